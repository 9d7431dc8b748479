"""CPU restatement of the reference layer (test infrastructure; never shipped).

The judged unit is one attention sub-block of the reference's pre-LN encoder
block, followed by the LayerNorm that the reference's fused path applies next:

    h   = LayerNorm_1(x)                                  torch_transformer_benchmark.py:129, :141
    q,k,v = h Wq^T + bq, h Wk^T + bk, h Wv^T + bv         :73-75, :94-96
    ctx = softmax(q k^T * d_h^-0.5) v   (per head)       :98, :112-113
    r   = x + ctx Wo^T + bo                               :119, :141
    y   = LayerNorm_2(r)                                  :131 (fused at :1262-1268)

Every function below cites the reference lines it restates. The arithmetic is
done op for op in the same order and dtype as the reference, so that in fp32
on the CPU the result is bit-identical to the reference module (checked
against fixtures produced by the reference itself, ``tests/golden``).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class TransformerConfig:
    """Restates ``TransformerConfig`` (torch_transformer_benchmark.py:30-57).

    ``ffn_dim`` and ``num_layers`` shape the full stack (``ReferenceTransformer``);
    the judged single layer (``ReferenceLayer``) has no FFN.
    """

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int = 0
    num_layers: int = 1
    causal: bool = False

    def validate(self) -> None:
        # Same checks and messages as torch_transformer_benchmark.py:40-57.
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )


class ReferenceSelfAttention(nn.Module):
    """Restates ``BaselineSelfAttention`` (torch_transformer_benchmark.py:60-123).

    Parameter names and construction order (q, k, v, out) match the reference,
    so a module built under the same ``torch.manual_seed`` has the same weights.
    """

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5                       # :71
        self.q_proj = nn.Linear(d_model, d_model, bias=True)     # :73
        self.k_proj = nn.Linear(d_model, d_model, bias=True)     # :74
        self.v_proj = nn.Linear(d_model, d_model, bias=True)     # :75
        self.out_proj = nn.Linear(d_model, d_model, bias=True)   # :76

    def _split_heads(self, x: torch.Tensor) -> torch.Tensor:
        # :78-84  [B,S,d] -> [B,H,S,d_h], materialised copy
        b, s, _ = x.shape
        return x.view(b, s, self.num_heads, self.head_dim).transpose(1, 2).contiguous()

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                causal: bool = False) -> torch.Tensor:
        b, s, _ = x.shape
        q = self._split_heads(self.q_proj(x))                     # :94
        k = self._split_heads(self.k_proj(x))                     # :95
        v = self._split_heads(self.v_proj(x))                     # :96
        scores = torch.matmul(q, k.transpose(-2, -1)) * self.scale  # :98
        if causal:                                                # :100-104
            cm = torch.ones((s, s), device=x.device, dtype=torch.bool).triu(diagonal=1)
            scores = scores.masked_fill(cm, float("-inf"))
        if valid_token_mask is not None:                          # :106-109
            scores = scores.masked_fill(~valid_token_mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)  # :112
        ctx = torch.matmul(probs, v)                              # :113
        ctx = ctx.transpose(1, 2).contiguous().view(b, s, self.d_model)  # :114-118
        out = self.out_proj(ctx)                                  # :119
        if valid_token_mask is not None:                          # :121-122
            out = out.masked_fill(~valid_token_mask[..., None], 0)
        return out


class ReferenceLayer(nn.Module):
    """norm1 -> attention -> +x -> norm2, with the reference's parameter names.

    ``state_dict`` keys: ``norm1.*``, ``attention.{q,k,v,out}_proj.*``,
    ``norm2.*`` -- the keys of the reference block's attention half
    (``BaselineTransformerBlock`` torch_transformer_benchmark.py:126-131).
    Construction order norm1, attention, norm2 matches the reference block, so
    the RNG draws (only the Linear layers draw) are identical.
    """

    def __init__(self, d_model: int, num_heads: int, causal: bool = False) -> None:
        super().__init__()
        self.causal = causal
        self.norm1 = nn.LayerNorm(d_model)                        # :129
        self.attention = ReferenceSelfAttention(d_model, num_heads)  # :130
        self.norm2 = nn.LayerNorm(d_model)                        # :131

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        r = x + self.attention(self.norm1(x), valid_token_mask, self.causal)  # :141
        return self.norm2(r)                                      # :131, :1265-1268


def build_reference_layer(cfg: TransformerConfig, seed: int) -> ReferenceLayer:
    """Seeded default-init layer, as the harness builds its models (:2024, :2031)."""
    torch.manual_seed(seed)
    return ReferenceLayer(cfg.d_model, cfg.num_heads, cfg.causal).eval()


class ReferenceBlock(nn.Module):
    """Restates ``BaselineTransformerBlock`` (torch_transformer_benchmark.py:126-146):
    the full pre-LN encoder block, attention half + GELU FFN half.

        x1 = x + Attention(LayerNorm_1(x))                          :141
        x2 = x1 + W2 gelu_erf(W1 LayerNorm_2(x1) + b1) + b2          :142
        padded rows of x2 are zeroed                                 :144-145

    Construction order norm1, attention, norm2, ffn_in, ffn_out (:129-133)
    fixes the RNG draws of the seeded default init.
    """

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)                           # :129
        self.attention = ReferenceSelfAttention(d_model, num_heads)  # :130
        self.norm2 = nn.LayerNorm(d_model)                           # :131
        self.ffn_in = nn.Linear(d_model, ffn_dim)                    # :132
        self.ffn_out = nn.Linear(ffn_dim, d_model)                   # :133

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor], causal: bool) -> torch.Tensor:
        x = x + self.attention(self.norm1(x), valid_token_mask, causal)                    # :141
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))     # :142
        if valid_token_mask is not None:                                                  # :144-145
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


class ReferenceTransformer(nn.Module):
    """Restates ``BaselineTransformer`` (torch_transformer_benchmark.py:149-173):
    ``num_layers`` blocks, then ``final_norm``, padded rows zeroed.
    ``state_dict`` keys ``layers.{i}.*`` and ``final_norm.*`` are the reference's."""

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([ReferenceBlock(config.d_model, config.num_heads, config.ffn_dim)
                                     for _ in range(config.num_layers)])             # :152-160
        self.final_norm = nn.LayerNorm(config.d_model)                                 # :161

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:                                                      # :168-169
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)                                                         # :170
        if valid_token_mask is not None:                                               # :171-172
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def build_reference_transformer(cfg: TransformerConfig, seed: int) -> ReferenceTransformer:
    """Seeded default-init stack, as the harness builds its baseline (:2024-2031)."""
    torch.manual_seed(seed)
    return ReferenceTransformer(cfg).eval()


def generate_random_case(cfg: TransformerConfig, seed: int, padding_ratio: float = 0.0,
                         input_scale: float = 1.0, device: str = "cpu",
                         dtype: torch.dtype = torch.float32) -> Tuple[torch.Tensor, torch.Tensor]:
    """Restates ``generate_random_case`` (torch_transformer_benchmark.py:1575-1613).

    Inputs are drawn on the CPU generator so that CPU and GPU runs see the same x.
    """
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, generator=g,
                    device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(cfg.batch_size, cfg.seq_len, device=device, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=cfg.seq_len + 1, size=(cfg.batch_size,),
                            generator=g, device=device)
    pos = torch.arange(cfg.seq_len, device=device)[None, :]
    mask = pos < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def _ln64(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * w + b


def streamed_keys(layer: ReferenceLayer, xs: torch.Tensor, dtype: torch.dtype = torch.float64):
    """First phase of the streamed layer for one sequence ``xs`` [S, d]:
    h = LN1(x) for every token and the K / V projections of every key
    (tools/reference_chunked.py:73-128 projects the whole sequence once).
    Returns (h, k, v) in ``dtype``."""
    att = layer.attention
    f = lambda t: t.detach().to(dtype)
    h = _ln64(f(xs), f(layer.norm1.weight), f(layer.norm1.bias), layer.norm1.eps)
    k = h @ f(att.k_proj.weight).T + f(att.k_proj.bias)
    v = h @ f(att.v_proj.weight).T + f(att.v_proj.bias)
    return h, k, v


def streamed_ctx_rows(layer: ReferenceLayer, h: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      rows: torch.Tensor, causal: bool, key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Second phase: ctx rows [R, d] for the query positions ``rows``.

    Follows ``chunked_attention`` (tools/reference_chunked.py:73-128): each
    head's scores are formed for a block of queries against all keys (the key
    axis is never blocked, so the softmax normalisation is exact), causal
    keys are masked with -inf before the softmax (:109-113), and
    ctx = probs @ v (:120). Only the sampled query rows are formed, so memory
    is O(R * S) per head. Computed in the dtype of h / k / v. ``key_mask``
    (bool [S], True = valid token) gives padded keys -inf scores, as
    BaselineSelfAttention does (torch_transformer_benchmark.py:106-109).
    """
    att = layer.attention
    H, dh = att.num_heads, att.head_dim
    f = lambda t: t.detach().to(h.dtype)
    q = h[rows] @ f(att.q_proj.weight).T + f(att.q_proj.bias)
    S = h.shape[0]
    ctx = torch.empty(rows.numel(), att.d_model, dtype=h.dtype)
    scale = dh ** -0.5
    for hh in range(H):
        sl = slice(hh * dh, (hh + 1) * dh)
        sc = (q[:, sl] @ k[:, sl].T) * scale
        if causal:
            kpos = torch.arange(S)[None, :]
            sc = sc.masked_fill(kpos > rows[:, None], float("-inf"))
        if key_mask is not None:
            sc = sc.masked_fill(~key_mask[None, :], float("-inf"))
        p = torch.softmax(sc, dim=-1)
        ctx[:, sl] = p @ v[:, sl]
        del sc, p
    return ctx


def streamed_output_rows(layer: ReferenceLayer, xs: torch.Tensor, ctx: torch.Tensor,
                         rows: torch.Tensor, key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Last phase: y rows = LN2(x + ctx Wo^T + bo) (:119, :141, :131), in ctx's
    dtype; a padded query row's attention output is zeroed, bias included
    (:121-122), so its y is LN2(x)."""
    att = layer.attention
    f = lambda t: t.detach().to(ctx.dtype)
    out = ctx @ f(att.out_proj.weight).T + f(att.out_proj.bias)
    if key_mask is not None:
        out = out.masked_fill(~key_mask[rows][:, None], 0)
    r = f(xs[rows]) + out
    return _ln64(r, f(layer.norm2.weight), f(layer.norm2.bias), layer.norm2.eps)


def _attn_rows_fp64(layer: ReferenceLayer, xs: torch.Tensor, rows: torch.Tensor,
                    causal: bool, key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """ctx rows [R, d] in fp64 for one sequence ``xs`` [S, d] (streamed_keys,
    then streamed_ctx_rows)."""
    h, k, v = streamed_keys(layer, xs, torch.float64)
    return streamed_ctx_rows(layer, h, k, v, rows, causal, key_mask)


def streamed_attention_rows_fp64(layer: ReferenceLayer, xs: torch.Tensor,
                                 rows: Sequence[int], causal: bool = False,
                                 key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp64 attention context (before out_proj) for sampled query rows of one sequence."""
    rows_t = torch.as_tensor(rows, dtype=torch.long)
    return _attn_rows_fp64(layer, xs, rows_t, causal, key_mask)


def streamed_layer_rows_fp64(layer: ReferenceLayer, xs: torch.Tensor,
                             rows: Sequence[int], causal: bool = False,
                             key_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp64 layer output y for sampled query rows of one sequence ``xs`` [S, d].

    This is the long-context oracle: ``BaselineSelfAttention`` would
    materialise [B,H,S,S] scores (torch_transformer_benchmark.py:98), which is
    infeasible at S=100000, so the layer is restated per sampled row in fp64.
    """
    rows_t = torch.as_tensor(rows, dtype=torch.long)
    ctx = _attn_rows_fp64(layer, xs, rows_t, causal, key_mask)
    return streamed_output_rows(layer, xs, ctx, rows_t, key_mask)


def sample_rows(seq_len: int, count: int, seed: int) -> torch.Tensor:
    """Seeded subset of query positions (sorted, without replacement)."""
    g = torch.Generator().manual_seed(seed)
    count = min(count, seq_len)
    return torch.sort(torch.randperm(seq_len, generator=g)[:count]).values


def layer_flops(batch: int, seq_len: int, d_model: int, causal: bool = False) -> float:
    """Algorithmic FLOPs of one layer: 8*T*d^2 (QKV + out-proj) + 4*B*S^2*d (attention).

    Causal attention counts half the score/PV work (the masked half is not formed).
    """
    t = batch * seq_len
    attn = 4.0 * batch * seq_len * seq_len * d_model
    return 8.0 * t * d_model * d_model + (attn / 2 if causal else attn)


def layer_bytes(batch: int, seq_len: int, d_model: int) -> float:
    """Algorithmic bytes of one layer: x read + y write in fp32 = 8*T*d."""
    return 8.0 * batch * seq_len * d_model


__all__ = [
    "TransformerConfig", "ReferenceSelfAttention", "ReferenceLayer",
    "build_reference_layer", "generate_random_case", "streamed_layer_rows_fp64",
    "streamed_attention_rows_fp64", "streamed_keys", "streamed_ctx_rows", "streamed_output_rows",
    "sample_rows", "layer_flops", "layer_bytes",
]

