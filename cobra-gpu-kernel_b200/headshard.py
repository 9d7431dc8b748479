"""Head-sharded layer forward, one process per GPU over ``torch.distributed``.

Batch sharding (``sharding.py``) leaves ranks idle when the batch has fewer
sequences than there are ranks (the cfg1 benchmark shape: B = 4 on 8 GPUs). The heads of
one layer are independent up to the out-projection
(torch_transformer_benchmark.py:94-118: q, k, v and the softmax are per head),
so they can be split instead: rank r computes LN1, the q / k / v projections
and the attention of heads [h0, h1) for the whole batch, and the caller's rank
gathers every rank's ctx columns, after which the out-projection, which mixes
all heads (:119), the residual and LN2 run there. Unlike batch sharding this
needs a data-path exchange: the caller broadcasts x, and every rank sends its
ctx columns (T x (h1 - h0) * d_h fp16) back.

Contiguous head ranges of ceil(H / n) heads per rank; ranks past the last
range only take part in the broadcasts. Failure behaviour is that of
``sharded_forward``: the input is validated on the caller's rank and the
verdict is broadcast, so a bad input raises the same ``ValueError`` on every
rank; a rank that fails later leaves its peers in a transfer that the process
group's timeout ends.

The per-rank compute comes from two methods of the layer:
``_head_ctx(x, mask, h0, h1)`` -> ctx columns of heads [h0, h1) as
[B*S, (h1 - h0) * d_h] of dtype ``layer.ctx_dtype`` (fp16 when absent), and
``_finish_from_ctx(x, mask, ctx)`` -> y from the full ctx [B*S, d].
``B200TransformerLayer`` implements them with the C ABI (K1 and K2 with
``local_heads``, then K3).
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .sharding import _HDR_MESSAGES, _HDR_OK, _default_device, _validate

__all__ = ["head_shards", "head_sharded_forward", "HeadShardedLayer"]


def head_shards(heads: int, world: int) -> List[Tuple[int, int]]:
    """Half-open head ranges [h0, h1) for ranks 0..world-1: contiguous runs
    of ceil(heads / world) heads; ranks past the last run get an empty range."""
    if heads <= 0 or world <= 0:
        raise ValueError(f"bad heads/world: {heads}, {world}")
    per = -(-heads // world)
    out = []
    for r in range(world):
        a = min(heads, r * per)
        b = min(heads, a + per)
        out.append((a, b))
    return out


def head_sharded_forward(layer, x: Optional[torch.Tensor] = None,
                         valid_token_mask: Optional[torch.Tensor] = None, *, src: int = 0,
                         group: Optional[dist.ProcessGroup] = None,
                         device: Optional[torch.device] = None) -> Optional[torch.Tensor]:
    """Run ``layer`` on the batch of ``x`` with its heads split across the ranks of ``group``.

    Collective: every rank of ``group`` calls it with the same (replicated)
    layer; ``x`` (fp32 [B, S, d] on this rank's device) and the optional
    ``valid_token_mask`` ([B, S] bool) are read on ``src`` only. Returns y
    [B, S, d] on ``src`` and ``None`` on every other rank.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    src_g = dist.get_global_rank(group, src) if group is not None else src
    backend = dist.get_backend(group)
    if rank == src:
        device = x.device if x is not None else (device or _default_device(backend))
    elif device is None:
        device = _default_device(backend)

    hdr = torch.zeros(5, dtype=torch.int64, device=device)
    if rank == src:
        status = _validate(x, valid_token_mask)
        hdr[0] = status
        if status == _HDR_OK:
            hdr[1:4] = torch.tensor(x.shape, dtype=torch.int64)
            hdr[4] = 1 if valid_token_mask is not None else 0
    dist.broadcast(hdr, src_g, group=group)
    status, B, S, d, has_mask = (int(v) for v in hdr.tolist())
    if status != _HDR_OK:
        raise ValueError(f"head_sharded_forward: {_HDR_MESSAGES[status]} (validated on rank {src})")

    # Every rank needs the whole batch (and its mask): broadcast from src.
    if rank == src:
        xb = x.contiguous()
        mb = valid_token_mask.to(torch.uint8).contiguous() if has_mask else None
    else:
        xb = torch.empty(B, S, d, dtype=torch.float32, device=device)
        mb = torch.empty(B, S, dtype=torch.uint8, device=device) if has_mask else None
    dist.broadcast(xb, src_g, group=group)
    if mb is not None:
        dist.broadcast(mb, src_g, group=group)
    mask = mb.bool() if mb is not None else None

    H = layer.attention.num_heads
    dh = d // H
    shards = head_shards(H, world)
    h0, h1 = shards[rank]
    part = layer._head_ctx(xb, mask, h0, h1) if h1 > h0 else None

    if rank != src:
        if part is not None:
            dist.send(part.contiguous(), src_g, group=group)
        return None
    T = B * S
    ctx = None
    for r, (a, b) in enumerate(shards):
        if b == a:
            continue
        if r == src:
            piece = part
        else:
            peer = dist.get_global_rank(group, r) if group is not None else r
            piece = torch.empty(T, (b - a) * dh, dtype=getattr(layer, "ctx_dtype", torch.float16), device=device)
            dist.recv(piece, peer, group=group)
        if ctx is None:
            ctx = torch.empty(T, d, dtype=piece.dtype, device=device)
        ctx[:, a * dh:b * dh].copy_(piece)
    return layer._finish_from_ctx(xb, mask, ctx)


class HeadShardedLayer(torch.nn.Module):
    """``forward(x, valid_token_mask=None)`` of a replicated layer with its heads
    split over the ranks of a process group; see ``head_sharded_forward``."""

    def __init__(self, layer: torch.nn.Module, *, src: int = 0,
                 group: Optional[dist.ProcessGroup] = None) -> None:
        super().__init__()
        self.layer = layer
        self.src = src
        self.group = group

    def forward(self, x: Optional[torch.Tensor] = None,
                valid_token_mask: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        return head_sharded_forward(self.layer, x, valid_token_mask, src=self.src, group=self.group)
