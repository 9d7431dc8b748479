"""Drop-in ``nn.Module`` for the reference's single transformer-layer forward.

``B200TransformerLayer`` has the parameter names of the reference's block
(``norm1``, ``attention.{q,k,v,out}_proj``, ``norm2``;
torch_transformer_benchmark.py:126-131, :73-76), loads the reference's
``state_dict`` with ``strict=True`` and registers nothing else, packs weights
lazily on the first forward (as ``UserOptimizedTransformer._prepare`` does,
:948-1081, :1524-1525), and computes

    y = LayerNorm_2(x + Attention(LayerNorm_1(x)))

through the sm_100a library (``include/cobra_b200.h``): one persistent
whole-layer kernel for d_model 64/128 with head_dim 32 and S <= 128, else K1
LN1+QKV GEMM, K2 flash attention, K3 out-proj + residual + LN2. Inputs up to
64 MiB replay a captured CUDA graph (the reference's ``_run_graphed``,
:1331-1360). An optional key-padding mask follows BaselineSelfAttention
(:106-109, :121-122).

The computation always runs on the GPU that holds the parameters: a
host-resident x is streamed through it in chunks (the reference's
``_run_streamed``, :1418-1508) and comes back as a host tensor; a layer whose
parameters are on the CPU raises (there is no CPU path).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from . import _lib

GRAPH_MAX_INPUT_BYTES = 64 * 1024 * 1024   # reference gate, torch_transformer_benchmark.py:1077-1079
_REDUCED = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}   # converted at the boundary
HOST_CHUNK_BYTES = 16 * 1024 * 1024        # about this many x bytes per chunk when streaming a host batch


def host_chunk_seqs(B: int, S: int, d: int, H: int, sms: int) -> int:
    """Sequences per chunk when a host-resident batch streams through the GPU.

    About HOST_CHUNK_BYTES of x per chunk, shaped so that each launch fills
    the GPU: the whole-layer kernel (short sequences) walks sequence pairs,
    one pair per SM at a time, so a chunk is a multiple of 2 x SMs sequences;
    for longer sequences a chunk holds at least two sequences when the batch
    has four or more, so the next chunk's copy overlaps a launch with enough
    work items that its last wave is a small share."""
    per_seq = max(1, S * d * 4)
    if _lib.fused_shape(S, d, H):
        unit = 2 * max(1, sms)
        cb = unit * max(1, round(HOST_CHUNK_BYTES / (unit * per_seq)))
    else:
        cb = max(1, HOST_CHUNK_BYTES // per_seq)
        if cb == 1 and B >= 4:
            cb = 2
    return max(1, min(B, cb))


@dataclass(frozen=True)
class TransformerConfig:
    """Mirror of the reference's ``TransformerConfig`` (:30-57).

    Only ``d_model``, ``num_heads`` and ``causal`` shape the layer; the batch
    and sequence sizes come from the input. ``ffn_dim``/``num_layers`` are
    accepted for signature compatibility and must describe a single layer
    without FFN (0 or 1)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int = 0
    num_layers: int = 1
    causal: bool = False

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by num_heads ({self.num_heads})")
        if self.num_layers != 1:
            raise ValueError("B200TransformerLayer is a single layer (num_layers must be 1)")


class SelfAttentionWeights(nn.Module):
    """Parameter holder with ``BaselineSelfAttention``'s names (:60-76).

    The attention itself runs inside the fused kernels, so this module has no
    forward of its own."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)


class _Pack:
    """Device-resident packed weights (plain attributes, not registered:
    the reference keeps them out of ``state_dict`` for the same reason,
    :857-865)."""

    __slots__ = ("wqkv16", "bqkv32", "wo16", "ln", "device", "versions")


class B200TransformerLayer(nn.Module):
    """LN1 -> MHA -> +x -> LN2 on B200, with the reference's API.

    ``forward(x, valid_token_mask=None)``: x is fp32 [B, S, d] on an sm_100
    device; ``valid_token_mask`` is an optional [B, S] bool key-padding mask
    on the same device (True = valid): invalid keys get probability 0 and an
    invalid query row's attention output is zeroed, so its y is LN2(x)
    (BaselineSelfAttention :106-109, :121-122). The returned tensor may be an
    internal static buffer that the next call overwrites (as the reference's
    graph path returns, :1356-1360): copy it if it must outlive the next call.
    """

    # forward(..., out=y) writes into a caller-provided tensor (used by the
    # batch-sharded path to write each slice straight into its gather buffer).
    accepts_out = True
    # dtype of the ctx columns _head_ctx returns (head sharding).
    ctx_dtype = torch.float16

    def __init__(self, d_model: int, num_heads: int, causal: bool = False, *,
                 use_graphs: bool = True) -> None:
        super().__init__()
        self.causal = bool(causal)
        self.use_graphs = use_graphs
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = SelfAttentionWeights(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self._pack: Optional[_Pack] = None
        self._ws: Optional[torch.Tensor] = None
        self._ws_off = 0
        self._ws_bytes = 0
        self._sig = None
        self._graph = None
        self._static_x = None
        self._static_y = None
        self._static_m = None
        self._host_out = None
        self._io_streams = None
        self._warm = set()
        self._head_packs = {}
        self._hws: Optional[torch.Tensor] = None
        self.register_load_state_dict_post_hook(lambda mod, _keys: mod.invalidate())

    @classmethod
    def from_config(cls, config, **kw) -> "B200TransformerLayer":
        if hasattr(config, "validate"):
            config.validate()
        return cls(config.d_model, config.num_heads, bool(getattr(config, "causal", False)), **kw)

    # ------------------------------------------------------------ state
    def invalidate(self) -> None:
        """Drop packed weights and captured graphs (weights changed)."""
        self._pack = None
        self._head_packs = {}
        self._graph = None
        self._static_x = self._static_y = self._static_m = None
        self._sig = None

    def _param_versions(self):
        # Parameters created under torch.inference_mode() carry no version
        # counter; their storage address still identifies a replaced tensor
        # (in-place edits of such weights need an explicit invalidate()).
        return tuple((p.data_ptr(), 0 if p.is_inference() else p._version) for p in self.parameters())

    def _ensure_pack(self, device: torch.device) -> _Pack:
        pk = self._pack
        if pk is not None and pk.device == device and pk.versions == self._param_versions():
            return pk
        self._graph = None
        att = self.attention
        d = att.d_model
        L = _lib.lib()

        def dev32(t: torch.Tensor) -> torch.Tensor:
            return t.detach().to(device=device, dtype=torch.float32).contiguous()

        wq, wk, wv, wo = (dev32(m.weight) for m in (att.q_proj, att.k_proj, att.v_proj, att.out_proj))
        bq, bk, bv = (dev32(m.bias) for m in (att.q_proj, att.k_proj, att.v_proj))
        pk = _Pack()
        pk.wqkv16 = torch.empty(3 * d, d, dtype=torch.float16, device=device)
        pk.bqkv32 = torch.empty(3 * d, dtype=torch.float32, device=device)
        pk.wo16 = torch.empty(d, d, dtype=torch.float16, device=device)
        pk.ln = tuple(dev32(t) for t in (self.norm1.weight, self.norm1.bias, att.out_proj.bias,
                                          self.norm2.weight, self.norm2.bias))
        stream = torch.cuda.current_stream(device).cuda_stream
        with torch.cuda.device(device):
            _lib.check(L.b200l_pack_weights(
                d, wq.data_ptr(), wk.data_ptr(), wv.data_ptr(), bq.data_ptr(), bk.data_ptr(),
                bv.data_ptr(), wo.data_ptr(), pk.wqkv16.data_ptr(), pk.bqkv32.data_ptr(),
                pk.wo16.data_ptr(), stream))
        # Keep the fp32 staging copies alive until the pack kernel has run.
        torch.cuda.current_stream(device).synchronize()
        pk.device = device
        pk.versions = self._param_versions()
        self._pack = pk
        return pk

    def _desc(self, B: int, S: int, pk: _Pack, mask: Optional[torch.Tensor] = None) -> _lib.LayerDesc:
        att = self.attention
        ln1w, ln1b, bo, ln2w, ln2b = pk.ln
        return _lib.LayerDesc(
            batch=B, seq_len=S, d_model=att.d_model, num_heads=att.num_heads,
            causal=1 if self.causal else 0, eps1=float(self.norm1.eps), eps2=float(self.norm2.eps),
            wqkv=pk.wqkv16.data_ptr(), bqkv=pk.bqkv32.data_ptr(), wo=pk.wo16.data_ptr(),
            bo=bo.data_ptr(), ln1_w=ln1w.data_ptr(), ln1_b=ln1b.data_ptr(),
            ln2_w=ln2w.data_ptr(), ln2_b=ln2b.data_ptr(),
            valid_mask=mask.data_ptr() if mask is not None else None)

    def _ensure_workspace(self, desc: _lib.LayerDesc, device: torch.device, stepwise: bool = False) -> None:
        """Grow the workspace to what ``b200l_layer_forward`` needs for this
        shape (the status block alone for the whole-layer kernel), or with
        ``stepwise`` to what the per-kernel entry points need."""
        L = _lib.lib()
        fn = L.b200l_kernel_workspace_bytes if stepwise else L.b200l_layer_workspace_bytes
        need = fn(ctypes.byref(desc))
        if need == 0:
            raise _lib.B200LError(-1, _lib.last_error())
        if self._ws is None or self._ws.device != device or self._ws_bytes < need:
            self._ws = None
            buf = torch.empty(need + 1024, dtype=torch.uint8, device=device)
            off = (-buf.data_ptr()) % 1024
            self._ws, self._ws_off, self._ws_bytes = buf, off, need
            with torch.cuda.device(device):
                _lib.check(L.b200l_clear_status(self.workspace_ptr,
                                                torch.cuda.current_stream(device).cuda_stream))

    @property
    def workspace_ptr(self) -> int:
        return self._ws.data_ptr() + self._ws_off

    # ------------------------------------------------------------ compute
    def _launch(self, x: torch.Tensor, y: torch.Tensor, desc: _lib.LayerDesc) -> None:
        L = _lib.lib()
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(L.b200l_layer_forward(ctypes.byref(desc), x.data_ptr(), y.data_ptr(),
                                         self.workspace_ptr, self._ws_bytes, stream))

    def check_status(self) -> None:
        """Synchronise and raise if a kernel recorded a device-side failure."""
        if self._ws is None:
            return
        L = _lib.lib()
        with torch.cuda.device(self._ws.device):
            rc = L.b200l_read_status(self.workspace_ptr,
                                     torch.cuda.current_stream(self._ws.device).cuda_stream)
        _lib.check(rc)

    # ------------------------------------------------------------ head sharding
    def _head_pack(self, device: torch.device, h0: int, h1: int):
        """fp16 q|k|v weight rows and fp32 biases of heads [h0, h1) on ``device``."""
        versions = self._param_versions()
        key = (device, h0, h1)
        hp = self._head_packs.get(key)
        if hp is not None and hp[2] == versions:
            return hp
        att = self.attention
        sl = slice(h0 * att.head_dim, h1 * att.head_dim)
        w = torch.cat([m.weight[sl] for m in (att.q_proj, att.k_proj, att.v_proj)]).detach()
        w = w.to(device=device, dtype=torch.float32).contiguous()
        b = torch.cat([m.bias[sl] for m in (att.q_proj, att.k_proj, att.v_proj)]).detach()
        b = b.to(device=device, dtype=torch.float32).contiguous()
        w16 = torch.empty(w.shape, dtype=torch.float16, device=device)
        with torch.cuda.device(device):
            _lib.check(_lib.lib().b200l_cast_f16(w.data_ptr(), w16.data_ptr(), w.numel(),
                                                 torch.cuda.current_stream(device).cuda_stream))
        torch.cuda.current_stream(device).synchronize()   # w (fp32 staging) is read
        hp = (w16, b, versions)
        self._head_packs[key] = hp
        return hp

    def _head_ctx(self, x: torch.Tensor, mask: Optional[torch.Tensor], h0: int, h1: int) -> torch.Tensor:
        """ctx columns of heads [h0, h1) for the whole batch, fp16 [B*S, (h1-h0)*d_h]:
        K1 (LN1 + the q / k / v projections of those heads) and K2 through the
        C ABI with ``local_heads`` (used by ``headshard.head_sharded_forward``)."""
        B, S, _ = x.shape
        dev = x.device
        L = _lib.lib()
        m8 = mask.to(torch.bool).contiguous().view(torch.uint8) if mask is not None else None
        with torch.cuda.device(dev):
            pk = self._ensure_pack(dev)
            w16, b32, _ = self._head_pack(dev, h0, h1)
            desc = self._desc(B, S, pk, m8)
            desc.wqkv, desc.bqkv, desc.local_heads = w16.data_ptr(), b32.data_ptr(), h1 - h0
            need = L.b200l_kernel_workspace_bytes(ctypes.byref(desc))
            if need == 0:
                raise _lib.B200LError(-1, _lib.last_error())
            if self._hws is None or self._hws.device != dev or self._hws.numel() < need + 1024:
                self._hws = None
                self._hws = torch.zeros(need + 1024, dtype=torch.uint8, device=dev)
            off = (-self._hws.data_ptr()) % 1024
            ws = self._hws.data_ptr() + off
            st = torch.cuda.current_stream(dev).cuda_stream
            _lib.check(L.b200l_clear_status(ws, st))
            _lib.check(L.b200l_qkv_ln_gemm(ctypes.byref(desc), x.data_ptr(), ws, need, st))
            _lib.check(L.b200l_flash_attn(ctypes.byref(desc), ws, need, st))
            _lib.check(L.b200l_read_status(ws, st))
            lay = _lib.workspace_layout(B, S, self.attention.d_model, self.attention.num_heads, h1 - h0)
            n = B * S * lay["dq"]
            ctx = self._hws[off + lay["ctx"]:off + lay["ctx"] + 2 * n].view(torch.float16)
            return ctx.view(B * S, lay["dq"]).clone()

    def _finish_from_ctx(self, x: torch.Tensor, mask: Optional[torch.Tensor], ctx: torch.Tensor) -> torch.Tensor:
        """y = LN2(x + ctx Wo^T + bo) from every head's ctx (fp16 [B*S, d]): K3
        through the C ABI on this layer's own workspace."""
        B, S, d = x.shape
        dev = x.device
        L = _lib.lib()
        m8 = mask.to(torch.bool).contiguous().view(torch.uint8) if mask is not None else None
        with torch.cuda.device(dev):
            pk = self._ensure_pack(dev)
            desc = self._desc(B, S, pk, m8)
            self._ensure_workspace(desc, dev, stepwise=True)
            lay = _lib.workspace_layout(B, S, d, self.attention.num_heads)
            base = self._ws[self._ws_off + lay["ctx"]:self._ws_off + lay["ctx"] + 2 * B * S * d]
            base.view(torch.float16).view(B * S, d).copy_(ctx)
            y = torch.empty_like(x)
            _lib.check(L.b200l_outproj_res_ln(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), self.workspace_ptr,
                                              self._ws_bytes, torch.cuda.current_stream(dev).cuda_stream))
            return y

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None, *,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = LN2(x + Attn(LN1(x))); ``out`` (optional, device x only): a
        contiguous fp32 tensor of x's shape on x's device that receives y
        (no CUDA-graph replay, no static buffer); it is returned."""
        if x.dim() != 3 or x.shape[-1] != self.attention.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.attention.d_model}], got {tuple(x.shape)}")
        if x.dtype in _REDUCED:
            return self._forward_reduced(x, valid_token_mask, out)
        if x.dtype != torch.float32:
            raise TypeError(f"B200TransformerLayer takes fp32, fp16 or bf16 x; got {x.dtype}")
        if out is not None and (not x.is_cuda or out.device != x.device or out.shape != x.shape
                                or out.dtype != torch.float32 or not out.is_contiguous()):
            raise ValueError("out must be a contiguous fp32 tensor of x's shape on x's (CUDA) device")
        if not x.is_cuda:
            if self.norm1.weight.is_cuda:
                # Host-resident input, parameters on the GPU: stream it through
                # the device (the reference's _run_streamed, :1418-1508).
                return self._forward_host(x, valid_token_mask)
            raise RuntimeError("B200TransformerLayer runs only on CUDA (sm_100a) devices; there is no CPU path")
        B, S, _ = x.shape
        mask = None
        if valid_token_mask is not None:
            # [B, S], True = valid token. Used as its raw bytes (0 / nonzero),
            # as the reference's fused path does (:1205-1207); no host sync.
            if tuple(valid_token_mask.shape) != (B, S):
                raise ValueError(f"valid_token_mask must have shape {(B, S)}, got {tuple(valid_token_mask.shape)}")
            if valid_token_mask.device != x.device:
                raise ValueError("valid_token_mask must be on the same device as x")
            mask = valid_token_mask.to(torch.bool).contiguous().view(torch.uint8)
        x = x.contiguous()
        with torch.cuda.device(x.device):
            pk = self._ensure_pack(x.device)
            desc = self._desc(B, S, pk, mask)
            self._ensure_workspace(desc, x.device)
            sig = (B, S, x.device, mask is not None)
            if sig != self._sig:
                self._sig = sig
                self._graph = None
                self._static_x = self._static_y = self._static_m = None
            small = x.numel() * x.element_size() <= GRAPH_MAX_INPUT_BYTES
            if self.use_graphs and small and out is None:
                return self._run_graphed(x, mask, pk)
            y = out if out is not None else torch.empty_like(x)
            self._launch(x, y, desc)
            return y

    def _forward_reduced(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                         out: Optional[torch.Tensor]) -> torch.Tensor:
        """fp16 / bf16 x (the reference's --dtype float16 / bfloat16 modes,
        torch_transformer_benchmark.py:952-962): converted to fp32 on the GPU
        by b200l_convert, run through the fp32 layer, and y converted back to
        x's dtype (round to nearest even). A host-resident x is widened on the
        host and streamed as fp32."""
        code = _REDUCED[x.dtype]
        if not x.is_cuda:
            if out is not None:
                raise ValueError("out= needs a CUDA x")
            return self.forward(x.float(), valid_token_mask).to(x.dtype)
        if out is not None and (out.device != x.device or out.shape != x.shape or out.dtype != x.dtype
                                or not out.is_contiguous()):
            raise ValueError("out must be a contiguous tensor of x's shape, dtype and device")
        x = x.contiguous()
        L = _lib.lib()
        n = x.numel()
        with torch.cuda.device(x.device):
            st = torch.cuda.current_stream(x.device).cuda_stream
            x32 = torch.empty(x.shape, dtype=torch.float32, device=x.device)
            _lib.check(L.b200l_convert(x.data_ptr(), code, x32.data_ptr(), _lib.DTYPE_F32, n, st))
            y32 = self.forward(x32, valid_token_mask)
            y = out if out is not None else torch.empty(x.shape, dtype=x.dtype, device=x.device)
            _lib.check(L.b200l_convert(y32.data_ptr(), _lib.DTYPE_F32, y.data_ptr(), code, n, st))
        return y

    def warmup(self, seq_len: int, device: torch.device, with_mask: bool = False) -> None:
        """Pack the weights and run one single-sequence forward of this shape
        class on ``device`` (zeros), so that the kernels it launches are
        loaded before the caller starts other device work -- e.g. NCCL
        transfers in flight, which a lazily loaded kernel must not wait on.
        Runs once per (seq_len, device, mask) combination."""
        key = (int(seq_len), torch.device(device), bool(with_mask))
        if key in self._warm:
            return
        d = self.attention.d_model
        x = torch.zeros(1, seq_len, d, dtype=torch.float32, device=device)
        m = torch.ones(1, seq_len, dtype=torch.bool, device=device) if with_mask else None
        saved, self.use_graphs = self.use_graphs, False
        try:
            with torch.inference_mode():
                self.forward(x, m)
            torch.cuda.current_stream(device).synchronize()
        finally:
            self.use_graphs = saved
        self._warm.add(key)

    def _forward_host(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
        """Host x -> host y through the GPU that holds the parameters.

        Sequences are independent (:1446-1447), so the batch moves in chunks
        (``host_chunk_seqs``) through a three-stream pipeline: host-to-
        device copies on one stream, the layer on the caller's current stream,
        device-to-host copies on a third, with two device buffers for each of
        x and y. Both PCIe directions and the kernels overlap, so the call
        costs about one direction's transfer time. Pinned host memory makes
        the copies asynchronous; the result is a pinned host buffer owned by
        the module (overwritten by the next host call), complete on return.
        """
        dev = self.norm1.weight.device
        B, S, d = x.shape
        mask = None
        if valid_token_mask is not None:
            if tuple(valid_token_mask.shape) != (B, S):
                raise ValueError(f"valid_token_mask must have shape {(B, S)}, got {tuple(valid_token_mask.shape)}")
            mask = valid_token_mask.to(torch.bool).contiguous().view(torch.uint8)
        x = x.contiguous()
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        cb = host_chunk_seqs(B, S, d, self.attention.num_heads, sms)
        with torch.cuda.device(dev):
            pk = self._ensure_pack(dev)
            self._ensure_workspace(self._desc(cb, S, pk), dev)
            if self._host_out is None or self._host_out.shape != x.shape:
                self._host_out = None
                self._host_out = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
            out = self._host_out
            if self._io_streams is None or self._io_streams[0].device != dev:
                self._io_streams = (torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev))
            h2d, d2h = self._io_streams
            comp = torch.cuda.current_stream(dev)
            nbuf = 2 if B > cb else 1
            xb = [torch.empty(cb, S, d, dtype=torch.float32, device=dev) for _ in range(nbuf)]
            yb = [torch.empty(cb, S, d, dtype=torch.float32, device=dev) for _ in range(nbuf)]
            mb = [torch.empty(cb, S, dtype=torch.uint8, device=dev) for _ in range(nbuf)] if mask is not None else None
            ev_in = [torch.cuda.Event() for _ in range(nbuf)]
            ev_comp = [torch.cuda.Event() for _ in range(nbuf)]
            ev_out = [torch.cuda.Event() for _ in range(nbuf)]
            h2d.wait_stream(comp)      # device buffers were just allocated on comp
            for i, b0 in enumerate(range(0, B, cb)):
                b1 = min(B, b0 + cb)
                n, k = b1 - b0, i % nbuf
                with torch.cuda.stream(h2d):
                    if i >= nbuf:
                        h2d.wait_event(ev_comp[k])        # the layer is done reading xb[k]
                    xb[k][:n].copy_(x[b0:b1], non_blocking=True)
                    if mb is not None:
                        mb[k][:n].copy_(mask[b0:b1], non_blocking=True)
                    ev_in[k].record(h2d)
                comp.wait_event(ev_in[k])
                if i >= nbuf:
                    comp.wait_event(ev_out[k])            # yb[k] has been copied out
                self._launch(xb[k][:n], yb[k][:n], self._desc(n, S, pk, mb[k][:n] if mb is not None else None))
                ev_comp[k].record(comp)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_comp[k])
                    out[b0:b1].copy_(yb[k][:n], non_blocking=True)
                    ev_out[k].record(d2h)
            comp.wait_stream(d2h)
            comp.wait_stream(h2d)
            comp.synchronize()         # y is complete on the host; the buffers are idle
        return out

    def _run_graphed(self, x: torch.Tensor, mask: Optional[torch.Tensor], pk: _Pack) -> torch.Tensor:
        """Capture the layer once per shape (and mask / no mask), then copy x
        (and the mask) into the static buffers and replay."""
        if self._graph is None:
            self._static_x = x.clone()
            self._static_y = torch.empty_like(x)
            self._static_m = mask.clone() if mask is not None else None
            B, S, _ = x.shape
            desc = self._desc(B, S, pk, self._static_m)
            side = torch.cuda.Stream(device=x.device)
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                self._launch(self._static_x, self._static_y, desc)   # sets kernel attributes
            torch.cuda.current_stream(x.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            # thread_local: other threads (e.g. a NCCL watchdog) may keep
            # making CUDA calls while this thread captures.
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._launch(self._static_x, self._static_y, desc)
            self._graph = g
        self._static_x.copy_(x)
        if mask is not None:
            self._static_m.copy_(mask)
        self._graph.replay()
        return self._static_y
