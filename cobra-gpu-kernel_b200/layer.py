"""Drop-in ``nn.Module`` for the reference's single transformer-layer forward.

``B200TransformerLayer`` has the parameter names of the reference's block
(``norm1``, ``attention.{q,k,v,out}_proj``, ``norm2``;
torch_transformer_benchmark.py:126-131, :73-76), loads the reference's
``state_dict`` with ``strict=True`` and registers nothing else, packs weights
lazily on the first forward (as ``UserOptimizedTransformer._prepare`` does,
:948-1081, :1524-1525), and computes

    y = LayerNorm_2(x + Attention(LayerNorm_1(x)))

through the sm_100a library (``include/cobra_b200.h``): K1 LN1+QKV GEMM,
K2 flash attention, K3 out-proj + residual + LN2. Small inputs replay a CUDA
graph of the three launches (the reference's ``_run_graphed``, :1331-1360).

There is no CPU path: inputs must be fp32 CUDA tensors on an sm_100 device.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from . import _lib

GRAPH_MAX_INPUT_BYTES = 64 * 1024 * 1024   # reference gate, torch_transformer_benchmark.py:1077-1079


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
    device. The returned tensor may be an internal static buffer that the
    next call overwrites (as the reference's graph path returns,
    :1356-1360): copy it if it must outlive the next call.
    """

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
        self._graph = None
        self._static_x = self._static_y = None
        self._sig = None

    def _param_versions(self):
        return tuple(p._version for p in self.parameters())

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

    def _desc(self, B: int, S: int, pk: _Pack) -> _lib.LayerDesc:
        att = self.attention
        ln1w, ln1b, bo, ln2w, ln2b = pk.ln
        return _lib.LayerDesc(
            batch=B, seq_len=S, d_model=att.d_model, num_heads=att.num_heads,
            causal=1 if self.causal else 0, eps1=float(self.norm1.eps), eps2=float(self.norm2.eps),
            wqkv=pk.wqkv16.data_ptr(), bqkv=pk.bqkv32.data_ptr(), wo=pk.wo16.data_ptr(),
            bo=bo.data_ptr(), ln1_w=ln1w.data_ptr(), ln1_b=ln1b.data_ptr(),
            ln2_w=ln2w.data_ptr(), ln2_b=ln2b.data_ptr())

    def _ensure_workspace(self, desc: _lib.LayerDesc, device: torch.device) -> None:
        L = _lib.lib()
        need = L.b200l_layer_workspace_bytes(ctypes.byref(desc))
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

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dim() != 3 or x.shape[-1] != self.attention.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.attention.d_model}], got {tuple(x.shape)}")
        if not x.is_cuda:
            raise RuntimeError("B200TransformerLayer runs only on CUDA (sm_100a) devices; there is no CPU path")
        if x.dtype != torch.float32:
            raise TypeError(f"B200TransformerLayer computes fp32-in/fp32-out; got {x.dtype}")
        if valid_token_mask is not None and not bool(valid_token_mask.all()):
            raise NotImplementedError("key-padding masks with padded positions are not supported yet")
        B, S, _ = x.shape
        x = x.contiguous()
        with torch.cuda.device(x.device):
            pk = self._ensure_pack(x.device)
            desc = self._desc(B, S, pk)
            self._ensure_workspace(desc, x.device)
            sig = (B, S, x.device)
            if sig != self._sig:
                self._sig = sig
                self._graph = None
                self._static_x = self._static_y = None
            small = x.numel() * x.element_size() <= GRAPH_MAX_INPUT_BYTES
            if self.use_graphs and small:
                return self._run_graphed(x, desc)
            y = torch.empty_like(x)
            self._launch(x, y, desc)
            return y

    def _run_graphed(self, x: torch.Tensor, desc: _lib.LayerDesc) -> torch.Tensor:
        """Capture K1->K2->K3 once per shape, then copy x in and replay."""
        if self._graph is None:
            self._static_x = x.clone()
            self._static_y = torch.empty_like(x)
            side = torch.cuda.Stream(device=x.device)
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                self._launch(self._static_x, self._static_y, desc)   # sets kernel attributes
            torch.cuda.current_stream(x.device).wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch(self._static_x, self._static_y, desc)
            self._graph = g
        self._static_x.copy_(x)
        self._graph.replay()
        return self._static_y
