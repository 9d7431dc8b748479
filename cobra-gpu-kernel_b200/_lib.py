"""ctypes binding of the C ABI in ``include/cobra_b200.h``.

The library is the only compute path: if it cannot be loaded (or built from
the in-tree sources when nvcc is present) every entry point raises. There is
no CPU or PyTorch fallback.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int, c_int32, c_size_t, c_void_p

from . import build as _build

EXPORTED = (
    "b200l_version", "b200l_last_error", "b200l_layer_workspace_bytes",
    "b200l_clear_status", "b200l_read_status", "b200l_pack_weights",
    "b200l_layer_forward", "b200l_qkv_ln_gemm", "b200l_flash_attn",
    "b200l_outproj_res_ln", "b200l_layer_forward_noalloc", "b200l_block_workspace_bytes",
    "b200l_block_forward", "b200l_row_layernorm", "b200l_cast_f16",
    "b200l_kernel_workspace_bytes", "b200l_debug_arm", "b200l_noalloc_read_status",
    "b200l_convert",
)

# Element types of b200l_convert.
DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2

ABI_VERSION = 4

# Fault-injection sites of b200l_debug_arm (test hook for the bounded waits).
DEBUG_SITE_NONE = 0
DEBUG_SITE_ATTN_KV = 1
DEBUG_SITE_GEMM_OPERAND = 2

# Size of the library's built-in scratch used by b200l_layer_forward_noalloc.
NOALLOC_MAX_SCRATCH_BYTES = 64 * 1024 * 1024

ERRORS = {
    -1: "B200L_ERR_BAD_SHAPE",
    -2: "B200L_ERR_UNSUPPORTED_HEAD_DIM",
    -3: "B200L_ERR_NULL_POINTER",
    -4: "B200L_ERR_WORKSPACE_TOO_SMALL",
    -5: "B200L_ERR_LAUNCH",
    -6: "B200L_ERR_DEVICE",
    -7: "B200L_ERR_TIMEOUT",
    -8: "B200L_ERR_ALIGNMENT",
}


class LayerDesc(ctypes.Structure):
    """Mirror of ``b200l_layer_desc``."""

    _fields_ = [
        ("batch", c_int32), ("seq_len", c_int32), ("d_model", c_int32),
        ("num_heads", c_int32), ("causal", c_int32), ("eps1", c_float), ("eps2", c_float),
        ("wqkv", c_void_p), ("bqkv", c_void_p), ("wo", c_void_p), ("bo", c_void_p),
        ("ln1_w", c_void_p), ("ln1_b", c_void_p), ("ln2_w", c_void_p), ("ln2_b", c_void_p),
        ("valid_mask", c_void_p), ("local_heads", c_int32),
    ]


class BlockDesc(ctypes.Structure):
    """Mirror of ``b200l_block_desc``."""

    _fields_ = [
        ("layer", LayerDesc), ("ffn_dim", c_int32),
        ("w1", c_void_p), ("b1", c_void_p), ("w2", c_void_p), ("b2", c_void_p),
    ]


class B200LError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def _declare(lib: ctypes.CDLL) -> None:
    P = c_void_p
    sig = {
        "b200l_version": (c_int, []),
        "b200l_last_error": (c_int, [ctypes.c_char_p, c_size_t]),
        "b200l_layer_workspace_bytes": (c_size_t, [P]),
        "b200l_clear_status": (c_int, [P, P]),
        "b200l_read_status": (c_int, [P, P]),
        "b200l_pack_weights": (c_int, [c_int32, P, P, P, P, P, P, P, P, P, P, P]),
        "b200l_layer_forward": (c_int, [P, P, P, P, c_size_t, P]),
        "b200l_qkv_ln_gemm": (c_int, [P, P, P, c_size_t, P]),
        "b200l_flash_attn": (c_int, [P, P, c_size_t, P]),
        "b200l_outproj_res_ln": (c_int, [P, P, P, P, c_size_t, P]),
        "b200l_layer_forward_noalloc": (c_int, [P, P, P, P]),
        "b200l_block_workspace_bytes": (c_size_t, [P]),
        "b200l_block_forward": (c_int, [P, P, P, P, c_size_t, P]),
        "b200l_row_layernorm": (c_int, [P, P, P, P, c_float, ctypes.c_int64, c_int32, P, P]),
        "b200l_cast_f16": (c_int, [P, P, ctypes.c_int64, P]),
        "b200l_kernel_workspace_bytes": (c_size_t, [P]),
        "b200l_debug_arm": (c_int, [P, c_int32, ctypes.c_uint64, P]),
        "b200l_noalloc_read_status": (c_int, [P]),
        "b200l_convert": (c_int, [P, c_int32, P, c_int32, ctypes.c_int64, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib() -> ctypes.CDLL:
    """Load (building first if stale and nvcc exists) the sm_100a library."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            path = _build.build()
            h = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
            _declare(h)
            v = h.b200l_version()
            if v != ABI_VERSION:
                raise RuntimeError(f"libcobra_b200 ABI version {v}, expected {ABI_VERSION}")
            _handle = h
    return _handle


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().b200l_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != 0:
        raise B200LError(rc, last_error())


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def fused_shape(S: int, d: int, H: int) -> bool:
    """b200l_layer_forward runs the whole-layer kernel for these shapes
    (mirror of ``fused_shape`` in csrc/capi.cu)."""
    return d in (64, 128) and d // H == 32 and d % H == 0 and S <= 128


def workspace_layout(B: int, S: int, d: int, H: int, local_heads: int = 0) -> dict:
    """Byte offsets of the workspace regions (mirror of ``make_plan`` in csrc/capi.cu).

    q, k: fp16 [B*H, S, dhp]; vt: fp16 [B*H, dhp, sp]; ctx: fp16 [B*S, d];
    h: fp16 [B*S, d] (only for d > 256). ``total`` is the full layout (what
    the per-kernel entry points need), ``layer_total`` what
    b200l_layer_forward needs (the status block alone for the whole-layer
    kernel)."""
    dh = d // H
    Hl = local_heads or H
    dhp = 32 if dh <= 32 else 64 if dh <= 64 else 128 if dh <= 128 else 256
    sp = _align(S, 8)
    T = B * S
    off = 1024
    lay = {"dh": dh, "dhp": dhp, "sp": sp, "heads": Hl, "dq": Hl * dh}
    qk = B * Hl * S * dhp * 2
    lay["q"] = off; off = _align(off + qk, 1024)
    lay["k"] = off; off = _align(off + qk, 1024)
    lay["vt"] = off; off = _align(off + B * Hl * dhp * sp * 2, 1024)
    lay["ctx"] = off; off = _align(off + T * Hl * dh * 2, 1024)
    lay["h"] = off
    if d > 256:
        off = _align(off + T * d * 2, 1024)
    lay["total"] = off
    lay["layer_total"] = 1024 if (fused_shape(S, d, H) and Hl == H) else off
    return lay
