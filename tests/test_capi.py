"""CPU tests of the C ABI: the library builds, loads, exports every declared
symbol, and validates shapes before touching a device."""

import ctypes
import re

import pytest

from tests.conftest import ROOT


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"B200L_API\s+[\w\s\*]+?\b(b200l_\w+)\s*\(", h.read_text()))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for n in ("b200l_layer_forward", "b200l_qkv_ln_gemm", "b200l_flash_attn",
              "b200l_outproj_res_ln", "b200l_pack_weights", "b200l_last_error", "b200l_version"):
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.lib()
    handle = ctypes.CDLL(lib._name)
    for n in declared_symbols():
        assert hasattr(handle, n), f"{n} declared in include/ but not exported"
    assert set(pkg._lib.EXPORTED) == declared_symbols()
    assert lib.b200l_version() == pkg._lib.ABI_VERSION


def _desc(pkg, B, S, d, H):
    return pkg._lib.LayerDesc(batch=B, seq_len=S, d_model=d, num_heads=H, causal=0, eps1=1e-5, eps2=1e-5)


@pytest.mark.parametrize("B,S,d,H", [(4, 128, 128, 4), (3, 17, 96, 3), (10000, 128, 128, 4),
                                     (32, 100000, 1024, 16), (2, 96, 256, 1), (2, 200, 512, 4)])
def test_workspace_bytes_matches_python_layout(pkg, B, S, d, H):
    lib = pkg._lib.lib()
    d_ = _desc(pkg, B, S, d, H)
    lay = pkg._lib.workspace_layout(B, S, d, H)
    n = lib.b200l_kernel_workspace_bytes(ctypes.byref(d_))
    assert n == lay["total"]
    assert n % 1024 == 0
    # b200l_layer_forward's workspace follows the path it takes: the status
    # block alone for the whole-layer kernel, the full layout otherwise.
    nl = lib.b200l_layer_workspace_bytes(ctypes.byref(d_))
    assert nl == lay["layer_total"]
    assert nl == (1024 if pkg._lib.fused_shape(S, d, H) else n)


@pytest.mark.parametrize("B,S,d,H,code,msg", [
    (0, 128, 128, 4, -1, "positive"),
    (2, 128, 130, 4, -1, "divisible"),
    (2, 128, 48, 3, -2, "head_dim 16"),
    (2, 128, 640, 1, -2, "head_dim 640"),
    (2, 128, 4096, 16, -1, "2048"),
])
def test_bad_shapes_are_rejected_on_the_host(pkg, B, S, d, H, code, msg):
    lib = pkg._lib.lib()
    d_ = _desc(pkg, B, S, d, H)
    assert lib.b200l_layer_workspace_bytes(ctypes.byref(d_)) == 0
    assert lib.b200l_kernel_workspace_bytes(ctypes.byref(d_)) == 0
    rc = lib.b200l_layer_forward(ctypes.byref(d_), None, None, None, 0, None)
    assert rc == code
    assert msg in pkg._lib.last_error()


def test_null_descriptor(pkg):
    lib = pkg._lib.lib()
    assert lib.b200l_layer_forward(None, None, None, None, 0, None) == -3
    assert lib.b200l_flash_attn(None, None, 0, None) == -3


def test_no_cpu_fallback(pkg):
    import torch
    layer = pkg.B200TransformerLayer(128, 4)
    with pytest.raises(RuntimeError, match="no CPU path"):
        layer(torch.zeros(1, 4, 128))


@pytest.mark.parametrize("struct,cls", [("b200l_layer_desc", "LayerDesc"), ("b200l_block_desc", "BlockDesc")])
def test_descriptor_layout_matches_header(pkg, tmp_path, struct, cls):
    """The ctypes mirrors of the descriptors have the C structs' sizes and
    field offsets (compiled from include/cobra_b200.h with the host C compiler)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    D = getattr(pkg._lib, cls)
    names = [f[0] for f in D._fields_]
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "cobra_b200.h"\nint main(void) {\n'
        f'  printf("%zu\\n", sizeof({struct}));\n'
        + "".join(f'  printf("%zu\\n", offsetof({struct}, {n}));\n' for n in names)
        + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(ROOT / "include"), "-o", str(exe), str(src)], check=True)
    out = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    assert out[0] == ctypes.sizeof(D)
    assert out[1:] == [getattr(D, n).offset for n in names]


def _align(v, a=1024):
    return (v + a - 1) // a * a


@pytest.mark.parametrize("B,S,d,H,f", [(2, 128, 128, 4, 512), (3, 17, 96, 3, 200), (64, 128, 1024, 4, 4096)])
def test_block_workspace_bytes_layout(pkg, B, S, d, H, f):
    """The block's workspace is the layer's plus the fp32 residual x1, the
    fp16 LN2 output h2 and the fp16 FFN hidden h1, each 1024-byte aligned."""
    lib = pkg._lib.lib()
    bd = pkg._lib.BlockDesc(layer=_desc(pkg, B, S, d, H), ffn_dim=f)
    T = B * S
    off = _align(pkg._lib.workspace_layout(B, S, d, H)["total"])
    off = _align(off + T * d * 4)
    off = _align(off + T * d * 2)
    off = _align(off + T * f * 2)
    assert lib.b200l_block_workspace_bytes(ctypes.byref(bd)) == off


@pytest.mark.parametrize("f", [0, -8, 100, 65544])
def test_block_rejects_bad_ffn_dim(pkg, f):
    lib = pkg._lib.lib()
    bd = pkg._lib.BlockDesc(layer=_desc(pkg, 2, 128, 128, 4), ffn_dim=f)
    assert lib.b200l_block_workspace_bytes(ctypes.byref(bd)) == 0
    assert lib.b200l_block_forward(ctypes.byref(bd), None, None, None, 0, None) == -1
    assert "ffn_dim" in pkg._lib.last_error()
