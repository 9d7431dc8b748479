"""GPU test of ``b200l_layer_forward_noalloc``, the allocation-free entry point.

Some callers cannot call cudaMalloc: a plugin whose host process owns all
device memory through its own pool, or a latency-critical service that
forbids allocation after start-up because cudaMalloc/cudaFree synchronise
the device. For them the library runs the layer out of a fixed 64 MiB scratch
array of its own instead of a caller-provided workspace.

The test calls that entry point through the C ABI twice in a row and checks
each output against ``b200l_layer_forward`` (caller-provided workspace) on the
same inputs, with the tolerance the kernel tests use for the final output
(abs 1e-4 + rel 1e-4; the kernels are the same, so the results are expected
to be identical). It also checks that a problem too large for the built-in
scratch is refused with a clear error instead of running.

This file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu

SHAPES = [
    (4, 128, 128, 4, False),   # cfg1: LN-fused K1, fused LN2 epilogue
    (3, 17, 96, 3, True),      # odd shape, causal
    (2, 200, 512, 4, False),   # d > 256: uses the h region of the scratch too
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_S{}_d{}_H{}{}".format(*s[:4], "_causal" if s[4] else ""))
def test_noalloc_matches_workspace_entry_point(pkg, cuda_ok, shape):
    B, S, d, H, causal = shape
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    ref = build_reference_layer(cfg, 1234)
    layer = pkg.B200TransformerLayer(d, H, causal, use_graphs=False).cuda().eval()
    layer.load_state_dict(ref.state_dict(), strict=True)
    L = pkg._lib.lib()
    dev = torch.device("cuda", 0)
    pk = layer._ensure_pack(dev)
    desc = layer._desc(B, S, pk)
    layer._ensure_workspace(desc, dev)
    assert layer._ws_bytes <= pkg._lib.NOALLOC_MAX_SCRATCH_BYTES
    st = torch.cuda.current_stream(dev).cuda_stream

    xs = [generate_random_case(cfg, seed=100 + i)[0].to(dev) for i in range(2)]
    with torch.inference_mode():
        # Outputs of the existing entry point (caller-provided workspace).
        y_ws = []
        for x in xs:
            y = torch.empty_like(x)
            pkg._lib.check(L.b200l_layer_forward(ctypes.byref(desc), x.data_ptr(), y.data_ptr(),
                                                 layer.workspace_ptr, layer._ws_bytes, st))
            y_ws.append(y)
        # Two allocation-free calls in a row.
        y_na = [torch.full_like(x, float("nan")) for x in xs]
        for x, y in zip(xs, y_na):
            pkg._lib.check(L.b200l_layer_forward_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), st))
        torch.cuda.synchronize(dev)
    layer.check_status()
    for i in range(2):
        torch.testing.assert_close(y_na[i], y_ws[i], atol=1e-4, rtol=1e-4)
        with torch.inference_mode():
            y_cpu = ref(xs[i].cpu())
        assert compare_outputs(y_cpu, y_na[i].cpu()).passed


def test_noalloc_rejects_problems_beyond_its_scratch(pkg, cuda_ok):
    L = pkg._lib.lib()
    desc = pkg._lib.LayerDesc(batch=10000, seq_len=128, d_model=128, num_heads=4, causal=0,
                              eps1=1e-5, eps2=1e-5)
    need = L.b200l_layer_workspace_bytes(ctypes.byref(desc))
    assert need > pkg._lib.NOALLOC_MAX_SCRATCH_BYTES
    rc = L.b200l_layer_forward_noalloc(ctypes.byref(desc), None, None, None)
    assert rc == -4                       # B200L_ERR_WORKSPACE_TOO_SMALL
    assert "built-in scratch" in pkg._lib.last_error()
