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
to be identical). After the calls it reads the status block inside the
library's scratch (``b200l_noalloc_read_status``), which is where a kernel
of a no-alloc call records a device-side failure. It also checks that a
problem too large for the built-in scratch is refused with a clear error
instead of running. The whole-layer kernel (d_model 128, head_dim 32,
S <= 128) needs only the status block, so the full cfg2 batch
(10000 sequences) runs through the no-alloc entry point too.

This file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu

SHAPES = [
    (4, 128, 128, 4, False),   # cfg1: the whole-layer kernel
    (3, 17, 96, 3, True),      # odd shape, causal: K1 -> K2 -> K3
    (2, 200, 512, 4, False),   # d > 256: uses the h region of the scratch too
    (10000, 128, 128, 4, False),  # cfg2 at full size: the whole-layer kernel, status block only
]
ORACLE_SEQS = 16   # sequences checked against the CPU oracle (all of them when B is smaller)


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
    pkg._lib.check(L.b200l_clear_status(layer.workspace_ptr, st))   # start from a clean status block

    xs = [generate_random_case(cfg, seed=100 + i)[0].to(dev) for i in range(2)]
    with torch.inference_mode():
        # Outputs of the existing entry point (caller-provided workspace).
        y_ws = []
        for x in xs:
            y = torch.empty_like(x)
            pkg._lib.check(L.b200l_layer_forward(ctypes.byref(desc), x.data_ptr(), y.data_ptr(),
                                                 layer.workspace_ptr, layer._ws_bytes, st))
            y_ws.append(y)
        pkg._lib.check(L.b200l_read_status(layer.workspace_ptr, st))
        # Two allocation-free calls in a row; after each, the status block in
        # the library's scratch must be clean.
        y_na = [torch.full_like(x, float("nan")) for x in xs]
        for x, y in zip(xs, y_na):
            pkg._lib.check(L.b200l_layer_forward_noalloc(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), st))
            rc = L.b200l_noalloc_read_status(st)
            assert rc == 0, f"no-alloc call recorded device status {rc}: {pkg._lib.last_error()}"
        torch.cuda.synchronize(dev)
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(3))[:ORACLE_SEQS]
    for i in range(2):
        torch.testing.assert_close(y_na[i], y_ws[i], atol=1e-4, rtol=1e-4)
        with torch.inference_mode():
            y_cpu = ref(xs[i][idx].cpu())
        assert compare_outputs(y_cpu, y_na[i][idx].cpu()).passed


def test_noalloc_rejects_problems_beyond_its_scratch(pkg, cuda_ok):
    L = pkg._lib.lib()
    # d_model 256 does not take the whole-layer kernel, so q, k, v^T and ctx
    # (about 2.6 GB here) would have to fit in the scratch.
    desc = pkg._lib.LayerDesc(batch=10000, seq_len=128, d_model=256, num_heads=8, causal=0,
                              eps1=1e-5, eps2=1e-5)
    need = L.b200l_layer_workspace_bytes(ctypes.byref(desc))
    assert need > pkg._lib.NOALLOC_MAX_SCRATCH_BYTES
    rc = L.b200l_layer_forward_noalloc(ctypes.byref(desc), None, None, None)
    assert rc == -4                       # B200L_ERR_WORKSPACE_TOO_SMALL
    assert "built-in scratch" in pkg._lib.last_error()
