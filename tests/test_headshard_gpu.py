"""Head sharding's per-rank compute on one GPU: K1 and K2 with ``local_heads``.

A rank of ``headshard.head_sharded_forward`` runs LN1, the q / k / v
projections and the attention of a contiguous range of heads only
(``B200TransformerLayer._head_ctx``, the C ABI's ``local_heads``), and the
caller finishes the layer from every rank's ctx columns
(``_finish_from_ctx``). Emulating the ranks in one process: the ctx columns of
every head range must equal the same columns of the all-heads run of
K1 -> K2, and the layer finished from them must equal the three-kernel path
bit for bit (every output element is computed by the same arithmetic) and
pass the reference gate. The NCCL run on two GPUs is in
tests/test_sharding_gpu.py.
"""

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case
from tests.test_layer_gpu import make_layer, run_stepwise, ws_views

pytestmark = pytest.mark.gpu

CASES = [
    # (B, S, d, H, causal, padding, head ranges)
    (4, 128, 128, 4, False, 0.0, [(0, 1), (1, 2), (2, 3), (3, 4)]),   # cfg1 split over 4 ranks
    (2, 300, 256, 4, True, 0.0, [(0, 3), (3, 4)]),                     # dh 64, causal, uneven
    (3, 130, 512, 4, False, 0.3, [(0, 2), (2, 4)]),                    # d > 256 (row LN + TMA GEMM), mask
    (1, 160, 1024, 16, False, 0.0, [(0, 6), (6, 12), (12, 16)]),       # cfg5 family
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_S{}_d{}_H{}".format(*c[:4]))
def test_local_heads_match_all_heads(pkg, cuda_ok, case):
    B, S, d, H, causal, pad, ranges = case
    cfg, ref, lay = make_layer(pkg, B, S, d, H, causal)
    x, mask = generate_random_case(cfg, seed=91, padding_ratio=pad)
    m = mask.cuda() if pad > 0 else None
    xg = x.cuda()
    dh = d // H
    with torch.inference_mode():
        if m is None:
            y3 = run_stepwise(pkg, lay, xg).clone()
            _, _, _, ctx_all, _, _ = ws_views(pkg, lay, B, S, d, H)
            ctx_all = ctx_all.clone()
        parts = [lay._head_ctx(xg, m, a, b) for a, b in ranges]
        ctx = torch.cat(parts, dim=1)
        torch.cuda.synchronize()
        if m is None:
            for (a, b), p in zip(ranges, parts):
                assert torch.equal(p, ctx_all[:, a * dh:b * dh]), f"heads [{a}, {b}): ctx differs"
        y = lay._finish_from_ctx(xg, m, ctx).clone()
        torch.cuda.synchronize()
        lay.check_status()
        if m is None:
            assert torch.equal(y, y3), "finished layer differs from the three-kernel path"
        y_ref = ref(x, mask if pad > 0 else None)
    res = compare_outputs(y_ref, y.cpu())
    assert res.passed, res


def test_local_heads_are_validated(pkg, cuda_ok):
    import ctypes
    L = pkg._lib.lib()
    desc = pkg._lib.LayerDesc(batch=2, seq_len=64, d_model=128, num_heads=4, causal=0, eps1=1e-5, eps2=1e-5,
                              local_heads=5)
    assert L.b200l_kernel_workspace_bytes(ctypes.byref(desc)) == 0
    assert "local_heads" in pkg._lib.last_error()
    desc.local_heads = 2
    assert L.b200l_layer_workspace_bytes(ctypes.byref(desc)) > 1024     # not the whole-layer kernel
    rc = L.b200l_layer_forward(ctypes.byref(desc), None, None, None, 0, None)
    assert rc in (-1, -3)
