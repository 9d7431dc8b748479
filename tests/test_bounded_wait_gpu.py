"""Bounded device waits: a wait that runs out ends the kernel with an error
status instead of a hang, and the next call on the same workspace is clean.

Every mbarrier wait in the kernels is bounded (2 s by default) and, when it
runs out, raises a CTA-wide abort flag: the CTA unwinds, drains the copies it
issued, frees its tensor memory and records B200L_ERR_TIMEOUT in the
workspace's status block. The reference has no device-side failure handling
at all (its only recovery is the eager fallback after a failed graph capture,
torch_transformer_benchmark.py:1527-1534).

The test arms the library's fault hook (``b200l_debug_arm``): in CTA 0 of the
named kernel the TMA producer leaves out its first operand load -- a barrier
that nothing will complete -- and every wait is limited to 20 ms. Nothing
faults, traps or spins without bound. The status must read
B200L_ERR_TIMEOUT; after ``b200l_clear_status`` the same layer on the same
workspace must reproduce its earlier output bit for bit and pass the
reference gate.
"""

import ctypes
import time

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu

WAIT_NS = 20_000_000   # 20 ms per wait while armed

CASES = [
    # (fault site, B, S, d, H): attention for head_dim 32 runs attn2_kernel;
    # d = 512 runs the TMA-fed GEMM for both the QKV and the out-projection.
    ("ATTN_KV", 2, 300, 128, 4),
    ("GEMM_OPERAND", 2, 200, 512, 4),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_wait_runs_out_then_next_call_is_clean(pkg, cuda_ok, case):
    site_name, B, S, d, H = case
    site = getattr(pkg._lib, f"DEBUG_SITE_{site_name}")
    cfg = TransformerConfig(B, S, d, H)
    ref = build_reference_layer(cfg, 1234)
    lay = pkg.B200TransformerLayer(d, H, use_graphs=False).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    x, _ = generate_random_case(cfg, seed=31)
    xg = x.cuda()
    L = pkg._lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    with torch.inference_mode():
        y_good = lay(xg).clone()
        torch.cuda.synchronize()
        lay.check_status()

        pkg._lib.check(L.b200l_debug_arm(lay.workspace_ptr, site, WAIT_NS, st))
        t0 = time.perf_counter()
        lay(xg)                                   # launches return at once
        rc = L.b200l_read_status(lay.workspace_ptr, st)
        elapsed = time.perf_counter() - t0
        msg = pkg._lib.last_error()
        assert rc == -7, f"expected B200L_ERR_TIMEOUT, got {rc} ({msg})"
        assert "block 0" in msg, msg
        # The aborted CTA gave up after about one 20 ms limit, not the 2 s default.
        assert elapsed < 1.5, f"armed forward took {elapsed:.3f} s"

        pkg._lib.check(L.b200l_clear_status(lay.workspace_ptr, st))
        y_after = lay(xg).clone()
        torch.cuda.synchronize()
        lay.check_status()
    assert torch.equal(y_after, y_good), "the call after the timeout differs from the call before it"
    with torch.inference_mode():
        y_ref = ref(x)
    res = compare_outputs(y_ref, y_after.cpu())
    assert res.passed, res


def test_debug_arm_validates_its_arguments(pkg, cuda_ok):
    L = pkg._lib.lib()
    buf = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert L.b200l_debug_arm(None, 1, WAIT_NS, st) == -3
    assert L.b200l_debug_arm(buf.data_ptr(), 99, WAIT_NS, st) == -1
    assert L.b200l_debug_arm(buf.data_ptr(), 1, 1000, st) == -1      # below 1 ms
    assert "below 1 ms" in pkg._lib.last_error()
