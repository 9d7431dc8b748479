"""fp16 / bf16 inputs: the reference harness's --dtype float16 / bfloat16 modes.

In those modes the reference builds its models in the reduced dtype and runs
the layer on x of that dtype (torch_transformer_benchmark.py:952-962,
:1091-1094, :2033-2040). ``B200TransformerLayer`` takes such x (and parameters),
converts x to fp32 on the GPU with its own kernel (``b200l_convert``), runs the
fp32 layer and rounds y to x's dtype. Two checks per case:

* against the layer's exact value: the fp32 oracle evaluated on the same
  (rounded) inputs and parameters, with the reference's gate
  ``abs <= 2e-3 OR rel <= 2e-2`` -- our only added error is the final rounding
  to fp16 / bf16 (2^-11 / 2^-8 relative);
* against the reference module run in that dtype (its own rounding at every
  op): fp16 passes the same gate; for bf16 the reference itself notes that any
  reordering of its arithmetic costs ~4e-3 (:952-962), so that comparison is
  reported as the maximum error instead of gated.
"""

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu

SHAPES = [
    (4, 128, 128, 4, False),    # cfg1: the whole-layer kernel
    (2, 300, 128, 4, True),     # three-kernel path, causal
    (2, 200, 512, 4, False),    # d > 256
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_S{}_d{}_H{}{}".format(*s[:4], "_causal" if s[4] else ""))
def test_reduced_precision_inputs(pkg, cuda_ok, dtype, shape):
    B, S, d, H, causal = shape
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    ref = build_reference_layer(cfg, 1234).to(dtype)          # the harness's model.to(dtype)
    lay = pkg.B200TransformerLayer(d, H, causal).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    lay.to(dtype)
    x, _ = generate_random_case(cfg, seed=55)
    x = x.to(dtype)
    with torch.inference_mode():
        y = lay(x.cuda()).clone()
        torch.cuda.synchronize()
        lay.check_status()
        assert y.dtype == dtype and y.shape == x.shape
        # exact value on the rounded inputs and parameters
        ref32 = build_reference_layer(cfg, 1234)
        ref32.load_state_dict({k: v.float() for k, v in ref.state_dict().items()})
        y_exact = ref32(x.float())
        res = compare_outputs(y_exact, y.float().cpu())
        assert res.passed, f"vs the exact layer: {res}"
        # the reference module run in the reduced dtype
        y_red = ref(x)
        res2 = compare_outputs(y_red.float(), y.float().cpu())
        print(f"{dtype} {shape}: vs exact max_abs {res.max_abs_error:.2e}; vs reference in {dtype} "
              f"max_abs {res2.max_abs_error:.2e}, {res2.failed_elements} of {res2.total_elements} outside the gate")
        if dtype == torch.float16:
            assert res2.passed, f"vs the reference module in fp16: {res2}"


def test_convert_round_trip(pkg, cuda_ok):
    import ctypes  # noqa: F401
    L = pkg._lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(3)
    for n in (1, 7, 8, 9, 1000, 4096 + 3):
        x = torch.randn(n, generator=g, device="cuda") * 100
        for dt, code in ((torch.float16, pkg._lib.DTYPE_F16), (torch.bfloat16, pkg._lib.DTYPE_BF16)):
            h = torch.empty(n, dtype=dt, device="cuda")
            pkg._lib.check(L.b200l_convert(x.data_ptr(), pkg._lib.DTYPE_F32, h.data_ptr(), code, n, st))
            assert torch.equal(h, x.to(dt)), (n, dt)          # round to nearest even, like torch
            back = torch.empty(n, dtype=torch.float32, device="cuda")
            pkg._lib.check(L.b200l_convert(h.data_ptr(), code, back.data_ptr(), pkg._lib.DTYPE_F32, n, st))
            assert torch.equal(back, h.float())
    assert L.b200l_convert(None, 0, None, 1, 4, st) == -3
