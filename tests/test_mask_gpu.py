"""Key-padding masks on the GPU against the CPU oracle.

Semantics (BaselineSelfAttention, torch_transformer_benchmark.py:106-109 and
:121-122): invalid keys get probability 0 in every query's softmax, and an
invalid query row's attention output (after the out-projection, bias
included) is zeroed, so that row's y is LN2(x). Rows whose every visible key
is invalid are NaN inside the reference's softmax and then zeroed by the same
row mask; the kernels must give LN2(x) there too, with no NaN anywhere.

Gate: the reference's abs_err <= 2e-3 OR rel_err <= 2e-2 per element.
"""

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu

# (B, S, d, H, causal): whole-layer kernel (d 64/128, dh 32, S <= 128), the
# two-tile attention (dh 32 / 64, S > 128), the one-tile attention (dh 128 /
# 256), the d > 256 residual path, causal.
SHAPES = [
    (6, 128, 128, 4, False),
    (5, 77, 64, 2, False),
    (4, 128, 128, 4, True),
    (3, 300, 128, 4, False),
    (3, 390, 256, 4, False),
    (2, 200, 256, 2, False),
    (2, 150, 256, 1, False),
    (2, 260, 512, 4, False),
    (2, 333, 128, 4, True),
]


def _ids(s):
    B, S, d, H, c = s
    return f"B{B}_S{S}_d{d}_H{H}" + ("_causal" if c else "")


def _layer(pkg, B, S, d, H, causal, graphs=False):
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    ref = build_reference_layer(cfg, 4321)
    lay = pkg.B200TransformerLayer(d, H, causal, use_graphs=graphs).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    return cfg, ref, lay


def _masks(B, S, seed):
    """A prefix mask per sequence (the harness's kind), a scattered mask with
    whole invalid 128-key tiles, a mask whose first keys are invalid (causal
    rows with no visible valid key) and one fully invalid sequence."""
    g = torch.Generator().manual_seed(seed)
    prefix = torch.arange(S)[None, :] < torch.randint(1, S + 1, (B, 1), generator=g)
    scattered = torch.rand(B, S, generator=g) > 0.35
    if S > 256:
        scattered[:, 128:256] = False
    head_gap = torch.ones(B, S, dtype=torch.bool)
    head_gap[:, : min(5, S)] = False
    head_gap[-1, :] = False
    return {"prefix": prefix, "scattered": scattered, "head_gap": head_gap}


def _check(ref, lay, x, mask, what):
    with torch.inference_mode():
        y = lay(x.cuda(), mask.cuda()).clone()
        y_ref = ref(x, mask)
    torch.cuda.synchronize()
    lay.check_status()
    y = y.cpu()
    assert torch.isfinite(y).all(), f"{what}: non-finite output"
    res = compare_outputs(y_ref, y)
    assert res.passed, f"{what}: {res}"
    return y


@pytest.mark.parametrize("shape", SHAPES, ids=_ids)
def test_masked_layer_matches_oracle(pkg, cuda_ok, shape):
    B, S, d, H, causal = shape
    cfg, ref, lay = _layer(pkg, B, S, d, H, causal)
    x, _ = generate_random_case(cfg, seed=17)
    for name, mask in _masks(B, S, seed=18).items():
        y = _check(ref, lay, x, mask, f"{_ids(shape)} {name}")
        # An invalid query row is exactly LN2(x) of that row.
        if not bool(mask.all()):
            ln2 = torch.nn.functional.layer_norm(x, (d,), lay.norm2.weight.cpu(), lay.norm2.bias.cpu(),
                                                 lay.norm2.eps)
            torch.testing.assert_close(y[~mask], ln2[~mask], atol=2e-5, rtol=2e-5)


def test_harness_padding_cases(pkg, cuda_ok):
    """generate_random_case's padded inputs (x zeroed at padded positions)."""
    for B, S, d, H in ((4, 128, 128, 4), (3, 513, 128, 4), (2, 200, 1024, 16)):
        cfg, ref, lay = _layer(pkg, B, S, d, H, False)
        for ratio in (0.1, 0.5):
            x, mask = generate_random_case(cfg, seed=31, padding_ratio=ratio)
            assert not bool(mask.all())
            _check(ref, lay, x, mask, f"B{B} S{S} d{d} padding {ratio}")


def test_all_true_mask_equals_no_mask(pkg, cuda_ok):
    for B, S, d, H in ((3, 128, 128, 4), (2, 300, 256, 4)):
        cfg, ref, lay = _layer(pkg, B, S, d, H, False)
        x, _ = generate_random_case(cfg, seed=3)
        ones = torch.ones(B, S, dtype=torch.bool, device="cuda")
        with torch.inference_mode():
            a = lay(x.cuda()).clone()
            b = lay(x.cuda(), ones).clone()
        assert torch.equal(a, b)


def test_graph_replay_with_changing_masks(pkg, cuda_ok):
    B, S, d, H = 4, 128, 128, 4
    cfg, ref, eager = _layer(pkg, B, S, d, H, False, graphs=False)
    graphed = pkg.B200TransformerLayer(d, H, use_graphs=True).cuda().eval()
    graphed.load_state_dict(ref.state_dict(), strict=True)
    x, _ = generate_random_case(cfg, seed=8)
    for name, mask in _masks(B, S, seed=9).items():
        with torch.inference_mode():
            ye = eager(x.cuda(), mask.cuda()).clone()
            yg = graphed(x.cuda(), mask.cuda()).clone()
        assert torch.equal(ye, yg), name
    assert graphed._graph is not None and graphed._static_m is not None
    with torch.inference_mode():     # back to no mask: a separate capture
        assert torch.equal(graphed(x.cuda()).clone(), eager(x.cuda()).clone())


def test_mask_shape_and_device_are_checked(pkg, cuda_ok):
    _, _, lay = _layer(pkg, 2, 16, 64, 2, False)
    x = torch.randn(2, 16, 64, device="cuda")
    with pytest.raises(ValueError, match="shape"):
        lay(x, torch.ones(2, 15, dtype=torch.bool, device="cuda"))
    with pytest.raises(ValueError, match="device"):
        lay(x, torch.ones(2, 16, dtype=torch.bool))
