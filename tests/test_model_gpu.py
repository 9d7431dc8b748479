"""The full stack on the GPU (blocks with the GELU FFN, final_norm) against the
reference: fixtures made by the reference's own BaselineTransformer
(tests/golden/model_*.pt) and the CPU oracle on further shapes.

Gate: the reference's abs_err <= 2e-3 OR rel_err <= 2e-2 per element. The FFN
half rounds LN2(x1) and the GELU output to fp16 before its GEMMs, as the
reference's fused path does (:1274-1292).
"""

import pytest
import torch

from oracle import TransformerConfig, build_reference_transformer, compare_outputs, generate_random_case
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

MODEL_FIXTURES = sorted(p.name for p in GOLDEN.glob("model_*.pt"))


def _ours(pkg, g_or_cfg, state_dict):
    c = g_or_cfg
    cfg = pkg.TransformerConfig(c.batch_size, c.seq_len, c.d_model, c.num_heads, ffn_dim=c.ffn_dim,
                                num_layers=c.num_layers, causal=c.causal)
    m = pkg.B200Transformer(cfg).cuda().eval()
    m.load_state_dict(state_dict, strict=True)
    return m


@pytest.mark.parametrize("name", MODEL_FIXTURES)
def test_stack_matches_reference_fixture(pkg, cuda_ok, name):
    g = torch.load(GOLDEN / name)
    cfg = TransformerConfig(g["B"], g["S"], g["d"], g["H"], ffn_dim=g["ffn_dim"],
                            num_layers=g["num_layers"], causal=g["causal"])
    ref = build_reference_transformer(cfg, g["weight_seed"])
    if "state_dict" in g:
        ref.load_state_dict(g["state_dict"], strict=True)
    model = _ours(pkg, cfg, ref.state_dict())
    for t in g["trials"]:
        mask = t["mask"].cuda() if t["mask"] is not None else None
        with torch.inference_mode():
            y = model(t["x"].cuda(), mask)
        torch.cuda.synchronize()
        model.check_status()
        res = compare_outputs(t["y"], y.cpu())
        assert res.passed, f"{name}: {res}"


@pytest.mark.parametrize("B,S,d,H,f,L,causal,pad", [
    (2, 128, 128, 4, 512, 2, False, 0.0),     # dh 32 (two-tile attention), fused-size layer shape
    (2, 200, 256, 4, 1024, 2, False, 0.3),    # dh 64, ragged S, padding
    (2, 150, 512, 4, 2048, 1, True, 0.0),     # dh 128, d > 256 (row-pass LN2), causal
    (1, 96, 256, 1, 200, 1, False, 0.0),      # dh 256, f not a multiple of 32 (GELU epilogue tail)
    (3, 64, 1024, 16, 4096, 1, False, 0.2),   # cfg5 family width, padding
])
def test_stack_matches_oracle(pkg, cuda_ok, B, S, d, H, f, L, causal, pad):
    cfg = TransformerConfig(B, S, d, H, ffn_dim=f, num_layers=L, causal=causal)
    ref = build_reference_transformer(cfg, 4242)
    model = _ours(pkg, cfg, ref.state_dict())
    x, mask = generate_random_case(cfg, seed=7, padding_ratio=pad)
    m = mask if pad > 0 else None
    with torch.inference_mode():
        y = model(x.cuda(), m.cuda() if m is not None else None)
        y_ref = ref(x, m)
    torch.cuda.synchronize()
    model.check_status()
    assert torch.isfinite(y).all()
    res = compare_outputs(y_ref, y.cpu())
    assert res.passed, f"{(B, S, d, H, f, L, causal, pad)}: {res}"
    if m is not None:   # padded rows are exactly zero after final_norm's mask
        assert torch.count_nonzero(y.cpu()[~m]) == 0


def test_stack_weights_change_is_picked_up(pkg, cuda_ok):
    cfg = TransformerConfig(2, 64, 128, 4, ffn_dim=256, num_layers=1)
    ref = build_reference_transformer(cfg, 1)
    model = _ours(pkg, cfg, ref.state_dict())
    x, _ = generate_random_case(cfg, seed=2)
    with torch.inference_mode():
        y1 = model(x.cuda()).clone()
        ref.layers[0].ffn_out.bias.add_(1.0)
        model.load_state_dict(ref.state_dict(), strict=True)
        y2 = model(x.cuda()).clone()
        y_ref = ref(x)
    assert not torch.equal(y1, y2)
    assert compare_outputs(y_ref, y2.cpu()).passed
