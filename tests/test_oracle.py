"""CPU tests of the oracle: pinned to the reference's own outputs (tests/golden)."""

import hashlib

import pytest
import torch

from oracle import (ReferenceLayer, TransformerConfig, build_reference_layer, build_reference_transformer,
                    compare_outputs, generate_random_case, streamed_attention_rows_fp64,
                    streamed_layer_rows_fp64)
from oracle.ref_layer import sample_rows
from tests.conftest import GOLDEN

FIXTURES = sorted(p.name for p in GOLDEN.glob("*.pt") if not p.name.startswith("model_"))
MODEL_FIXTURES = sorted(p.name for p in GOLDEN.glob("model_*.pt"))


def _sha(sd):
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().contiguous().float().numpy().tobytes())
    return h.hexdigest()


def test_fixtures_present():
    assert len(FIXTURES) >= 8
    assert len(MODEL_FIXTURES) >= 4


@pytest.mark.parametrize("name", MODEL_FIXTURES)
def test_stack_oracle_bit_exact_vs_reference_fixture(name):
    """Full stacks (blocks with the GELU FFN, final_norm) produced by the
    reference's own BaselineTransformer (tests/golden/make_golden.py)."""
    g = torch.load(GOLDEN / name)
    cfg = TransformerConfig(g["B"], g["S"], g["d"], g["H"], ffn_dim=g["ffn_dim"],
                            num_layers=g["num_layers"], causal=g["causal"])
    model = build_reference_transformer(cfg, g["weight_seed"])
    assert _sha(model.state_dict()) == g["state_sha"]
    if "state_dict" in g:
        model.load_state_dict(g["state_dict"], strict=True)
    for t in g["trials"]:
        x_again, _ = generate_random_case(cfg, t["seed"], g["padding"])
        assert torch.equal(x_again, t["x"])
        with torch.inference_mode():
            y = model(t["x"], t["mask"])
        assert torch.equal(y, t["y"]), f"{name}: stack oracle differs from the reference output"


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_bit_exact_vs_reference_fixture(name):
    g = torch.load(GOLDEN / name)
    cfg = TransformerConfig(g["B"], g["S"], g["d"], g["H"], causal=g["causal"])
    layer = build_reference_layer(cfg, g["weight_seed"])
    # Weights regenerated from the seed must be the reference's weights.
    assert _sha(layer.state_dict()) == g["state_sha"]
    if "state_dict" in g:
        layer.load_state_dict(g["state_dict"], strict=True)
    for t in g["trials"]:
        x_again, mask_again = generate_random_case(cfg, t["seed"], g["padding"])
        assert torch.equal(x_again, t["x"]), "input generator drifted from the reference's"
        with torch.inference_mode():
            y = layer(t["x"], t["mask"])
        assert torch.equal(y, t["y"]), f"{name}: oracle differs from the reference output"


def test_state_dict_keys_match_reference_block_half():
    keys = set(ReferenceLayer(128, 4).state_dict())
    expected = {"norm1.weight", "norm1.bias", "norm2.weight", "norm2.bias"}
    for p in ("q", "k", "v", "out"):
        expected |= {f"attention.{p}_proj.weight", f"attention.{p}_proj.bias"}
    assert keys == expected


@pytest.mark.parametrize("B,S,d,H,causal", [(2, 128, 128, 4, False), (2, 333, 96, 3, True),
                                            (1, 257, 256, 4, False), (1, 130, 128, 2, True)])
def test_streamed_fp64_oracle_matches_full_layer(B, S, d, H, causal):
    """Mirrors tools/reference_chunked.py:146-177: the row-sampled fp64 oracle
    equals the full reference layer evaluated in fp64 (whose softmax still runs
    in fp32, torch_transformer_benchmark.py:112), within the reference's own
    oracle tolerance of 1e-5 (tools/reference_chunked.py:167)."""
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    layer = build_reference_layer(cfg, 1234)
    x, _ = generate_random_case(cfg, 1234)
    full = ReferenceLayer(d, H, causal).double()
    full.load_state_dict(layer.state_dict())
    with torch.inference_mode():
        y_full = full(x.double())
        ctx_rows_seen = []
        for b in range(B):
            rows = sample_rows(S, 37, seed=b)
            y_rows = streamed_layer_rows_fp64(layer, x[b], rows, causal)
            assert (y_rows - y_full[b, rows]).abs().max() <= 1e-5
            ctx_rows_seen.append(streamed_attention_rows_fp64(layer, x[b], rows, causal))
    assert all(torch.isfinite(c).all() for c in ctx_rows_seen)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_streamed_fp64_oracle_with_key_mask_matches_full_layer(causal):
    """The streamed oracle with a key-padding mask (the long-context masked
    check's oracle) equals the full reference layer given the same
    valid_token_mask: padded keys get no probability (:106-109) and a padded
    query row's attention output is zeroed (:121-122), sampled rows including
    padded ones."""
    B, S, d, H = 2, 333, 64, 2
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    layer = build_reference_layer(cfg, 1234)
    x, _ = generate_random_case(cfg, 1234)
    g = torch.Generator().manual_seed(5)
    mask = torch.stack([torch.arange(S) < 250,                       # padded tail
                        torch.rand(S, generator=g) > 0.3])           # scattered
    mask[1, 0] = True   # causal rows always see at least key 0
    full = ReferenceLayer(d, H, causal).double()
    full.load_state_dict(layer.state_dict())
    with torch.inference_mode():
        y_full = full(x.double(), mask)
        for b in range(B):
            rows = sample_rows(S, 41, seed=b)
            y_rows = streamed_layer_rows_fp64(layer, x[b], rows, causal, key_mask=mask[b])
            assert (y_rows - y_full[b, rows]).abs().max() <= 1e-5


def test_fp32_oracle_within_gate_of_fp64():
    cfg = TransformerConfig(4, 128, 128, 4)
    layer = build_reference_layer(cfg, 1234)
    x, _ = generate_random_case(cfg, 1234)
    with torch.inference_mode():
        y32 = layer(x)
        y64 = torch.stack([streamed_layer_rows_fp64(layer, x[b], range(128)) for b in range(4)])
    assert compare_outputs(y64, y32, rtol=1e-4, atol=1e-5).passed


def test_compare_outputs_semantics():
    ref = torch.tensor([1.0, 100.0, 0.0, 1.0])
    ok = torch.tensor([1.0019, 101.9, 0.0019, 1.0])
    assert compare_outputs(ref, ok).passed
    bad = torch.tensor([1.0, 100.0, 0.0021, float("nan")])
    r = compare_outputs(ref, bad)
    assert not r.passed and r.failed_elements == 2
