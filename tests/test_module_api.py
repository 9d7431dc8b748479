"""CPU tests of the drop-in module's API (no kernels run)."""

import pytest
import torch

from oracle import ReferenceLayer, TransformerConfig, build_reference_layer


def test_state_dict_identical_keys_and_strict_load(pkg):
    ref = build_reference_layer(TransformerConfig(2, 8, 128, 4), 1234)
    lay = pkg.B200TransformerLayer(128, 4)
    assert set(lay.state_dict()) == set(ref.state_dict())
    lay.load_state_dict(ref.state_dict(), strict=True)      # must not raise
    for k, v in ref.state_dict().items():
        assert torch.equal(lay.state_dict()[k], v)


def test_same_seed_same_init_as_reference(pkg):
    torch.manual_seed(42)
    a = ReferenceLayer(96, 3)
    torch.manual_seed(42)
    b = pkg.B200TransformerLayer(96, 3)
    for k, v in a.state_dict().items():
        assert torch.equal(b.state_dict()[k], v)


def test_from_config_mirrors_reference_config(pkg):
    cfg = pkg.TransformerConfig(4, 128, 128, 4, causal=True)
    lay = pkg.B200TransformerLayer.from_config(cfg)
    assert lay.causal and lay.attention.head_dim == 32
    with pytest.raises(ValueError):
        pkg.TransformerConfig(4, 128, 130, 4).validate()
    with pytest.raises(ValueError):
        pkg.TransformerConfig(4, 128, 128, 4, num_layers=2).validate()


def test_load_state_dict_invalidates_pack(pkg):
    lay = pkg.B200TransformerLayer(64, 2)
    lay._pack = object()
    lay.load_state_dict(ReferenceLayer(64, 2).state_dict())
    assert lay._pack is None


def test_module_built_under_inference_mode_tracks_parameters(pkg):
    """A layer constructed inside torch.inference_mode() has inference-tensor
    parameters (no version counter); weight-change tracking must still work."""
    import torch
    with torch.inference_mode():
        lay = pkg.B200TransformerLayer(64, 2)
        v1 = lay._param_versions()
    v2 = lay._param_versions()
    assert v1 == v2
    with torch.inference_mode():
        lay.norm1.weight = torch.nn.Parameter(torch.ones(64))
    assert lay._param_versions() != v1


def test_stack_state_dict_and_seeded_init_match_reference(pkg):
    """B200Transformer has the reference BaselineTransformer's module tree:
    identical state_dict keys, and seeded construction draws identical weights
    (the harness copies baseline weights with strict=True, :1544-1554)."""
    import torch
    from oracle import TransformerConfig as OCfg, build_reference_transformer
    ocfg = OCfg(2, 16, 64, 2, ffn_dim=96, num_layers=3, causal=True)
    ref = build_reference_transformer(ocfg, seed=5)
    cfg = pkg.TransformerConfig(2, 16, 64, 2, ffn_dim=96, num_layers=3, causal=True)
    torch.manual_seed(5)
    ours = pkg.B200Transformer(cfg)
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert list(rs) == list(os_)
    assert all(torch.equal(rs[k], os_[k]) for k in rs)
    ours.load_state_dict(rs, strict=True)
    assert pkg.UserOptimizedTransformer is pkg.B200Transformer
    with pytest.raises(RuntimeError, match="no CPU path"):
        ours(torch.zeros(2, 16, 64))


def test_stack_config_validation(pkg):
    with pytest.raises(ValueError, match="ffn_dim"):
        pkg.B200Transformer(pkg.TransformerConfig(1, 8, 64, 2, ffn_dim=0, num_layers=1))
    with pytest.raises(ValueError, match="num_layers"):
        pkg.B200Transformer(pkg.TransformerConfig(1, 8, 64, 2, ffn_dim=64, num_layers=0))
