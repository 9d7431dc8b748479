"""Host-resident input with the parameters on the GPU: the module streams the
batch through the device in chunks (the reference's _run_streamed,
torch_transformer_benchmark.py:1418-1508) and returns a host tensor.

Every sequence runs the same kernels as on the device path, so the streamed
result must equal the device-resident result bit for bit, whatever the chunk
boundaries.
"""

import pytest
import torch

from oracle import TransformerConfig, build_reference_layer, compare_outputs, generate_random_case

pytestmark = pytest.mark.gpu


def _layer(pkg, B, S, d, H, causal=False):
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    ref = build_reference_layer(cfg, 99)
    lay = pkg.B200TransformerLayer(d, H, causal, use_graphs=False).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    return cfg, ref, lay


@pytest.mark.parametrize("B,S,d,H,causal", [
    (600, 128, 128, 4, False),   # whole-layer kernel, 3 chunks (the last ragged)
    (120, 300, 256, 4, False),   # three-kernel path, 3 chunks
    (70, 257, 128, 4, True),     # causal
    (3, 17, 96, 3, False),       # one chunk
])
def test_host_input_streams_and_matches_device_path(pkg, cuda_ok, B, S, d, H, causal):
    cfg, ref, lay = _layer(pkg, B, S, d, H, causal)
    x, _ = generate_random_case(cfg, seed=5)
    with torch.inference_mode():
        y_dev = lay(x.cuda()).cpu()
        for pinned in (True, False):
            xh = x.pin_memory() if pinned else x.clone()
            y = lay(xh)
            assert y.device.type == "cpu" and y.shape == x.shape
            assert torch.equal(y, y_dev), f"pinned={pinned}"
    lay.check_status()
    idx = torch.arange(0, B, max(1, B // 4))
    with torch.inference_mode():
        assert compare_outputs(ref(x[idx]), y_dev[idx]).passed


def test_host_input_with_mask(pkg, cuda_ok):
    B, S, d, H = 520, 128, 128, 4
    cfg, ref, lay = _layer(pkg, B, S, d, H)
    x, mask = generate_random_case(cfg, seed=6, padding_ratio=0.3)
    with torch.inference_mode():
        y_dev = lay(x.cuda(), mask.cuda()).cpu()
        y = lay(x.pin_memory(), mask).clone()
    assert torch.equal(y, y_dev)
    with torch.inference_mode():
        assert compare_outputs(ref(x[:8], mask[:8]), y[:8]).passed


def test_host_output_buffer_is_reused(pkg, cuda_ok):
    cfg, ref, lay = _layer(pkg, 300, 128, 128, 4)
    x1, _ = generate_random_case(cfg, seed=1)
    x2, _ = generate_random_case(cfg, seed=2)
    with torch.inference_mode():
        y1 = lay(x1)
        y1c = y1.clone()
        y2 = lay(x2)
    assert y2.data_ptr() == y1.data_ptr()       # documented: the next call overwrites it
    assert not torch.equal(y1c, y2)
    assert y2.is_pinned()
