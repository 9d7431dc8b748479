"""GPU parity tests: the sm_100a path through the C ABI against the CPU oracle.

Gate (torch_transformer_benchmark.py:1959-1960): every output
element satisfies abs_err <= 2e-3 OR rel_err <= 2e-2 against the reference
layer (the fp32 CPU oracle, itself pinned bit-exactly to the reference).

Per-kernel tests compare each kernel with a torch fp32 reference of the same
op computed from the same fp16-rounded operands, so a failure names the
kernel that broke:
  K1  q/k/v = fp16(LN1(x)) @ fp16(Wqkv)^T + b         tol: abs 2e-3 + 4e-3*|ref|
  K2  ctx = softmax(q k^T / sqrt(dh)) v  (fp32 math)   tol: abs 2e-3 + 1e-2*|ref|
  K3  y = LN2(x + ctx @ fp16(Wo)^T + bo)  (fp32 math)  tol: abs 1e-4 + 1e-4*|ref|
"""

import ctypes
import math

import pytest
import torch

from oracle import (TransformerConfig, build_reference_layer, compare_outputs,
                    generate_random_case)
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

# (B, S, d, H, causal) -- covers every kernel template:
# K1 KP in {64,128,192,256} + the d>256 TMA path; K2 dhp in {32,64,128,256};
# K3 BN in {64,128,192,256}, the clusters for d = 256 NC (NC 2, 3, 4, 6, 8)
# and the d>256 residual path.
SHAPES = [
    (4, 128, 128, 4, False),     # cfg1
    (3, 17, 96, 3, False),       # odd shape (tools/validate.py:96-97)
    (2, 64, 64, 2, False),
    (2, 130, 256, 4, False),     # dh 64, S not a multiple of 128
    (2, 96, 256, 1, False),      # dh 256
    (2, 70, 160, 5, False),      # d 160 -> KP 192
    (2, 200, 512, 4, False),     # dh 128, d > 256 path
    (2, 150, 768, 6, False),     # K3 cluster of 3 CTAs, last row tile partial
    (1, 130, 1536, 12, False),   # K3 cluster of 6
    (1, 140, 2048, 16, False),   # K3 cluster of 8
    (2, 100, 640, 5, False),     # d > 256 but not 256 * NC: residual epilogue + row LayerNorm
    (1, 160, 1024, 16, False),   # cfg5 family, short S
    (2, 300, 128, 4, True),      # causal, 3 query tiles
    (1, 1, 128, 4, False),       # S = 1 (tools/validate.py:94-95)
    (2, 257, 128, 4, True),
]


def _ids(s):
    B, S, d, H, c = s
    return f"B{B}_S{S}_d{d}_H{H}" + ("_causal" if c else "")


def make_layer(pkg, B, S, d, H, causal, seed=1234):
    cfg = TransformerConfig(B, S, d, H, causal=causal)
    ref = build_reference_layer(cfg, seed)
    lay = pkg.B200TransformerLayer(d, H, causal, use_graphs=False).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    return cfg, ref, lay


def ws_views(pkg, lay, B, S, d, H):
    L = pkg._lib.workspace_layout(B, S, d, H)
    base = lay._ws[lay._ws_off:]
    dh, dhp, sp = L["dh"], L["dhp"], L["sp"]

    def f16(off, n):
        return base[off:off + 2 * n].view(torch.float16)

    q = f16(L["q"], B * H * S * dhp).view(B * H, S, dhp)
    k = f16(L["k"], B * H * S * dhp).view(B * H, S, dhp)
    vt = f16(L["vt"], B * H * dhp * sp).view(B * H, dhp, sp)
    ctx = f16(L["ctx"], B * S * d).view(B * S, d)
    return q, k, vt, ctx, dh, dhp


def run_stepwise(pkg, lay, x):
    """Run K1, K2, K3 one entry point at a time; returns y."""
    B, S, d = x.shape
    pk = lay._ensure_pack(x.device)
    desc = lay._desc(B, S, pk)
    lay._ensure_workspace(desc, x.device, stepwise=True)
    L = pkg._lib.lib()
    st = torch.cuda.current_stream().cuda_stream
    y = torch.empty_like(x)
    pkg._lib.check(L.b200l_qkv_ln_gemm(ctypes.byref(desc), x.data_ptr(), lay.workspace_ptr, lay._ws_bytes, st))
    pkg._lib.check(L.b200l_flash_attn(ctypes.byref(desc), lay.workspace_ptr, lay._ws_bytes, st))
    pkg._lib.check(L.b200l_outproj_res_ln(ctypes.byref(desc), x.data_ptr(), y.data_ptr(),
                                          lay.workspace_ptr, lay._ws_bytes, st))
    torch.cuda.synchronize()
    lay.check_status()
    return y


def _ln(x, w, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[-1],), w, b, eps)


def _close(name, got, ref, atol, rtol):
    err = (got.float() - ref.float()).abs()
    lim = atol + rtol * ref.float().abs()
    bad = ~(err <= lim)
    assert torch.isfinite(got.float()).all(), f"{name}: non-finite values"
    assert not bad.any(), (f"{name}: {int(bad.sum())}/{bad.numel()} elements out of tolerance, "
                           f"max_abs={err.max().item():.3e}")


@pytest.fixture(autouse=True)
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("shape", SHAPES, ids=_ids)
def test_kernels_stepwise(pkg, cuda_ok, shape):
    B, S, d, H, causal = shape
    cfg, ref, lay = make_layer(pkg, B, S, d, H, causal)
    x, _ = generate_random_case(cfg, seed=1234)
    xg = x.cuda()
    with torch.inference_mode():
        y = run_stepwise(pkg, lay, xg)
        q, k, vt, ctx, dh, dhp = ws_views(pkg, lay, B, S, d, H)
        att = lay.attention
        # ---- K1
        h16 = _ln(xg, lay.norm1.weight, lay.norm1.bias, lay.norm1.eps).half().float()
        w = torch.cat([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight]).half().float()
        b = torch.cat([att.q_proj.bias, att.k_proj.bias, att.v_proj.bias]).float()
        qkv = (h16.view(B * S, d) @ w.T + b).view(B, S, 3, H, dh).permute(2, 0, 3, 1, 4)
        qkv = qkv.reshape(3, B * H, S, dh)
        _close("K1 q", q[..., :dh], qkv[0], 2e-3, 4e-3)
        _close("K1 k", k[..., :dh], qkv[1], 2e-3, 4e-3)
        _close("K1 v", vt[:, :dh, :S].transpose(1, 2), qkv[2], 2e-3, 4e-3)
        if dhp > dh:
            assert (q[..., dh:] == 0).all() and (k[..., dh:] == 0).all() and (vt[:, dh:, :S] == 0).all()
        # ---- K2 (from the kernel's own fp16 q/k/v)
        qf, kf, vf = q[..., :dh].float(), k[..., :dh].float(), vt[:, :dh, :S].transpose(1, 2).float()
        sc = (qf @ kf.transpose(1, 2)) * dh ** -0.5
        if causal:
            sc = sc.masked_fill(torch.ones(S, S, device=sc.device, dtype=torch.bool).triu(1), float("-inf"))
        ctx_ref = (torch.softmax(sc, -1) @ vf).view(B, H, S, dh).permute(0, 2, 1, 3).reshape(B * S, d)
        _close("K2 ctx", ctx, ctx_ref, 2e-3, 1e-2)
        # ---- K3 (from the kernel's own fp16 ctx)
        r = xg.view(B * S, d) + ctx.float() @ att.out_proj.weight.half().float().T + att.out_proj.bias
        y_ref = _ln(r, lay.norm2.weight, lay.norm2.bias, lay.norm2.eps).view(B, S, d)
        _close("K3 y", y, y_ref, 1e-4, 1e-4)
        # ---- whole layer against the CPU oracle (the reference's gate)
        y_cpu = ref(x)
    res = compare_outputs(y_cpu, y.cpu())
    assert res.passed, f"layer gate failed: {res}"


@pytest.mark.parametrize("path", sorted(p.name for p in GOLDEN.glob("*.pt") if not p.name.startswith("model_")))
def test_golden_fixtures(pkg, cuda_ok, path):
    """The reference's own outputs (tests/golden, produced by make_golden.py)."""
    g = torch.load(GOLDEN / path)
    cfg = TransformerConfig(g["B"], g["S"], g["d"], g["H"], causal=g["causal"])
    ref = build_reference_layer(cfg, g["weight_seed"])
    if "state_dict" in g:
        ref.load_state_dict(g["state_dict"], strict=True)
    lay = pkg.B200TransformerLayer(g["d"], g["H"], g["causal"]).cuda().eval()
    lay.load_state_dict(ref.state_dict(), strict=True)
    for t in g["trials"]:
        mask = t["mask"].cuda() if g["padding"] > 0 else None
        with torch.inference_mode():
            y = lay(t["x"].cuda(), mask).clone()
        torch.cuda.synchronize()
        lay.check_status()
        res = compare_outputs(t["y"], y.cpu())
        assert res.passed, f"{path} seed {t['seed']}: {res}"


def test_graph_replay_matches_eager(pkg, cuda_ok):
    B, S, d, H = 4, 128, 128, 4
    cfg = TransformerConfig(B, S, d, H)
    ref = build_reference_layer(cfg, 7)
    eager = pkg.B200TransformerLayer(d, H, use_graphs=False).cuda().eval()
    graphed = pkg.B200TransformerLayer(d, H, use_graphs=True).cuda().eval()
    eager.load_state_dict(ref.state_dict())
    graphed.load_state_dict(ref.state_dict())
    for seed in (1, 2, 3):
        x, _ = generate_random_case(cfg, seed=seed)
        with torch.inference_mode():
            ye = eager(x.cuda()).clone()
            yg = graphed(x.cuda()).clone()
        assert torch.equal(ye, yg), f"graph replay differs from eager (seed {seed})"
    assert graphed._graph is not None


def test_deterministic_repeat(pkg, cuda_ok):
    cfg, ref, lay = make_layer(pkg, 8, 256, 128, 4, False)
    x, _ = generate_random_case(cfg, seed=99)
    with torch.inference_mode():
        y1 = lay(x.cuda()).clone()
        y2 = lay(x.cuda()).clone()
    assert torch.equal(y1, y2)


def test_all_true_mask_is_accepted(pkg, cuda_ok):
    cfg, ref, lay = make_layer(pkg, 2, 64, 128, 4, False)
    x, mask = generate_random_case(cfg, seed=5)
    with torch.inference_mode():
        y = lay(x.cuda(), mask.cuda()).clone()
        y_ref = ref(x)
    assert compare_outputs(y_ref, y.cpu()).passed


@pytest.mark.parametrize("cfg_name,B,S,d,H", [
    ("cfg3", 64, 128, 1024, 4),
    ("cfg4", 64, 1024, 128, 4),
])
def test_baseline_configs_full(pkg, cuda_ok, cfg_name, B, S, d, H):
    """cfg3 / cfg4 at full size against the CPU fp32 oracle, 5 seeds
    (the harness default trial count, torch_transformer_benchmark.py:1958-1961)."""
    cfg, ref, lay = make_layer(pkg, B, S, d, H, False)
    for t in range(5):
        x, _ = generate_random_case(cfg, seed=1234 + t)
        with torch.inference_mode():
            y = lay(x.cuda()).clone()
            y_ref = ref(x)
        torch.cuda.synchronize()
        lay.check_status()
        res = compare_outputs(y_ref, y.cpu())
        assert res.passed, f"{cfg_name} trial {t}: {res}"


def test_cfg2_full_size_sampled(pkg, cuda_ok):
    """cfg2 (B=10000) on the GPU; the CPU oracle checks 64 sampled sequences
    (sequences are independent, torch_transformer_benchmark.py:1446-1447)."""
    B, S, d, H = 10000, 128, 128, 4
    cfg, ref, lay = make_layer(pkg, B, S, d, H, False)
    x, _ = generate_random_case(cfg, seed=1234)
    with torch.inference_mode():
        y = lay(x.cuda()).cpu()
    lay.check_status()
    idx = torch.randperm(B, generator=torch.Generator().manual_seed(0))[:64]
    with torch.inference_mode():
        y_ref = ref(x[idx])
    res = compare_outputs(y_ref, y[idx])
    assert res.passed, res


def test_error_codes(pkg, cuda_ok):
    lay = pkg.B200TransformerLayer(128, 4).cuda()
    with pytest.raises(ValueError):
        lay(torch.zeros(2, 3, 64, device="cuda"))
    with pytest.raises(TypeError):
        lay(torch.zeros(2, 3, 128, device="cuda", dtype=torch.float64))
    bad = pkg.B200TransformerLayer(48, 3).cuda()      # head_dim 16: unsupported
    with pytest.raises(pkg._lib.B200LError, match="head_dim 16 unsupported"):
        bad(torch.zeros(1, 4, 48, device="cuda"))


FUSED_SHAPES = [
    (4, 128, 128, 4, False),    # cfg1
    (3, 128, 128, 4, False),    # odd batch: the last pair has one sequence
    (5, 77, 128, 4, True),      # S < 128, causal
    (1, 1, 128, 4, False),      # S = 1
    (2, 100, 64, 2, False),     # d = 64
    (300, 128, 128, 4, False),  # more pairs than SMs: persistent loop
    (301, 128, 128, 4, False),  # odd batch over more pairs than SMs: slot 1 idle in the last pair
    (299, 100, 64, 2, True),    # the same at d = 64, S < 128, causal
]


@pytest.mark.parametrize("shape", FUSED_SHAPES, ids=_ids)
def test_fused_layer_matches_three_kernel_path(pkg, cuda_ok, shape):
    """b200l_layer_forward runs the whole-layer kernel for d in {64, 128},
    head_dim 32, S <= 128; the per-kernel entry points run K1 -> K2 -> K3.
    Both must pass the reference gate and agree with each other."""
    B, S, d, H, causal = shape
    cfg, ref, lay = make_layer(pkg, B, S, d, H, causal)
    x, _ = generate_random_case(cfg, seed=4321)
    xg = x.cuda()
    with torch.inference_mode():
        y3 = run_stepwise(pkg, lay, xg)
        yf = lay(xg).clone()
        torch.cuda.synchronize()
        lay.check_status()
        y_ref = ref(x)
    _close("fused vs three-kernel", yf, y3, 1e-3, 1e-3)
    res = compare_outputs(y_ref, yf.cpu())
    assert res.passed, f"fused layer gate failed: {res}"


def test_fused_cfg2_every_sequence_matches_three_kernel_path(pkg, cuda_ok):
    """Full-size cfg2 (10000 sequences, ~34 sequence pairs per persistent CTA):
    every output row of the whole-layer kernel against the three-kernel path,
    three runs, so a rare ordering bug in the long persistent loop shows."""
    B, S, d, H = 10000, 128, 128, 4
    cfg, ref, lay = make_layer(pkg, B, S, d, H, False)
    x, _ = generate_random_case(cfg, seed=77)
    xg = x.cuda()
    with torch.inference_mode():
        y3 = run_stepwise(pkg, lay, xg).clone()
        bad_rows = []
        for _ in range(3):
            yf = lay(xg).clone()
            torch.cuda.synchronize()
            lay.check_status()
            err = (yf - y3).abs().amax(dim=-1)               # [B, S]
            bad = torch.nonzero(err > 1e-3)
            bad_rows.append(bad[:8].tolist())
            assert bad.shape[0] == 0, f"{bad.shape[0]} rows differ, first {bad_rows[-1]}, max {err.max():.3e}"
