"""Generate golden fixtures from the reference's own PyTorch classes.

Run in a container where the reference source tree is mounted (read-only):

    python tests/golden/make_golden.py --reference-root <path to COBRA-GPU-Kernel>

It loads ``torch_transformer_benchmark.py`` by path, as the reference's own
tools do (tools/sweep.py:23-29), builds the judged layer from the reference's
``nn.LayerNorm`` + ``BaselineSelfAttention`` + ``nn.LayerNorm`` under
``torch.manual_seed(seed)`` (the harness's construction, :2024-2031), draws
inputs with the reference's ``generate_random_case`` on the CPU (:1575-1613),
runs the forward in fp32 on the CPU, and stores x, mask, y and the weights.

It also builds full stacks with the reference's own ``BaselineTransformer``
(blocks with the GELU FFN, final_norm; :126-173) for the ``model_*`` fixtures.

The fixtures are what ``tests/test_oracle.py`` pins the CPU oracle against
and what the GPU parity tests compare the CUDA path with. The reference is
never needed at test time.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))

# name, B, S, d, H, causal, padding, n_trials, store_weights
CASES = [
    ("cfg1_tiny", 4, 128, 128, 4, False, 0.0, 2, True),
    ("cfg1_tiny_causal", 4, 128, 128, 4, True, 0.0, 1, True),
    ("odd_b3_s17_d96_h3", 3, 17, 96, 3, False, 0.0, 1, True),
    ("odd_b3_s17_d96_h3_causal", 3, 17, 96, 3, True, 0.0, 1, True),
    ("seq1_b2_d128_h4", 2, 1, 128, 4, False, 0.0, 1, True),
    ("hd64_b2_s130_d256_h4", 2, 130, 256, 4, False, 0.0, 1, True),
    ("hd256_b2_s96_d256_h1", 2, 96, 256, 1, False, 0.0, 1, True),
    ("hd32_b2_s300_d128_h4_causal", 2, 300, 128, 4, True, 0.0, 1, True),
    ("pad03_b4_s128_d128_h4", 4, 128, 128, 4, False, 0.3, 1, True),
    ("d1024_h16_b1_s160", 1, 160, 1024, 16, False, 0.0, 1, False),
]
# Full stacks (the reference's BaselineTransformer: blocks with GELU FFN, final_norm):
# name, B, S, d, H, ffn_dim, num_layers, causal, padding, store_weights
MODEL_CASES = [
    ("model_b2_s64_d128_h4_f512_l2", 2, 64, 128, 4, 512, 2, False, 0.0, True),
    ("model_causal_b2_s100_d128_h4_f256_l1", 2, 100, 128, 4, 256, 1, True, 0.0, True),
    ("model_pad03_b3_s128_d256_h4_f1024_l2", 3, 128, 256, 4, 1024, 2, False, 0.3, False),
    ("model_odd_b2_s37_d96_h3_f160_l1", 2, 37, 96, 3, 160, 1, False, 0.0, True),
]
WEIGHT_SEED = 1234      # torch_transformer_benchmark.py:1961 default seed
INPUT_SEED = 1234       # trials use seed + t (:1724-1731)


def load_reference(root: str):
    spec = importlib.util.spec_from_file_location(
        "bm", os.path.join(root, "torch_transformer_benchmark.py"))
    bm = importlib.util.module_from_spec(spec)
    sys.modules["bm"] = bm
    spec.loader.exec_module(bm)
    return bm


def state_sha(sd) -> str:
    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].detach().contiguous().float().numpy().tobytes())
    return h.hexdigest()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True)
    args = ap.parse_args()
    bm = load_reference(args.reference_root)

    class RefLayer(nn.Module):
        """The judged unit assembled from the reference's own classes."""

        def __init__(self, d, h, causal):
            super().__init__()
            self.causal = causal
            self.norm1 = nn.LayerNorm(d)
            self.attention = bm.BaselineSelfAttention(d, h)
            self.norm2 = nn.LayerNorm(d)

        def forward(self, x, mask=None):
            return self.norm2(x + self.attention(self.norm1(x), mask, self.causal))

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, B, S, d, H, causal, pad, trials, store_w in CASES:
        cfg = bm.TransformerConfig(B, S, d, H, d, 1, causal)
        cfg.validate()
        torch.manual_seed(WEIGHT_SEED)
        layer = RefLayer(d, H, causal).eval()
        sd = {k: v.detach().clone() for k, v in layer.state_dict().items()}
        out = {"name": name, "B": B, "S": S, "d": d, "H": H, "causal": causal,
               "padding": pad, "weight_seed": WEIGHT_SEED, "state_sha": state_sha(sd),
               "trials": []}
        if store_w:
            out["state_dict"] = sd
        with torch.inference_mode():
            for t in range(trials):
                x, mask = bm.generate_random_case(cfg, torch.device("cpu"), torch.float32,
                                                  INPUT_SEED + t, pad, 1.0)
                m = mask if pad > 0 else None
                y = layer(x, m)
                out["trials"].append({"seed": INPUT_SEED + t, "x": x.clone(),
                                      "mask": mask.clone() if pad > 0 else None,
                                      "y": y.clone()})
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(out, path)
        print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB)")

    # Full stacks, straight from the reference's BaselineTransformer (:149-173).
    for name, B, S, d, H, f, L, causal, pad, store_w in MODEL_CASES:
        cfg = bm.TransformerConfig(B, S, d, H, f, L, causal)
        cfg.validate()
        torch.manual_seed(WEIGHT_SEED)
        model = bm.BaselineTransformer(cfg).eval()
        sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
        out = {"name": name, "B": B, "S": S, "d": d, "H": H, "ffn_dim": f, "num_layers": L,
               "causal": causal, "padding": pad, "weight_seed": WEIGHT_SEED,
               "state_sha": state_sha(sd), "trials": []}
        if store_w:
            out["state_dict"] = sd
        with torch.inference_mode():
            x, mask = bm.generate_random_case(cfg, torch.device("cpu"), torch.float32,
                                              INPUT_SEED, pad, 1.0)
            m = mask if pad > 0 else None
            y = model(x, m)
            out["trials"].append({"seed": INPUT_SEED, "x": x.clone(),
                                  "mask": mask.clone() if pad > 0 else None, "y": y.clone()})
        path = os.path.join(HERE, f"{name}.pt")
        torch.save(out, path)
        print(f"wrote {path} ({os.path.getsize(path) / 1e6:.2f} MB)")


if __name__ == "__main__":
    main()
