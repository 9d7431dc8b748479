#!/usr/bin/env python3
"""Benchmark of the B200 single transformer-layer forward (one JSON line).

Metric: layer tokens/s = B*S / latency, the reference
harness's definition (torch_transformer_benchmark.py:1906-1908).

Default workload: BASELINE cfg2 -- B=10000, S=128, d_model=128, H=4 (d_h=32),
x fp32 ~ N(0,1), seeded default nn.Linear init, LayerNorm gamma=1 beta=0, no
mask, non-causal. One step = one layer forward over the batch. The input
(655 MB) and output are larger than the 126 MB L2, so no flush is needed
between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

Multi-GPU (one process per GPU under torchrun): sequences are independent,
so every rank runs its own full cfg batch (weak scaling) with no data-path
collective; the timed region is bracketed by barriers and the reported time
is the max over ranks of the CUDA-event time.

``--impl reference`` times the reference's PyTorch layer on the host CPU
(all threads) -- the oracle port of BaselineSelfAttention + nn.LayerNorm --
on a bounded sample of the same workload; only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "cfg1": dict(B=4, S=128, d=128, H=4),
    "cfg2": dict(B=10000, S=128, d=128, H=4),
    "cfg3": dict(B=64, S=128, d=1024, H=4),
    "cfg4": dict(B=64, S=1024, d=128, H=4),
    "cfg5": dict(B=32, S=100000, d=1024, H=16),
}
METRIC = "layer tokens/s (B*S/latency)"
L2_BYTES = 126 * 1024 * 1024


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": j["hbm_gbs"], "bf16_tflops": j["bf16_tflops"],
                "bf16_tflops_sustained": j.get("bf16_tflops_sustained", j["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def fused_eligible(cfg) -> bool:
    """b200l_layer_forward runs the whole-layer kernel for these shapes."""
    return cfg["d"] in (64, 128) and cfg["d"] // cfg["H"] == 32 and cfg["S"] <= 128


def kernel_work(cfg):
    """Algorithmic bytes and FLOPs per launch of each kernel (per-token figures x T)."""
    B, S, d = cfg["B"], cfg["S"], cfg["d"]
    T = B * S
    return {
        # whole layer in one kernel: x read + y write (8d B/token); 8*T*d^2 + 4*B*S^2*d FLOP
        "fused_layer": {"bytes": 8.0 * T * d, "flops": 8.0 * T * d * d + 4.0 * B * S * S * d},
        # K1: x read (4d B/token) + q,k,v fp16 written (6d); 6*T*d^2 FLOP
        "qkv_ln_gemm": {"bytes": 10.0 * T * d, "flops": 6.0 * T * d * d},
        # K2: q,k,v read (6d) + ctx written (2d); 4*B*S^2*d FLOP (non-causal)
        "flash_attn": {"bytes": 8.0 * T * d, "flops": 4.0 * B * S * S * d},
        # K3: ctx (2d) + x (4d) read, y (4d) written; 2*T*d^2 FLOP
        "outproj_res_ln": {"bytes": 10.0 * T * d, "flops": 2.0 * T * d * d},
    }


def read_traffic(kernel: str, cfg_name: str):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    p = ROOT / "profiles" / "dram_traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[0] == kernel and parts[1] == cfg_name:
            try:
                return float(parts[2])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ["clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def start(self):
        import tempfile
        try:
            self.out = tempfile.NamedTemporaryFile("w", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(self.FIELDS):
                rows.append(parts)
        try:
            os.unlink(self.out.name)
        except OSError:
            pass
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower().startswith("active")})
        loaded = [s for s in sm if mx and s >= 0.3 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_reference(cfg, cfg_name, steps, warmup, budget_s=20.0):
    """The reference's PyTorch layer on the host CPU (oracle port), bounded sample."""
    from oracle import TransformerConfig, build_reference_layer, generate_random_case
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    B, S, d, H = cfg["B"], cfg["S"], cfg["d"], cfg["H"]
    # Score tensor [b,H,S,S] fp32 must fit: cfg5 materialises 19,073 GiB -> infeasible.
    if 4.0 * H * S * S > 64e9:
        return None
    sample_b = B
    tc = TransformerConfig(1, S, d, H)
    layer = build_reference_layer(tc, 1234)
    # Calibrate: time one sequence, size the per-step sample to ~budget/(steps+warmup).
    x1, _ = generate_random_case(tc, 1234 + 100000)
    with torch.inference_mode():
        layer(x1)
        t0 = time.perf_counter()
        layer(x1)
        per_seq = max(time.perf_counter() - t0, 1e-6)
    per_step = budget_s / max(1, steps + warmup)
    sample_b = int(max(1, min(B, per_step / per_seq)))
    tcs = TransformerConfig(sample_b, S, d, H)
    xs, _ = generate_random_case(tcs, 1234 + 100000)
    times = []
    with torch.inference_mode():
        for i in range(warmup + steps):
            t0 = time.perf_counter_ns()
            layer(xs)
            dt = (time.perf_counter_ns() - t0) / 1e9
            if i >= warmup:
                times.append(dt)
    med = statistics.median(times)
    cpu_model = ""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                cpu_model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"value": sample_b * S / med, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample_b} of {B} sequences of {cfg_name} per step (S={S}, d={d}, H={H}), fp32, "
                      f"median of {steps} after {warmup} warm-up, {cpu_model}",
            "ms_per_step": med * 1e3}


def run_reference_arm(args, cfg):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    r = cpu_reference(cfg, args.config, args.steps, args.warmup)
    if r is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"{args.config}: the reference materialises [B,H,S,S] scores "
                          f"({4.0 * cfg['H'] * cfg['S'] ** 2 * cfg['B'] / 2**30:.0f} GiB), infeasible on the host"}))
        return 0
    line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: x ~ N(0,1) fp32, seeded default nn.Linear init",
            "config": {"workload": args.config, **cfg, "causal": False, "sample_sequences_note": r["sample"]},
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def run_stack(args, cfg) -> int:
    """Full stack (blocks with the GELU FFN + final_norm) on one GPU: device-
    resident x, CUDA events around each forward, inputs larger than L2 or the
    L2 flushed between steps."""
    import __graft_entry__
    from oracle import TransformerConfig as OCfg, build_reference_transformer

    pkg = __graft_entry__.load_package()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S, d, H = cfg["B"], cfg["S"], cfg["d"], cfg["H"]
    f = args.ffn or 4 * d
    L = args.layers
    ocfg = OCfg(B, S, d, H, ffn_dim=f, num_layers=L)
    ref = build_reference_transformer(ocfg, 1234)
    model = pkg.B200Transformer(pkg.TransformerConfig(B, S, d, H, ffn_dim=f, num_layers=L)).to(dev).eval()
    model.load_state_dict(ref.state_dict(), strict=True)
    g = torch.Generator(device="cpu").manual_seed(1234 + 100000)
    x = torch.randn(B, S, d, generator=g).to(dev)
    big = x.numel() * 4 > L2_BYTES
    flush = None if big else torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x)
        torch.cuda.synchronize(dev)
        model.check_status()
        times = []
        for _ in range(args.steps):
            if flush is not None:
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            model(x)
            e1.record()
            times.append((e0, e1))
        torch.cuda.synchronize(dev)
        model.check_status()
    ms = statistics.fmean(a.elapsed_time(b) for a, b in times)
    T = B * S
    flops = L * (8.0 * T * d * d + 4.0 * B * S * S * d + 4.0 * T * d * f)
    pk_ = peaks()
    tflops = flops / (ms / 1e3) / 1e12
    launches = L * (6 + (1 if d > 256 else 0)) + 1
    print(json.dumps({
        "metric": "stack tokens/s (B*S/latency)", "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 operands / fp32 accumulate, fp32 in/out",
        "data": "synthetic: x ~ N(0,1) fp32, seeded default init of the reference's BaselineTransformer",
        "config": {"workload": f"{args.config} shape, {L} blocks, ffn_dim {f}", **cfg, "layers": L, "ffn_dim": f,
                   "l2": "inputs larger than L2" if big else "L2 flushed between steps"},
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk_["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tflops / pk_["bf16_tflops"], "kernel": "whole forward (all GEMMs + attention)",
                     "traffic": None, "peak_source": pk_["source"]},
        "gpu_launches": launches * args.steps,
    }))
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard-chunks", type=int, default=2,
                    help="pieces per rank for the scatter/gather measurement (N > 1)")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the config's batch (smaller cases for ncu captures)")
    ap.add_argument("--model", default="layer", choices=["layer", "stack"],
                    help="layer: the judged single layer (default); stack: full blocks with the GELU FFN")
    ap.add_argument("--layers", type=int, default=2, help="--model stack: number of blocks")
    ap.add_argument("--ffn", type=int, default=0, help="--model stack: ffn_dim (default 4*d)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = dict(CONFIGS[args.config])
    if args.batch > 0:
        cfg["B"] = args.batch

    if args.impl == "reference":
        return run_reference_arm(args, cfg)
    if args.model == "stack":
        return run_stack(args, cfg)

    import ctypes
    import datetime
    import torch.distributed as dist
    import __graft_entry__
    from oracle import TransformerConfig, build_reference_layer, generate_random_case

    world, rank, local = dist_env()
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pkg = __graft_entry__.load_package()
    L = pkg._lib.lib()

    B, S, d, H = cfg["B"], cfg["S"], cfg["d"], cfg["H"]
    T = B * S
    tc = TransformerConfig(B, S, d, H)
    ref = build_reference_layer(tc, 1234)
    layer = pkg.B200TransformerLayer(d, H, use_graphs=False).to(dev).eval()
    layer.load_state_dict(ref.state_dict(), strict=True)
    x_host, _ = generate_random_case(tc, 1234 + 100000 + rank)
    x = x_host.to(dev)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream(dev)
    pk = layer._ensure_pack(dev)
    desc = layer._desc(B, S, pk)
    layer._ensure_workspace(desc, dev)
    wsp, wsb, st = layer.workspace_ptr, layer._ws_bytes, stream.cuda_stream

    fused = fused_eligible(cfg)

    def step_kernels(ev=None):
        if fused:   # the product path: one whole-layer kernel
            if ev is not None:
                ev[0].record(stream)
            pkg._lib.check(L.b200l_layer_forward(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), wsp, wsb, st))
            if ev is not None:
                ev[3].record(stream)
            return
        if ev is not None:
            ev[0].record(stream)
        pkg._lib.check(L.b200l_qkv_ln_gemm(ctypes.byref(desc), x.data_ptr(), wsp, wsb, st))
        if ev is not None:
            ev[1].record(stream)
        pkg._lib.check(L.b200l_flash_attn(ctypes.byref(desc), wsp, wsb, st))
        if ev is not None:
            ev[2].record(stream)
        pkg._lib.check(L.b200l_outproj_res_ln(ctypes.byref(desc), x.data_ptr(), y.data_ptr(), wsp, wsb, st))
        if ev is not None:
            ev[3].record(stream)

    launches_per_step = 1 if fused else 3 + (2 if d > 256 else 0)

    with torch.inference_mode():
        for _ in range(args.warmup):
            step_kernels()
        torch.cuda.synchronize(dev)
        layer.check_status()

        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
        clk = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                           if os.environ.get("CUDA_VISIBLE_DEVICES") else local) if rank == 0 else None
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        if clk:
            clk.start()
            time.sleep(0.3)
        for i in range(args.steps):
            step_kernels(evs[i])
        torch.cuda.synchronize(dev)
        clocks = clk.stop() if clk else None
        total_ms = evs[0][0].elapsed_time(evs[-1][3])
        if fused:
            k_ms = {"fused_layer": statistics.fmean(e[0].elapsed_time(e[3]) for e in evs)}
        else:
            k_ms = {name: statistics.fmean(e[i].elapsed_time(e[i + 1]) for e in evs)
                    for i, name in enumerate(["qkv_ln_gemm", "flash_attn", "outproj_res_ln"])}
        layer.check_status()
        if world > 1:
            t = torch.tensor([total_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total_ms = float(t.item())
            dist.barrier()

        # ---- end to end through the public API: pinned host x -> forward ->
        # host y (the module streams a host-resident batch through the GPU,
        # copies in both directions overlapped with the kernels).
        xh = x_host.pin_memory()
        for _ in range(2):
            yh = layer(xh)
        torch.cuda.synchronize(dev)
        e2e_steps = max(3, min(args.steps, 10))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(e2e_steps):
            yh = layer(xh)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = e0.elapsed_time(e1) / e2e_steps
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())

        # ---- N > 1: the config's own batch held on rank 0's device, split by
        # ShardedLayer (x slices sent, y slices gathered back over NCCL
        # send/recv). Strong scaling; reported beside the weak-scaling value.
        sharded = None
        if world > 1:
            del xh, yh
            sl = pkg.ShardedLayer(layer, src=0, chunks=args.shard_chunks)
            xg = x if rank == 0 else None
            for _ in range(2):
                sl(xg)
            torch.cuda.synchronize(dev)
            sh_steps = max(3, min(args.steps, 10))
            dist.barrier()
            torch.cuda.synchronize(dev)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            for _ in range(sh_steps):
                sl(xg)
            s1.record(stream)
            torch.cuda.synchronize(dev)
            layer.check_status()
            t = torch.tensor([s0.elapsed_time(s1) / sh_steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sh_ms = float(t.item())
            sharded = {"value": T / (sh_ms / 1e3), "unit": "tokens/s", "ms_per_step": sh_ms,
                       "global_batch": B, "per_gpu_batch": -(-B // world), "chunks": args.shard_chunks,
                       "scaling": "strong", "steps": sh_steps,
                       "path": "ShardedLayer.forward: x on rank 0's device, slices over NCCL "
                               "send/recv, y gathered into rank 0's output"}

    ms_per_step = total_ms / args.steps
    value = world * T / (ms_per_step / 1e3)
    pk_ = peaks()
    work = kernel_work(cfg)
    flops_layer = 8.0 * T * d * d + 4.0 * B * S * S * d
    bytes_layer = 8.0 * T * d
    # Dominant kernel = the one with the largest share of the step.
    dom = max(k_ms, key=k_ms.get)
    hbm_bound = args.config in ("cfg1", "cfg2")
    if hbm_bound:
        achieved = work[dom]["bytes"] / (k_ms[dom] / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": pk_["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / pk_["hbm_gbs"], "kernel": dom,
                "traffic": read_traffic(dom, args.config), "peak_source": pk_["source"]}
    else:
        achieved = work[dom]["flops"] / (k_ms[dom] / 1e3) / 1e12
        pk_t = pk_["bf16_tflops_sustained"] if ms_per_step > 100 else pk_["bf16_tflops"]
        roof = {"bound": "tensor", "achieved": achieved, "peak": pk_t, "unit": "TFLOP/s",
                "frac": achieved / pk_t, "kernel": dom,
                "traffic": read_traffic(dom, args.config), "peak_source": pk_["source"]}

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return 0

    cpu = None
    if not args.no_cpu_baseline and world == 1:
        c = cpu_reference(cfg, args.config, steps=3, warmup=1, budget_s=20.0)
        cpu = None if c is None else {k: c[k] for k in ("value", "unit", "cores", "kind", "sample")}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 operands / fp32 accumulate, fp32 in/out",
        "data": "synthetic: x ~ N(0,1) fp32 seeded per rank, seeded default nn.Linear init, no mask",
        "config": {"workload": args.config, **cfg, "causal": False, "per_gpu_batch": B,
                   "global_batch": B * world, "parallelism": f"batch shards x{world} (no collective)",
                   "l2": "inputs larger than L2" if T * d * 4 > L2_BYTES else "inputs smaller than L2 (no flush)"},
        "e2e": {"value": world * T / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": T * d * 4, "d2h_bytes_per_step": T * d * 4,
                "ms_per_step": e2e_ms, "path": "B200TransformerLayer.forward(pinned host x) -> host y, streamed in chunks with both copy directions overlapped"},
        "roofline": roof,
        "layer_roofline": {"hbm_gbs": bytes_layer / (ms_per_step / 1e3) / 1e9,
                           "hbm_frac": bytes_layer / (ms_per_step / 1e3) / 1e9 / pk_["hbm_gbs"],
                           "tflops": flops_layer / (ms_per_step / 1e3) / 1e12,
                           "tflops_frac": flops_layer / (ms_per_step / 1e3) / 1e12 / pk_["bf16_tflops"]},
        "kernel_ms": k_ms,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if sharded is not None:
        line["sharded_from_rank0"] = sharded
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
