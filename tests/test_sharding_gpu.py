"""Batch and head sharding over NCCL on two B200s: the gathered output is
bitwise equal to the one-GPU output (every sequence runs the same kernels
either way), also when x starts in rank 0's host memory; head sharding
(ctx columns gathered from both ranks) equals the same head ranges computed
on one GPU and passes the reference gate.

Skipped unless two sm_100 devices are visible. Ranks are spawned processes,
one per GPU, with a short process-group timeout.
"""

import socket
import sys
from pathlib import Path

import pytest
import torch

from tests.conftest import spawn_ranks

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu

CASES = [
    # (B, S, d, H, causal, chunks): whole-layer kernel, three-kernel path, causal, B < world
    (37, 128, 128, 4, False, 1),
    (37, 128, 128, 4, False, 3),
    (6, 300, 256, 4, False, 2),
    (5, 200, 128, 2, True, 1),
    (1, 64, 128, 4, False, 1),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, root: str) -> None:
    import datetime
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    from oracle import TransformerConfig, build_reference_layer, generate_random_case

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        with torch.inference_mode():
            for B, S, d, H, causal, chunks in CASES:
                cfg = TransformerConfig(B, S, d, H, causal=causal)
                ref = build_reference_layer(cfg, seed=21)
                layer = pkg.B200TransformerLayer(d, H, causal).to(dev).eval()
                layer.load_state_dict(ref.state_dict(), strict=True)
                x, _ = generate_random_case(cfg, seed=22)
                x = x.to(dev)
                print(f"rank {rank}: case {(B, S, d, H, causal, chunks)}", flush=True)
                y = pkg.sharded_forward(layer, x if rank == 0 else None, chunks=chunks)
                torch.cuda.synchronize(dev)
                layer.check_status()
                if rank == 0:
                    single = layer(x).clone()
                    torch.cuda.synchronize(dev)
                    assert torch.equal(y, single), f"case {(B, S, d, H, causal, chunks)}"
                else:
                    assert y is None
            # Host-resident x on rank 0: pieces staged through rank 0's GPU.
            cfg = TransformerConfig(6, 300, 256, 4)
            ref = build_reference_layer(cfg, seed=23)
            layer = pkg.B200TransformerLayer(256, 4).to(dev).eval()
            layer.load_state_dict(ref.state_dict(), strict=True)
            x, _ = generate_random_case(cfg, seed=24)
            xh = x.pin_memory() if rank == 0 else None
            y = pkg.ShardedLayer(layer, chunks=2)(xh)
            torch.cuda.synchronize(dev)
            layer.check_status()
            if rank == 0:
                assert y.device.type == "cpu"
                single = layer(x.to(dev)).cpu()
                assert torch.equal(y, single), "host-resident sharded output differs"
            # Head sharding (B smaller than the number of ranks' work): cfg1 shape.
            for B, S, d, H, pad in ((4, 128, 128, 4, 0.0), (2, 200, 256, 4, 0.3)):
                cfg = TransformerConfig(B, S, d, H)
                ref = build_reference_layer(cfg, seed=25)
                layer = pkg.B200TransformerLayer(d, H).to(dev).eval()
                layer.load_state_dict(ref.state_dict(), strict=True)
                x, mask = generate_random_case(cfg, seed=26, padding_ratio=pad)
                m = mask.to(dev) if pad > 0 else None
                y = pkg.head_sharded_forward(layer, x.to(dev) if rank == 0 else None,
                                             m if rank == 0 else None)
                torch.cuda.synchronize(dev)
                if rank == 0:
                    from oracle import compare_outputs
                    res = compare_outputs(ref(x, mask if pad > 0 else None), y.cpu())
                    assert res.passed, f"head-sharded {(B, S, d, H)}: {res}"
                    parts = [layer._head_ctx(x.to(dev), m, a, b) for a, b in pkg.head_shards(H, world)]
                    single = layer._finish_from_ctx(x.to(dev), m, torch.cat(parts, 1))
                    assert torch.equal(y, single), "head-sharded output differs from one GPU"
                else:
                    assert y is None
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        # Leave at once: a rank that failed with transfers in flight must not
        # wait in destroy_process_group for peers that will never answer.
        import os
        import traceback
        traceback.print_exc()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(1)


def test_sharded_forward_two_gpus_bitwise(pkg):
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if any(torch.cuda.get_device_capability(i)[0] != 10 for i in range(2)):
        pytest.skip("needs sm_100 devices")
    spawn_ranks(_worker, (2, _free_port(), str(ROOT)), 2, 240)
