"""Batch sharding over one process per device: host logic on CPU (gloo, world 2).

The per-rank compute here is the CPU oracle layer (the checker), so these
tests cover the scatter / gather plumbing of ``sharding.sharded_forward``:
slice bounds, chunked point-to-point transfers, mask transport, idle ranks,
a non-zero source rank and input validation that raises on every rank.
The same function runs over NCCL in ``tests/test_sharding_gpu.py``.
"""

import socket
import sys
from pathlib import Path

import pytest
import torch

from tests.conftest import spawn_ranks

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_batch_shards_bounds(pkg):
    from cobra_gpu_kernel_b200.sharding import batch_shards
    assert batch_shards(10000, 8) == [(i * 1250, (i + 1) * 1250) for i in range(8)]
    assert batch_shards(32, 8) == [(4 * i, 4 * i + 4) for i in range(8)]
    assert batch_shards(5, 2) == [(0, 3), (3, 5)]
    assert batch_shards(4, 8) == [(0, 1), (1, 2), (2, 3), (3, 4)] + [(4, 4)] * 4
    assert batch_shards(7, 3) == [(0, 3), (3, 6), (6, 7)]
    assert batch_shards(0, 2) == [(0, 0), (0, 0)]
    for B in range(0, 40):
        for n in range(1, 9):
            sh = batch_shards(B, n)
            assert len(sh) == n
            assert sh[0][0] == 0 and sh[-1][1] == B
            assert all(a <= b for a, b in sh)
            assert all(sh[i][1] == sh[i + 1][0] for i in range(n - 1))
            assert max(b - a for a, b in sh) == -(-B // n)
    with pytest.raises(ValueError):
        batch_shards(3, 0)


def _worker(rank: int, world: int, port: int, root: str) -> None:
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from cobra_gpu_kernel_b200.sharding import ShardedLayer, sharded_forward
    from oracle import TransformerConfig, build_reference_layer, generate_random_case

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        def layer_for(cfg):
            return build_reference_layer(cfg, seed=77)

        def local_chunks(layer, x, mask, shards_, chunks):
            from cobra_gpu_kernel_b200.sharding import _chunk_ranges
            out = torch.empty_like(x)
            for a, b in shards_:
                for c0, c1 in _chunk_ranges(a, b, chunks):
                    m = mask[c0:c1] if mask is not None else None
                    out[c0:c1] = layer(x[c0:c1], m)
            return out

        from cobra_gpu_kernel_b200.sharding import batch_shards
        with torch.inference_mode():
            # 1. ragged batch, several chunkings: bitwise equal to the same
            #    slices computed in one process; close to the whole batch.
            cfg = TransformerConfig(5, 9, 32, 2)
            layer = layer_for(cfg)
            x, _ = generate_random_case(cfg, seed=5)
            full = layer(x)
            for chunks in (1, 2, 5):
                y = sharded_forward(layer, x if rank == 0 else None, chunks=chunks)
                if rank == 0:
                    exp = local_chunks(layer, x, None, batch_shards(5, world), chunks)
                    assert torch.equal(y, exp), f"chunks={chunks}"
                    torch.testing.assert_close(y, full, atol=1e-5, rtol=1e-5)
                else:
                    assert y is None

            # 2. B < world: rank 1 idle, rank 0 computes everything.
            cfg1 = TransformerConfig(1, 6, 32, 4)
            layer1 = layer_for(cfg1)
            x1, _ = generate_random_case(cfg1, seed=6)
            y = sharded_forward(layer1, x1 if rank == 0 else None)
            if rank == 0:
                assert torch.equal(y, layer1(x1))

            # 3. key-padding mask travels with its slice.
            cfgm = TransformerConfig(4, 8, 32, 2)
            layerm = layer_for(cfgm)
            xm, mask = generate_random_case(cfgm, seed=9, padding_ratio=0.5)
            assert not bool(mask.all())
            y = sharded_forward(layerm, xm if rank == 0 else None,
                                mask if rank == 0 else None, chunks=2)
            if rank == 0:
                exp = local_chunks(layerm, xm, mask, batch_shards(4, world), 2)
                assert torch.equal(y, exp)

            # 4. source rank 1, causal layer, through the module wrapper.
            cfgc = TransformerConfig(3, 7, 32, 2, causal=True)
            layerc = layer_for(cfgc)
            xc, _ = generate_random_case(cfgc, seed=11)
            y = ShardedLayer(layerc, src=1)(xc if rank == 1 else None)
            if rank == 1:
                exp = local_chunks(layerc, xc, None, batch_shards(3, world), 1)
                assert torch.equal(y, exp)
            else:
                assert y is None

            # 5. a bad input on the source raises the same error on every rank,
            #    and the group is still usable afterwards.
            for bad, msg in ((x.half(), "float32"), (x[0], "[B, S, d]"),
                             (None, "no input tensor")):
                with pytest.raises(ValueError, match=msg.replace("[", r"\[").replace("]", r"\]")):
                    sharded_forward(layer, bad if rank == 0 else None)
            with pytest.raises(ValueError, match="valid_token_mask"):
                sharded_forward(layer, x if rank == 0 else None,
                                torch.ones(5, 8, dtype=torch.bool) if rank == 0 else None)
            y = sharded_forward(layer, x if rank == 0 else None)
            if rank == 0:
                assert torch.equal(y, local_chunks(layer, x, None, batch_shards(5, world), 1))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_forward_gloo_world2(pkg, monkeypatch):
    port = _free_port()
    monkeypatch.setenv("GLOO_SOCKET_IFNAME", "lo")
    spawn_ranks(_worker, (2, port, str(ROOT)), 2, 120)


def _failing_worker(rank: int, world: int, port: int, root: str) -> None:
    """Rank 1's layer raises after the header: rank 0 must not wait forever."""
    import datetime
    import time
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from cobra_gpu_kernel_b200.sharding import sharded_forward

    def layer(x, mask=None):
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        return x * 2.0

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=3))
    x = torch.randn(4, 3, 8)
    t0 = time.monotonic()
    try:
        sharded_forward(layer, x if rank == 0 else None)
    except RuntimeError as e:
        if rank == 1:
            assert "injected failure" in str(e)
        else:
            assert time.monotonic() - t0 < 60, "rank 0 waited past the group timeout"
        return
    raise AssertionError(f"rank {rank}: the failure was not reported")


def test_sharded_forward_peer_failure_times_out(pkg, monkeypatch):
    port = _free_port()
    monkeypatch.setenv("GLOO_SOCKET_IFNAME", "lo")
    spawn_ranks(_failing_worker, (2, port, str(ROOT)), 2, 120)
