"""Head sharding over one process per device: host logic on CPU (gloo, world 2).

``headshard.head_sharded_forward`` broadcasts x from the caller's rank, lets
each rank compute the ctx columns of its heads, gathers them on the caller and
finishes the layer there. Here the per-rank compute is a CPU restatement of
the reference layer's per-head math (the checker), so these tests cover the
plumbing: head ranges, the broadcasts, the column gather, masks, a non-zero
source rank, idle ranks (fewer heads than ranks) and input validation that
raises on every rank. The CUDA per-rank compute (K1 / K2 with local_heads, K3)
is checked in tests/test_headshard_gpu.py.
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


def test_head_shards_bounds(pkg):
    from cobra_gpu_kernel_b200.headshard import head_shards
    assert head_shards(4, 8) == [(0, 1), (1, 2), (2, 3), (3, 4)] + [(4, 4)] * 4
    assert head_shards(16, 8) == [(2 * i, 2 * i + 2) for i in range(8)]
    assert head_shards(16, 3) == [(0, 6), (6, 12), (12, 16)]
    for H in range(1, 33):
        for n in range(1, 9):
            sh = head_shards(H, n)
            assert sh[0][0] == 0 and sh[-1][1] == H
            assert all(sh[i][1] == sh[i + 1][0] for i in range(n - 1))
    with pytest.raises(ValueError):
        head_shards(0, 2)


class _OracleHeads:
    """The reference layer's math split by head (CPU, fp32): the checker
    standing in for the CUDA per-rank compute."""

    ctx_dtype = torch.float32

    def __init__(self, ref):
        self.ref = ref
        self.attention = ref.attention

    def _head_ctx(self, x, mask, h0, h1):
        att, B, S, d = self.ref.attention, *x.shape
        dh = att.head_dim
        h = self.ref.norm1(x)
        out = []
        for hh in range(h0, h1):
            sl = slice(hh * dh, (hh + 1) * dh)
            q = h @ att.q_proj.weight[sl].T + att.q_proj.bias[sl]
            k = h @ att.k_proj.weight[sl].T + att.k_proj.bias[sl]
            v = h @ att.v_proj.weight[sl].T + att.v_proj.bias[sl]
            sc = (q @ k.transpose(1, 2)) * att.scale
            if self.ref.causal:
                sc = sc.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
            if mask is not None:
                sc = sc.masked_fill(~mask[:, None, :], float("-inf"))
            out.append(torch.softmax(sc, -1) @ v)
        return torch.cat(out, -1).reshape(B * S, (h1 - h0) * dh)

    def _finish_from_ctx(self, x, mask, ctx):
        att, B, S, d = self.ref.attention, *x.shape
        o = att.out_proj(ctx.view(B, S, d))
        if mask is not None:
            o = o.masked_fill(~mask[..., None], 0)
        return self.ref.norm2(x + o)


def _worker(rank: int, world: int, port: int, root: str) -> None:
    sys.path.insert(0, root)
    import torch.distributed as dist
    import __graft_entry__
    __graft_entry__.load_package()
    from cobra_gpu_kernel_b200.headshard import HeadShardedLayer, head_sharded_forward
    from oracle import TransformerConfig, build_reference_layer, generate_random_case

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        with torch.inference_mode():
            # 1. B=3 < world... and heads split 2 + 2
            for causal in (False, True):
                cfg = TransformerConfig(3, 10, 32, 4, causal=causal)
                ref = build_reference_layer(cfg, seed=3)
                x, _ = generate_random_case(cfg, seed=4)
                y = head_sharded_forward(_OracleHeads(ref), x if rank == 0 else None)
                if rank == 0:
                    torch.testing.assert_close(y, ref(x), atol=1e-5, rtol=1e-5)
                else:
                    assert y is None
            # 2. key-padding mask travels to every rank
            cfg = TransformerConfig(2, 12, 32, 2)
            ref = build_reference_layer(cfg, seed=5)
            x, mask = generate_random_case(cfg, seed=6, padding_ratio=0.5)
            y = head_sharded_forward(_OracleHeads(ref), x if rank == 0 else None, mask if rank == 0 else None)
            if rank == 0:
                torch.testing.assert_close(y, ref(x, mask), atol=1e-5, rtol=1e-5)
            # 3. one head: rank 1 idle; source rank 1 through the module wrapper
            cfg = TransformerConfig(2, 8, 32, 1)
            ref = build_reference_layer(cfg, seed=7)
            x, _ = generate_random_case(cfg, seed=8)
            y = HeadShardedLayer(_OracleHeads(ref), src=1)(x if rank == 1 else None)
            if rank == 1:
                torch.testing.assert_close(y, ref(x), atol=1e-5, rtol=1e-5)
            else:
                assert y is None
            # 4. a bad input raises the same error on every rank
            with pytest.raises(ValueError, match="float32"):
                head_sharded_forward(_OracleHeads(ref), x.half() if rank == 0 else None)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_head_sharded_forward_gloo_world2(pkg, monkeypatch):
    monkeypatch.setenv("GLOO_SOCKET_IFNAME", "lo")
    spawn_ranks(_worker, (2, _free_port(), str(ROOT)), 2, 120)
