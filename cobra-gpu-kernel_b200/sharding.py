"""Batch-sharded layer forward, one process per GPU over ``torch.distributed``.

Every op of the layer works on one sequence at a time
(torch_transformer_benchmark.py:1446-1447, ``tools/sweep.py:62-65``), so the
batch splits into contiguous slices of ceil(B / n) sequences, one per rank,
with no reduction collective. The caller's rank (``src``) holds x; it sends
each rank its slice, runs its own slice, and receives the other ranks' y
slices straight into its output tensor. Transfers are point-to-point
(NCCL send/recv over NVLink/NVSwitch with the ``nccl`` backend; the same code
runs on ``gloo`` for CPU tests) and are split into ``chunks`` pieces per
rank so that a rank computes piece i while piece i+1 is still arriving.

Weights are replicated: every rank builds or loads the same layer. With
B < n only the first B ranks receive work; the rest still take part in the
header broadcast and return at once (``head_sharded_forward`` in
``headshard.py`` splits heads instead for that case).

Host-resident input (the reference's ``_run_streamed``,
torch_transformer_benchmark.py:1418-1508, spread over GPUs): with the NCCL
backend, ``x`` on the source rank may be a CPU tensor (pinned, for
asynchronous copies). The source then copies each piece host-to-device just
before sending it -- the other ranks' pieces first, round-robin, so every rank
starts computing as early as possible -- and copies each returned y piece
device-to-host on a separate stream as soon as it lands, overlapped with its
own compute. The result is a CPU tensor; both host copies run over the source
GPU's own host link.

Layers that accept ``out=`` (``B200TransformerLayer`` does) write each result
straight into its place in the gathered output or in the send buffer.

Failure behaviour: the caller's input is validated on ``src`` before any data
moves and the verdict is broadcast, so a bad input raises the same
``ValueError`` on every rank. A rank that fails after the header (a kernel
error, an exception in ``layer``) leaves its peers waiting on a transfer that
never comes; the process group's timeout ends their wait with an error.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

__all__ = ["batch_shards", "sharded_forward", "ShardedLayer"]

# Header broadcast from src: status, B, S, d, has_mask.
_HDR_OK = 0
_HDR_BAD_RANK = 1
_HDR_BAD_SHAPE = 2
_HDR_BAD_DTYPE = 3
_HDR_BAD_MASK = 4
_HDR_MESSAGES = {
    _HDR_BAD_RANK: "src rank passed no input tensor",
    _HDR_BAD_SHAPE: "x must be a [B, S, d] tensor with B, S, d > 0",
    _HDR_BAD_DTYPE: "x must be float32",
    _HDR_BAD_MASK: "valid_token_mask must be a [B, S] bool tensor",
}


def batch_shards(batch: int, world: int) -> List[Tuple[int, int]]:
    """Half-open sequence ranges [start, stop) for ranks 0..world-1.

    Contiguous slices of ceil(batch / world) sequences; ranks past the last
    slice get an empty range (start == stop == batch)."""
    if batch < 0 or world <= 0:
        raise ValueError(f"bad batch/world: {batch}, {world}")
    per = -(-batch // world) if batch else 0
    out = []
    for r in range(world):
        a = min(batch, r * per)
        b = min(batch, a + per)
        out.append((a, b))
    return out


def _chunk_ranges(a: int, b: int, chunks: int) -> List[Tuple[int, int]]:
    n = b - a
    if n <= 0:
        return []
    k = max(1, min(chunks, n))
    per = -(-n // k)
    return [(a + i, min(b, a + i + per)) for i in range(0, n, per)]


def _default_device(backend: str) -> torch.device:
    if backend == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def _validate(x: Optional[torch.Tensor], mask: Optional[torch.Tensor]) -> int:
    if x is None:
        return _HDR_BAD_RANK
    if x.dim() != 3 or min(x.shape) <= 0:
        return _HDR_BAD_SHAPE
    if x.dtype != torch.float32:
        return _HDR_BAD_DTYPE
    if mask is not None and (mask.dtype != torch.bool or tuple(mask.shape) != tuple(x.shape[:2])):
        return _HDR_BAD_MASK
    return _HDR_OK


def _run_into(layer, x: torch.Tensor, m: Optional[torch.Tensor], out: torch.Tensor) -> None:
    """out <- layer(x, m), written in place when the layer supports ``out=``."""
    if getattr(layer, "accepts_out", False):
        layer(x, m, out=out)
    else:
        out.copy_(layer(x, m))


def sharded_forward(layer: Callable[..., torch.Tensor], x: Optional[torch.Tensor] = None,
                    valid_token_mask: Optional[torch.Tensor] = None, *, src: int = 0,
                    group: Optional[dist.ProcessGroup] = None, device: Optional[torch.device] = None,
                    chunks: int = 1, out: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Run ``layer`` over the batch of ``x`` split across the ranks of ``group``.

    Collective: every rank of ``group`` calls it; ``x`` (fp32 [B, S, d]) and
    the optional ``valid_token_mask`` ([B, S] bool) are read on ``src`` only.
    ``x`` lives on this rank's device, or -- with the NCCL backend -- on the
    host (see the module docstring). ``layer(x_slice, mask_slice)`` must map
    [b, S, d] to [b, S, d] sequence by sequence (``B200TransformerLayer``
    does). Returns y [B, S, d] on ``src`` (the slices computed by the ranks,
    gathered into one tensor on x's device, or into ``out`` when given) and
    ``None`` on every other rank.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    src_g = dist.get_global_rank(group, src) if group is not None else src
    backend = dist.get_backend(group)
    if rank == src:
        if x is not None and x.device.type == "cpu" and backend == "nccl":
            device = device or _default_device(backend)    # host input staged through this GPU
        else:
            device = x.device if x is not None else (device or _default_device(backend))
    elif device is None:
        device = _default_device(backend)

    hdr = torch.zeros(5, dtype=torch.int64, device=device)
    if rank == src:
        status = _validate(x, valid_token_mask)
        hdr[0] = status
        if status == _HDR_OK:
            hdr[1:4] = torch.tensor(x.shape, dtype=torch.int64)
            hdr[4] = 1 if valid_token_mask is not None else 0
    dist.broadcast(hdr, src_g, group=group)
    status, B, S, d, has_mask = (int(v) for v in hdr.tolist())
    if status != _HDR_OK:
        raise ValueError(f"sharded_forward: {_HDR_MESSAGES[status]} (validated on rank {src})")

    # Before any transfer is posted: a layer that can warm up packs its
    # weights and loads its kernels now, so that no first-use work (weight
    # packing, lazy kernel loading) waits behind NCCL kernels in flight.
    warm = getattr(layer, "warmup", None)
    if warm is not None and batch_shards(B, world)[rank][1] > batch_shards(B, world)[rank][0]:
        warm(S, device, bool(has_mask))
    # Run the layer eagerly while transfers are in flight: a CUDA-graph
    # capture (B200TransformerLayer captures on the first call per shape, and
    # ragged chunks change the shape) must not overlap NCCL work.
    saved_graphs = getattr(layer, "use_graphs", None)
    if saved_graphs:
        layer.use_graphs = False
    try:
        if rank == src:
            return _source(layer, x, valid_token_mask, world, src, group, device, B, has_mask, chunks, out)
        return _exchange(layer, rank, world, src_g, group, device, B, S, d, has_mask, chunks)
    finally:
        if saved_graphs:
            layer.use_graphs = saved_graphs


def _peer_pieces(shards, src, group, chunks):
    """(global peer rank, c0, c1) of every piece that leaves the source, in
    round-robin order over the peers, so each peer's first piece goes out
    before any peer's second."""
    per_peer = []
    for r, (a, b) in enumerate(shards):
        if r == src or a == b:
            continue
        peer = dist.get_global_rank(group, r) if group is not None else r
        per_peer.append([(peer, c0, c1) for c0, c1 in _chunk_ranges(a, b, chunks)])
    order = []
    for i in range(max((len(p) for p in per_peer), default=0)):
        order.extend(p[i] for p in per_peer if i < len(p))
    return order


def _source(layer, x, valid_token_mask, world, src, group, device, B, has_mask, chunks, out):
    shards = batch_shards(B, world)
    pieces = _peer_pieces(shards, src, group, chunks)
    host_io = x.device.type == "cpu" and device.type == "cuda"
    x = x.contiguous()
    mask = valid_token_mask.to(torch.uint8).contiguous() if has_mask else None
    works = []
    if not host_io:
        y = out if out is not None else torch.empty_like(x)
        # Post every transfer first: x slices out, y slices back into y.
        for peer, c0, c1 in pieces:
            works.append(dist.isend(x[c0:c1], peer, group=group))
            if mask is not None:
                works.append(dist.isend(mask[c0:c1], peer, group=group))
        for peer, c0, c1 in pieces:
            works.append(dist.irecv(y[c0:c1], peer, group=group))
        a, b = shards[src]
        for c0, c1 in _chunk_ranges(a, b, chunks):
            m = mask[c0:c1].bool() if mask is not None else None
            _run_into(layer, x[c0:c1], m, y[c0:c1])
        for w in works:
            w.wait()
        return y

    # Host input: stage through this GPU. Copies and NCCL transfers are
    # ordered on the current stream (an NCCL send waits for the work queued on
    # it), the returned pieces go device-to-host on a separate stream.
    comp = torch.cuda.current_stream(device)
    d2h = torch.cuda.Stream(device=device)
    xd = torch.empty(x.shape, dtype=x.dtype, device=device)
    yd = torch.empty_like(xd)
    md = mask.to(device, non_blocking=True) if mask is not None else None
    y = out if out is not None else torch.empty(x.shape, dtype=x.dtype, pin_memory=x.is_pinned())
    for peer, c0, c1 in pieces:
        xd[c0:c1].copy_(x[c0:c1], non_blocking=True)
        works.append(dist.isend(xd[c0:c1], peer, group=group))
        if md is not None:
            works.append(dist.isend(md[c0:c1], peer, group=group))
    recvs = [(dist.irecv(yd[c0:c1], peer, group=group), c0, c1) for peer, c0, c1 in pieces]
    a, b = shards[src]
    own = _chunk_ranges(a, b, chunks)
    for c0, c1 in own:
        xd[c0:c1].copy_(x[c0:c1], non_blocking=True)
    # d2h_stream: each returned piece goes to the host once it has landed.
    with torch.cuda.stream(d2h):
        for w, c0, c1 in recvs:
            w.wait()
            y[c0:c1].copy_(yd[c0:c1], non_blocking=True)
    for c0, c1 in own:
        m = md[c0:c1].bool() if md is not None else None
        _run_into(layer, xd[c0:c1], m, yd[c0:c1])
    d2h.wait_stream(comp)
    with torch.cuda.stream(d2h):
        for c0, c1 in own:
            y[c0:c1].copy_(yd[c0:c1], non_blocking=True)
    for w in works:
        w.wait()
    comp.wait_stream(d2h)
    xd.record_stream(d2h)
    yd.record_stream(d2h)
    comp.synchronize()     # y is complete on the host
    return y


def _exchange(layer, rank, world, src_g, group, device, B, S, d, has_mask, chunks):
    shards = batch_shards(B, world)
    works = []

    a, b = shards[rank]
    if a == b:
        return None
    xs = torch.empty(b - a, S, d, dtype=torch.float32, device=device)
    ms = torch.empty(b - a, S, dtype=torch.uint8, device=device) if has_mask else None
    ys = torch.empty_like(xs)
    pieces = []
    for c0, c1 in _chunk_ranges(a, b, chunks):
        wx = dist.irecv(xs[c0 - a:c1 - a], src_g, group=group)
        wm = dist.irecv(ms[c0 - a:c1 - a], src_g, group=group) if ms is not None else None
        pieces.append((c0 - a, c1 - a, wx, wm))
    for c0, c1, wx, wm in pieces:
        wx.wait()
        if wm is not None:
            wm.wait()
        m = ms[c0:c1].bool() if ms is not None else None
        # Into the send buffer (never the layer's static output buffer, which
        # the next call would overwrite while the send still reads it).
        _run_into(layer, xs[c0:c1], m, ys[c0:c1])
        works.append(dist.isend(ys[c0:c1], src_g, group=group))
    for w in works:
        w.wait()
    return None


class ShardedLayer(torch.nn.Module):
    """``forward(x, valid_token_mask=None)`` of a replicated layer, sharded by batch.

    Wraps a layer (every rank holds the same weights) so that the caller's
    rank sees the reference module's API; see ``sharded_forward``. For a
    host-resident x the result is a pinned host buffer owned by this module
    and overwritten by the next host call of the same shape (as the layer's
    own host path returns)."""

    def __init__(self, layer: torch.nn.Module, *, src: int = 0,
                 group: Optional[dist.ProcessGroup] = None, chunks: int = 1) -> None:
        super().__init__()
        self.layer = layer
        self.src = src
        self.group = group
        self.chunks = chunks
        self._host_out: Optional[torch.Tensor] = None

    def forward(self, x: Optional[torch.Tensor] = None,
                valid_token_mask: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        out = None
        if x is not None and x.device.type == "cpu" and dist.get_backend(self.group) == "nccl":
            if self._host_out is None or self._host_out.shape != x.shape:
                self._host_out = None
                self._host_out = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
            out = self._host_out
        return sharded_forward(self.layer, x, valid_token_mask, src=self.src, group=self.group,
                               chunks=self.chunks, out=out)
