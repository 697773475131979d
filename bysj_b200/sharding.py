"""Multi-GPU decompositions of the segmented-operator path.

Two modes, one process per GPU:

* **Frames** (independent systems): rank r takes frames r, r+P, r+2P, ... and
  runs every operator locally; there is no collective on the data path.
* **Destination-range partition** of one large system: atoms are split into P
  contiguous ranges holding about the same number of *edges* (binary search on
  the destination offsets), so rank r owns the edges whose destination lies in
  its range -- a contiguous slice of the dst-sorted edge list.  The segmented
  operators (RMSNorm, segment softmax / sum, attention, zonal scatter) are
  then purely local.  ``force_assembly`` is not: an edge's source may live in
  another rank's range.  Each rank therefore computes the source-side partial
  sums ``[-sum g, -sum g (x) v]`` (12 floats) for *all* atoms from its own
  edges, the partials are summed across ranks by one reduce-scatter (NCCL over
  NVLink) into each rank's atom range, and the destination-side sums of the
  local edges are added on top.  Atoms are expected in a spatial (Morton)
  order so that a range is a compact slab.

The reduce-scatter wants equal blocks, so partials live in a *padded* atom
index space: rank r's atoms occupy rows ``[r*chunk, r*chunk + n_r)`` with
``chunk = max_r n_r``.  The partition's source offsets are built directly in
that space (padding rows are empty segments), so the partial kernel writes
the exchange buffer itself -- no gather or copy before the collective.

The communication step is injectable so the host logic runs with gloo ranks
on CPU (where the reduce-scatter is an all-reduce and a slice).
"""
from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass
from typing import Callable

import torch


def init_process_group(backend: str = "nccl", *, timeout_s: float = 60.0, **kwargs):
    """``torch.distributed.init_process_group`` with a bounded timeout.

    Every collective of the partition (the force reduce-scatter) then ends
    within ``timeout_s`` seconds: with a peer that died or left between steps
    it raises on the host instead of waiting forever.  For NCCL the
    asynchronous error handling is switched on (``TORCH_NCCL_ASYNC_ERROR_HANDLING=1``
    unless the caller set it), so a timed-out or failed communicator aborts
    and the waiting ``work.wait()`` raises.  No kernel of this library waits on
    another rank: only NCCL's own kernels do, and their wait is bounded here.
    """
    import datetime
    import os

    import torch.distributed as dist

    if backend == "nccl":
        os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=float(timeout_s)),
                            **kwargs)
    return dist


def frame_share(frames: int, rank: int, world: int) -> list[int]:
    """Frames handled by ``rank``: ``rank, rank + world, ...``."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return list(range(rank, frames, world))


def edge_balanced_bounds(offsets: torch.Tensor, parts: int) -> list[int]:
    """Atom boundaries ``b[0] = 0 <= ... <= b[parts] = N`` splitting the edges evenly.

    ``b[r]`` is the first atom whose first edge is at or past ``ceil(E * r / parts)``
    (a binary search on the exclusive prefix sum ``offsets``).
    """
    if parts <= 0:
        raise ValueError("parts must be positive")
    off = offsets.detach().to("cpu", torch.int64)
    n = int(off.numel()) - 1
    e = int(off[-1])
    targets = torch.tensor([(e * r + parts - 1) // parts for r in range(parts + 1)],
                           dtype=torch.int64)
    bounds = torch.searchsorted(off[:-1].contiguous(), targets, right=False).tolist()
    bounds[0], bounds[-1] = 0, n
    for r in range(1, parts + 1):  # monotone even with empty ranges
        bounds[r] = max(bounds[r], bounds[r - 1])
    return [int(b) for b in bounds]


def padded_offsets(offsets: torch.Tensor, bounds: list[int], chunk: int) -> torch.Tensor:
    """Offsets over the padded atom space: row ``r*chunk + i`` is atom ``bounds[r] + i``.

    Rows past a rank's last atom are empty segments (their offset repeats the
    next real one), so ``[world*chunk + 1]`` entries describe the same edges.
    """
    world = len(bounds) - 1
    dev = offsets.device
    i = torch.arange(chunk, device=dev)
    rows = []
    for r in range(world):
        n_r = bounds[r + 1] - bounds[r]
        rows.append(bounds[r] + torch.clamp(i, max=n_r))
    index = torch.cat(rows + [torch.tensor([bounds[-1]], device=dev)])
    return offsets[index].contiguous()


@dataclass
class DstPartition:
    """One rank's share of a dst-sorted graph."""

    rank: int
    world: int
    bounds: list[int]          # atom boundaries of all ranks
    atom_begin: int
    atom_end: int
    edge_begin: int
    edge_end: int
    chunk: int                 # rows per rank in the padded exchange buffer
    dst_offsets: torch.Tensor  # [n_local + 1], relative to edge_begin
    src_offsets: torch.Tensor  # [world*chunk + 1] over the padded atom space, local edges
    src_order: torch.Tensor    # [E_local] local edges grouped by source

    @property
    def n_local(self) -> int:
        return self.atom_end - self.atom_begin

    @property
    def n_edges(self) -> int:
        return self.edge_end - self.edge_begin

    def edges(self, tensor: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a per-edge tensor (a view)."""
        return tensor[self.edge_begin:self.edge_end]

    def atoms(self, tensor: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a per-atom tensor (a view)."""
        return tensor[self.atom_begin:self.atom_end]


def make_partition(offsets: torch.Tensor, src: torch.Tensor, rank: int, world: int,
                   group_by_source: Callable | None = None) -> DstPartition:
    """Partition a dst-sorted graph (``offsets`` [N+1], ``src`` [E]) for ``rank``.

    ``src`` may be the whole source column or only this rank's slice of it.
    ``group_by_source(src_local, N) -> (order, offsets)`` groups the local
    edges by source; it defaults to :func:`bysj_b200.kernels.group_by_source`.
    """
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    bounds = edge_balanced_bounds(offsets, world)
    a0, a1 = bounds[rank], bounds[rank + 1]
    off_cpu = offsets.detach().to("cpu", torch.int64)
    e0, e1 = int(off_cpu[a0]), int(off_cpu[a1])
    n = int(off_cpu.numel()) - 1
    local_src = src[e0:e1] if src.numel() == int(off_cpu[-1]) else src
    if local_src.numel() != e1 - e0:
        raise ValueError("src must hold all edges or exactly this rank's edges")
    if group_by_source is None:
        from .kernels import group_by_source as group_by_source
    order, src_off = group_by_source(local_src.contiguous(), n)
    chunk = max(1, max(bounds[r + 1] - bounds[r] for r in range(world)))
    return DstPartition(rank, world, bounds, a0, a1, e0, e1, chunk,
                        (offsets[a0:a1 + 1] - e0).contiguous(),
                        padded_offsets(src_off, bounds, chunk), order)


def reduce_scatter_sum(padded: torch.Tensor, part: DstPartition, group=None,
                       async_op: bool = False):
    """Sum ``[world*chunk, 12]`` over ranks into this rank's ``[chunk, 12]`` block.

    Returns ``(block, work)``; with ``async_op`` the caller waits on ``work``
    (NCCL runs on its own stream, after the current stream's pending work).
    """
    import torch.distributed as dist

    if part.world == 1:  # one partition: nothing to exchange
        return padded[:part.chunk], None
    block = padded.new_empty((part.chunk, padded.shape[1]))
    if dist.get_backend(group) == "nccl":
        work = dist.reduce_scatter_tensor(block, padded, op=dist.ReduceOp.SUM, group=group,
                                          async_op=async_op)
        return block, work
    total = padded.clone()
    dist.all_reduce(total, op=dist.ReduceOp.SUM, group=group)
    block.copy_(total[part.rank * part.chunk:(part.rank + 1) * part.chunk])
    return block, None


class ForceExchange:
    """Partitioned ``force_assembly`` in two halves around other local work.

    ``start`` launches the source-partial kernel and the reduce-scatter
    (asynchronous on NCCL); ``finish`` waits for it and adds the local
    destination sums.  On CUDA the whole exchange runs on a side stream that
    first waits for the caller's stream, so the kernels the caller launches
    between ``start`` and ``finish`` (e.g. the local attention) overlap all of
    it; ``finish`` makes the caller's stream wait for the side stream again.
    """

    def __init__(self, part: DstPartition, *, src_partial: Callable | None = None,
                 dst_add: Callable | None = None, combine: Callable | None = None,
                 group=None, side_stream: bool = True):
        if src_partial is None or dst_add is None:
            from ._C import force_assembly_dst_add, force_assembly_src_partial

            src_partial = src_partial or force_assembly_src_partial
            dst_add = dst_add or force_assembly_dst_add
        self.part, self.group = part, group
        self._src_partial, self._dst_add, self._combine = src_partial, dst_add, combine
        self._use_side = side_stream
        self._side = None
        self._pending = None

    def _stream_for(self, tensor: torch.Tensor):
        if not (self._use_side and tensor.is_cuda):
            return None
        if self._side is None or self._side.device != tensor.device:
            self._side = torch.cuda.Stream(device=tensor.device)
        return self._side

    def start(self, grad_edge: torch.Tensor, edge_vec: torch.Tensor) -> None:
        """``grad_edge`` / ``edge_vec``: this rank's edges, ``[E_local, 3]`` fp32."""
        if self._pending is not None:
            raise RuntimeError("ForceExchange.start called twice without finish")
        p = self.part
        side = self._stream_for(grad_edge)
        main = torch.cuda.current_stream(grad_edge.device) if side is not None else None
        if side is not None:
            side.wait_stream(main)
        with torch.cuda.stream(side) if side is not None else nullcontext():
            partial = self._src_partial(grad_edge, edge_vec, p.src_offsets, p.src_order)
            if self._combine is not None:
                block, work = self._combine(partial, p), None
            else:
                block, work = reduce_scatter_sum(partial, p, self.group, async_op=True)
        if side is not None:
            for t in (grad_edge, edge_vec, p.src_offsets, p.src_order, p.dst_offsets):
                t.record_stream(side)
        self._pending = (grad_edge, partial, block, work, side, main)

    def finish(self):
        """``(force [n_local, 3], virial [n_local, 9])`` of this rank's atoms."""
        if self._pending is None:
            raise RuntimeError("ForceExchange.finish called before start")
        grad_edge, _partial, block, work, side, main = self._pending
        self._pending = None
        p = self.part
        with torch.cuda.stream(side) if side is not None else nullcontext():
            if work is not None:
                work.wait()
            force, virial = self._dst_add(grad_edge, p.dst_offsets, block[:p.n_local])
        if side is not None:
            main.wait_stream(side)
            force.record_stream(main)
            virial.record_stream(main)
        return force, virial


def force_assembly_partitioned(grad_edge: torch.Tensor, edge_vec: torch.Tensor,
                               part: DstPartition, **kwargs):
    """Forces and virials of this rank's atoms from this rank's edges (one call)."""
    ex = ForceExchange(part, **kwargs)
    ex.start(grad_edge, edge_vec)
    return ex.finish()


__all__ = [
    "DstPartition",
    "ForceExchange",
    "edge_balanced_bounds",
    "force_assembly_partitioned",
    "frame_share",
    "init_process_group",
    "make_partition",
    "padded_offsets",
    "reduce_scatter_sum",
]
