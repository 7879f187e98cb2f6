"""Data-parallel training: the batch is sharded over one process per GPU and the parameter gradients are
averaged with an all-reduce (NCCL over NVLink on the GPUs, gloo on CPU), bucket by bucket, while the backward
of the earlier layers is still running.

Two forms: DataParallel drives the exchange from Python with torch.distributed (any backend, gloo on CPU);
NcclDataParallel runs it inside the library (osam_dp_*: buckets, NCCL all-reduce with ncclAvg on a
communication stream, non-blocking communicator with a host-side abort guard) — the path a C++ trainer
calls directly.

This is the gradient exchange of the reference's multi-GPU plan (ncclAllReduce, sum then ÷ world, over the
fp32 gradient arenas, bucketed in reverse layer order on a communication stream after each bucket's
weight-gradient work; it must finish before the optimizer step).  The model's fp32 gradient arena keeps the
nodes in reverse order, so the gradients of nodes [first, n) form one contiguous range: a bucket is a node
range whose backward has been issued; its all-reduce waits on an event recorded after that backward, on a
separate stream, so it overlaps with the backward of the nodes before it.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Bucket:
    first: int   # first node (lowest index) of the bucket
    count: int   # nodes [first, first + count)
    off: int     # element offset of the bucket's gradients in the arena
    n: int       # elements


def plan_buckets(node_ranges: list[tuple[int, int]], bucket_elems: int) -> list[Bucket]:
    """node_ranges[i] = (offset, count) of node i's gradients in the arena (count 0: no parameters).  Walks the
    nodes from the last one (the first whose gradients are ready) and closes a bucket once it holds at least
    bucket_elems gradients; the buckets come out in backward order and tile the arena."""
    out: list[Bucket] = []
    hi = len(node_ranges)
    lo_off, hi_end, acc = None, None, 0
    for i in range(len(node_ranges) - 1, -1, -1):
        off, n = node_ranges[i]
        if n:
            lo_off = off if lo_off is None else min(lo_off, off)
            hi_end = off + n if hi_end is None else max(hi_end, off + n)
            acc += n
        if (acc >= bucket_elems and lo_off is not None) or i == 0:
            if lo_off is not None:
                out.append(Bucket(i, hi - i, lo_off, hi_end - lo_off))
            elif out:  # trailing nodes without parameters join the previous bucket's backward
                out[-1] = Bucket(i, out[-1].count + hi - i, out[-1].off, out[-1].n)
            hi, lo_off, hi_end, acc = i, None, None, 0
    # the arena's alignment padding between buckets: extend each bucket to the next one's start
    out.sort(key=lambda b: b.off)
    for a, b in zip(out, out[1:]):
        a.n = b.off - a.off
    out.sort(key=lambda b: -b.first)
    return out


class DataParallel:
    """backward(): the model's backward in buckets with the gradient all-reduce (average) overlapped.

    model: anything with num_launches(), node_grad_range(i), grad_arena() and backward_nodes(first, count)
    (objectsam_b200.model.Model after train_init).  group: a torch.distributed process group or None (the
    default group; world size 1 without one)."""

    def __init__(self, model, group=None, bucket_mb: float = 25.0):
        self.m = model
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.arena = model.grad_arena()
        ranges = [model.node_grad_range(i) for i in range(model.num_launches())]
        self.buckets = plan_buckets(ranges, max(1, int(bucket_mb * (1 << 20) / 4)))
        tail = max(b.off + b.n for b in self.buckets)
        if tail < self.arena.numel():  # alignment padding at the end of the arena
            last = max(self.buckets, key=lambda b: b.off)
            last.n = self.arena.numel() - last.off
        self.cuda = self.arena.is_cuda
        self.comm = torch.cuda.Stream(device=self.arena.device) if self.cuda else None

    def backward(self, stream=None) -> None:
        pending = []
        for b in self.buckets:
            self.m.backward_nodes(b.first, b.count, stream) if stream is not None else \
                self.m.backward_nodes(b.first, b.count)
            if self.world == 1:
                continue
            view = self.arena[b.off:b.off + b.n]
            if self.cuda:
                ev = torch.cuda.Event()
                ev.record(stream if stream is not None else torch.cuda.current_stream(self.arena.device))
                self.comm.wait_event(ev)
                with torch.cuda.stream(self.comm):
                    work = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                    work.wait()  # the communication stream (not the host) waits for the collective
                    view.mul_(1.0 / self.world)
            else:
                work = dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
                pending.append((work, view))
        for work, view in pending:
            work.wait()
            view.mul_(1.0 / self.world)
        if self.cuda and self.world > 1:
            (stream if stream is not None else torch.cuda.current_stream(self.arena.device)).wait_stream(self.comm)


class NcclDataParallel:
    """The library's own data-parallel exchange (include/osam.h osam_dp_*) for one process per GPU.

    The NCCL communicator id is made by rank 0 and passed to the other ranks through the torch.distributed
    group (any backend); the communicator itself belongs to the library.  backward() runs the model's whole
    backward with the bucketed, overlapped all-reduce (average) on the current stream; wait(timeout_ms)
    guards a step: it raises (after aborting the communicator) if the exchange fails or does not finish in
    time."""

    def __init__(self, model, bucket_mb: float = 4.0, group=None, init_timeout_ms: int = 120000):
        import ctypes
        from ._lib import check, lib
        self.m = model
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        uid = ctypes.create_string_buffer(128)
        if self.world > 1:
            if self.rank == 0:
                check(lib().osam_dp_unique_id(uid))
            box = [bytes(uid.raw)]
            dist.broadcast_object_list(box, src=0, group=group)
            uid = ctypes.create_string_buffer(box[0], 128)
        self._dp = ctypes.c_void_p()
        check(lib().osam_dp_create(model._m, self.world, self.rank, uid, int(bucket_mb * (1 << 20)),
                                   init_timeout_ms, ctypes.byref(self._dp)))

    @property
    def num_buckets(self) -> int:
        from ._lib import lib
        return lib().osam_dp_num_buckets(self._dp)

    def buckets(self) -> list[Bucket]:
        import ctypes
        from ._lib import check, lib
        out = []
        for i in range(self.num_buckets):
            f, c, o, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
            check(lib().osam_dp_bucket(self._dp, i, ctypes.byref(f), ctypes.byref(c), ctypes.byref(o), ctypes.byref(n)))
            out.append(Bucket(f.value, c.value, o.value, n.value))
        return out

    def backward(self, stream=None) -> None:
        from ._lib import check, lib, stream_ptr
        check(lib().osam_dp_backward(self._dp, stream_ptr(stream)))

    def wait(self, timeout_ms: int = 60000) -> None:
        from ._lib import check, lib
        check(lib().osam_dp_wait(self._dp, timeout_ms))

    def close(self) -> None:
        from ._lib import lib
        if getattr(self, "_dp", None):
            lib().osam_dp_destroy(self._dp)
            self._dp = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
