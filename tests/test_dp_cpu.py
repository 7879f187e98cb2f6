"""Data-parallel gradient exchange (objectsam_b200/dp.py) on CPU with gloo, world size 2: the bucket plan
tiles the arena in backward order, and after DataParallel.backward every rank holds the average of the
ranks' gradients (the reference's allreduce-sum then ÷ world)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from objectsam_b200.dp import DataParallel, plan_buckets


def _ranges():
    # 12 nodes, arena in reverse node order with 64-element alignment, two nodes without parameters
    sizes = [300, 0, 5000, 70, 1200, 0, 64, 9000, 128, 640, 33, 2000]
    ranges, off = [None] * len(sizes), 0
    for i in range(len(sizes) - 1, -1, -1):
        ranges[i] = (off if sizes[i] else 0, sizes[i])
        off = (off + sizes[i] + 63) // 64 * 64 if sizes[i] else off
    return ranges, off


def test_plan_buckets_tiles_arena_in_backward_order():
    ranges, total = _ranges()
    for elems in (1, 1000, 4000, 10 ** 6):
        bs = plan_buckets(ranges, elems)
        assert [b.first for b in bs] == sorted([b.first for b in bs], reverse=True)
        assert sum(b.count for b in bs) == len(ranges) and bs[-1].first == 0
        spans = sorted((b.off, b.off + b.n) for b in bs)
        assert spans[0][0] == 0 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        for b in bs:  # every node's gradients lie inside its bucket
            for i in range(b.first, b.first + b.count):
                off, n = ranges[i]
                if n:
                    assert b.off <= off and off + n <= b.off + b.n


class _FakeModel:
    """Stands in for Model: backward_nodes writes rank-dependent gradients into its nodes' ranges."""

    def __init__(self, rank):
        self.ranges, n = _ranges()
        self.arena = torch.zeros(n)
        self.rank = rank
        self.order = []

    def num_launches(self):
        return len(self.ranges)

    def node_grad_range(self, i):
        return self.ranges[i]

    def grad_arena(self):
        return self.arena

    def backward_nodes(self, first, count):
        self.order.append(first)
        for i in range(first + count - 1, first - 1, -1):
            off, n = self.ranges[i]
            self.arena[off:off + n] = torch.arange(n, dtype=torch.float32) * (self.rank + 1) + i


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    m = _FakeModel(rank)
    dp = DataParallel(m, bucket_mb=4000 * 4 / (1 << 20))
    dp.backward()
    out[rank] = (m.arena.clone(), m.order)
    dist.destroy_process_group()


def test_data_parallel_average_gloo_world2():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    ref = _FakeModel(0)
    for i in range(len(ref.ranges)):
        off, n = ref.ranges[i]
        ref.arena[off:off + n] = torch.arange(n, dtype=torch.float32) * 1.5 + i  # mean of ×1 and ×2
    for r in range(2):
        arena, order = out[r]
        assert torch.allclose(arena, ref.arena)
        assert order == sorted(order, reverse=True) and len(order) > 1
