"""Data-parallel training on 2 GPUs: the gradient exchange of the library (osam_dp_*, NCCL) and of the Python
DataParallel (torch.distributed NCCL), and the host-side abort guard.

Per-replica BN statistics (the reference has no SyncBN) make a rank's gradient depend on its own images only,
so the exchanged gradient must be the MEAN of the ranks' local gradients: each rank first runs the backward
alone (no exchange), the ranks all-gather those arenas, then the same step runs with the exchange and its
arena is compared with the mean (the weight gradients accumulate with fp32 atomics, so two runs of the same
backward differ in the last bits: relative L2 ≤ 1e-5).

Abort guard: one rank stops calling in (it stays alive, with nothing of its own in flight); the other rank's
osam_dp_wait must give up after its timeout, abort the communicator and return OSAM_ERR_TIMEOUT instead of
hanging.  NVLS is off for these child processes (NCCL_NVLS_ENABLE=0), as the pool requires for a test where a
rank leaves a collective.  Needs 2 GPUs; skipped with fewer.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _run_ranks(fn, args, deadline_s):
    """Starts the 2 ranks as child processes and joins them; kills them (their own process ids) and fails if
    they have not finished after deadline_s."""
    import time

    import torch.multiprocessing as mp
    ctx = mp.start_processes(fn, args=args, nprocs=2, join=False, start_method="spawn")
    t0 = time.time()
    while not ctx.join(timeout=5):
        if time.time() - t0 > deadline_s:
            for p in ctx.processes:
                if p.is_alive():
                    p.kill()
            pytest.fail(f"ranks did not finish within {deadline_s} s")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, N, S):
    import sys
    sys.path.insert(0, ROOT)
    from objectsam_b200.model import Model
    from oracle import yolo_params, yolo_ref
    w = yolo_ref.calibrated_weights(5, 128)
    m = Model(N, S)
    m.load(w)
    m.sync_weights()
    m.train_init()
    m.input().copy_(torch.from_numpy(yolo_params.make_images(N, S, 30 + rank)).half())
    g = torch.Generator(device="cpu").manual_seed(70 + rank)
    for n in [f"out.{k}{l}" for k in ("box", "cls", "coef") for l in range(3)] + ["out.proto"]:
        t = m.act_grad(n)
        t.copy_((torch.randn(t.shape, generator=g) * 0.05).half().to(t.device))
    return m


def _worker_exchange(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from objectsam_b200.dp import DataParallel, NcclDataParallel
        m = _setup(rank, 2, 128)
        m.forward_train(0.0)  # momentum 0: the running statistics stay as they are across the three passes
        m.backward()
        torch.cuda.synchronize()
        local = m.grad_arena().clone()
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        mean = torch.stack(parts).mean(0)
        res = {}
        for name, make in (("library", lambda: NcclDataParallel(m, bucket_mb=2.0)),
                           ("python", lambda: DataParallel(m, bucket_mb=2.0))):
            dp = make()
            m.forward_train(0.0)
            dp.backward()
            if name == "library":
                dp.wait(60000)
                res["buckets"] = dp.num_buckets
            torch.cuda.synchronize()
            got = m.grad_arena()
            res[name] = (torch.norm(got - mean) / torch.norm(mean)).item()
            res[name + "_vs_local"] = (torch.norm(got - local) / torch.norm(local)).item()
            if name == "library":
                dp.close()
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.array([res["library"], res["python"],
                                                                 res["library_vs_local"], res["buckets"]]))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@two_gpus
def test_exchanged_gradient_is_the_mean_of_the_ranks(cuda_lib):
    with tempfile.TemporaryDirectory() as td:
        _run_ranks(_worker_exchange, (2, _port(), td), 300)
        for r in range(2):
            lib_err, py_err, vs_local, buckets = np.load(os.path.join(td, f"r{r}.npy"))
            assert buckets > 3, "the exchange should overlap the backward in several buckets"
            assert lib_err <= 1e-5, f"rank {r}: library exchange relL2 {lib_err:.2e} from the mean"
            assert py_err <= 1e-5, f"rank {r}: Python exchange relL2 {py_err:.2e} from the mean"
            assert vs_local > 1e-3, "the ranks' gradients should differ (different images)"


def _worker_abort(rank, world, port, out_dir):
    import time

    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from objectsam_b200 import _lib
    from objectsam_b200.dp import NcclDataParallel
    m = _setup(rank, 2, 64)
    dp = NcclDataParallel(m, bucket_mb=2.0)
    # one good step on both ranks
    m.forward_train(0.0)
    dp.backward()
    dp.wait(60000)
    torch.cuda.synchronize()
    dist.barrier()  # host-side: both ranks are between steps, nothing in flight
    rc = None
    if rank == 0:
        m.forward_train(0.0)
        dp.backward()  # rank 1 never joins this step's collectives
        t0 = time.time()
        rc = _lib.lib().osam_dp_wait(dp._dp, 3000)
        waited = time.time() - t0
        msg = _lib.lib().osam_last_error().decode()
        np.save(os.path.join(out_dir, "abort.npy"), np.array([rc, waited]))
        with open(os.path.join(out_dir, "abort.txt"), "w") as f:
            f.write(msg)
    dist.barrier()  # rank 1 waits here (alive, nothing in flight) until rank 0 has aborted
    # rank 1's communicator cannot finalize with its peer gone: close() bounds the finalize and aborts it
    dp.close()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()


@two_gpus
def test_wait_aborts_when_a_rank_stops_calling_in(cuda_lib):
    with tempfile.TemporaryDirectory() as td:
        _run_ranks(_worker_abort, (2, _port(), td), 240)
        rc, waited = np.load(os.path.join(td, "abort.npy"))
        msg = open(os.path.join(td, "abort.txt")).read()
        from objectsam_b200 import _lib
        assert int(rc) == _lib.OSAM_ERR_TIMEOUT, msg
        assert 2.5 <= waited <= 30, f"waited {waited:.1f} s"
        assert "aborted" in msg
