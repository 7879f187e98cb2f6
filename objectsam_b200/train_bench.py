"""Training pass of the conv stack at BASELINE config 4 (batch 16 per GPU, 640²): forward in training mode
(batch-statistics BN), then the backward of every node from given head gradients, with the data-parallel
gradient all-reduce (objectsam_b200/dp.py) overlapped when more than one GPU runs.  The loss and the
optimizer step are outside the conv path and not included; the reference is timed on the same work —
its own Model::forward(true) + Model::backward (oracle/_ref/ref_train, built from its sources) from seeded
head gradients.

    python -m objectsam_b200.train_bench [--batch 16] [--imgsz 640] [--steps 10] [--warmup 3]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 -m objectsam_b200.train_bench

Timing: CUDA events around the K steps after W warm-up steps, barrier + synchronize on both sides, max over
ranks.  Weights are seeded He-normal (BN γ = 1, β = 0), images U[0,1], head gradients N(0, 0.05²) — fixed
over the steps.  Rank 0 prints one JSON line: images/s of the whole job, the per-step time, the same step
without the all-reduce (its overlap cost), and the reference's time for one GPU's share.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--bucket-mb", type=float, default=25.0)
    ap.add_argument("--ref", default=os.path.join(ROOT, "oracle", "_ref", "ref_train"))
    ap.add_argument("--graph", action="store_true",
                    help="one GPU: replay the step as a captured CUDA graph (launch overhead removed)")
    a = ap.parse_args()
    import torch
    import torch.distributed as dist

    from objectsam_b200.dp import DataParallel
    from objectsam_b200.model import Model
    from oracle import fsow, yolo_params

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    weights = yolo_params.make_weights(0)
    m = Model(a.batch, a.imgsz)
    m.load(weights)
    m.sync_weights()
    m.train_init()
    m.input().copy_(torch.from_numpy(yolo_params.make_images(a.batch, a.imgsz, 1 + rank)).half())
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for n in [f"out.{k}{l}" for k in ("box", "cls", "coef") for l in range(3)] + ["out.proto"]:
        t = m.act_grad(n)
        t.copy_((torch.randn(t.shape, generator=g, device="cuda") * 0.05).half())
    dp = DataParallel(m, bucket_mb=a.bucket_mb)

    def step(allreduce=True):
        m.forward_train(0.03)
        if allreduce:
            dp.backward()
        else:
            m.backward()

    graph = None
    if a.graph and world == 1:
        step(False)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            step(False)
        torch.cuda.synchronize()

    def timed(allreduce):
        run = graph.replay if graph is not None else (lambda: step(allreduce))
        for _ in range(a.warmup):
            run()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            run()
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / a.steps], device="cuda")
        if world > 1:
            dist.barrier()
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    t_dp = timed(True)
    t_local = timed(False) if world > 1 else t_dp
    ref = None
    if rank == 0 and a.ref and os.path.exists(a.ref):
        with tempfile.TemporaryDirectory() as td:
            wp = os.path.join(td, "w.fsow")
            fsow.save(wp, weights)
            r = subprocess.run([a.ref, wp, "-", "-", str(a.steps), str(a.batch), str(a.imgsz)], capture_output=True,
                               text=True, timeout=900)
            for line in r.stdout.splitlines():
                if line.startswith("{"):
                    ref = json.loads(line)
    if rank == 0:
        line = {"metric": "conv-stack training pass img/s (forward train + backward, no loss / optimizer)",
                "value": round(world * a.batch / (t_dp / 1e3), 2), "unit": "img/s", "n_gpus": world,
                "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(t_dp, 4),
                "ms_per_step_without_allreduce": round(t_local, 4), "scaling": "weak",
                "cuda_graph": graph is not None,
                "config": {"workload": "BASELINE config 4 conv path", "batch_per_gpu": a.batch, "imgsz": a.imgsz,
                           "bucket_mb": a.bucket_mb, "grad_elems": int(m.grad_arena().numel()),
                           "buckets": len(dp.buckets)},
                "dtype": "fp16 activations, fp32 accumulation and gradients", "data": "synthetic"}
        if ref:
            line["reference_cudnn"] = {"ms_per_gpu_step": ref["ms"], "img_per_s_per_gpu": ref["img_per_s"],
                                       "speedup_per_gpu": round(ref["ms"] / t_local, 3)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
