"""Per-layer sweep: forward, dgrad and wgrad of every conv of the network, one by one.

    python -m objectsam_b200.sweep --batch 128 [--reps 10] [--ops fwd,dgrad,wgrad] [--ref oracle/_ref/ref_forward_fp16]
                                   [--json out]

Each op runs on seeded U[-1,1] NHWC fp16 tensors of the layer's shape (He-normal weights) and is timed
with CUDA events over `reps` launches after two warm-up launches; TFLOP/s use the reference's FLOP
formula 2·N·P·Q·K·C·R·S (src/model.cpp:483; the transposed conv counts H·W).  With --ref, the reference's
own cuDNN build prints its tuned fwd/dgrad/wgrad times for the same layers at the same batch
(OSAM_REF_PRINT_CONVS), joined here by layer name.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def reference_table(binary: str, batch: int, imgsz: int) -> dict:
    """{layer name: (fwd_ms, dgrad_ms, wgrad_ms)} from the reference cuDNN build's tuned-timing table."""
    from oracle import fsow, yolo_params
    with tempfile.TemporaryDirectory() as td:
        wp = os.path.join(td, "w.fsow")
        fsow.save(wp, yolo_params.make_weights(0))
        env = dict(os.environ, OSAM_REF_PRINT_CONVS="1")
        out = subprocess.run([binary, wp, "-", "-", "0", str(batch), str(imgsz)], capture_output=True, text=True,
                             env=env, timeout=900).stdout
    tab = {}
    for line in out.splitlines():
        m = re.match(r"^(\S+)\s+\d+\s+\d+\s+\d+\s+\d+\s+\d+\s+\d+\s+\|\s+([\d.]+)\s+([\d.]+)\s+([\d.]+)", line)
        if m:
            tab[m.group(1)] = tuple(float(m.group(i)) for i in (2, 3, 4))
    return tab


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--ref", default=None, help="reference cuDNN harness binary (oracle/_ref/ref_forward_fp16)")
    ap.add_argument("--json", default=None, help="write the table as JSON")
    ap.add_argument("--ops", default="fwd,dgrad,wgrad", help="comma list of the passes to time")
    a = ap.parse_args()
    ops = set(a.ops.split(","))
    import torch

    from objectsam_b200.conv import ConvGeom, ConvOp
    from objectsam_b200.model import Model

    from oracle import yolo_params  # seeded synthetic weights only: the layer geometry comes from the model

    dev = "cuda"
    m = Model(a.batch, a.imgsz)
    m.load(yolo_params.make_weights(0))
    m.sync_weights()  # the per-node conv plans (and their geometry) are built here
    nodes = [n for n in m.nodes() if n["kind"] in (0, 1, 2)]  # convs, head convs, the transposed conv
    del m
    torch.cuda.empty_cache()
    g = torch.Generator(device="cpu").manual_seed(0)
    rows = []

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.reps

    for n in nodes:
        N, H, W, C, K, R, s = n["N"], n["H"], n["W"], n["C"], n["K"], n["R"], n["stride"]
        tr = n["kind"] == 2
        pad = 0 if tr else R // 2
        op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, pad), transposed=tr)
        oshape = op.out_shape()
        x = (torch.rand(N, H, W, C, generator=g) * 2 - 1).half().to(dev)
        w_shape = (C, R, R, K) if tr else (K, R, R, C)
        w = (torch.randn(*w_shape, generator=g) * (2.0 / (C * R * R)) ** 0.5).half().to(dev)
        y = torch.empty(oshape, dtype=torch.half, device=dev)
        ws = torch.empty(max(op.workspace_size(), 256), dtype=torch.uint8, device=dev)
        flops = 2.0 * N * (H * W if tr else oshape[1] * oshape[2]) * K * C * R * R
        row = {"name": n["name"], "N": N, "H": H, "W": W, "C": C, "K": K, "R": R, "stride": s, "gflop": flops / 1e9}
        if "fwd" in ops:
            row["fwd_ms"] = timed(lambda: op.fwd(x, w, y, ws=ws))
        if not tr and n["index"] > 0 and "dgrad" in ops:  # the stem has no input gradient (need_grad = false, src/model.cpp:177)
            dx = torch.empty_like(x)
            try:
                row["dgrad_ms"] = timed(lambda: op.dgrad(y, w, dx, ws=ws))
            except RuntimeError as e:
                row["dgrad_ms"] = None
                row["dgrad_note"] = str(e)[:80]
        if not tr and "wgrad" in ops:
            dw = torch.empty(w_shape, dtype=torch.half, device=dev)
            try:
                row["wgrad_ms"] = timed(lambda: op.wgrad(x, y, dw, ws=ws))
            except RuntimeError as e:
                row["wgrad_ms"] = None
                row["wgrad_note"] = str(e)[:80]
        for k in ("fwd", "dgrad", "wgrad"):
            t = row.get(k + "_ms")
            if t:
                row[k + "_tflops"] = flops / (t / 1e3) / 1e12
        rows.append(row)
        op.close()
        del x, w, y, ws
        torch.cuda.empty_cache()

    ref = reference_table(a.ref, a.batch, a.imgsz) if a.ref and os.path.exists(a.ref) else {}
    tot = {"fwd": 0.0, "dgrad": 0.0, "wgrad": 0.0}
    rtot = {"fwd": 0.0, "dgrad": 0.0, "wgrad": 0.0}
    hdr = f"{'layer':26s} {'shape':28s} {'fwd ms':>8s} {'TF':>6s} {'dgrad':>8s} {'TF':>6s} {'wgrad':>8s} {'TF':>6s}"
    if ref:
        hdr += f" | {'ref fwd':>8s} {'dgrad':>8s} {'wgrad':>8s}"
    print(hdr)
    for r in rows:
        shape = f"{r['H']}x{r['W']} {r['C']}->{r['K']} {r['R']}x{r['R']} s{r['stride']}"
        cells = []
        for k in ("fwd", "dgrad", "wgrad"):
            t = r.get(k + "_ms")
            cells.append(f"{t:8.3f} {r[k + '_tflops']:6.0f}" if t else f"{'-':>8s} {'-':>6s}")
            if t and (not ref or r["name"] in ref):
                tot[k] += t
        line = f"{r['name']:26s} {shape:28s} " + " ".join(cells)
        if r["name"] in ref:
            rf = ref[r["name"]]
            r["ref_ms"] = rf
            for i, k in enumerate(("fwd", "dgrad", "wgrad")):
                if r.get(k + "_ms"):
                    rtot[k] += rf[i]
            line += f" | {rf[0]:8.3f} {rf[1]:8.3f} {rf[2]:8.3f}"
        print(line)
    print("total ms (layers with both sides when --ref):", {k: round(v, 3) for k, v in tot.items()})
    if ref:
        print("reference total ms (same layers):", {k: round(v, 3) for k, v in rtot.items()})
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"batch": a.batch, "imgsz": a.imgsz, "rows": rows, "total": tot, "ref_total": rtot}, f, indent=1)


if __name__ == "__main__":
    main()
