"""Training-side passes at BASELINE config 4 (batch 16 per GPU, 640²): BatchNorm statistics / apply / backward
for every distinct conv+BN+SiLU output shape of the network, the stem weight gradient and the mask loss,
each timed alone and compared with the reference's own kernels on the same shapes.

    python -m objectsam_b200.train_sweep [--batch 16] [--imgsz 640] [--iters 10] [--ref oracle/_ref/ref_bn]
                                          [--json out]

Timing: CUDA events around each call, after two warm-up calls, with a 256 MiB read before every call so
that L2 (126 MB) holds none of the inputs and no dirty lines; the reference harness times its kernels the
same way.
Algorithmic bytes (the minimum HBM traffic of each pass, fp16 activations):
  stats     read z                               = 2·M·C
  apply     read z, write one destination        = 4·M·C
  backward  read z and dA once, write dz         = 6·M·C      (two passes: the sums need all of z first)
  fwd       statistics then apply back to back   = 4·M·C      (as in a training step: z read once from HBM
                                                               when the apply finds it in L2)
  stem wgrad read x and dz once                  = 2·(N·H·W·3 + N·P·Q·32)
  mask loss read proto, write dproto, read the mask bits = 2·(2·B·Hp·Wp·32) + B·G·Hp·Wp/8; its useful
            work is 3 × 64 flop per (positive, crop pixel) pair (z, dproto, dcoef), reported as GFLOP/s
GB/s are those bytes ÷ time; the fraction is of the measured copy bandwidth (MEASURED_PEAKS.json).
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


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def reference_times(binary, cases):
    """cases: list of meta int lists → list of ms arrays from the reference harness (timing ops)."""
    import numpy as np
    from oracle import fsow
    ins = {f"c{i}.meta": np.array(m, np.int32) for i, m in enumerate(cases)}
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([binary, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=900)
        out = fsow.load(os.path.join(td, "out.fsow"))
    return [out[f"c{i}.ms"] for i in range(len(cases))]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--ref", default=os.path.join(ROOT, "oracle", "_ref", "ref_bn"))
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    import torch

    from objectsam_b200 import bn
    from objectsam_b200.conv import ConvGeom, ConvOp, DestSpec
    from objectsam_b200.model import Model
    from oracle import yolo_params

    dev = "cuda"
    flush = torch.ones(64 << 20, dtype=torch.float32, device=dev)  # 256 MiB, read (not written) between calls

    def timed(fn):
        fn()
        fn()
        tot = 0.0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(a.iters):
            flush.sum()
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / a.iters

    m = Model(a.batch, a.imgsz)
    m.load(yolo_params.make_weights(0))
    m.sync_weights()
    shapes = []
    for n in m.nodes():
        if n["kind"] == 0:
            g = ConvGeom(n["N"], n["H"], n["W"], n["C"], n["K"], n["R"], n["R"], n["stride"], n["R"] // 2)
            s = (n["N"], g.P(), g.Q(), n["K"])
            if s not in shapes:
                shapes.append(s)
    del m
    torch.cuda.empty_cache()
    peak, peak_kind = hbm_peak()
    gen = torch.Generator(device=dev).manual_seed(0)
    rows = []
    for (N, H, W, C) in shapes:
        M = N * H * W
        z = (torch.rand(N, H, W, C, generator=gen, device=dev) * 5 - 2).half()
        dA = ((torch.rand(N, H, W, C, generator=gen, device=dev) - 0.5) * 0.2).half()
        ones, zeros = torch.ones(C, device=dev), torch.zeros(C, device=dev)
        rm, rv = zeros.clone(), ones.clone()
        mean, istd, scale, shift = (torch.empty(C, device=dev) for _ in range(4))
        out, dz = torch.empty_like(z), torch.empty_like(z)
        gwg, gwb = torch.empty(C, device=dev), torch.empty(C, device=dev)
        ws = bn.workspace(C, dev)
        t_stats = timed(lambda: bn.bn_forward_stats(z, ones, zeros, rm, rv, 0.0, 1e-3, mean, istd, scale, shift, ws=ws))
        t_apply = timed(lambda: bn.bn_forward_apply(z, scale, shift, None, [DestSpec(out)], True))
        t_bwd = timed(lambda: bn.bn_backward(z, mean, istd, scale, shift, [DestSpec(dA)], True, dz, gwg, gwb, ws=ws))

        def fwd_pair():
            bn.bn_forward_stats(z, ones, zeros, rm, rv, 0.0, 1e-3, mean, istd, scale, shift, ws=ws)
            bn.bn_forward_apply(z, scale, shift, None, [DestSpec(out)], True)
        t_pair = timed(fwd_pair)
        mc2 = 2.0 * M * C
        rows.append({"op": "bn", "shape": [N, H, W, C], "ms": [t_stats, t_apply, t_bwd, t_pair],
                     "gbs": [mc2 / t_stats / 1e6, 2 * mc2 / t_apply / 1e6, 3 * mc2 / t_bwd / 1e6,
                             2 * mc2 / t_pair / 1e6]})
        del z, dA, out, dz
        torch.cuda.empty_cache()
    # stem weight gradient
    N, H, W = a.batch, a.imgsz, a.imgsz
    op = ConvOp().init(ConvGeom(N, H, W, 3, 32, 3, 3, 2, 1))
    P, Q = op.geom().P(), op.geom().Q()
    x = torch.rand(N, H, W, 3, generator=gen, device=dev).half()
    dzs = (torch.rand(N, P, Q, 32, generator=gen, device=dev) * 2 - 1).half()
    dw = torch.empty(32, 3, 3, 3, dtype=torch.half, device=dev)
    wsw = torch.empty(op.workspace_size(), dtype=torch.uint8, device=dev)
    t_wg = timed(lambda: op.wgrad(x, dzs, dw, ws=wsw))
    wbytes = 2.0 * (N * H * W * 3 + N * P * Q * 32)
    rows.append({"op": "stem_wgrad", "shape": [N, H, W, 3, 32], "ms": [t_wg], "gbs": [wbytes / t_wg / 1e6]})
    op.close()

    # mask loss: 1–30 boxes per image (sides 8–400 px), 10 positives per box, random mask bits
    from objectsam_b200 import loss as mloss
    S, B = a.imgsz, a.batch
    Hp = Wp = S // 4
    lv = [(S // 8, S // 8), (S // 16, S // 16), (S // 32, S // 32)]
    A = sum(h * w for h, w in lv)
    G = 32
    cg = torch.Generator(device="cpu").manual_seed(1)
    n_gt = torch.randint(1, 31, (B,), generator=cg)
    side = torch.rand(B, G, 2, generator=cg) * 392 + 8
    xy = torch.rand(B, G, 2, generator=cg) * (S - side)
    gt_box = torch.cat([xy, xy + side], -1).float().contiguous()
    npos = (n_gt * 10).int()
    pos = torch.zeros(B, A, dtype=torch.int32)
    agt = torch.full((B, A), -1, dtype=torch.int32)
    for b in range(B):
        sel = torch.randperm(A, generator=cg)[: int(npos[b])].sort().values
        pos[b, : len(sel)] = sel.int()
        agt[b, sel] = (torch.arange(len(sel)) // 10).int()
    words = torch.randint(-2**31, 2**31 - 1, (B, G, Hp * Wp // 32), generator=cg, dtype=torch.int64).int()
    coef = [((torch.rand(B, h, w, 32, generator=gen, device=dev) * 2 - 1)).half() for h, w in lv]
    proto = (torch.rand(B, Hp, Wp, 32, generator=gen, device=dev) * 2 - 1).half()
    dproto = torch.empty_like(proto)
    dcoef = [torch.empty_like(c) for c in coef]
    lsum = torch.zeros(1, device=dev)
    fg = torch.tensor([float(npos.sum())], device=dev)
    one = torch.ones(1, device=dev)
    args = [t.to(dev) for t in (npos.int(), pos, agt, gt_box, words)]
    t_ml = timed(lambda: mloss.mask_loss(coef, proto, *args, fg, one, S, 7.5, dproto, dcoef, lsum))
    pairs = 0
    for b in range(B):  # positive × crop-pixel pairs: the work of the reference's per-pixel loops
        for i in range(int(npos[b])):
            x1, y1, x2, y2 = (gt_box[b, int(agt[b, int(pos[b, i])])] / 4).tolist()
            pairs += max(0, min(Wp, int(-(-x2 // 1))) - max(0, int(-(-x1 // 1)))) * \
                max(0, min(Hp, int(-(-y2 // 1))) - max(0, int(-(-y1 // 1))))
    mbytes = 2.0 * (B * Hp * Wp * 32 * 2) + B * G * Hp * Wp / 8
    rows.append({"op": "mask_loss", "shape": [B, Hp, Wp, int(npos.sum())], "ms": [t_ml], "gbs": [mbytes / t_ml / 1e6],
                 "pairs": pairs, "gflops": 3 * 2 * 32 * pairs / t_ml / 1e6})

    ref = {}
    if a.ref and os.path.exists(a.ref):
        cases = [[10, *r["shape"], a.iters] for r in rows if r["op"] == "bn"] + [[13, N, H, W, a.iters]]
        for r, t in zip(rows, reference_times(a.ref, cases)):
            r["ref_ms"] = [float(v) for v in t]

    print(f"HBM peak {peak:.0f} GB/s ({peak_kind})")
    print(f"{'pass':12s} {'shape':24s} {'stats':>8s} {'apply':>8s} {'bwd':>8s} {'fwd':>8s}   {'GB/s (frac)':>48s}   "
          f"{'ref stats':>9s} {'apply':>8s} {'bwd':>8s} {'fwd':>8s}")
    tot, rtot = 0.0, 0.0
    for r in rows:
        shp = "x".join(map(str, r["shape"]))
        ms = " ".join(f"{v:8.3f}" for v in r["ms"]) + " " * 9 * (4 - len(r["ms"]))
        gb = " ".join(f"{g:6.0f} ({g / peak:4.2f})" for g in r["gbs"])
        rs = " ".join(f"{v:8.3f}" for v in r.get("ref_ms", []))
        print(f"{r['op']:12s} {shp:24s} {ms}   {gb:>48s}   {rs}")
        tot += sum(r["ms"][:3])  # stats + apply + backward (the back-to-back pair is shown, not summed)
        rtot += sum(r.get("ref_ms", [0.0])[:3])
    print(f"total ms: ours {tot:.3f}" + (f", reference {rtot:.3f}" if ref is not None and rtot else ""))
    if a.json:
        with open(a.json, "w") as f:
            json.dump({"batch": a.batch, "imgsz": a.imgsz, "peak_gbs": peak, "peak_kind": peak_kind, "rows": rows},
                      f, indent=1)


if __name__ == "__main__":
    main()
