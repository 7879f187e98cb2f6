"""Generates tests/golden/network_golden.npz from the reference's own network (its cuDNN build).

Runs on a machine with a B200 and the binaries of oracle/Makefile (oracle/_ref/ref_forward_fp32 and
ref_forward_fp16, built from the reference sources).  The weights and images are regenerated from their
seeds by oracle/yolo_ref.calibrated_weights / oracle/yolo_params.make_images, so only the reference's
outputs are stored:

    python tests/golden/make_network_golden.py [out.npz]

Cases: (seed, batch, imgsz) below; per case the raw heads (box/cls/coef × 3 levels) and proto, NHWC,
from the fp32 build (act_t = float, FMA math, no TF32 — the reference's parity precision) and from the
fp16 build (its production precision), stored as float16 to keep the fixture small.
"""
from __future__ import annotations

import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import fsow, yolo_params, yolo_ref  # noqa: E402

CASES = [(3, 2, 128), (5, 1, 192)]
KEYS = [f"out.{k}{l}" for k in ("box", "cls", "coef") for l in range(3)] + ["out.proto"]


def run_reference(binary: str, weights: dict, images: np.ndarray) -> dict:
    with tempfile.TemporaryDirectory() as td:
        wp, ip, op = (os.path.join(td, n) for n in ("w.fsow", "x.fsow", "o.fsow"))
        fsow.save(wp, weights)
        fsow.save(ip, {"images": images.astype(np.float32)})
        subprocess.run([binary, wp, ip, op], check=True)
        return fsow.load(op)


def main(out=os.path.join(HERE, "network_golden.npz")):
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    res = {}
    for ci, (seed, n, s) in enumerate(CASES):
        w = yolo_ref.calibrated_weights(seed, 128)
        imgs = yolo_params.make_images(n, s, seed + 100)
        res[f"c{ci}_cfg"] = np.array([seed, n, s], np.int64)
        for prec in ("fp32", "fp16"):
            o = run_reference(os.path.join(ref_dir, f"ref_forward_{prec}"), w, imgs)
            for k in KEYS:
                res[f"c{ci}_{prec}_{k}"] = o[k].astype(np.float16 if prec == "fp16" else np.float32)
    res["n_cases"] = np.array(len(CASES))
    np.savez_compressed(out, **res)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main(*sys.argv[1:])
