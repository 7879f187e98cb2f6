"""Profiling driver: one eager forward of the fused model, then one node of it `--repeat` more times.

Used to point Nsight Compute at a single conv of the network on a realistic activation:

    python -m objectsam_b200.profile_case --batch 32 --node model.22.proto.cv2 --repeat 3

wraps the repeated launches in the NVTX range "osam_profile", so that
`ncu --nvtx --nvtx-include osam_profile/ -c <repeat> …` captures exactly the repeated node.
"""
from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--imgsz", type=int, default=640)
    ap.add_argument("--node", default="model.22.proto.cv2")
    ap.add_argument("--repeat", type=int, default=1)
    ap.add_argument("--list", action="store_true")
    a = ap.parse_args()
    import numpy as np
    import torch

    from objectsam_b200.model import Model
    from oracle import yolo_params

    m = Model(a.batch, a.imgsz)
    m.load(yolo_params.make_weights(0))
    m.sync_weights()
    rng = np.random.Generator(np.random.PCG64(0))
    m.input().copy_(torch.from_numpy(rng.random((a.batch, a.imgsz, a.imgsz, 3), dtype=np.float32)).half())
    nodes = m.nodes()
    idx = {n["name"]: n["index"] for n in nodes}
    if a.list:
        for n in nodes:
            print(n["index"], n["name"], n["kind"], n["N"], n["H"], n["W"], n["C"], n["K"], n["R"], n["stride"])
    kinds = {0: "k_conv_fprop", 1: "k_conv_fprop", 2: "k_conv_fprop", 3: "k_sppf"}
    per_kernel = {}
    for n in nodes:
        kname = "k_conv_stem" if (n["kind"] == 0 and n["C"] * n["R"] * n["S"] <= 32 and n["C"] % 32) else kinds[n["kind"]]
        per_kernel[kname] = per_kernel.get(kname, 0) + 1
    m.forward()
    torch.cuda.synchronize()
    i = idx[a.node]
    torch.cuda.nvtx.range_push("osam_profile")  # `ncu --nvtx --nvtx-include osam_profile/` captures only these
    for _ in range(a.repeat):
        m.forward_nodes(i, 1)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print("launches per forward:", per_kernel, "| repeated node", a.node, "index", i)


if __name__ == "__main__":
    main()
