"""Detection part of the training loss (DFL decode, top-10 task-aligned assignment, CIoU / DFL / BCE and their
gradients) and the whole segment-head loss, on the GPU through the C ABI, against the reference's own
SegLoss::run (src/loss.cu, compiled here as oracle/_ref/ref_bn op 5) on the same heads and ground truth.

Checks and tolerances (written per check below):
  assignment    agt identical (the same top-10 ranking by the same fp32 CIoU and metric); positives = items[4]
  target scores |Δ| ≤ 1e-5·(|ref| + 1e-3)  at the positives
  loss sums     items[5], [8], [10], [11] relative 1e-4 (fp32 sums in a different order)
  gradients     dbox, dcls |Δ| ≤ 2e-3·|ref| + 2e-3·max|ref| (fp16 outputs of fp32 math)
  whole loss    items[0..3] relative 2e-3 (the mask loss's tensor-core BCE included), dproto / dcoef as the
                mask-loss test's bar
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from objectsam_b200 import loss as L
from oracle import det_loss_ref, fsow

from test_mask_loss_gpu import fp16, gt_batch, level_hw

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BN = os.path.join(ROOT, "oracle", "_ref", "ref_bn")
need_ref = pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")


def make_case(seed, B, S, G, n_range, side, head_sd=1.0):
    r = np.random.default_rng(seed)
    lv = level_hw(S)
    n_gt, box, words = gt_batch(r, B, S, G, n_range, side)
    c = dict(B=B, S=S, G=G, n_gt=n_gt, box=box, words=words, lv=lv)
    c["box_h"] = [fp16(r.normal(0, head_sd, (B, h, w, 64))) for h, w in lv]
    c["cls_h"] = [fp16(r.normal(0, head_sd, (B, h, w, 1))) for h, w in lv]
    c["coef_h"] = [fp16(r.uniform(-1, 1, (B, h, w, 32))) for h, w in lv]
    c["proto"] = fp16(r.uniform(-1, 1, (B, S // 4, S // 4, 32)))
    return c


def run_reference(c):
    ins = {"c0.meta": np.array([5, c["B"], c["S"], c["G"]], np.int32), "c0.n_gt": c["n_gt"], "c0.gt_box": c["box"],
           "c0.gt_mask": c["words"], "c0.scale": np.array([1.0], np.float32), "c0.proto": c["proto"]}
    for l in range(3):
        ins[f"c0.box{l}"], ins[f"c0.cls{l}"], ins[f"c0.coef{l}"] = c["box_h"][l], c["cls_h"][l], c["coef_h"][l]
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        return fsow.load(os.path.join(td, "out.fsow"))


def run_ours(c, whole=True):
    t16 = lambda a: torch.from_numpy(a).half().to(DEV)  # noqa: E731
    box = [t16(x) for x in c["box_h"]]
    cls = [t16(x) for x in c["cls_h"]]
    coef = [t16(x) for x in c["coef_h"]]
    proto = t16(c["proto"])
    dbox = [torch.full_like(x, 7.0) for x in box]
    dcls = [torch.full_like(x, 7.0) for x in cls]
    dcoef = [torch.full_like(x, 7.0) for x in coef]
    dproto = torch.full_like(proto, 7.0)
    n_gt = torch.from_numpy(c["n_gt"]).to(DEV)
    gt_box = torch.from_numpy(c["box"]).to(DEV)
    words = torch.from_numpy(c["words"]).to(DEV)
    scale = torch.ones(1, device=DEV)
    if whole:
        out = L.seg_loss(box, cls, coef, proto, n_gt, gt_box, words, scale, c["S"], dbox, dcls, dcoef, dproto)
    else:
        out = L.det_loss(box, cls, n_gt, gt_box, scale, c["S"], dbox, dcls, dcoef)
    torch.cuda.synchronize()
    res = {k: v.cpu().numpy() for k, v in out.items()}
    res["dbox"] = [x.float().cpu().numpy() for x in dbox]
    res["dcls"] = [x.float().cpu().numpy() for x in dcls]
    res["dcoef"] = [x.float().cpu().numpy() for x in dcoef]
    res["dproto"] = dproto.float().cpu().numpy()
    return res


def close(a, b, what, rel):
    err = np.abs(a - b)
    lim = rel * np.abs(b) + rel * (np.abs(b).max() + 1e-12)
    assert (err <= lim).all(), f"{what}: {(err > lim).sum()} out of tolerance, max err {err.max():.3e}"


CASES = {  # seed, B, S, G, gt count range, box side range (px)
    "b2_256_small": (3, 2, 256, 8, (3, 8), (16, 200)),
    "b3_320_tiny_boxes": (5, 3, 320, 12, (4, 12), (4, 40)),
    "b3_256_empty_and_full_image": (29, 3, 256, 6, (0, 6), (24, 180)),  # n_gt = 6 (all slots), 0, 4
}


@need_ref
@pytest.mark.parametrize("name", list(CASES))
def test_det_loss_matches_reference_segloss(cuda_lib, name):
    seed, B, S, G, nr, side = CASES[name]
    c = make_case(seed, B, S, G, nr, side)
    ref = run_reference(c)
    got = run_ours(c)
    A = got["agt"].shape[1]
    # assignment
    np.testing.assert_array_equal(got["agt"], ref["c0.agt"].reshape(B, A))
    items, ritems = got["items"], ref["c0.items"]
    assert items[4] == ritems[4] == float((got["agt"] >= 0).sum())
    assert (got["npos"] == (got["agt"] >= 0).sum(1)).all()
    for b in range(B):  # positives in anchor order
        n = got["npos"][b]
        np.testing.assert_array_equal(got["pos"][b, :n], np.nonzero(got["agt"][b] >= 0)[0])
    posm = got["agt"] >= 0
    rt = ref["c0.tsc"].reshape(B, A)
    assert (np.abs(got["tsc"][posm] - rt[posm]) <= 1e-5 * (np.abs(rt[posm]) + 1e-3)).all()
    assert (got["tsc"][~posm] == 0).all()
    for k in (5, 8, 10, 11):
        assert abs(items[k] - ritems[k]) <= 1e-4 * abs(ritems[k]) + 1e-6, f"items[{k}] {items[k]} vs {ritems[k]}"
    for k in range(4):
        assert abs(items[k] - ritems[k]) <= 2e-3 * abs(ritems[k]) + 1e-6, f"items[{k}] {items[k]} vs {ritems[k]}"
    for l in range(3):
        close(got["dbox"][l], ref[f"c0.dbox{l}"], f"dbox{l}", 2e-3)
        close(got["dcls"][l], ref[f"c0.dcls{l}"], f"dcls{l}", 2e-3)
        close(got["dcoef"][l], ref[f"c0.dcoef{l}"], f"dcoef{l}", 3e-3)
    close(got["dproto"], ref["c0.dproto"], "dproto", 3e-3)


def test_det_loss_workspace_any_contents_and_repeats(cuda_lib):
    """The workspace needs no zeroing (here: filled with 0xFF bytes, i.e. −1 counts and NaN floats): a second
    call on the same inputs gives the same result."""
    seed, B, S, G, nr, side = CASES["b2_256_small"]
    c = make_case(seed, B, S, G, nr, side)
    A = sum(h * w for h, w in level_hw(S))
    ws = torch.full((int(L.lib().osam_det_loss_workspace_size(B, A, G)),), 255, dtype=torch.uint8, device=DEV)
    first, second = None, None
    for i in range(2):
        t16 = lambda a: torch.from_numpy(a).half().to(DEV)  # noqa: E731
        box, cls = [t16(x) for x in c["box_h"]], [t16(x) for x in c["cls_h"]]
        dbox, dcls = [torch.zeros_like(x) for x in box], [torch.zeros_like(x) for x in cls]
        dcoef = [torch.zeros(B, h, w, 32, dtype=torch.half, device=DEV) for h, w in level_hw(S)]
        out = L.det_loss(box, cls, torch.from_numpy(c["n_gt"]).to(DEV), torch.from_numpy(c["box"]).to(DEV),
                         torch.ones(1, device=DEV), S, dbox, dcls, dcoef, ws=ws)
        torch.cuda.synchronize()
        res = (out["agt"].cpu(), out["items"].cpu(), [x.cpu() for x in dbox])
        if i == 0:
            first = res
        else:
            second = res
    assert torch.equal(first[0], second[0])
    assert torch.allclose(first[1], second[1], rtol=1e-5, atol=1e-6)
    for a, b in zip(first[2], second[2]):
        assert torch.equal(a, b)


def test_det_loss_no_ground_truth(cuda_lib):
    """No gt anywhere: every anchor negative, class loss only, zero box gradients, items[4] = 0."""
    seed, B, S, G, nr, side = CASES["b2_256_small"]
    c = make_case(seed, B, S, G, (0, 0), side)
    got = run_ours(c, whole=True)
    assert (got["agt"] == -1).all() and got["items"][4] == 0 and got["items"][1] == 0
    for l in range(3):
        assert (got["dbox"][l] == 0).all()
        assert (got["dcoef"][l] == 0).all()
    assert got["items"][2] > 0


@pytest.mark.parametrize("seed", [11, 12])
def test_det_loss_matches_cpu_restatement(cuda_lib, seed):
    """Against oracle/det_loss_ref.py (float32 numpy in the reference's order; no fused multiply-adds, so an
    anchor whose rank sits on a rounding-level tie may go the other way: ≥ 99 % of the assignment identical,
    the rest compared where both agree)."""
    c = make_case(seed, 2, 128, 6, (2, 6), (12, 100))
    got = run_ours(c, whole=False)
    ref = det_loss_ref.det_loss(c["box_h"], c["cls_h"], c["n_gt"], c["box"], c["S"])
    agree = got["agt"] == ref["agt"]
    assert agree.mean() >= 0.99, f"assignment agrees on {agree.mean():.4f}"
    assert (got["agt"] >= 0).sum() > 0
    both = agree & (got["agt"] >= 0)
    assert np.allclose(got["tsc"][both], ref["tsc"][both], rtol=1e-4, atol=1e-6)
    if agree.all():
        for k in (4, 5, 8, 10, 11):
            assert abs(got["items"][k] - ref["items"][k]) <= 1e-3 * abs(ref["items"][k]) + 1e-5, k
        for l in range(3):  # fp16 outputs: also one fp16 subnormal step (6e-8) of absolute slack
            for k, want in (("dbox", ref["dbox"][l]), ("dcls", ref["dcls"][l])):
                err = np.abs(got[k][l] - want)
                lim = 3e-3 * np.abs(want) + 3e-3 * np.abs(want).max() + 6e-8
                assert (err <= lim).all(), f"{k}{l}: {(err > lim).sum()} out of tolerance, max err {err.max():.3e}"
