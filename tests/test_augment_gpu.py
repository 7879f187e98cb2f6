"""Training-batch augmentation (osam_augment, ≙ the reference's augment(), src/augment.cu) on the GPU through
the C ABI, against the reference's own kernels (oracle/_ref/ref_bn op 6) on the same seeded batches, and
against the CPU restatement (oracle/augment_ref.py).

Checks and tolerances:
  reference kernels   bit-exact: every fp16 pixel, n_gt, the boxes and instance indices of the targets, every
                      mask and ignore word (the same float steps under the same fast-math flags)
  CPU restatement     float32 without fast-math division or fused multiply-adds: at most 1 % of pixel values
                      off, by at most 8 u8 levels (a bilinear value one level apart before the HSV round
                      trip can move the quantised hue, which shifts the other channels by a few levels);
                      targets identical; at most 1 % of mask cells different
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from aug_batch import make_batch
from objectsam_b200 import augment as A
from oracle import augment_ref, fsow

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BN = os.path.join(ROOT, "oracle", "_ref", "ref_bn")
need_ref = pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")

# seed, B (even: the reference's one-block record layout needs it), S, G, Hp, Wp, tile overlap (px)
CASES = {
    "b4_256_g16": (1, 4, 256, 16, 64, 64, 0),
    "b2_640_g256_train_grid": (2, 2, 640, 256, 160, 160, 0),
    "b6_320_g8_cap": (3, 6, 320, 8, 64, 64, 0),
    "b4_256_overlapping_tiles": (4, 4, 256, 16, 64, 64, 37),
}


def on_device(bt):
    return (torch.from_numpy(bt["meta"]).to(DEV), torch.from_numpy(bt["img"]).to(DEV),
            torch.from_numpy(bt["mask"].view(np.int32)).to(DEV))


def run_reference(bt, G, Hp, Wp, ignore=True, iters=0):
    ins = {"c0.meta": np.array([6, bt["B"], bt["S"], G, Hp, Wp, int(ignore), iters], np.int32),
           "c0.blob": bt["meta"], "c0.img": bt["img"], "c0.mask": bt["mask"].view(np.int32)}
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        return fsow.load(os.path.join(td, "out.fsow"))


def run_ours(bt, G, Hp, Wp, ignore=True, out=None):
    meta, img, mask = on_device(bt)
    o = A.augment(meta, img, mask, bt["B"], bt["S"], G, Hp, Wp, ignore=ignore, out=out)
    torch.cuda.synchronize()
    return {k: (v.cpu().numpy() if v is not None else None) for k, v in o.items()}


@need_ref
@pytest.mark.parametrize("name", list(CASES))
def test_augment_matches_reference_kernels(cuda_lib, name):
    seed, B, S, G, Hp, Wp, ov = CASES[name]
    bt = make_batch(seed, B, S, overlap=ov)
    ref = run_reference(bt, G, Hp, Wp)
    got = run_ours(bt, G, Hp, Wp)
    np.testing.assert_array_equal(got["img"].astype(np.float32), ref["c0.img"])
    n = ref["c0.n_gt"]
    np.testing.assert_array_equal(got["n_gt"], n)
    assert n.sum() > 0
    rbox = ref["c0.box"].reshape(B, G, 4)
    rmask = ref["c0.mask"].reshape(B, G, -1)
    for b in range(B):
        k = n[b]
        np.testing.assert_array_equal(got["box"][b, :k], rbox[b, :k])
        np.testing.assert_array_equal(got["gt_inst"][b, :k], ref["c0.gt_inst"][b, :k])
        np.testing.assert_array_equal(got["mask"][b, :k], rmask[b, :k])
        assert (got["mask"][b, k:] == 0).all() and (got["gt_inst"][b, k:] == -1).all()
    np.testing.assert_array_equal(got["ignore"], ref["c0.ignore"].reshape(B, -1))
    if name == "b6_320_g8_cap":
        assert (n == G).any(), "the case should reach the per-image target cap"


@need_ref
def test_augment_extreme_hsv_gains_match_reference(cuda_lib):
    """Gains outside the training range: a negative hue gain (negative H), hue products of 360 and more, zero
    and saturating saturation/value gains."""
    from objectsam_b200.augment import pack_meta
    B, S, G, Hp, Wp = 4, 128, 8, 32, 32
    bt = make_batch(31, B, S)
    bt["samples"]["hsv"] = [[-0.7, 1.9, 0.2], [2.6, 0.0, 1.9], [7.3, 3.0, 0.0], [1.0, 1.0, 1.0]]
    bt["meta"] = pack_meta(B, S, bt["samples"], bt["sources"], bt["insts"], bt["img"].size, bt["mask"].size)
    ref = run_reference(bt, G, Hp, Wp)
    got = run_ours(bt, G, Hp, Wp)
    np.testing.assert_array_equal(got["img"].astype(np.float32), ref["c0.img"])


def test_augment_writes_every_output_word(cuda_lib):
    """Outputs filled with 0xFF bytes beforehand (and a second call on the same buffers) give the same
    result: nothing depends on prior zeroing."""
    seed, B, S, G, Hp, Wp, _ = CASES["b4_256_g16"]
    bt = make_batch(seed, B, S)
    first = run_ours(bt, G, Hp, Wp)
    out = {"img": torch.full((B, S, S, 3), float("nan"), dtype=torch.half, device=DEV),
           "n_gt": torch.full((B,), -1, dtype=torch.int32, device=DEV),
           "box": torch.full((B, G, 4), float("nan"), device=DEV),
           "gt_inst": torch.full((B, G), 123, dtype=torch.int32, device=DEV),
           "mask": torch.full((B, G, Hp * Wp // 32), -1, dtype=torch.int32, device=DEV),
           "ignore": torch.full((B, Hp * Wp // 32), -1, dtype=torch.int32, device=DEV)}
    for _ in range(2):
        again = run_ours(bt, G, Hp, Wp, out=out)
        for k in first:
            np.testing.assert_array_equal(np.nan_to_num(again[k]), np.nan_to_num(first[k]), err_msg=k)


def test_augment_without_ignore_output(cuda_lib):
    seed, B, S, G, Hp, Wp, _ = CASES["b4_256_g16"]
    bt = make_batch(seed, B, S)
    a = run_ours(bt, G, Hp, Wp, ignore=True)
    b = run_ours(bt, G, Hp, Wp, ignore=False)
    assert b["ignore"] is None
    for k in ("img", "n_gt", "box", "gt_inst", "mask"):
        np.testing.assert_array_equal(a[k], b[k])


@pytest.mark.parametrize("seed", [21, 22])
def test_augment_matches_cpu_restatement(cuda_lib, seed):
    B, S, G, Hp, Wp = 2, 128, 8, 32, 32
    bt = make_batch(seed, B, S)
    got = run_ours(bt, G, Hp, Wp)
    want = augment_ref.augment(bt["samples"], bt["sources"], bt["insts"], bt["img"], bt["mask"], S, G, Hp, Wp)
    d = np.abs(got["img"].astype(np.float32) - want["img"].astype(np.float32))
    assert d.max() <= 8 / 255 + 1e-3 and (d > 0).mean() <= 0.01, (d.max(), (d > 0).mean())
    np.testing.assert_array_equal(got["n_gt"], want["n_gt"])
    for b in range(B):
        k = want["n_gt"][b]
        np.testing.assert_array_equal(got["gt_inst"][b, :k], want["gt_inst"][b, :k])
        np.testing.assert_allclose(got["box"][b, :k], want["box"][b, :k], rtol=1e-5, atol=1e-4)
    bits = np.unpackbits(got["mask"].view(np.uint8), bitorder="little").reshape(B, G, Hp, Wp).astype(bool)
    assert (bits != want["mask"]).mean() <= 0.01
    ibits = np.unpackbits(got["ignore"].view(np.uint8), bitorder="little").reshape(B, Hp, Wp).astype(bool)
    assert (ibits != want["ignore"]).mean() <= 0.01
