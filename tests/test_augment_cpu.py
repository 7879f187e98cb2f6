"""The CPU restatement of the training-batch augmentation (oracle/augment_ref.py) against the reference's own
kernels' outputs (tests/golden/augment_golden.npz, made by tests/golden/make_augment_golden.py on a GPU),
hand-made known-answer cases, and osam_augment's argument checks (which return before any CUDA call).

Tolerance against the golden outputs (the restatement computes without the reference's fast-math division
and fused multiply-adds): at most 1 % of pixel values off, by at most 8 u8 levels (one level apart before the
HSV round trip can move the quantised hue, which shifts the other channels by a few levels), targets
identical, at most 1 % of mask and ignore cells different.
"""
import ctypes
import os

import numpy as np
import pytest

from aug_batch import make_batch
from objectsam_b200 import _lib
from objectsam_b200.augment import HEADER_DT, INST_DT, SAMPLE_DT, SRC_DT, pack_meta
from oracle import augment_ref as R

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "augment_golden.npz")


def test_restatement_matches_reference_golden():
    g = np.load(GOLDEN)
    seed, B, S, G, Hp, Wp = (int(v) for v in g["case"])
    bt = make_batch(seed, B, S)
    want = R.augment(bt["samples"], bt["sources"], bt["insts"], bt["img"], bt["mask"], S, G, Hp, Wp)
    d = np.abs(want["img"].astype(np.float32) - g["img"].astype(np.float32))
    assert d.max() <= 8 / 255 + 1e-3 and (d > 0).mean() <= 0.01, (d.max(), (d > 0).mean())
    np.testing.assert_array_equal(want["n_gt"], g["n_gt"])
    assert g["n_gt"].sum() > 0
    for b in range(B):
        k = int(g["n_gt"][b])
        np.testing.assert_array_equal(want["gt_inst"][b, :k], g["gt_inst"][b, :k])
        np.testing.assert_allclose(want["box"][b, :k], g["box"][b, :k], rtol=1e-5, atol=1e-4)
    bits = np.unpackbits(g["mask"].astype(np.int32).view(np.uint8), bitorder="little").reshape(B, G, Hp, Wp)
    for b in range(B):
        k = int(g["n_gt"][b])
        assert (bits[b, :k].astype(bool) != want["mask"][b, :k]).mean() <= 0.01
    assert bits.any()
    ign = np.unpackbits(g["ignore"].astype(np.int32).view(np.uint8), bitorder="little").reshape(B, Hp, Wp)
    assert (ign.astype(bool) != want["ignore"]).mean() <= 0.01


def one_tile_sample(S, w, h, s=0.5, tx=0.0, ty=0.0, flip=0, hsv=(1.0, 1.0, 1.0)):
    sm = np.zeros(1, SAMPLE_DT)[0]
    sm["src"] = (0, -1, -1, -1)
    sm["ta"][0] = (0, 0, w, h)
    sm["tb"][0] = (0, 0)
    sm["s"], sm["tx"], sm["ty"], sm["hsv"], sm["flip"] = s, tx, ty, hsv, flip
    return sm


def gray_source(w, h, seed=0):
    r = np.random.default_rng(seed)
    v = r.integers(0, 256, (h, w), dtype=np.uint8)
    src = np.zeros(1, SRC_DT)
    src["img_off"], src["iw"], src["ih"], src["mw"], src["mh"] = 0, w, h, w, h
    return np.repeat(v[..., None], 3, -1).reshape(-1), src, v


def test_half_scale_samples_canvas_pixels_exactly():
    """s = 0.5, t = 0 on a gray source covering the canvas: output (x, y) reads canvas (2x, 2y) with zero
    bilinear weight on the neighbours, and gray survives the HSV round trip at unit gains."""
    S = 16
    img, src, v = gray_source(2 * S, 2 * S)
    out = R.image(one_tile_sample(S, 2 * S, 2 * S), src, img, S)
    np.testing.assert_array_equal(out[..., 0], (v[::2, ::2].astype(np.float32) / 255).astype(np.float16))
    assert (out[..., 0] == out[..., 2]).all()


def test_no_tile_is_fill_value():
    S = 8
    sm = one_tile_sample(S, 4, 4)
    sm["src"][0] = -1
    out = R.image(sm, np.zeros(0, SRC_DT), np.zeros(3, np.uint8), S)
    assert (out == np.float16(114 / 255)).all()


def test_flip_mirrors_the_image():
    S = 16
    img, src, _ = gray_source(2 * S, 2 * S, seed=3)
    a = R.image(one_tile_sample(S, 2 * S, 2 * S, s=0.43, tx=1.5, ty=-0.7), src, img, S)
    b = R.image(one_tile_sample(S, 2 * S, 2 * S, s=0.43, tx=1.5, ty=-0.7, flip=1), src, img, S)
    np.testing.assert_array_equal(b, a[:, ::-1])


def test_hsv_known_values():
    r, g, b = np.array([255, 0, 0, 128, 10]), np.array([0, 255, 0, 128, 200]), np.array([0, 0, 255, 128, 30])
    h, s, v = R.rgb2hsv(r, g, b)
    np.testing.assert_array_equal(h, [0, 60, 120, 0, 63])  # (120 + 60·20/190) / 2 = 63.16
    np.testing.assert_array_equal(s, [255, 255, 255, 0, 242])
    np.testing.assert_array_equal(v, [255, 255, 255, 128, 200])
    rr, gg, bb = R.hsv2rgb(h[:4], s[:4], v[:4])
    np.testing.assert_array_equal(rr, r[:4])
    np.testing.assert_array_equal(gg, g[:4])
    np.testing.assert_array_equal(bb, b[:4])


def test_target_box_known_answer():
    """A box inside tile 0 of a canvas placed at (10, 20) from source offset (0, 0), mapped by s = 0.5,
    t = (4, −2), then flipped in a 64-pixel image."""
    S = 64
    sm = one_tile_sample(S, 80, 90, s=0.5, tx=4.0, ty=-2.0, flip=1)
    sm["ta"][0] = (10, 20, 90, 110)
    inst = np.zeros(1, INST_DT)[0]
    inst["box"] = (10.0, 12.0, 50.0, 40.0)
    X1, Y1, X2, Y2, w1, h1 = R.map_box(sm, inst, S)
    # canvas box (20, 32, 60, 60) → output (14, 14, 34, 28) → flipped x: (30, 50)
    assert (X1, Y1, X2, Y2) == (30.0, 14.0, 50.0, 28.0)
    assert (w1, h1) == (20.0, 14.0)
    boxes, idx = R.targets(0, sm, np.array([inst], INST_DT), S, 4)
    np.testing.assert_array_equal(boxes, [[30, 14, 50, 28]])
    inst["box"] = (100.0, 100.0, 120.0, 120.0)  # beyond the tile: dropped
    assert R.map_box(sm, inst, S) is None


def test_osam_augment_rejects_bad_arguments():
    """Validated on the host before any launch (no GPU needed): S not a multiple of 8, Wp not a multiple of
    32, misaligned records."""
    L = _lib.lib()
    fake = 1 << 20  # never dereferenced: every call below fails its checks first

    def call(S=64, Wp=32, src_off=0):
        bt = _lib.AugBatch(fake, fake + 32, fake + 4096 + src_off, fake + 8192, fake, fake)
        ao = _lib.AugOut(fake, fake, fake, fake, None, fake, 4, 16, Wp)
        return L.osam_augment(ctypes.byref(bt), 2, S, ctypes.byref(ao), None)

    assert call(S=60) == _lib.OSAM_ERR_INVALID
    assert call(Wp=48) == _lib.OSAM_ERR_INVALID
    assert call(src_off=4) == _lib.OSAM_ERR_INVALID
    assert b"aligned" in L.osam_last_error()


def test_pack_meta_layout():
    """The one-block layout: header (32 B), B samples (148 B each), 4B sources (24 B each), instances (64 B)."""
    bt = make_batch(5, 2, 64)
    m = bt["meta"]
    assert m.size == 32 + 2 * 148 + 8 * 24 + len(bt["insts"]) * 64
    assert m[:32].view(np.int32)[3] == len(bt["insts"])
    assert SAMPLE_DT.itemsize == 148 and SRC_DT.itemsize == 24 and INST_DT.itemsize == 64
    with pytest.raises(AssertionError):
        pack_meta(3, 64, bt["samples"], bt["sources"], bt["insts"], 0, 0)


def test_record_dtypes_match_the_c_header(tmp_path):
    """The numpy record layouts of objectsam_b200.augment against include/osam.h itself: a C program built
    with gcc prints every field's offset and each record's size (the reference harness asserts the header
    against the reference's own structs at compile time)."""
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    fields = {"osam_aug_src": SRC_DT, "osam_aug_inst": INST_DT, "osam_aug_sample": SAMPLE_DT,
              "osam_aug_header": HEADER_DT}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "osam.h"', "int main(void) {"]
    for st, dt in fields.items():
        lines.append(f'  printf("{st} size %zu\\n", sizeof({st}));')
        for name in dt.names:
            lines.append(f'  printf("{st} {name} %zu\\n", offsetof({st}, {name}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(HERE), "include")
    subprocess.run(["gcc", "-std=c11", "-I", inc, str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        st, name, v = line.split()
        got[(st, name)] = int(v)
    for st, dt in fields.items():
        assert got[(st, "size")] == dt.itemsize, st
        for name in dt.names:
            assert got[(st, name)] == dt.fields[name][1], (st, name)
