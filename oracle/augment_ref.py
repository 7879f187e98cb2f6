"""Test infrastructure: CPU restatement (numpy, float32) of the reference's training-batch augmentation,
src/augment.cu (declared in src/augment.cuh:19), for checking objectsam_b200's osam_augment on small batches.

Used only by tests/ (and the golden-vector script beside them); the product path never imports it.

Parity: this restatement computes in IEEE float32 with separately rounded operations.  The reference (and
the CUDA path, built with the same flags) runs under --use_fast_math — approximate division, fused
multiply-adds — so a value that lands within an ulp of a rounding or floor boundary may come out one u8
level or one cell apart, and a pixel one level apart before the HSV round trip may move its quantised hue
and end a few levels apart.  The bit-exact pin is the reference's own kernels (oracle/_ref/ref_bn op 6, on
the GPU); this restatement is pinned against their committed outputs (tests/golden/augment_golden.npz)
within that tolerance.

Batch records are numpy structured arrays with the layouts of include/osam.h (osam_aug_*), which are
the reference's (src/dataset.h:19-47); objectsam_b200.augment builds them.
"""
from __future__ import annotations

import numpy as np

F = np.float32
FILL = 114  # canvas value outside every tile (src/augment.cu:10)


def canvas_px(sm, srcs, img: np.ndarray, S: int, px: np.ndarray, py: np.ndarray) -> np.ndarray:
    """Canvas pixels (src/augment.cu:7-23): the first present tile whose rectangle holds (px, py), read from
    its source; FILL outside the 2S × 2S canvas or every tile.  Returns float32 (n, 3)."""
    out = np.full(px.shape + (3,), FILL, F)
    done = (px < 0) | (py < 0) | (px >= 2 * S) | (py >= 2 * S)
    for t in range(4):
        s = int(sm["src"][t])
        if s < 0:
            continue
        a = sm["ta"][t]
        hit = ~done & (px >= a[0]) & (px < a[2]) & (py >= a[1]) & (py < a[3])
        if not hit.any():
            continue
        x = px[hit] - a[0] + sm["tb"][t][0]
        y = py[hit] - a[1] + sm["tb"][t][1]
        si = srcs[s]
        off = int(si["img_off"]) + (y.astype(np.int64) * int(si["iw"]) + x) * 3
        out[hit] = np.stack([img[off], img[off + 1], img[off + 2]], -1).astype(F)
        done |= hit
    return out


def rnd_u8(v: np.ndarray) -> np.ndarray:
    """min(255, max(0, round-half-even(v))) (src/augment.cu:25)."""
    return np.clip(np.rint(v), 0, 255).astype(np.int64)


def rgb2hsv(r, g, b):
    """OpenCV u8 RGB → HSV, H in 0..179 (src/augment.cu:28-44)."""
    mx = np.maximum(r, np.maximum(g, b))
    mn = np.minimum(r, np.minimum(g, b))
    d = mx - mn
    with np.errstate(divide="ignore", invalid="ignore"):
        s = np.where(mx > 0, np.rint(F(255) * d.astype(F) / mx.astype(F)), 0).astype(np.int64)
        df = d.astype(F)
        h_r = F(60) * (g - b).astype(F) / df
        h_g = F(120) + F(60) * (b - r).astype(F) / df
        h_b = F(240) + F(60) * (r - g).astype(F) / df
    hh = np.where(mx == r, h_r, np.where(mx == g, h_g, h_b))
    hh = np.where(d > 0, hh, F(0)).astype(F)
    hh = np.where(hh < 0, hh + F(360), hh).astype(F)
    h = np.rint(hh * F(0.5)).astype(np.int64)
    h = np.where(h >= 180, h - 180, h)
    return h, s, mx


def hsv2rgb(h, s, v):
    """OpenCV u8 HSV → RGB (src/augment.cu:47-63)."""
    H = (h.astype(F) * F(2)) / F(60)
    S_ = s.astype(F) / F(255)
    V = v.astype(F)
    fl = np.floor(H)
    i = fl.astype(np.int64) % 6
    f = (H - fl).astype(F)
    p = V * (F(1) - S_)
    q = V * (F(1) - S_ * f)
    t = V * (F(1) - S_ * (F(1) - f))
    R = np.select([i == 0, i == 1, i == 2, i == 3, i == 4], [V, q, p, p, t], V)
    G = np.select([i == 0, i == 1, i == 2, i == 3, i == 4], [t, V, V, q, p], p)
    B = np.select([i == 0, i == 1, i == 2, i == 3, i == 4], [p, p, t, V, V], q)
    return rnd_u8(R), rnd_u8(G), rnd_u8(B)


def image(sm, srcs, img: np.ndarray, S: int) -> np.ndarray:
    """One output image (src/augment.cu:65-97): flip, inverse affine, bilinear over the canvas, HSV gains,
    fp16 in 0..1.  Returns float16 (S, S, 3)."""
    y, x = np.meshgrid(np.arange(S), np.arange(S), indexing="ij")
    xs = np.where(sm["flip"], S - 1 - x, x)
    u = (xs.astype(F) - F(sm["tx"])) / F(sm["s"])
    v = (y.astype(F) - F(sm["ty"])) / F(sm["s"])
    x0 = np.floor(u).astype(np.int64)
    y0 = np.floor(v).astype(np.int64)
    fx = (u - x0.astype(F)).astype(F)[..., None]
    fy = (v - y0.astype(F)).astype(F)[..., None]
    a = canvas_px(sm, srcs, img, S, x0, y0)
    b = canvas_px(sm, srcs, img, S, x0 + 1, y0)
    c = canvas_px(sm, srcs, img, S, x0, y0 + 1)
    e = canvas_px(sm, srcs, img, S, x0 + 1, y0 + 1)
    one = F(1)
    val = (a * (one - fx) + b * fx) * (one - fy) + (c * (one - fx) + e * fx) * fy
    rgb = rnd_u8(val)
    h, s, vv = rgb2hsv(rgb[..., 0], rgb[..., 1], rgb[..., 2])
    g = sm["hsv"].astype(F)
    h = np.fmod(h.astype(F) * g[0], F(180)).astype(np.int64)
    s = np.minimum(np.maximum(s.astype(F) * g[1], F(0)), F(255)).astype(np.int64)
    vv = np.minimum(np.maximum(vv.astype(F) * g[2], F(0)), F(255)).astype(np.int64)
    r, gg, bb = hsv2rgb(h, s, vv)
    return (np.stack([r, gg, bb], -1).astype(F) / F(255)).astype(np.float16)


def map_box(sm, inst, S: int):
    """An instance's box in output pixels, clipped to its tile, mapped, clipped, flipped (src/augment.cu:123-134,
    :200-206); None when nothing of it lies in its tile.  Also the mapped size before the clip."""
    t = int(inst["tile"])
    ta, tb = sm["ta"][t], sm["tb"][t]
    dx, dy = F(int(ta[0]) - int(tb[0])), F(int(ta[1]) - int(tb[1]))
    bx = inst["box"].astype(F)
    x1 = max(F(bx[0] + dx), F(ta[0]))
    y1 = max(F(bx[1] + dy), F(ta[1]))
    x2 = min(F(bx[2] + dx), F(ta[2]))
    y2 = min(F(bx[3] + dy), F(ta[3]))
    if not (x2 > x1 and y2 > y1):
        return None
    s, tx, ty = F(sm["s"]), F(sm["tx"]), F(sm["ty"])
    w1, h1 = F((x2 - x1) * s), F((y2 - y1) * s)
    X1 = min(max(F(s * x1 + tx), F(0)), F(S))
    X2 = min(max(F(s * x2 + tx), F(0)), F(S))
    Y1 = min(max(F(s * y1 + ty), F(0)), F(S))
    Y2 = min(max(F(s * y2 + ty), F(0)), F(S))
    if sm["flip"]:
        X1, X2 = F(F(S) - X2), F(F(S) - X1)
    return X1, Y1, X2, Y2, w1, h1


def targets(i: int, sm, insts, S: int, G: int):
    """Targets of image i (src/augment.cu:116-152): kept non-ignore instances in instance order, at most G.
    Returns (boxes (n, 4) float32, instance indices (n,))."""
    boxes, idx = [], []
    for k in range(len(insts)):
        if len(idx) >= G:
            break
        inst = insts[k]
        if int(inst["sample"]) != i or int(inst["ignore"]):
            continue
        m = map_box(sm, inst, S)
        if m is None:
            continue
        X1, Y1, X2, Y2, w1, h1 = m
        w2, h2 = F(X2 - X1), F(Y2 - Y1)
        ar = max(F(w2 / F(h2 + F(1e-16))), F(h2 / F(w2 + F(1e-16))))
        if w2 > 2 and h2 > 2 and F(F(w2 * h2) / F(w1 * h1 + F(1e-16))) > F(0.1) and ar < 100:
            boxes.append((X1, Y1, X2, Y2))
            idx.append(k)
    return np.array(boxes, F).reshape(-1, 4), np.array(idx, np.int64)


def box_cells(x1, y1, x2, y2, cs, Hp: int, Wp: int):
    """Loss-grid window of a box, one cell of margin (src/augment.cu:163-164, :207-208)."""
    c0 = max(0, int(np.floor(F(x1 / cs))) - 1)
    c1 = min(Wp, int(np.ceil(F(x2 / cs))) + 1)
    r0 = max(0, int(np.floor(F(y1 / cs))) - 1)
    r1 = min(Hp, int(np.ceil(F(y2 / cs))) + 1)
    return c0, c1, r0, r1


def cell_bits(sm, inst, src, mask: np.ndarray, S: int, cs, rows: np.ndarray, cols: np.ndarray) -> np.ndarray:
    """Mask bit of each (row, col) cell: the cell centre followed back through flip, affine and tile to the
    instance's bitmap (src/augment.cu:174-185)."""
    t = int(inst["tile"])
    ta, tb = sm["ta"][t], sm["tb"][t]
    x = (cols.astype(F) + F(0.5)) * cs - F(0.5)
    y = (rows.astype(F) + F(0.5)) * cs - F(0.5)
    xs = np.where(sm["flip"], F(S - 1) - x, x).astype(F)
    u = (xs - F(sm["tx"])) / F(sm["s"])
    v = (y - F(sm["ty"])) / F(sm["s"])
    inside = (u >= ta[0]) & (u < ta[2]) & (v >= ta[1]) & (v < ta[3])
    sx = (u - F(ta[0])) + F(tb[0])
    sy = (v - F(ta[1])) + F(tb[1])
    kx = F(src["mw"]) / F(src["iw"])
    ky = F(src["mh"]) / F(src["ih"])
    mx = np.floor((sx + F(0.5)) * kx).astype(np.int64) - int(inst["mx0"])
    my = np.floor((sy + F(0.5)) * ky).astype(np.int64) - int(inst["my0"])
    ok = inside & (mx >= 0) & (my >= 0) & (mx < int(inst["mcw"])) & (my < int(inst["mch"]))
    bits = np.zeros(rows.shape, bool)
    if ok.any():
        wd = mask[int(inst["mask_off"]) + my[ok] * int(inst["wpr"]) + (mx[ok] >> 5)].astype(np.uint64)
        bits[ok] = ((wd >> (mx[ok] & 31).astype(np.uint64)) & 1) == 1
    return bits


def augment(smp, srcs, insts, img: np.ndarray, mask: np.ndarray, S: int, G: int, Hp: int, Wp: int):
    """The whole batch (src/augment.cu:243-252).  Returns img (B, S, S, 3) fp16, n_gt (B,), box (B, G, 4),
    gt_inst (B, G) (−1 past n_gt), mask (B, G, Hp, Wp) bool, ignore (B, Hp, Wp) bool."""
    B = len(smp)
    cs = F(F(S) / F(Wp))
    out_img = np.stack([image(smp[i], srcs, img, S) for i in range(B)])
    n_gt = np.zeros(B, np.int64)
    box = np.zeros((B, G, 4), F)
    gi = np.full((B, G), -1, np.int64)
    gmask = np.zeros((B, G, Hp, Wp), bool)
    ign = np.zeros((B, Hp, Wp), bool)
    for i in range(B):
        sm = smp[i]
        bx, idx = targets(i, sm, insts, S, G)
        n_gt[i] = len(idx)
        box[i, :len(idx)] = bx
        gi[i, :len(idx)] = idx
        for j, k in enumerate(idx):
            c0, c1, r0, r1 = box_cells(*bx[j], cs, Hp, Wp)
            if c1 <= c0 or r1 <= r0:
                continue
            rr, cc = np.meshgrid(np.arange(r0, r1), np.arange(c0, c1), indexing="ij")
            gmask[i, j, r0:r1, c0:c1] = cell_bits(sm, insts[k], srcs[int(insts[k]["src"])], mask, S, cs, rr, cc)
        for k in range(len(insts)):  # ignore regions (src/augment.cu:190-241)
            inst = insts[k]
            if int(inst["sample"]) != i or not int(inst["ignore"]):
                continue
            m = map_box(sm, inst, S)
            if m is None:
                continue
            c0, c1, r0, r1 = box_cells(m[0], m[1], m[2], m[3], cs, Hp, Wp)
            if c1 <= c0 or r1 <= r0:
                continue
            rr, cc = np.meshgrid(np.arange(r0, r1), np.arange(c0, c1), indexing="ij")
            ign[i, r0:r1, c0:c1] |= cell_bits(sm, inst, srcs[int(inst["src"])], mask, S, cs, rr, cc)
    return dict(img=out_img, n_gt=n_gt, box=box, gt_inst=gi, mask=gmask, ignore=ign)
