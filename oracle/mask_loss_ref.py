"""CPU restatement of the reference's training mask loss (TEST INFRASTRUCTURE: only tests/ use it; the
product path never does).

Follows the mask part of SegLoss::run in the reference (src/loss.cu:393-543):
  crop_of (:409-415)   box / imgsz → normalised; area = (nx2−nx1)(ny2−ny1); crop on the proto grid
                       x1 = nx1·Wp … ; pixel (px, py) is inside when px ≥ x1, px < x2, py ≥ y1, py < y2,
                       i.e. the integer ranges [ceil(x1), ceil(x2)) ∩ [0, Wp) (k_mask_coef, :519-522)
  k_mask_tile (:417-491)  z = coef·proto, y = gt mask bit, loss += bce(z, y)/(Hp·Wp·area),
                       g = (σ(z) − y)/(Hp·Wp·area)·box_gain·B/max(fg, 1)·scale, dproto += g·coef
  k_mask_coef (:494-543)  dcoef = Σ_crop g·proto
Sums and products here are fp64; the per-positive constants are fp32 as in the reference.  Pinned against
the reference's own loss kernels built from its sources (oracle/ref_bn_harness.cpp op 5, tests/test_mask_loss_gpu.py).
"""
from __future__ import annotations

import numpy as np


def unpack_bits(words, n):
    """int32 words [..., n/32] → bool [..., n]; pixel 32·w + k is bit k of word w."""
    u = np.ascontiguousarray(words).view(np.uint32)
    bits = (u[..., :, None] >> np.arange(32, dtype=np.uint32)) & 1
    return bits.reshape(*u.shape[:-1], -1)[..., :n].astype(bool)


def anchor_of(level_hw, a):
    off = 0
    for l in range(3):
        h, w = level_hw[l]
        if a < off + h * w:
            r = a - off
            return l, r // w, r % w
        off += h * w
    raise ValueError(a)


def mask_loss(coef, proto, npos, pos, agt, gt_box, gt_mask, fg, scale, imgsz, box_gain):
    """coef: list of 3 arrays (B, h, w, 32); proto (B, Hp, Wp, 32); npos (B,); pos, agt (B, A); gt_box (B, G, 4);
    gt_mask (B, G, Hp·Wp/32) int32.  Returns dproto (B, Hp, Wp, 32) f64, dcoef {(b, anchor): (32,) f64}, loss."""
    B, Hp, Wp, _ = proto.shape
    level_hw = [(c.shape[1], c.shape[2]) for c in coef]
    bits = unpack_bits(gt_mask, Hp * Wp).reshape(B, gt_box.shape[1], Hp, Wp)
    f32 = np.float32
    gk = f32(box_gain) * f32(B) / max(f32(fg), f32(1)) * f32(scale)
    hw = f32(Hp) * f32(Wp)
    dproto = np.zeros(proto.shape, np.float64)
    dcoef, loss = {}, 0.0
    for b in range(B):
        for i in range(int(npos[b])):
            a = int(pos[b, i])
            j = int(agt[b, a])
            s = f32(imgsz)
            nx1, ny1, nx2, ny2 = (f32(v) / s for v in gt_box[b, j])
            area = (nx2 - nx1) * (ny2 - ny1)
            x1, x2, y1, y2 = nx1 * f32(Wp), nx2 * f32(Wp), ny1 * f32(Hp), ny2 * f32(Hp)
            inv = f32(1) / (hw * area)
            c0, c1 = max(0, int(np.ceil(x1))), min(Wp, int(np.ceil(x2)))
            r0, r1 = max(0, int(np.ceil(y1))), min(Hp, int(np.ceil(y2)))
            l, h, w = anchor_of(level_hw, a)
            cf = coef[l][b, h, w].astype(np.float64)
            if c1 <= c0 or r1 <= r0:
                dcoef[(b, a)] = np.zeros(32)
                continue
            P = proto[b, r0:r1, c0:c1].astype(np.float64)
            z = P @ cf
            y = bits[b, j, r0:r1, c0:c1].astype(np.float64)
            loss += float((np.maximum(z, 0) - z * y + np.log1p(np.exp(-np.abs(z)))).sum()) * float(inv)
            g = (1 / (1 + np.exp(-z)) - y) * float(inv) * float(gk)
            dproto[b, r0:r1, c0:c1] += g[..., None] * cf
            dcoef[(b, a)] = (g[..., None] * P).sum((0, 1))
    return dproto, dcoef, loss
