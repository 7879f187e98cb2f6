"""CPU restatement of the detection part of the segment head's training loss — test infrastructure (a checker
for the CUDA path), never the product path.

Follows the reference's SegLoss::run before its mask part (src/loss.cu:123-390, :590-612; Ultralytics 8.4
v8SegmentationLoss with one class, reg_max 16, top-10 task-aligned assignment).  float32 numpy arithmetic in
the reference's order of operations; small sizes only (loops over images and ground-truth boxes).  Pinned on
the GPU against the reference's own SegLoss (tests/test_det_loss_gpu.py); the CPU tests check it against
hand-made cases (tests/test_det_loss_cpu.py).
"""
from __future__ import annotations

import numpy as np

F = np.float32
CIOU_EPS = F(1e-7)   # bbox_iou eps (src/loss.cu:7)
TAL_EPS = F(1e-9)    # assigner eps (src/loss.cu:8)
K4 = F(0.40528473456935108)  # 4/π²
TOPK = 10


def levels(S: int):
    """(h, w, stride, first anchor) of the three head levels (src/loss.cu:9-20, :568-578)."""
    out, off = [], 0
    for s in (8, 16, 32):
        out.append((S // s, S // s, s, off))
        off += (S // s) ** 2
    return out, off


def decode(box, cls, S):
    """DFL expectation and score per anchor (src/loss.cu:128-147): box heads (B, h, w, 64), cls (B, h, w, 1)
    → pbox (B, A, 4) xyxy grid units, score (B, A)."""
    lv, A = levels(S)
    B = box[0].shape[0]
    pbox = np.zeros((B, A, 4), F)
    score = np.zeros((B, A), F)
    for l, (h, w, s, off) in enumerate(lv):
        p = box[l].astype(F).reshape(B, h * w, 4, 16)
        m = p.max(-1, keepdims=True)
        t = np.exp(p - m).astype(F)
        d = (t * np.arange(16, dtype=F)).sum(-1, dtype=F) / t.sum(-1, dtype=F)
        yy, xx = np.divmod(np.arange(h * w), w)
        ax, ay = (xx + F(0.5)).astype(F), (yy + F(0.5)).astype(F)
        pbox[:, off:off + h * w] = np.stack([ax - d[..., 0], ay - d[..., 1], ax + d[..., 2], ay + d[..., 3]], -1)
        score[:, off:off + h * w] = (F(1) / (F(1) + np.exp(-cls[l].astype(F).reshape(B, h * w)))).astype(F)
    return pbox, score


def ciou(b1, b2):
    """Ultralytics bbox_iou(CIoU=True) of xyxy boxes (src/loss.cu:57-70), float32, broadcasting."""
    b1, b2 = np.asarray(b1, F), np.asarray(b2, F)
    w1, h1 = b1[..., 2] - b1[..., 0], b1[..., 3] - b1[..., 1] + CIOU_EPS
    w2, h2 = b2[..., 2] - b2[..., 0], b2[..., 3] - b2[..., 1] + CIOU_EPS
    iw = np.maximum(np.minimum(b1[..., 2], b2[..., 2]) - np.maximum(b1[..., 0], b2[..., 0]), F(0))
    ih = np.maximum(np.minimum(b1[..., 3], b2[..., 3]) - np.maximum(b1[..., 1], b2[..., 1]), F(0))
    inter = iw * ih
    iou = inter / (w1 * h1 + w2 * h2 - inter + CIOU_EPS)
    cw = np.maximum(b1[..., 2], b2[..., 2]) - np.minimum(b1[..., 0], b2[..., 0])
    ch = np.maximum(b1[..., 3], b2[..., 3]) - np.minimum(b1[..., 1], b2[..., 1])
    c2 = cw * cw + ch * ch + CIOU_EPS
    sx = b2[..., 0] + b2[..., 2] - b1[..., 0] - b1[..., 2]
    sy = b2[..., 1] + b2[..., 3] - b1[..., 1] - b1[..., 3]
    rho2 = (sx * sx + sy * sy) * F(0.25)
    dv = np.arctan(w2 / h2) - np.arctan(w1 / h1)
    v = K4 * dv * dv
    alpha = v / (F(1) - iou + v + CIOU_EPS)
    return (iou - (rho2 / c2 + v * alpha)).astype(F)


def ciou_value_grad(b1, b2):
    """CIoU and d CIoU / d b1 with α constant (src/loss.cu:73-121), float32 scalars."""
    b1, b2 = np.asarray(b1, F), np.asarray(b2, F)
    w1, h1 = b1[2] - b1[0], b1[3] - b1[1] + CIOU_EPS
    w2, h2 = b2[2] - b2[0], b2[3] - b2[1] + CIOU_EPS
    iw0 = min(b1[2], b2[2]) - max(b1[0], b2[0])
    ih0 = min(b1[3], b2[3]) - max(b1[1], b2[1])
    iw, ih = max(iw0, F(0)), max(ih0, F(0))
    inter = iw * ih
    uni = w1 * h1 + w2 * h2 - inter + CIOU_EPS
    iou = inter / uni
    cw = max(b1[2], b2[2]) - min(b1[0], b2[0])
    ch = max(b1[3], b2[3]) - min(b1[1], b2[1])
    c2 = cw * cw + ch * ch + CIOU_EPS
    sx = b2[0] + b2[2] - b1[0] - b1[2]
    sy = b2[1] + b2[3] - b1[1] - b1[3]
    rho2 = (sx * sx + sy * sy) * F(0.25)
    r1 = w1 / h1
    dv = np.arctan(w2 / h2) - np.arctan(r1)
    v = K4 * dv * dv
    alpha = v / (F(1) - iou + v + CIOU_EPS)
    out = iou - (rho2 / c2 + v * alpha)
    dx1 = dy1 = dx2 = dy2 = dw1 = dh1 = F(0)
    dinter, da1 = (uni + inter) / (uni * uni), -inter / (uni * uni)
    dw1 += da1 * h1
    dh1 += da1 * w1
    diw = dinter * ih if iw0 > 0 else F(0)
    dih = dinter * iw if ih0 > 0 else F(0)
    if b1[2] < b2[2]:
        dx2 += diw
    if b1[0] > b2[0]:
        dx1 -= diw
    if b1[3] < b2[3]:
        dy2 += dih
    if b1[1] > b2[1]:
        dy1 -= dih
    drho2, dc2 = -F(1) / c2, rho2 / (c2 * c2)
    dx1 += drho2 * (-sx * F(0.5))
    dx2 += drho2 * (-sx * F(0.5))
    dy1 += drho2 * (-sy * F(0.5))
    dy2 += drho2 * (-sy * F(0.5))
    dcw, dch = dc2 * F(2) * cw, dc2 * F(2) * ch
    if b1[2] > b2[2]:
        dx2 += dcw
    if b1[0] < b2[0]:
        dx1 -= dcw
    if b1[3] > b2[3]:
        dy2 += dch
    if b1[1] < b2[1]:
        dy1 -= dch
    dr1 = -alpha * K4 * F(2) * dv * (-F(1) / (F(1) + r1 * r1))
    dw1 += dr1 / h1
    dh1 += dr1 * (-w1 / (h1 * h1))
    dx2 += dw1
    dx1 -= dw1
    dy2 += dh1
    dy1 -= dh1
    return F(out), np.array([dx1, dy1, dx2, dy2], F)


def enlarged(g):
    """select_candidates_in_gts' widening of sides < 16 px (src/loss.cu:149-155)."""
    cx, cy = (g[0] + g[2]) * F(0.5), (g[1] + g[3]) * F(0.5)
    w, h = max(g[2] - g[0], F(16)), max(g[3] - g[1], F(16))
    return np.array([cx - w * F(0.5), cy - h * F(0.5), cx + w * F(0.5), cy + h * F(0.5)], F)


def centre_in(e, px, py):
    return (px - e[0] > TAL_EPS) & (py - e[1] > TAL_EPS) & (e[2] - px > TAL_EPS) & (e[3] - py > TAL_EPS)


def assign(pbox, score, n_gt, gt_box, S):
    """Top-10 per gt, resolution per anchor, target scores (src/loss.cu:160-278) → agt (B, A; −1 negative),
    tsc (B, A)."""
    lv, A = levels(S)
    B, G = gt_box.shape[:2]
    centres = np.concatenate([np.stack(np.meshgrid((np.arange(w) + 0.5) * s, (np.arange(h) + 0.5) * s), -1)
                              .reshape(-1, 2) for h, w, s, _ in lv]).astype(F)  # (A, 2) pixel x, y
    stride = np.concatenate([np.full(h * w, s, F) for h, w, s, _ in lv])
    agt = np.full((B, A), -1, np.int32)
    tsc = np.zeros((B, A), F)
    for b in range(B):
        pp = pbox[b] * stride[:, None]
        cnt = np.zeros(A, np.int32)
        who = np.zeros(A, np.int32)
        for j in range(int(n_gt[b])):
            g = gt_box[b, j].astype(F)
            cand = np.nonzero(centre_in(enlarged(g), centres[:, 0], centres[:, 1]))[0]
            ov = np.maximum(ciou(g[None], pp[cand]), F(0))
            o2 = ov * ov
            m = np.sqrt(score[b, cand]) * o2 * o2 * o2
            order = np.lexsort((cand, -m))[:TOPK]  # metric descending, then the lower anchor
            cnt[cand[order]] += 1
            who[cand[order]] = j
        galign = np.zeros(G, F)
        govl = np.zeros(G, F)
        amet = np.zeros(A, F)
        for a in np.nonzero(cnt)[0]:
            j = who[a]
            if cnt[a] > 1:  # the most-overlapping gt (first maximum); outside its widened box the overlap is 0
                best = F(-1)
                for k in range(int(n_gt[b])):
                    g = gt_box[b, k].astype(F)
                    ov = max(ciou(g, pp[a]), F(0)) if centre_in(enlarged(g), *centres[a]) else F(0)
                    if ov > best:
                        best, j = ov, k
            g = gt_box[b, j].astype(F)
            ov, m = F(0), F(0)
            if centre_in(enlarged(g), *centres[a]):
                ov = max(ciou(g, pp[a]), F(0))
                m = np.sqrt(score[b, a]) * (ov * ov) * (ov * ov) * (ov * ov)
            agt[b, a] = j
            amet[a] = m
            galign[j] = max(galign[j], m)
            govl[j] = max(govl[j], ov)
        for a in np.nonzero(agt[b] >= 0)[0]:
            j = agt[b, a]
            tsc[b, a] = amet[a] * govl[j] / (galign[j] + TAL_EPS)
    return agt, tsc


def bce(x, y):
    return np.maximum(x, F(0)) - x * y + np.log1p(np.exp(-np.abs(x)))


def det_loss(box, cls, n_gt, gt_box, S, scale=1.0, gains=(7.5, 0.5, 1.5)):
    """Losses and head gradients (src/loss.cu:290-390): returns dict(agt, tsc, items (16), dbox [l], dcls [l])
    in float32; items[4] positives, [5] target-score sum, [8] Σ(1−CIoU)·t, [10] Σ BCE, [11] Σ DFL·t."""
    lv, A = levels(S)
    B = box[0].shape[0]
    pbox, score = decode(box, cls, S)
    agt, tsc = assign(pbox, score, n_gt, gt_box, S)
    items = np.zeros(16, np.float64)
    items[4] = float((agt >= 0).sum())
    items[5] = float(tsc.sum(dtype=np.float64))
    sc = F(B / max(items[5], 1.0) * scale)
    bg, cg, dg = (F(v) for v in gains)
    dbox = [np.zeros_like(x, dtype=F) for x in box]
    dcls = [np.zeros_like(x, dtype=F) for x in cls]
    for l, (h, w, s, off) in enumerate(lv):
        x = cls[l].astype(F).reshape(B, h * w)
        t = tsc[:, off:off + h * w]
        items[10] += float(bce(x, t).sum(dtype=np.float64))
        dcls[l][...] = ((F(1) / (F(1) + np.exp(-x)) - t) * cg * sc).reshape(dcls[l].shape)
        for b in range(B):
            for r in np.nonzero(agt[b, off:off + h * w] >= 0)[0]:
                j, tt = agt[b, off + r], tsc[b, off + r]
                yy, xx = divmod(int(r), w)
                p = box[l][b, yy, xx].astype(F).reshape(4, 16)
                pr = np.exp(p - p.max(-1, keepdims=True)).astype(F)
                pr = (pr / pr.sum(-1, keepdims=True)).astype(F)
                dist = (pr * np.arange(16, dtype=F)).sum(-1).astype(F)
                ax, ay = F(xx + 0.5), F(yy + 0.5)
                pb = np.array([ax - dist[0], ay - dist[1], ax + dist[2], ay + dist[3]], F)
                tb = (gt_box[b, j] / F(s)).astype(F)
                ci, gb = ciou_value_grad(pb, tb)
                items[8] += float((F(1) - ci) * tt)
                gi = -tt * bg * sc
                dd = np.array([-gb[0] * gi, -gb[1] * gi, gb[2] * gi, gb[3] * gi], F)
                tl = np.array([ax - tb[0], ay - tb[1], tb[2] - ax, tb[3] - ay], F)
                gd = tt * F(0.25) * dg * sc
                g = np.zeros((4, 16), F)
                for side in range(4):
                    tv = min(max(tl[side], F(0)), F(16 - 1 - 0.01))
                    il = int(tv)
                    ir = il + 1
                    wl = F(ir) - tv
                    wr = F(1) - wl
                    items[11] += float(-(np.log(pr[side, il]) * wl + np.log(pr[side, ir]) * wr) * F(0.25) * tt)
                    onehot = np.zeros(16, F)
                    onehot[il] += wl
                    onehot[ir] += wr
                    g[side] = dd[side] * pr[side] * (np.arange(16, dtype=F) - dist[side]) + gd * (pr[side] - onehot)
                dbox[l][b, yy, xx] = g.reshape(64)
    return dict(agt=agt, tsc=tsc, items=items, dbox=dbox, dcls=dcls)
