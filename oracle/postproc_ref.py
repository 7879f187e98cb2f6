"""numpy restatement of the inference post-process (test infrastructure — the checker).

Decode follows the reference's DFL decode (src/loss.cu:128-147: softmax over reg_max bins, expectation,
anchor = cell + 0.5) and the exported head layout that archive/tools/ref_detect.py consumes
(xywh in pixels = Ultralytics dist2bbox(xywh=True) × stride, conf = sigmoid(cls)).
Detection follows archive/tools/ref_detect.py:37-81 for an S×S input with no letterbox padding:
  conf > conf_th → stable sort by −conf → greedy IoU NMS (strict >, union > 0 guard) → max_det;
  mask = (coef·proto > 0) ∩ box/4 ∩ image area on the 1/4 grid; optional area_min and mask-IoU dedup.
All arithmetic is float32 in the same operation order as ref_detect.py, so NMS indices are exactly
reproducible from the same decoded boxes/scores.
"""
from __future__ import annotations

import numpy as np

STRIDES = (8, 16, 32)


def _to_nhwc(t):
    a = t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)
    return a


def decode(box, cls, coef, reg_max: int = 16, strides=STRIDES, layout="nchw"):
    """box[l] (N,4·reg_max,H,W), cls[l] (N,1,H,W), coef[l] (N,32,H,W) (or NHWC with layout="nhwc").
    Returns xywh (N,A,4) px, conf (N,A), coefs (N,A,32), all float32; anchors level-major, row-major."""
    xs, confs, cfs = [], [], []
    for l, s in enumerate(strides):
        b = _to_nhwc(box[l]).astype(np.float32)
        c = _to_nhwc(cls[l]).astype(np.float32)
        m = _to_nhwc(coef[l]).astype(np.float32)
        if layout == "nchw":
            b, c, m = b.transpose(0, 2, 3, 1), c.transpose(0, 2, 3, 1), m.transpose(0, 2, 3, 1)
        N, H, W, _ = b.shape
        logits = b.reshape(N, H * W, 4, reg_max)
        mx = logits.max(-1, keepdims=True)
        e = np.exp(logits - mx, dtype=np.float32)
        d = (e * np.arange(reg_max, dtype=np.float32)).sum(-1) / e.sum(-1)  # (N, HW, 4)
        yy, xx = np.meshgrid(np.arange(H, dtype=np.float32), np.arange(W, dtype=np.float32), indexing="ij")
        ax = (xx + np.float32(0.5)).reshape(1, -1)
        ay = (yy + np.float32(0.5)).reshape(1, -1)
        x1, y1 = ax - d[..., 0], ay - d[..., 1]
        x2, y2 = ax + d[..., 2], ay + d[..., 3]
        xywh = np.stack([(x1 + x2) / np.float32(2), (y1 + y2) / np.float32(2), x2 - x1, y2 - y1], -1)
        xs.append((xywh * np.float32(s)).astype(np.float32))
        confs.append((1 / (1 + np.exp(-c.reshape(N, H * W)))).astype(np.float32))
        cfs.append(m.reshape(N, H * W, -1))
    return np.concatenate(xs, 1), np.concatenate(confs, 1), np.concatenate(cfs, 1)


def xywh_to_xyxy(xywh):
    """ref_detect.py:44-45 (float32)."""
    x = xywh
    h = np.float32(2)
    return np.stack([x[:, 0] - x[:, 2] / h, x[:, 1] - x[:, 3] / h, x[:, 0] + x[:, 2] / h, x[:, 1] + x[:, 3] / h], 1)


def nms_order(conf, conf_th: float):
    """Candidates above the threshold in stable descending-confidence order (ref_detect.py:41-42)."""
    idx = np.nonzero(conf > np.float32(conf_th))[0]
    return idx[np.argsort(-conf[idx], kind="stable")]


def greedy_nms(boxes, nms_iou: float, max_det: int):
    """Greedy NMS over boxes already in score order (ref_detect.py:46-60): returns kept positions."""
    keep = []
    thr = np.float32(nms_iou)
    zero = np.float32(0)
    for i in range(len(boxes)):
        if len(keep) >= max_det:
            break
        b = boxes[i]
        ok = True
        for k in keep:
            c = boxes[k]
            iw = max(zero, min(b[2], c[2]) - max(b[0], c[0]))
            ih = max(zero, min(b[3], c[3]) - max(b[1], c[1]))
            inter = np.float32(iw * ih)
            u = np.float32(np.float32((b[2] - b[0]) * (b[3] - b[1])) + np.float32((c[2] - c[0]) * (c[3] - c[1]))) - inter
            if u > zero and np.float32(inter / u) > thr:
                ok = False
                break
        if ok:
            keep.append(i)
    return keep


def masks_for(coefs, proto, boxes, S: int):
    """Mask logits and binary masks on the proto grid (ref_detect.py:62-71, no letterbox).
    coefs (n,32) float32, proto (32,Ph,Pw), boxes (n,4) xyxy px."""
    nm, Ph, Pw = proto.shape
    g = np.float32(Pw / S)
    logits = (coefs.astype(np.float32) @ proto.reshape(nm, -1).astype(np.float32)).reshape(-1, Ph, Pw)
    yy, xx = np.mgrid[0:Ph, 0:Pw]
    masks = np.zeros(logits.shape, bool)
    for j in range(len(boxes)):
        b = boxes[j] * g
        masks[j] = (logits[j] > 0) & (xx >= b[0]) & (xx < b[2]) & (yy >= b[1]) & (yy < b[3])
    return logits, masks


def detect_one(xywh, conf, coefs, proto, S: int, conf_th=0.25, nms_iou=0.7, max_det=300, area_min=0,
               mask_iou=1.0):
    """One image: returns dict(order=candidate anchor ids, keep=kept positions in order, anchors=kept anchor
    ids, score, box (xyxy px), logits, masks) — the full ref_detect.py pipeline for an unpadded input."""
    idx = nms_order(conf, conf_th)
    boxes = xywh_to_xyxy(xywh[idx])
    keep = greedy_nms(boxes, nms_iou, max_det)
    anchors = idx[keep]
    kb = boxes[keep] if len(keep) else np.zeros((0, 4), np.float32)
    logits, masks = masks_for(coefs[anchors], proto, kb, S)
    sel = list(range(len(keep)))
    if area_min > 0 or mask_iou < 1.0:
        sel0 = [j for j in sel if masks[j].sum() >= area_min]
        sel = []
        for j in sel0:
            m = masks[j]
            a = m.sum()
            if all((m & masks[k]).sum() / max(a + masks[k].sum() - (m & masks[k]).sum(), 1) <= mask_iou for k in sel):
                sel.append(j)
    return dict(order=idx, keep=np.array(keep, np.int64), anchors=anchors, score=conf[anchors], box=kb,
                logits=logits, masks=masks, sel=np.array(sel, np.int64))


def topk_order(conf, k: int):
    """'Forced' mode (BASELINE config 2 variant): the k highest scores, stable order, no threshold."""
    idx = np.argsort(-conf, kind="stable")
    return idx[:k]


def greedy_nms_vec(boxes, nms_iou: float, max_det: int):
    """greedy_nms with each candidate tested against all kept boxes as one float32 vector: the same
    element-wise float32 operations (each correctly rounded), so the same kept positions, in a time that
    suits thousands of candidates."""
    boxes = np.asarray(boxes, np.float32)
    thr = np.float32(nms_iou)
    zero = np.float32(0)
    kept = np.zeros((max(max_det, 1), 4), np.float32)
    area_k = np.zeros(max(max_det, 1), np.float32)
    keep = []
    for i in range(len(boxes)):
        n = len(keep)
        if n >= max_det:
            break
        b = boxes[i]
        if n:
            c = kept[:n]
            iw = np.maximum(zero, np.minimum(b[2], c[:, 2]) - np.maximum(b[0], c[:, 0]))
            ih = np.maximum(zero, np.minimum(b[3], c[:, 3]) - np.maximum(b[1], c[:, 1]))
            inter = (iw * ih).astype(np.float32)
            ab = np.float32((b[2] - b[0]) * (b[3] - b[1]))
            u = ((ab + area_k[:n]).astype(np.float32) - inter).astype(np.float32)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = (inter / np.where(u > zero, u, np.float32(1))).astype(np.float32)
            if np.any((u > zero) & (q > thr)):
                continue
        kept[n] = b
        area_k[n] = np.float32((b[2] - b[0]) * (b[3] - b[1]))
        keep.append(i)
    return keep


def stress_boxes(kind: str, n: int, seed: int):
    """Boxes for NMS stress cases: "mixed" (sizes 20-200 px over 640²), "grid" (integer corners in
    0..12, so many IoUs land exactly on simple fractions such as 1/2 and 7/10), "dense" (jittered copies of
    a few boxes: heavy suppression), "sparse" (small disjoint-ish boxes: little suppression)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if kind == "grid":
        a = rng.integers(0, 12, (n, 2))
        wh = rng.integers(1, 6, (n, 2))
        return np.concatenate([a, a + wh], 1).astype(np.float32)
    if kind == "dense":
        base = rng.random((8, 4)) * 400
        base[:, 2:] = base[:, :2] + 80 + rng.random((8, 2)) * 120
        b = base[rng.integers(0, 8, n)] + rng.normal(0, 6, (n, 4))
        return np.concatenate([np.minimum(b[:, :2], b[:, 2:]), np.maximum(b[:, :2], b[:, 2:])], 1).astype(np.float32)
    c = rng.random((n, 2)) * 640
    wh = (rng.random((n, 2)) * (180 if kind == "mixed" else 6)) + (20 if kind == "mixed" else 1)
    return np.concatenate([c - wh / 2, c + wh / 2], 1).astype(np.float32)
