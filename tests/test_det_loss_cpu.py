"""The CPU restatement of the detection loss (oracle/det_loss_ref.py) on hand-made cases: CIoU and its
gradient (finite differences at fixed α), the DFL decode of flat logits, the top-10 ranking and its tie rule,
and the loss of an image without ground truth.  The restatement is pinned against the reference's own
SegLoss on the GPU (tests/test_det_loss_gpu.py); these cases need no GPU."""
import numpy as np

from oracle import det_loss_ref as R


def test_ciou_identical_and_disjoint():
    b = np.array([10, 20, 50, 60], np.float32)
    assert abs(R.ciou(b, b) - 1.0) < 1e-5
    far = np.array([200, 200, 240, 260], np.float32)
    assert R.ciou(b, far) < 0  # no overlap: IoU 0 minus the distance term


def test_ciou_gradient_matches_finite_differences():
    b1 = np.array([12.3, 18.1, 47.9, 66.2], np.float32)
    b2 = np.array([10.0, 20.0, 50.0, 60.0], np.float32)
    v, g = R.ciou_value_grad(b1, b2)
    assert abs(v - R.ciou(b1, b2)) < 1e-6
    c = b2.astype(np.float64)
    eps = 1e-7

    def terms(b):
        w1, h1, w2, h2 = b[2] - b[0], b[3] - b[1] + eps, c[2] - c[0], c[3] - c[1] + eps
        inter = max(min(b[2], c[2]) - max(b[0], c[0]), 0) * max(min(b[3], c[3]) - max(b[1], c[1]), 0)
        iou = inter / (w1 * h1 + w2 * h2 - inter + eps)
        cw, ch = max(b[2], c[2]) - min(b[0], c[0]), max(b[3], c[3]) - min(b[1], c[1])
        rho2 = ((c[0] + c[2] - b[0] - b[2]) ** 2 + (c[1] + c[3] - b[1] - b[3]) ** 2) / 4
        v_ = 4 / np.pi ** 2 * (np.arctan(w2 / h2) - np.arctan(w1 / h1)) ** 2
        return iou, rho2 / (cw * cw + ch * ch + eps), v_

    iou0, _, v0 = terms(b1.astype(np.float64))
    alpha = v0 / (1 - iou0 + v0 + eps)  # α is a constant in the gradient, as in the reference

    def ciou_fixed_alpha(b):
        iou, dist, v_ = terms(b)
        return iou - (dist + v_ * alpha)

    for k in range(4):
        d = np.zeros(4)
        d[k] = 1e-3
        fd = (ciou_fixed_alpha(b1.astype(np.float64) + d) - ciou_fixed_alpha(b1.astype(np.float64) - d)) / 2e-3
        assert abs(g[k] - fd) <= 2e-3 + 2e-2 * abs(fd), (k, g[k], fd)


def test_decode_of_flat_logits_is_the_middle_bin():
    S = 64
    lv, A = R.levels(S)
    box = [np.zeros((1, h, w, 64), np.float32) for h, w, _, _ in lv]
    cls = [np.zeros((1, h, w, 1), np.float32) for h, w, _, _ in lv]
    pbox, score = R.decode(box, cls, S)
    # uniform over bins 0..15: expectation 7.5 on every side; score σ(0) = 0.5
    assert np.allclose(pbox[0, 0], [0.5 - 7.5, 0.5 - 7.5, 0.5 + 7.5, 0.5 + 7.5], atol=1e-5)
    assert np.allclose(score, 0.5)


def test_topk_ranking_and_tie_rule():
    """One gt: of the in-box anchors the 10 with the highest metric are positives; equal metrics keep the
    lower anchor ids (here every predicted box equals the gt, and one anchor has a higher score)."""
    S = 128
    lv, A = R.levels(S)
    gt = np.array([[[16.0, 16.0, 80.0, 80.0]]], np.float32)
    stride = np.concatenate([np.full(h * w, s, np.float32) for h, w, s, _ in lv])
    pbox = (gt[0, 0] / stride[:, None])[None].astype(np.float32)  # every prediction exact: CIoU ≈ 1
    score = np.full((1, A), 0.25, np.float32)
    score[0, 100] = 0.9
    agt, tsc = R.assign(pbox, score, np.array([1]), gt, S)
    pos = np.nonzero(agt[0] >= 0)[0]
    assert len(pos) == 10
    inside = []
    for a in range(A):
        l = 0 if a < lv[1][3] else (1 if a < lv[2][3] else 2)
        h, w, s, off = lv[l]
        y, x = divmod(a - off, w)
        if 16 < (x + 0.5) * s < 80 and 16 < (y + 0.5) * s < 80:
            inside.append(a)
    expect = ([100] if 100 in inside else []) + [a for a in inside if a != 100]
    assert sorted(pos.tolist()) == sorted(expect[:10])
    assert tsc[0, pos].max() <= 1.0 + 1e-6


def test_no_ground_truth_is_class_loss_only():
    S = 64
    lv, A = R.levels(S)
    r = np.random.default_rng(0)
    box = [r.normal(0, 1, (2, h, w, 64)).astype(np.float32) for h, w, _, _ in lv]
    cls = [r.normal(0, 1, (2, h, w, 1)).astype(np.float32) for h, w, _, _ in lv]
    out = R.det_loss(box, cls, np.array([0, 0]), np.zeros((2, 4, 4), np.float32), S)
    assert (out["agt"] == -1).all() and out["items"][4] == 0 and out["items"][8] == 0 and out["items"][11] == 0
    for l in range(3):
        assert (out["dbox"][l] == 0).all()
        sig = 1 / (1 + np.exp(-cls[l]))
        assert np.allclose(out["dcls"][l], sig * 0.5 * 2, rtol=1e-5)  # cls_gain · B / max(Σt, 1)
    assert out["items"][10] > 0
