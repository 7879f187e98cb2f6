"""GPU post-process (decode / NMS / masks) against the oracle and the reference's ref_detect golden vectors.

Bars: NMS kept indices, scores and boxes bit-exact on the same boxes and scores (north star); decode within
1e-3 px and 1e-6 in conf (different exp/sum order); masks identical except where |logit| < 1e-4·max|logit|
(fp32 tensor-core accumulation order vs numpy's).
"""
import os

import numpy as np
import pytest
import torch

from objectsam_b200 import postproc
from objectsam_b200.model import Model
from oracle import postproc_ref, yolo_params, yolo_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "postproc_golden.npz")


def _cases():
    z = np.load(GOLDEN)
    for ci in range(int(z["n_cases"])):
        yield {k[len(f"c{ci}_"):]: z[k] for k in z.files if k.startswith(f"c{ci}_")}


def _heads(B, S, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    box, cls, coef = [], [], []
    for s in (8, 16, 32):
        h = S // s
        box.append((torch.randn(B, h, h, 64, generator=g) * 2).half().to(DEV))
        cls.append(torch.randn(B, h, h, 1, generator=g).half().to(DEV))
        coef.append(torch.randn(B, h, h, 32, generator=g).half().to(DEV))
    return box, cls, coef


def test_decode_matches_oracle(cuda_lib):
    B, S = 2, 256
    box, cls, coef = _heads(B, S, 1)
    xyxy, conf = postproc.decode(box, cls, S)
    torch.cuda.synchronize()
    xywh, conf_ref, _ = postproc_ref.decode([t.float().cpu().numpy() for t in box], [t.float().cpu().numpy() for t in cls],
                                            [t.float().cpu().numpy() for t in coef], layout="nhwc")
    for b in range(B):
        ref = postproc_ref.xywh_to_xyxy(xywh[b])
        np.testing.assert_allclose(xyxy[b].cpu().numpy(), ref, atol=1e-3, rtol=1e-5)
    np.testing.assert_allclose(conf.cpu().numpy(), conf_ref, atol=1e-6)


@pytest.mark.parametrize("ci", range(4))
def test_nms_bit_exact_on_reference_golden(cuda_lib, ci):
    case = list(_cases())[ci]
    o0 = case["o0"].astype(np.float32)
    S, cth, nth, mth, amin, mdet = case["cfg"]
    boxes = postproc_ref.xywh_to_xyxy(o0[:4].T)
    conf = o0[4]
    det = postproc.nms(torch.from_numpy(boxes)[None].to(DEV), torch.from_numpy(conf)[None].to(DEV), conf_th=cth,
                       iou_th=nth, max_det=int(mdet))
    torch.cuda.synchronize()
    idx = postproc_ref.nms_order(conf, cth)
    keep = postproc_ref.greedy_nms(boxes[idx], nth, int(mdet))
    anchors = idx[keep]
    n = int(det["n_det"][0])
    assert n == len(anchors)
    np.testing.assert_array_equal(det["keep"][0, :n].cpu().numpy(), anchors)
    np.testing.assert_array_equal(det["score"][0, :n].cpu().numpy(), conf[anchors])
    np.testing.assert_array_equal(det["box"][0, :n].cpu().numpy(), boxes[anchors])
    assert (det["keep"][0, n:] == -1).all()
    if amin == 0 and mth >= 1.0:  # no area / mask-IoU filtering: the reference's own outputs directly
        np.testing.assert_array_equal(det["score"][0, :n].cpu().numpy(), case["score"])
        np.testing.assert_array_equal(det["box"][0, :n].cpu().numpy(), case["box"])


def test_nms_forced_topk(cuda_lib):
    rng = np.random.Generator(np.random.PCG64(3))
    A = 8400
    conf = rng.random(A).astype(np.float32)
    conf[rng.integers(0, A, 500)] = 0.5  # ties resolve by anchor index
    boxes = np.sort(rng.random((A, 4)).astype(np.float32) * 640, axis=1)[:, [0, 1, 2, 3]]
    det = postproc.nms(torch.from_numpy(boxes)[None].to(DEV), torch.from_numpy(conf)[None].to(DEV), max_det=300,
                       forced=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(det["keep"][0].cpu().numpy(), postproc_ref.topk_order(conf, 300))
    assert int(det["n_det"][0]) == 300


@pytest.mark.parametrize("ci", [1, 2])
def test_masks_match_reference_golden(cuda_lib, ci):
    case = list(_cases())[ci]
    o0, o1 = case["o0"].astype(np.float32), case["o1"].astype(np.float32)
    S, cth, nth, mth, amin, mdet = case["cfg"]
    S, mdet = int(S), int(mdet)
    boxes = postproc_ref.xywh_to_xyxy(o0[:4].T)
    conf, coefs = o0[4], o0[5:].T
    det = postproc.nms(torch.from_numpy(boxes)[None].to(DEV), torch.from_numpy(conf)[None].to(DEV), conf_th=cth,
                       iou_th=nth, max_det=mdet)
    n = int(det["n_det"][0])
    pad = (mdet + 127) // 128 * 128
    coef_g = torch.zeros(1, pad, 32, dtype=torch.float16)
    coef_g[0, :n] = torch.from_numpy(coefs[det["keep"][0, :n].cpu().numpy()]).half()
    proto = torch.from_numpy(o1).permute(1, 2, 0).contiguous()[None].half().to(DEV)
    masks = postproc.mask_assemble(coef_g.to(DEV), proto, det, S)
    packed = postproc.mask_assemble(coef_g.to(DEV), proto, det, S, packed=True)
    torch.cuda.synchronize()
    assert torch.equal(postproc.unpack_masks(packed, proto.shape[1], proto.shape[2]), masks.bool())
    grid = np.unpackbits(case["grid"], axis=-1)[..., : int(case["grid_shape"][-1])].astype(bool)
    grid = grid.reshape(tuple(case["grid_shape"]))
    got = masks[0, :n].cpu().numpy().astype(bool)
    logits, _ = postproc_ref.masks_for(coefs[det["keep"][0, :n].cpu().numpy()], o1, det["box"][0, :n].cpu().numpy(), S)
    near0 = np.abs(logits) < 1e-4 * np.abs(logits).max()
    assert ((got != grid) & ~near0).sum() == 0
    assert masks[0, n:].sum().item() == 0


def test_detect_pipeline_on_model_heads(cuda_lib):
    """Model forward → GPU decode/NMS/masks; the oracle's NMS on the same decoded boxes/scores keeps exactly
    the same anchors, and the masks agree with the oracle's on the same coefficients/prototypes."""
    w = yolo_ref.calibrated_weights(4, 128)
    B, S = 2, 256
    imgs = yolo_params.make_images(B, S, 77)
    m = Model(B, S)
    m.load(w)
    m.sync_weights()
    m.input().copy_(torch.from_numpy(imgs).half())
    m.forward()
    det = postproc.detect(m, conf_th=0.25, iou_th=0.7, max_det=300)
    torch.cuda.synchronize()
    xyxy, conf = det["xyxy"].cpu().numpy(), det["conf"].cpu().numpy()
    coef_all = np.concatenate([m.head(2, l).float().cpu().numpy().reshape(B, -1, 32) for l in range(3)], 1)
    proto = m.proto().float().cpu().numpy().transpose(0, 3, 1, 2)
    for b in range(B):
        idx = postproc_ref.nms_order(conf[b], 0.25)
        keep = postproc_ref.greedy_nms(xyxy[b][idx], 0.7, 300)
        anchors = idx[keep]
        n = int(det["n_det"][b])
        assert n == len(anchors)
        np.testing.assert_array_equal(det["keep"][b, :n].cpu().numpy(), anchors)
        logits, ref_masks = postproc_ref.masks_for(coef_all[b][anchors], proto[b], xyxy[b][anchors], S)
        got = det["masks"][b, :n].cpu().numpy().astype(bool)
        near0 = np.abs(logits) < 1e-4 * (np.abs(logits).max() + 1e-12)
        assert ((got != ref_masks) & ~near0).sum() == 0


@pytest.mark.parametrize("kind,thr,max_det", [("mixed", 0.5, 300), ("mixed", 0.7, 1000), ("grid", 0.5, 300),
                                              ("grid", 0.7, 1000), ("dense", 0.45, 300), ("sparse", 0.7, 1000),
                                              ("sparse", 1 / 3, 300), ("mixed", 0.2, 1000), ("grid", 0.3, 1000)])
def test_nms_bit_exact_many_candidates(cuda_lib, kind, thr, max_det):
    """8400 anchors, ~6300 above the threshold, tied scores: several 1024-candidate rounds and several
    suppression-matrix blocks per round; kept anchors, scores and boxes identical to the greedy loop."""
    A = 8400
    rng = np.random.Generator(np.random.PCG64(11))
    boxes = postproc_ref.stress_boxes(kind, A, 12)
    conf = rng.random(A).astype(np.float32)
    conf[rng.integers(0, A, 800)] = np.float32(0.625)  # ties resolve by anchor index
    det = postproc.nms(torch.from_numpy(boxes)[None].to(DEV), torch.from_numpy(conf)[None].to(DEV), conf_th=0.25,
                       iou_th=thr, max_det=max_det)
    torch.cuda.synchronize()
    idx = postproc_ref.nms_order(conf, 0.25)
    anchors = idx[postproc_ref.greedy_nms_vec(boxes[idx], thr, max_det)]
    n = int(det["n_det"][0])
    assert n == len(anchors)
    np.testing.assert_array_equal(det["keep"][0, :n].cpu().numpy(), anchors)
    np.testing.assert_array_equal(det["score"][0, :n].cpu().numpy(), conf[anchors])
    np.testing.assert_array_equal(det["box"][0, :n].cpu().numpy(), boxes[anchors])
    assert (det["keep"][0, n:] == -1).all()


@pytest.mark.parametrize("use_graph", [False, True])
def test_detect_step_matches_separate_post_process(cuda_lib, use_graph):
    """The detect step (forward + decode + NMS + masks in one schedule, the post-process overlapping the proto
    branch) gives exactly the detections of the forward followed by the separate post-process launches."""
    w = yolo_ref.calibrated_weights(4, 128)
    B, S = 3, 192
    imgs = yolo_params.make_images(B, S, 79)
    m = Model(B, S)
    m.load(w)
    m.sync_weights()
    m.input().copy_(torch.from_numpy(imgs).half())
    m.forward()
    ref = postproc.detect(m, conf_th=0.25, iou_th=0.7, max_det=300, packed=True)
    torch.cuda.synchronize()
    ref = {k: v.clone() for k, v in ref.items()}
    m.detect_init(0.25, 0.7, 300, packed=True)
    for _ in range(2):  # the graph is recorded at the first call and replayed at the second
        m.forward_detect(use_graph=use_graph)
    torch.cuda.synchronize()
    got = m.detections()
    assert int(ref["n_det"].sum()) > 0
    for k in ("xyxy", "conf", "n_det", "keep", "box", "score", "masks"):
        if k in ("keep", "box", "score", "masks"):
            n = got["n_det"].cpu()
            for b in range(B):
                assert torch.equal(got[k][b, :n[b]].cpu(), ref[k][b, :n[b]].cpu()), f"{k} image {b}"
        else:
            assert torch.equal(got[k].cpu(), ref[k].cpu()), k
    m.close()
