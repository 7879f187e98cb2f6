"""BASELINE config 5 — 1024x1024 inference: 21,504 anchors (128² + 64² + 32²), proto 32 x 256 x 256,
up to 300 detections per image.

  * NMS at 21,504 anchors: one CTA per image holds every candidate of the image in shared memory
    (two 16-bit anchor orders + the radix-sort keys: 204,800 B of the 226 KiB plan at 21,504 anchors);
    kept anchors, scores and boxes bit-exact against the greedy loop of archive/tools/ref_detect.py:37-59
    (oracle/postproc_ref.py), with tied scores, and in the forced top-300 mode;
  * mask assembly on a 256 x 256 proto (2·300·32·65,536 = 1.26 GFLOP per image): identical to the oracle's
    float32 masks (ref_detect.py:62-71) except where |logit| < 1e-4·max|logit|;
  * the whole detect pipeline on the model's own 1024² heads.
The network itself at 1024² is checked against the reference's cuDNN build in
tests/test_reference_cudnn_gpu.py.
"""
import numpy as np
import pytest
import torch

from objectsam_b200 import postproc
from objectsam_b200.model import Model
from oracle import postproc_ref, yolo_params, yolo_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
S = 1024
A = (S // 8) ** 2 + (S // 16) ** 2 + (S // 32) ** 2


def test_anchor_count():
    assert A == 21504


@pytest.mark.parametrize("kind,thr", [("mixed", 0.7), ("grid", 0.5), ("dense", 0.45), ("sparse", 0.7)])
def test_nms_bit_exact_21504_anchors(cuda_lib, kind, thr):
    rng = np.random.Generator(np.random.PCG64(21))
    boxes = postproc_ref.stress_boxes(kind, A, 5) * np.float32(S / 640)
    conf = rng.random(A).astype(np.float32)
    conf[rng.integers(0, A, 2000)] = np.float32(0.625)  # ties resolve by anchor index
    B = 2
    det = postproc.nms(torch.from_numpy(np.stack([boxes] * B)).to(DEV),
                       torch.from_numpy(np.stack([conf, conf[::-1].copy()])).to(DEV), conf_th=0.25, iou_th=thr,
                       max_det=300)
    torch.cuda.synchronize()
    for b, c in enumerate((conf, conf[::-1].copy())):
        idx = postproc_ref.nms_order(c, 0.25)
        anchors = idx[postproc_ref.greedy_nms_vec(boxes[idx], thr, 300)]
        n = int(det["n_det"][b])
        assert n == len(anchors)
        np.testing.assert_array_equal(det["keep"][b, :n].cpu().numpy(), anchors)
        np.testing.assert_array_equal(det["score"][b, :n].cpu().numpy(), c[anchors])
        np.testing.assert_array_equal(det["box"][b, :n].cpu().numpy(), boxes[anchors])
        assert (det["keep"][b, n:] == -1).all()


def test_nms_forced_top300_21504_anchors(cuda_lib):
    rng = np.random.Generator(np.random.PCG64(22))
    conf = rng.random(A).astype(np.float32)
    conf[rng.integers(0, A, 1500)] = 0.5
    boxes = np.sort(rng.random((A, 4)).astype(np.float32) * S, axis=1)
    det = postproc.nms(torch.from_numpy(boxes)[None].to(DEV), torch.from_numpy(conf)[None].to(DEV), max_det=300,
                       forced=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(det["keep"][0].cpu().numpy(), postproc_ref.topk_order(conf, 300))
    assert int(det["n_det"][0]) == 300


def test_masks_256_proto_300_detections(cuda_lib):
    """300 detections (forced top-300) x 256² proto: the full-size mask GEMM of config 5."""
    g = torch.Generator(device="cpu").manual_seed(5)
    B, Hp = 2, S // 4
    proto = torch.randn(B, Hp, Hp, 32, generator=g).half()
    coef_all = torch.randn(B, A, 32, generator=g).half()
    conf = torch.rand(B, A, generator=g)
    c = torch.rand(B, A, 2, generator=g) * S
    wh = torch.rand(B, A, 2, generator=g) * 500 + 8
    boxes = torch.cat([c - wh / 2, c + wh / 2], -1).float()
    det = postproc.nms(boxes.to(DEV), conf.to(DEV), max_det=300, forced=True)
    n = det["n_det"].cpu()
    assert (n == 300).all()
    pad = 384
    coef_g = torch.zeros(B, pad, 32, dtype=torch.float16)
    keep = det["keep"].cpu().long()
    for b in range(B):
        coef_g[b, :300] = coef_all[b, keep[b]]
    masks = postproc.mask_assemble(coef_g.to(DEV), proto.to(DEV), det, S)
    packed = postproc.mask_assemble(coef_g.to(DEV), proto.to(DEV), det, S, packed=True)
    torch.cuda.synchronize()
    assert torch.equal(postproc.unpack_masks(packed, Hp, Hp), masks.bool())
    for b in range(B):
        kb = det["box"][b].cpu().numpy()
        logits, ref = postproc_ref.masks_for(coef_g[b, :300].float().numpy(),
                                             proto[b].permute(2, 0, 1).float().numpy(), kb, S)
        got = masks[b].cpu().numpy().astype(bool)
        near0 = np.abs(logits) < 1e-4 * np.abs(logits).max()
        assert ((got != ref) & ~near0).sum() == 0


def test_detect_pipeline_1024(cuda_lib):
    """Model forward at 1024² → GPU decode/NMS/masks; the oracle's NMS on the same decoded boxes/scores keeps
    exactly the same anchors and its masks agree on the same coefficients and 256² prototypes."""
    w = yolo_ref.calibrated_weights(4, 128)
    B = 2
    imgs = yolo_params.make_images(B, S, 78)
    m = Model(B, S)
    m.load(w)
    m.sync_weights()
    m.input().copy_(torch.from_numpy(imgs).half())
    m.forward(use_graph=True)
    det = postproc.detect(m, conf_th=0.25, iou_th=0.7, max_det=300)
    torch.cuda.synchronize()
    assert m.proto().shape == (B, 256, 256, 32)
    xyxy, conf = det["xyxy"].cpu().numpy(), det["conf"].cpu().numpy()
    assert xyxy.shape == (B, A, 4)
    coef_all = np.concatenate([m.head(2, l).float().cpu().numpy().reshape(B, -1, 32) for l in range(3)], 1)
    proto = m.proto().float().cpu().numpy().transpose(0, 3, 1, 2)
    for b in range(B):
        idx = postproc_ref.nms_order(conf[b], 0.25)
        anchors = idx[postproc_ref.greedy_nms_vec(xyxy[b][idx], 0.7, 300)]
        n = int(det["n_det"][b])
        assert n == len(anchors)
        np.testing.assert_array_equal(det["keep"][b, :n].cpu().numpy(), anchors)
        logits, ref_masks = postproc_ref.masks_for(coef_all[b][anchors], proto[b], xyxy[b][anchors], S)
        got = det["masks"][b, :n].cpu().numpy().astype(bool)
        near0 = np.abs(logits) < 1e-4 * (np.abs(logits).max() + 1e-12)
        assert ((got != ref_masks) & ~near0).sum() == 0
    m.close()
