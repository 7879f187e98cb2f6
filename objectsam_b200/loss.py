"""Host-side mirror of the reference's training loss of the segment head (SegLoss, src/loss.cuh:53-64,
src/loss.cu) over the C ABI: its detection part, its mask part, and the whole loss.

    det_loss(box, cls, n_gt, gt_box, scale, imgsz, dbox, dcls, dcoef, ignore=None, proto_hw=None)
    mask_loss(coef, proto, npos, pos, agt, gt_box, gt_mask, fg, scale, imgsz, box_gain, dproto, dcoef, loss)
    seg_loss(box, cls, coef, proto, n_gt, gt_box, gt_mask, scale, imgsz, dbox, dcls, dcoef, dproto)  # SegLoss::run

coef: three NHWC fp16 CUDA tensors (B, h_l, w_l, 32); proto / dproto: (B, Hp, Wp, 32) fp16; npos (B,) int32;
pos, agt: (B, A) int32; gt_box (B, G, 4) float32 xyxy pixels; gt_mask (B, G, Hp·Wp/32) int32 bit words;
fg, scale: one-element float32 CUDA tensors (positive count, loss scale); loss: one-element float32 tensor
that the call adds the mask BCE sum to (the reference's items[9]).  dcoef rows are written at the positive
anchors only, as in the reference (its detection-loss pass zeroes the others).
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib, stream_ptr

_ws_cache: dict = {}


def workspace(batch: int, anchors: int, device, stream=None) -> torch.Tensor:
    """Zero-filled workspace per (device, stream); every call returns it zeroed."""
    dev = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    nbytes = int(lib().osam_mask_loss_workspace_size(batch, anchors))
    key = (dev.index, s.cuda_stream)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _ws_cache[key] = buf
    return buf


def mask_loss(coef, proto, npos, pos, agt, gt_box, gt_mask, fg, scale, imgsz: int, box_gain: float, dproto, dcoef,
              loss, ws=None, stream=None) -> None:
    B, Hp, Wp, _ = proto.shape
    hw = (ctypes.c_int * 6)(*[v for t in coef for v in (t.shape[1], t.shape[2])])
    A = sum(t.shape[1] * t.shape[2] for t in coef)
    G = gt_box.shape[1]
    for t in (npos, pos, agt, gt_mask):
        assert t.dtype == torch.int32 and t.is_contiguous()
    assert gt_box.dtype == torch.float32 and gt_box.is_contiguous()
    ws = ws if ws is not None else workspace(B, A, proto.device, stream)
    cp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in coef])
    dp = (ctypes.c_void_p * 3)(*[t.data_ptr() for t in dcoef])
    check(lib().osam_mask_loss(cp, hw, proto.data_ptr(), B, Hp, Wp, imgsz, G, npos.data_ptr(), pos.data_ptr(),
                               agt.data_ptr(), gt_box.data_ptr(), gt_mask.data_ptr(), fg.data_ptr(), scale.data_ptr(),
                               float(box_gain), dproto.data_ptr(), dp, loss.data_ptr(), ws.data_ptr(),
                               ws.numel() * ws.element_size(), stream_ptr(stream)))


BOX_GAIN, CLS_GAIN, DFL_GAIN = 7.5, 0.5, 1.5  # the reference's LossCfg defaults (src/loss.cuh:18)
_det_ws_cache: dict = {}


def det_workspace(batch: int, anchors: int, max_gt: int, device, stream=None) -> torch.Tensor:
    dev = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    nbytes = int(lib().osam_det_loss_workspace_size(batch, anchors, max_gt))
    key = (dev.index, s.cuda_stream)
    buf = _det_ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        _det_ws_cache[key] = buf
    return buf


def det_loss(box, cls, n_gt, gt_box, scale, imgsz: int, dbox, dcls, dcoef, ignore=None, proto_hw=None,
             gains=(BOX_GAIN, CLS_GAIN, DFL_GAIN), ws=None, stream=None) -> dict:
    """The detection part of SegLoss::run (src/loss.cu:123-390): returns dict(agt, tsc, npos, pos, items) as
    CUDA tensors (items: the reference's 16-float layout).  box / cls / dbox / dcls / dcoef: three NHWC fp16
    CUDA tensors each; n_gt (B,) int32; gt_box (B, G, 4) float32 xyxy pixels; scale: one-element float32."""
    B = box[0].shape[0]
    hw = (ctypes.c_int * 6)(*[v for t in box for v in (t.shape[1], t.shape[2])])
    A = sum(t.shape[1] * t.shape[2] for t in box)
    G = gt_box.shape[1]
    dev = box[0].device
    assert n_gt.dtype == torch.int32 and gt_box.dtype == torch.float32 and gt_box.is_contiguous()
    out = dict(agt=torch.empty(B, A, dtype=torch.int32, device=dev), tsc=torch.empty(B, A, device=dev),
               npos=torch.empty(B, dtype=torch.int32, device=dev), pos=torch.zeros(B, A, dtype=torch.int32, device=dev),
               items=torch.zeros(16, device=dev))
    Hp, Wp = proto_hw if proto_hw is not None else (imgsz // 4, imgsz // 4)
    ws = ws if ws is not None else det_workspace(B, A, G, dev, stream)
    vp = lambda ts: (ctypes.c_void_p * 3)(*[t.data_ptr() for t in ts])  # noqa: E731
    check(lib().osam_det_loss(vp(box), vp(cls), hw, B, imgsz, box[0].shape[3] // 4, n_gt.data_ptr(),
                              gt_box.data_ptr(), G, None if ignore is None else ignore.data_ptr(), Hp, Wp,
                              scale.data_ptr(), float(gains[0]), float(gains[1]), float(gains[2]), vp(dbox), vp(dcls),
                              vp(dcoef), out["agt"].data_ptr(), out["tsc"].data_ptr(), out["npos"].data_ptr(),
                              out["pos"].data_ptr(), out["items"].data_ptr(), ws.data_ptr(),
                              ws.numel() * ws.element_size(), stream_ptr(stream)))
    return out


def seg_loss(box, cls, coef, proto, n_gt, gt_box, gt_mask, scale, imgsz: int, dbox, dcls, dcoef, dproto,
             ignore=None, gains=(BOX_GAIN, CLS_GAIN, DFL_GAIN), stream=None) -> dict:
    """SegLoss::run (src/loss.cu:590-621): the detection loss, then the mask loss on its positives (fg =
    items[4], the sum into items[9]), then items[0..3] = [box, seg, cls, dfl]; every gradient head written."""
    out = det_loss(box, cls, n_gt, gt_box, scale, imgsz, dbox, dcls, dcoef, ignore=ignore,
                   proto_hw=tuple(proto.shape[1:3]), gains=gains, stream=stream)
    items = out["items"]
    mask_loss(coef, proto, out["npos"], out["pos"], out["agt"], gt_box, gt_mask, items[4:5], scale, imgsz, gains[0],
              dproto, dcoef, items[9:10], stream=stream)
    check(lib().osam_seg_loss_items(items.data_ptr(), float(gains[0]), float(gains[1]), float(gains[2]),
                                    stream_ptr(stream)))
    return out
