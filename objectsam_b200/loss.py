"""Host-side mirror of the reference's training mask loss (the mask part of SegLoss::run, src/loss.cu:393-543)
over the C ABI.

    mask_loss(coef, proto, npos, pos, agt, gt_box, gt_mask, fg, scale, imgsz, box_gain, dproto, dcoef, loss)

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
