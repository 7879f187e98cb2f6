"""Inference post-process on the GPU (decode → NMS → masks) over the C ABI.

Mirrors the reference's post-process (archive/tools/ref_detect.py:37-81) for unpadded S×S inputs:
    xyxy, conf = decode(box_heads, cls_heads, imgsz)          # DFL decode (src/loss.cu:128-147)
    det = nms(xyxy, conf, conf_th, iou_th, max_det)            # stable score order, greedy IoU NMS
    masks = mask_assemble(det["coef_g"], proto, det, imgsz)    # coef · proto > 0, cropped to the box
or all at once with detect(model).  Tensors are torch CUDA tensors (heads/proto NHWC fp16).
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib, stream_ptr


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _level_hw(ts):
    return (ctypes.c_int * 6)(*[v for t in ts for v in (t.shape[1], t.shape[2])])


def decode(box, cls, imgsz: int, reg_max: int = 16, stream=None, out=None):
    """box[l] (B,H,W,4·reg_max), cls[l] (B,H,W,1) fp16 → xyxy (B,A,4) float32 px, conf (B,A) float32.
    out=(xyxy, conf) writes into existing tensors instead of allocating."""
    B = box[0].shape[0]
    A = sum(t.shape[1] * t.shape[2] for t in box)
    if out is not None:
        xyxy, conf = out
    else:
        xyxy = torch.empty(B, A, 4, dtype=torch.float32, device=box[0].device)
        conf = torch.empty(B, A, dtype=torch.float32, device=box[0].device)
    check(lib().osam_decode(_ptrs(box), _ptrs(cls), _level_hw(box), B, imgsz, reg_max, xyxy.data_ptr(),
                            conf.data_ptr(), stream_ptr(stream)))
    return xyxy, conf


def nms(xyxy, conf, conf_th: float = 0.25, iou_th: float = 0.7, max_det: int = 300, forced: bool = False,
        coef=None, stream=None, out=None) -> dict:
    """Per image: n_det, keep (anchor ids, −1 padded), box (xyxy), score; with coef heads also coef_g, the
    kept anchors' mask coefficients laid out for mask_assemble.  out= a dict of that form from an earlier
    call with the same shapes: written in place instead of allocated."""
    B, A = conf.shape
    dev = conf.device
    pad = (max_det + 127) // 128 * 128
    if out is None:
        out = dict(n_det=torch.empty(B, dtype=torch.int32, device=dev),
                   keep=torch.empty(B, max_det, dtype=torch.int32, device=dev),
                   box=torch.empty(B, max_det, 4, dtype=torch.float32, device=dev),
                   score=torch.empty(B, max_det, dtype=torch.float32, device=dev))
    coef_p, hw, cg = None, None, None
    if coef is not None:
        if "coef_g" not in out:
            out["coef_g"] = torch.empty(B, pad, 32, dtype=torch.float16, device=dev)
        coef_p, hw, cg = _ptrs(coef), _level_hw(coef), out["coef_g"].data_ptr()
    check(lib().osam_nms(xyxy.data_ptr(), conf.data_ptr(), B, A, float(conf_th), float(iou_th), max_det,
                         int(forced), coef_p, hw, out["n_det"].data_ptr(), out["keep"].data_ptr(),
                         out["box"].data_ptr(), out["score"].data_ptr(), cg, stream_ptr(stream)))
    return out


def mask_assemble(coef_g, proto, det: dict, imgsz: int, packed: bool = False, stream=None, out=None):
    """coef_g (B, ceil128(max_det), 32) fp16, proto (B, Hp, Wp, 32) fp16 → masks (B, max_det, Hp, Wp) u8, or
    with packed=True (B, max_det, ceil(Hp·Wp/32)) int32 bit words (pixel 32·j + k = bit k of word j).
    out= an existing tensor of that shape and type to write into."""
    B, Hp, Wp, _ = proto.shape
    max_det = det["keep"].shape[1]
    if out is not None:
        masks = out
    elif packed:
        masks = torch.empty(B, max_det, (Hp * Wp + 31) // 32, dtype=torch.int32, device=proto.device)
    else:
        masks = torch.empty(B, max_det, Hp, Wp, dtype=torch.uint8, device=proto.device)
    check(lib().osam_mask_assemble(coef_g.data_ptr(), proto.data_ptr(), det["box"].data_ptr(),
                                   det["n_det"].data_ptr(), B, Hp, Wp, imgsz, max_det, int(packed),
                                   masks.data_ptr(), stream_ptr(stream)))
    return masks


def unpack_masks(packed, Hp: int, Wp: int):
    """Packed bit masks (…, words) → bool (…, Hp, Wp)."""
    w = packed.to(torch.int64) & 0xFFFFFFFF
    bits = ((w.unsqueeze(-1) >> torch.arange(32, device=w.device)) & 1).flatten(-2)
    return bits[..., : Hp * Wp].reshape(*packed.shape[:-1], Hp, Wp).bool()


def detect(model, conf_th: float = 0.25, iou_th: float = 0.7, max_det: int = 300, forced: bool = False,
           packed: bool = False, stream=None) -> dict:
    """Decode, NMS and masks on the model's current heads (after Model.forward)."""
    box = [model.head(0, l) for l in range(3)]
    cls = [model.head(1, l) for l in range(3)]
    coef = [model.head(2, l) for l in range(3)]
    xyxy, conf = decode(box, cls, model.imgsz, model.reg_max, stream)
    det = nms(xyxy, conf, conf_th, iou_th, max_det, forced, coef=coef, stream=stream)
    det["masks"] = mask_assemble(det["coef_g"], model.proto(), det, model.imgsz, packed, stream)
    det["xyxy"], det["conf"] = xyxy, conf
    return det
