"""Host-side mirror of the reference's training-batch augmentation (augment(), src/augment.cuh:19) over
the C ABI osam_augment.

The loader's batch description is the reference's (src/dataset.h:19-47): numpy structured dtypes with the
layouts of include/osam.h's osam_aug_* records.  `pack_meta` lays out the header, sample, source and
instance records as one block, as the reference's BatchBuf does (header, then B samples, then 4B sources,
then the instances), so that one host→device copy moves it.

    meta = pack_meta(B, S, samples, sources, instances, img_bytes, mask_words)   # numpy uint8
    out = augment(meta_dev, img_dev, mask_dev, B, S, G, Hp, Wp, ignore=True)     # CUDA tensors in, dict out

Outputs: img (B, S, S, 3) fp16 in 0..1, n_gt (B,) int32, box (B, G, 4) float32 xyxy, gt_inst (B, G) int32
(−1 past n_gt), mask (B, G, Hp·Wp/32) int32 bit words, ignore (B, Hp·Wp/32) int32 bit words or None.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import AugBatch, AugOut, check, lib, stream_ptr

SRC_DT = np.dtype({"names": ["img_off", "iw", "ih", "mw", "mh"],
                   "formats": ["<i8", "<i4", "<i4", "<i4", "<i4"], "offsets": [0, 8, 12, 16, 20], "itemsize": 24})
INST_DT = np.dtype({"names": ["src", "sample", "tile", "box", "mx0", "my0", "mcw", "mch", "wpr", "mask_off",
                              "ignore"],
                    "formats": ["<i4", "<i4", "<i4", ("<f4", 4), "<i4", "<i4", "<i4", "<i4", "<i4", "<i8", "<i4"],
                    "offsets": [0, 4, 8, 12, 28, 32, 36, 40, 44, 48, 56], "itemsize": 64})
SAMPLE_DT = np.dtype({"names": ["src", "ta", "tb", "s", "tx", "ty", "hsv", "flip", "inst0", "ninst"],
                      "formats": [("<i4", 4), ("<i4", (4, 4)), ("<i4", (4, 2)), "<f4", "<f4", "<f4", ("<f4", 3),
                                  "<i4", "<i4", "<i4"],
                      "offsets": [0, 16, 80, 112, 116, 120, 124, 136, 140, 144], "itemsize": 148})
HEADER_DT = np.dtype({"names": ["B", "S", "nsrc", "ninst", "img_bytes", "mask_words"],
                      "formats": ["<i4", "<i4", "<i4", "<i4", "<i8", "<i8"], "offsets": [0, 4, 8, 12, 16, 24],
                      "itemsize": 32})


def pack_meta(B: int, S: int, samples: np.ndarray, sources: np.ndarray, instances: np.ndarray, img_bytes: int,
              mask_words: int) -> np.ndarray:
    """The batch's records as one block (uint8): header, B samples, 4B source slots, then the instances."""
    assert samples.dtype == SAMPLE_DT and len(samples) == B
    assert sources.dtype == SRC_DT and len(sources) <= 4 * B
    assert instances.dtype == INST_DT
    hdr = np.zeros(1, HEADER_DT)
    hdr["B"], hdr["S"], hdr["nsrc"], hdr["ninst"] = B, S, len(sources), len(instances)
    hdr["img_bytes"], hdr["mask_words"] = img_bytes, mask_words
    src_all = np.zeros(4 * B, SRC_DT)
    src_all[:len(sources)] = sources
    return np.concatenate([hdr.view(np.uint8), samples.view(np.uint8), src_all.view(np.uint8),
                           instances.view(np.uint8)])


def meta_offsets(B: int) -> tuple:
    """Byte offsets of the samples, sources and instances in a pack_meta block."""
    o_smp = HEADER_DT.itemsize
    o_src = o_smp + B * SAMPLE_DT.itemsize
    o_inst = o_src + 4 * B * SRC_DT.itemsize
    return o_smp, o_src, o_inst


def augment(meta: torch.Tensor, img: torch.Tensor, mask: torch.Tensor, B: int, S: int, G: int, Hp: int, Wp: int,
            ignore: bool = True, out: dict | None = None, stream=None) -> dict:
    """osam_augment on a batch already on the device: meta (uint8, pack_meta's block), img (uint8 source
    pixels), mask (int32 bitmap words).  `out` (from a previous call) is reused when given."""
    dev = meta.device
    if out is None:
        out = {"img": torch.empty(B, S, S, 3, dtype=torch.half, device=dev),
               "n_gt": torch.empty(B, dtype=torch.int32, device=dev),
               "box": torch.empty(B, G, 4, dtype=torch.float32, device=dev),
               "gt_inst": torch.empty(B, G, dtype=torch.int32, device=dev),
               "mask": torch.empty(B, G, Hp * Wp // 32, dtype=torch.int32, device=dev),
               "ignore": torch.empty(B, Hp * Wp // 32, dtype=torch.int32, device=dev) if ignore else None}
    o_smp, o_src, o_inst = meta_offsets(B)
    base = meta.data_ptr()
    bt = AugBatch(base, base + o_smp, base + o_src, base + o_inst, img.data_ptr(), mask.data_ptr())
    ao = AugOut(out["img"].data_ptr(), out["n_gt"].data_ptr(), out["box"].data_ptr(), out["mask"].data_ptr(),
                out["ignore"].data_ptr() if out["ignore"] is not None else None, out["gt_inst"].data_ptr(), G, Hp, Wp)
    check(lib().osam_augment(ctypes.byref(bt), B, S, ctypes.byref(ao), stream_ptr(stream)))
    return out
