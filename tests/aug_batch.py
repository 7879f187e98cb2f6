"""Seeded synthetic training batches for the augmentation tests: source images, mosaic plans, affine and
HSV parameters, instances with bitmaps and ignore regions, packed in the reference loader's record layouts
(objectsam_b200.augment's dtypes).  There is no dataset here (and no JPEG decoder): the sources are
pseudo-random u8 images with smooth structure, so that the bilinear and HSV steps see varied values.

Mosaic placement follows the four-quadrant rule around a random centre (xc, yc) of the 2S × 2S canvas:
tile 0 ends at the centre from the upper left, 1 from the upper right, 2 from the lower left, 3 from the
lower right, each cut to the canvas; tb is where the cut tile starts in its source.
"""
from __future__ import annotations

import numpy as np

from objectsam_b200.augment import INST_DT, SAMPLE_DT, SRC_DT, pack_meta


def make_batch(seed: int, B: int, S: int, max_inst: int = 6, p_missing: float = 0.15, p_ignore: float = 0.15,
               overlap: int = 0):
    """overlap > 0 starts tiles 1 and 3 that many pixels left of the centre, over tiles 0 and 2 (the first
    tile holding a canvas pixel wins)."""
    r = np.random.default_rng(seed)
    samples = np.zeros(B, SAMPLE_DT)
    sources, insts, imgs, masks = [], [], [], []
    img_off, mask_off = 0, 0
    for i in range(B):
        sm = samples[i]
        xc, yc = int(r.integers(S // 2, 3 * S // 2)), int(r.integers(S // 2, 3 * S // 2))
        for t in range(4):
            if r.random() < p_missing:
                sm["src"][t] = -1
                continue
            long_side = int(r.integers(S // 3, S + 1))
            asp = r.uniform(0.6, 1.0)
            w, h = (long_side, max(8, int(long_side * asp))) if r.random() < 0.5 else (max(8, int(long_side * asp)),
                                                                                       long_side)
            if t == 0:
                a = (max(xc - w, 0), max(yc - h, 0), xc, yc)
                b = (w - (a[2] - a[0]), h - (a[3] - a[1]))
            elif t == 1:
                a = (xc - overlap, max(yc - h, 0), min(xc - overlap + w, 2 * S), yc)
                b = (0, h - (a[3] - a[1]))
            elif t == 2:
                a = (max(xc - w, 0), yc, xc, min(2 * S, yc + h))
                b = (w - (a[2] - a[0]), 0)
            else:
                a = (xc - overlap, yc, min(xc - overlap + w, 2 * S), min(2 * S, yc + h))
                b = (0, 0)
            si = len(sources)
            sm["src"][t] = si
            sm["ta"][t] = a
            sm["tb"][t] = b
            # source pixels: smooth gradients + noise, all of 0..255
            yy, xx = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
            base = np.stack([(xx * 255 // max(w - 1, 1)), (yy * 255 // max(h - 1, 1)),
                             ((xx + yy) * 3) % 256], -1).astype(np.int64)
            pix = np.clip(base + r.integers(-40, 41, base.shape), 0, 255).astype(np.uint8)
            imgs.append(pix.reshape(-1))
            mw, mh = (w + 1) // 2, (h + 1) // 2
            src = np.zeros(1, SRC_DT)
            src["img_off"], src["iw"], src["ih"], src["mw"], src["mh"] = img_off, w, h, mw, mh
            sources.append(src[0])
            img_off += pix.size
            for _ in range(int(r.integers(0, max_inst + 1))):
                x1, x2 = np.sort(r.uniform(0, w, 2))
                y1, y2 = np.sort(r.uniform(0, h, 2))
                inst = np.zeros(1, INST_DT)[0]
                inst["src"], inst["sample"], inst["tile"] = si, i, t
                inst["box"] = (x1, y1, x2, y2)
                mx0, my0 = int(np.floor(x1 * mw / w)), int(np.floor(y1 * mh / h))
                mcw = max(1, min(mw, int(np.ceil(x2 * mw / w))) - mx0)
                mch = max(1, min(mh, int(np.ceil(y2 * mh / h))) - my0)
                wpr = (mcw + 31) // 32
                # an ellipse in the window, with a few flipped bits
                my_, mx_ = np.meshgrid(np.arange(mch), np.arange(wpr * 32), indexing="ij")
                cx, cy = (mcw - 1) / 2, (mch - 1) / 2
                on = ((mx_ - cx) / max(cx, 0.5)) ** 2 + ((my_ - cy) / max(cy, 0.5)) ** 2 <= 1.0
                on &= mx_ < mcw
                on ^= (r.random(on.shape) < 0.05) & (mx_ < mcw)
                words = np.packbits(on.reshape(mch, wpr, 32)[..., ::-1], axis=-1, bitorder="big").view(">u4")
                words = words.reshape(mch, wpr).astype(np.uint32)
                inst["mx0"], inst["my0"], inst["mcw"], inst["mch"], inst["wpr"] = mx0, my0, mcw, mch, wpr
                inst["mask_off"] = mask_off
                inst["ignore"] = int(r.random() < p_ignore)
                masks.append(words.reshape(-1))
                mask_off += words.size
                insts.append(inst)
        scale = r.uniform(0.5, 1.5)
        s = 0.5 * scale
        sm["s"] = s
        sm["tx"] = S / 2 - s * S + r.uniform(-0.1, 0.1) * S
        sm["ty"] = S / 2 - s * S + r.uniform(-0.1, 0.1) * S
        sm["hsv"] = 1.0 + r.uniform(-1, 1, 3) * np.array([0.015, 0.7, 0.4])
        sm["flip"] = int(r.random() < 0.5)
    # the loader lists instances sample by sample; shuffle within runs of three to exercise the filter
    insts = np.array(insts, INST_DT) if insts else np.zeros(0, INST_DT)
    if len(insts) > 1:
        insts = insts[np.argsort(r.random(len(insts)) + np.arange(len(insts)) // 3)]
    img = np.concatenate(imgs) if imgs else np.zeros(16, np.uint8)
    mask = np.concatenate(masks) if masks else np.zeros(4, np.uint32)
    srcs = np.array(sources, SRC_DT)
    meta = pack_meta(B, S, samples, srcs, insts, img.size, mask.size)
    return dict(B=B, S=S, samples=samples, sources=srcs, insts=insts, img=img, mask=mask, meta=meta)
