"""CPU restatement of the reference's SPPF pooling chain, forward and backward (TEST INFRASTRUCTURE: only
tests/ use it; the product path never does).

  pool5_fwd   reference k_pool5 (src/misc.cu:32-46): 5×5 / stride 1 / pad 2 max over the clipped window
  sppf_bwd    reference sppf_pool_bwd (src/misc.cu:155-166) with k_unpool5 (:48-73): every output position
              sends its gradient to the FIRST maximum of its window in row-major scan order (strict >);
              slice 3's gradient goes back through pool(slice 2), slice 2's total through pool(slice 1),
              slice 1's total through pool(slice 0), and the result is added into dcat slice 0 (fp16).
Sums are fp32, each input position adding its window's contributions in row-major order of the output
positions (the order the GPU kernel uses, so the two agree bit for bit; the reference's atomics add in any
order).  Arrays are NHWC float32 holding fp16 values.
"""
from __future__ import annotations

import numpy as np

_OFFS = [(dy, dx) for dy in range(-2, 3) for dx in range(-2, 3)]  # row-major window scan


def _shift(a, dy, dx, fill):
    """b[:, h, w] = a[:, h+dy, w+dx] (fill outside)."""
    N, H, W, C = a.shape
    b = np.full_like(a, fill)
    ys, yd = (slice(dy, H), slice(0, H - dy)) if dy >= 0 else (slice(0, H + dy), slice(-dy, H))
    xs, xd = (slice(dx, W), slice(0, W - dx)) if dx >= 0 else (slice(0, W + dx), slice(-dx, W))
    b[:, yd, xd] = a[:, ys, xs]
    return b


def pool5_fwd(x):
    best = np.full(x.shape, -np.inf, np.float32)
    for dy, dx in _OFFS:
        best = np.maximum(best, _shift(x, dy, dx, -np.inf))
    return best


def _argmax_codes(x):
    best = np.full(x.shape, -np.inf, np.float32)
    code = np.full(x.shape, 255, np.int32)
    for k, (dy, dx) in enumerate(_OFFS):
        v = _shift(x, dy, dx, -np.inf)
        upd = v > best
        best = np.where(upd, v, best)
        code = np.where(upd, k, code)
    return code


def _unpool(x, g):
    """Gradient at the pool input x of gradient g at the pool output."""
    code = _argmax_codes(x)
    acc = np.zeros(x.shape, np.float32)
    # input position p receives from output o = p − (dy, dx) when code[o] = (dy, dx); increasing o order
    for k, (dy, dx) in reversed(list(enumerate(_OFFS))):
        go = _shift(g, -dy, -dx, 0.0)
        co = _shift(code, -dy, -dx, -1)
        acc = acc + np.where(co == k, go, np.float32(0)).astype(np.float32)
    return acc


def sppf_bwd(cat, dcat, c):
    """cat, dcat (N, H, W, 4c) → new dcat (slice 0 updated, fp16-rounded)."""
    s = [cat[..., k * c:(k + 1) * c].astype(np.float32) for k in range(3)]
    g = dcat[..., 3 * c:4 * c].astype(np.float32)
    for L in (2, 1, 0):
        acc = _unpool(s[L], g)
        if L > 0:
            g = (acc + dcat[..., L * c:(L + 1) * c]).astype(np.float32)
    out = dcat.astype(np.float32).copy()
    out[..., :c] = (out[..., :c] + acc).astype(np.float16).astype(np.float32)
    return out
