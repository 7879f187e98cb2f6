"""CPU restatement of the reference's training-mode BatchNorm + SiLU passes and bias passes (TEST
INFRASTRUCTURE: only tests/, smoke() and bench.py's CPU legs use it; the product path never does).

Follows, step for step in numpy:
  bn_forward_stats  reference src/bn.cu:112-202 (MODE 0) and :311-322 — shifted sums Σ(z−K), Σ(z−K)² with
                    K = running mean, mean = K + E[z−K], biased var (clamped at 0) for normalising, unbiased
                    var·M/(M−1) for the running estimate, momentum update only when momentum > 0
  bn_eval_scale     src/bn.cu:277-284
  bn_forward_apply  src/bn.cu:204-238 — a = silu(scale·z + shift), residual added after the activation,
                    each destination gets channels [c0, c1) at choff, up = 2 writes the 2×2 block
  bn_backward       src/bn.cu:46-66 (gradient gather), :112-202 (MODE 1), :240-270 — g = dA·σ(y)(1 + y(1−σ(y))),
                    dβ = Σg, dγ = Σg·x̂, dz = scale·(g − Σg/M − x̂·Σg·x̂/M), residual gradient = dA
  chan_sum          src/misc.cu:103-113, :168-172
  add_bias          src/misc.cu:116-134
Sums are fp64 here (the reference: fp32 per thread/CTA, fp64 across CTAs); elementwise math is fp32.
Pinned against torch autograd of batch_norm + SiLU in fp64 (tests/test_oracle_cpu.py) and against the
reference's own kernels built from its sources (oracle/ref_bn_harness.cpp, tests/test_bn_gpu.py).
Arrays are NHWC float32 holding fp16 values: z (N, H, W, C).
"""
from __future__ import annotations

import numpy as np


def _f32(x):
    return np.asarray(x, dtype=np.float32)


def _fp16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def bn_forward_stats(z, gamma, beta, run_mean, run_var, momentum, eps):
    """Returns dict mean, istd, scale, shift, run_mean, run_var (all float32 (C,))."""
    C = z.shape[-1]
    zz = _f32(z).reshape(-1, C).astype(np.float64)
    M = zz.shape[0]
    K = _f32(run_mean)
    d = zz - K.astype(np.float64)
    sx, sy = d.sum(0), (d * d).sum(0)
    dm = (sx / M).astype(np.float32)
    var = (sy / M - dm.astype(np.float64) ** 2).astype(np.float32)
    var = np.maximum(var, np.float32(0))
    mean = (K + dm).astype(np.float32)
    istd = (np.float32(1) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    scale = (_f32(gamma) * istd).astype(np.float32)
    shift = (_f32(beta) - mean * scale).astype(np.float32)
    rm, rv = _f32(run_mean).copy(), _f32(run_var).copy()
    if momentum > 0:
        m = np.float32(momentum)
        rm = ((np.float32(1) - m) * K + m * mean).astype(np.float32)
        rv = ((np.float32(1) - m) * rv + m * (var.astype(np.float64) * M / (M - 1)).astype(np.float32)).astype(np.float32)
    return {"mean": mean, "istd": istd, "scale": scale, "shift": shift, "run_mean": rm, "run_var": rv}


def bn_eval_scale(gamma, beta, run_mean, run_var, eps):
    sc = (_f32(gamma) / np.sqrt(_f32(run_var) + np.float32(eps))).astype(np.float32)
    return sc, (_f32(beta) - _f32(run_mean) * sc).astype(np.float32)


def _sigmoid(y):
    return (1.0 / (1.0 + np.exp(-y.astype(np.float64)))).astype(np.float32)


def bn_forward_apply(z, scale, shift, res, dests, act=True):
    """dests: list of (buf (N, H·up, W·up, ctot) float32 array, choff, c0, c1, up); written in place with
    fp16-rounded values.  Returns a, the fp32 activation before rounding."""
    y = _f32(z) * _f32(scale) + _f32(shift)
    a = y * _sigmoid(y) if act else y
    if res is not None:
        a = a + _f32(res)
    C = z.shape[-1]
    for buf, choff, c0, c1, up in dests:
        c1 = c1 or C
        v = _fp16(a[..., c0:c1])
        if up == 2:
            v = v.repeat(2, axis=1).repeat(2, axis=2)
        buf[..., choff:choff + c1 - c0] = v
    return a


def gather_grad(grad_dests, shape):
    """dA (N, H, W, C): Σ over destinations of their gradient slices, 2×2 block sums for up = 2."""
    N, H, W, C = shape
    dA = np.zeros(shape, np.float32)
    for g, choff, c0, c1, up in grad_dests:
        c1 = c1 or C
        s = _f32(g)[..., choff:choff + c1 - c0]
        if up == 2:
            s = s.reshape(N, H, 2, W, 2, c1 - c0)
            s = ((s[:, :, 0, :, 0] + s[:, :, 0, :, 1]) + s[:, :, 1, :, 0]) + s[:, :, 1, :, 1]
        dA[..., c0:c1] += s
    return dA


def bn_backward(z, mean, istd, scale, shift, grad_dests, act, gw_gamma=None, gw_beta=None, accum=False,
                res_grad=None, res_accum=False):
    """Returns dict dz (fp16-rounded), gw_gamma, gw_beta, res_grad (fp16-rounded or None), sums."""
    z = _f32(z)
    C = z.shape[-1]
    dA = gather_grad(grad_dests, z.shape)
    g = dA
    if act:
        y = z * _f32(scale) + _f32(shift)
        s = _sigmoid(y)
        g = dA * (s * (np.float32(1) + y * (np.float32(1) - s)))
    xh = (z - _f32(mean)) * _f32(istd)
    M = z.size // C
    sg = g.reshape(-1, C).astype(np.float64).sum(0)
    sgx = (g * xh).reshape(-1, C).astype(np.float64).sum(0)
    m1, m2 = (sg / M).astype(np.float32), (sgx / M).astype(np.float32)
    dz = _fp16(_f32(scale) * (g - m1 - xh * m2))
    gb = sg.astype(np.float32)
    gg = sgx.astype(np.float32)
    if accum:
        gb = (_f32(gw_beta) + gb).astype(np.float32)
        gg = (_f32(gw_gamma) + gg).astype(np.float32)
    rg = None
    if res_grad is not None or res_accum:
        rg = _fp16(_f32(res_grad) + dA) if res_accum else _fp16(dA)
    return {"dz": dz, "gw_gamma": gg, "gw_beta": gb, "res_grad": rg, "sums": np.concatenate([m1, m2])}


def chan_sum(x, out=None, accum=False):
    C = x.shape[-1]
    s = _f32(x).reshape(-1, C).astype(np.float64).sum(0).astype(np.float32)
    return (_f32(out) + s).astype(np.float32) if accum else s


def add_bias(y, bias):
    return _fp16(_f32(y) + _f32(bias))
