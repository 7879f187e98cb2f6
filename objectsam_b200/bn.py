"""Host-side mirror of the reference's training-mode BatchNorm + SiLU passes (src/bn.cuh:23-50) and of the
head-conv bias passes (src/misc.cuh:13-17), over the C ABI.

Same function names and argument meaning as the reference:
    bn_forward_stats(z, gamma, beta, run_mean, run_var, momentum, eps, mean, istd, scale, shift)
    bn_eval_scale(gamma, beta, run_mean, run_var, eps, scale, shift)
    bn_forward_apply(z, scale, shift, res, dests, act)
    bn_backward(z, mean, istd, scale, shift, grad_dests, act, dz, gw_gamma, gw_beta, accum, res_grad, res_accum)
    chan_sum(x, out, accum)
    add_bias(y, bias)
z / res / dz / gradients are NHWC fp16 torch CUDA tensors (N, H, W, C); per-channel vectors are fp32 (C,).
Destinations are DestSpec (tensor, choff, c0, c1, up) exactly like the conv epilogue's; for bn_backward each
DestSpec's tensor is the GRADIENT of that forward destination.  The fp64 accumulators the reference keeps in
a global buffer (bn_init) live in a per-device, per-stream zeroed workspace that every call returns zeroed.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from ._lib import MAX_DEST, Dest, check, lib, stream_ptr
from .conv import DestSpec

__all__ = ["bn_forward_stats", "bn_eval_scale", "bn_forward_apply", "bn_backward", "chan_sum", "add_bias",
           "DestSpec", "workspace"]

_ws_cache: dict = {}


def workspace(C: int, device, stream=None, kind: str = "bn") -> torch.Tensor:
    """The zero-filled accumulator workspace for channel count C on `device`, one per (device, stream): calls
    in stream order may share it; every call leaves it zeroed (the reference's bn_init buffers)."""
    dev = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    nbytes = int(lib().osam_bn_workspace_size(C) if kind == "bn" else lib().osam_chan_sum_workspace_size(C))
    key = (dev.index, s.cuda_stream)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256 * 1024), dtype=torch.uint8, device=dev)
        _ws_cache[key] = buf
    return buf


def _nhwc(t) -> tuple:
    assert t.dtype == torch.float16 and t.is_cuda and t.is_contiguous() and t.dim() == 4, \
        "NHWC fp16 contiguous CUDA tensor expected"
    return tuple(t.shape)


def _dests(dests: Sequence[DestSpec], C: int):
    if not 1 <= len(dests) <= MAX_DEST:
        raise ValueError(f"1..{MAX_DEST} destinations")
    arr = (Dest * MAX_DEST)()
    for i, d in enumerate(dests):
        arr[i] = Dest(d.t.data_ptr(), d.t.shape[-1], d.choff, d.c0, d.c1 or C, d.up)
    return arr


def _p(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


def bn_eval_scale(gamma, beta, run_mean, run_var, eps, scale, shift, stream=None) -> None:
    """scale = γ/√(var+eps), shift = β − μ·scale (reference bn_eval_scale, src/bn.cu:306-309)."""
    check(lib().osam_bn_eval_scale(gamma.numel(), gamma.data_ptr(), beta.data_ptr(), run_mean.data_ptr(),
                                   run_var.data_ptr(), float(eps), scale.data_ptr(), shift.data_ptr(),
                                   stream_ptr(stream)))


def bn_forward_stats(z, gamma, beta, run_mean, run_var, momentum, eps, mean, istd, scale, shift, ws=None,
                     stream=None) -> None:
    """Batch statistics of z and the running-statistics update (reference bn_forward_stats, src/bn.cu:311-322)."""
    N, H, W, C = _nhwc(z)
    ws = ws if ws is not None else workspace(C, z.device, stream)
    check(lib().osam_bn_forward_stats(z.data_ptr(), N, H, W, C, gamma.data_ptr(), beta.data_ptr(),
                                      run_mean.data_ptr(), run_var.data_ptr(), float(momentum), float(eps),
                                      mean.data_ptr(), istd.data_ptr(), scale.data_ptr(), shift.data_ptr(),
                                      ws.data_ptr(), ws.numel() * ws.element_size(), stream_ptr(stream)))


def bn_forward_apply(z, scale, shift, res, dests: Sequence[DestSpec], act: bool = True, stream=None) -> None:
    """a = act(scale·z + shift) (+ res) → dests (reference bn_forward_apply, src/bn.cu:324-327)."""
    N, H, W, C = _nhwc(z)
    if res is not None:
        assert res.shape == z.shape and res.dtype == torch.float16 and res.is_contiguous()
    d = _dests(dests, C)
    check(lib().osam_bn_forward_apply(z.data_ptr(), N, H, W, C, scale.data_ptr(), shift.data_ptr(), _p(res), d,
                                      len(dests), int(act), stream_ptr(stream)))


def bn_forward_train(z, gamma, beta, run_mean, run_var, momentum, eps, mean, istd, scale, shift, res,
                     dests: Sequence[DestSpec], act: bool = True, ws=None, stream=None) -> None:
    """bn_forward_stats then bn_forward_apply in one call (the pair the reference's forward(true) runs per
    conv, src/model.cpp:389-400): same outputs and workspace as the two calls."""
    N, H, W, C = _nhwc(z)
    if res is not None:
        assert res.shape == z.shape and res.dtype == torch.float16 and res.is_contiguous()
    ws = ws if ws is not None else workspace(C, z.device, stream)
    d = _dests(dests, C)
    check(lib().osam_bn_forward_train(z.data_ptr(), N, H, W, C, gamma.data_ptr(), beta.data_ptr(),
                                      run_mean.data_ptr(), run_var.data_ptr(), float(momentum), float(eps),
                                      mean.data_ptr(), istd.data_ptr(), scale.data_ptr(), shift.data_ptr(), _p(res),
                                      d, len(dests), int(act), ws.data_ptr(), ws.numel() * ws.element_size(),
                                      stream_ptr(stream)))


def bn_backward(z, mean, istd, scale, shift, grad_dests: Sequence[DestSpec], act: bool, dz, gw_gamma, gw_beta,
                accum: bool = False, res_grad=None, res_accum: bool = False, ws=None, stream=None) -> None:
    """dz, dγ, dβ (and the residual's gradient) of BN+SiLU (reference bn_backward, src/bn.cu:329-344)."""
    N, H, W, C = _nhwc(z)
    assert dz.shape == z.shape and dz.dtype == torch.float16 and dz.is_contiguous()
    if res_grad is not None:
        assert res_grad.shape == z.shape and res_grad.dtype == torch.float16 and res_grad.is_contiguous()
    ws = ws if ws is not None else workspace(C, z.device, stream)
    d = _dests(grad_dests, C)
    check(lib().osam_bn_backward(z.data_ptr(), N, H, W, C, mean.data_ptr(), istd.data_ptr(), scale.data_ptr(),
                                 shift.data_ptr(), d, len(grad_dests), int(act), dz.data_ptr(), gw_gamma.data_ptr(),
                                 gw_beta.data_ptr(), int(accum), _p(res_grad), int(res_accum), ws.data_ptr(),
                                 ws.numel() * ws.element_size(), stream_ptr(stream)))


def chan_sum(x, out, accum: bool = False, ws=None, stream=None) -> None:
    """out[c] (=|+=) Σ_rows x[…, c] — the bias gradient (reference chan_sum, src/misc.cu:168-172)."""
    assert x.dtype == torch.float16 and x.is_contiguous()
    C = x.shape[-1]
    M = x.numel() // C
    ws = ws if ws is not None else workspace(C, x.device, stream, kind="chan")
    check(lib().osam_chan_sum(x.data_ptr(), M, C, out.data_ptr(), int(accum), ws.data_ptr(),
                              ws.numel() * ws.element_size(), stream_ptr(stream)))


def add_bias(y, bias, stream=None) -> None:
    """y += bias per channel (reference add_bias, src/misc.cu:174-177)."""
    assert y.dtype == torch.float16 and y.is_contiguous()
    C = y.shape[-1]
    check(lib().osam_add_bias(y.data_ptr(), y.numel() // C, C, bias.data_ptr(), stream_ptr(stream)))
