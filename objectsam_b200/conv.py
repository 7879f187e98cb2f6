"""Host-side mirror of the reference's conv operator (ConvOp, reference src/conv.h:16-53) over the C ABI.

Same method names and argument meaning as the reference: `init(geom, transposed)`, `tune(...)` returning
the workspace size, `fwd(x, w, y, ws, beta)`, `geom()`, `out_elems()`; plus `fwd_fused`, the conv with
its BN/SiLU/residual/DestList (or bias) epilogue that replaces ConvOp::fwd + bn_forward_apply / add_bias.
Tensors are torch CUDA tensors (NHWC fp16 activations, KRSC fp16 weights); errors raise OsamError the
way the reference aborts through CUDNN_CHECK / FSO_ASSERT.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

from . import _lib
from ._lib import ConvGeom, Dest, Epilogue, check, lib, stream_ptr

__all__ = ["ConvGeom", "ConvOp", "DestSpec", "sppf_pool_fwd", "sppf_pool_bwd", "EPI_STORE", "EPI_BN_ACT", "EPI_BIAS"]
EPI_STORE, EPI_BN_ACT, EPI_BIAS = _lib.EPI_STORE, _lib.EPI_BN_ACT, _lib.EPI_BIAS


def _ptr(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


@dataclass
class DestSpec:
    """One epilogue destination (reference Dest, src/bn.cuh:10-17): output channels [c0, c1) go to channels
    [choff, …) of an NHWC tensor `t`; up=2 writes the 2×2 nearest-upsampled block."""
    t: object
    choff: int = 0
    c0: int = 0
    c1: int = 0  # 0 = all output channels (as in the reference's DestSpec default, src/model.cpp:123)
    up: int = 1


class ConvOp:
    def __init__(self):
        self._plan = ctypes.c_void_p()
        self._g: Optional[ConvGeom] = None
        self.transposed = False
        self.tuned_ms = [0.0, 0.0, 0.0]

    def init(self, g: ConvGeom, transposed: bool = False) -> "ConvOp":
        self.close()
        self._g = ConvGeom(*[getattr(g, n) for n, _ in ConvGeom._fields_])
        self.transposed = bool(transposed)
        check(lib().osam_conv_plan_create(ctypes.byref(self._g), int(self.transposed), ctypes.byref(self._plan)))
        return self

    def close(self) -> None:
        if self._plan:
            lib().osam_conv_plan_destroy(self._plan)
            self._plan = ctypes.c_void_p()

    __del__ = close

    def tune(self, *unused, **kw) -> int:
        """The tile shape is a static function of the geometry; returns the workspace size (bytes)."""
        return int(lib().osam_conv_workspace_size(self._plan))

    workspace_size = tune

    def geom(self) -> ConvGeom:
        return self._g

    def out_elems(self) -> int:
        return int(lib().osam_conv_out_elems(self._plan))

    def out_shape(self):
        g = self._g
        if self.transposed:
            return (g.N, 2 * g.H, 2 * g.W, g.K)
        return (g.N, g.P(), g.Q(), g.K)

    def fwd(self, x, w, y, ws=None, beta: float = 0.0, stream=None) -> None:
        nbytes = 0 if ws is None else ws.numel() * ws.element_size()
        check(lib().osam_conv_fwd(self._plan, _ptr(x), _ptr(w), _ptr(y), float(beta), _ptr(ws), nbytes,
                                  stream_ptr(stream)))

    def dgrad(self, dy, w, dx, ws=None, beta: float = 0.0, stream=None) -> None:
        """dx = dgrad(dy, w) (+ beta·dx) — ConvOp::dgrad (src/conv.cpp:346-355).  `ws` must hold
        workspace_size() bytes (a torch uint8 CUDA tensor, 256-byte aligned as torch allocates)."""
        nbytes = 0 if ws is None else ws.numel() * ws.element_size()
        check(lib().osam_conv_dgrad(self._plan, _ptr(dy), _ptr(w), _ptr(dx), float(beta), _ptr(ws), nbytes,
                                    stream_ptr(stream)))

    def wgrad(self, x, dy, dw, ws=None, beta: float = 0.0, stream=None) -> None:
        """dw = wgrad(x, dy) (+ beta·dw), fp16 KRSC — ConvOp::wgrad (src/conv.cpp:357-366)."""
        nbytes = 0 if ws is None else ws.numel() * ws.element_size()
        check(lib().osam_conv_wgrad(self._plan, _ptr(x), _ptr(dy), _ptr(dw), float(beta), _ptr(ws), nbytes,
                                    stream_ptr(stream)))

    def fwd_fused(self, x, w, dests: Sequence[DestSpec], kind: int = EPI_BN_ACT, scale=None, shift=None,
                  bias=None, res=None, act: bool = True, round_z: bool = True, ws=None, stream=None) -> None:
        ep = make_epilogue(self._g.K, dests, kind, scale, shift, bias, res, act, round_z)
        nbytes = 0 if ws is None else ws.numel() * ws.element_size()
        check(lib().osam_conv_fwd_fused(self._plan, _ptr(x), _ptr(w), ctypes.byref(ep), _ptr(ws), nbytes,
                                        stream_ptr(stream)))


def make_epilogue(K: int, dests: Sequence[DestSpec], kind: int, scale=None, shift=None, bias=None, res=None,
                  act: bool = True, round_z: bool = True) -> Epilogue:
    if not 1 <= len(dests) <= _lib.MAX_DEST:
        raise ValueError("1..4 destinations")
    ep = Epilogue()
    ep.kind = kind
    ep.scale, ep.shift, ep.bias, ep.res = _ptr(scale), _ptr(shift), _ptr(bias), _ptr(res)
    ep.act = int(act)
    ep.round_z = int(round_z)
    ep.n_dest = len(dests)
    for i, d in enumerate(dests):
        ep.dest[i] = Dest(d.t.data_ptr(), d.t.shape[-1], d.choff, d.c0, d.c1 or K, d.up)
    return ep


def sppf_pool_fwd(cat, N: int, H: int, W: int, c: int, stream=None) -> None:
    """Reference sppf_pool_fwd (src/misc.cuh:6): slices 1..3 of `cat` ← chained 5×5 max-pools of slice 0."""
    check(lib().osam_sppf_fwd(_ptr(cat), N, H, W, c, stream_ptr(stream)))


def sppf_pool_bwd(cat, dcat, N: int, H: int, W: int, c: int, stream=None) -> None:
    """Reference sppf_pool_bwd (src/misc.cuh:9): dcat slice 0 += the gradients of slices 1..3 routed back through
    the chained pools (first maximum of each window).  The reference's fp32 scratch buffers are not needed."""
    check(lib().osam_sppf_bwd(_ptr(cat), _ptr(dcat), N, H, W, c, stream_ptr(stream)))
