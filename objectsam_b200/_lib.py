"""ctypes binding of the C ABI declared in include/osam.h (libosam.so, built in-tree for sm_100a).

The library is the product path: there is no Python or CPU fallback.  Loading fails loudly when the
shared object is missing or does not export every symbol the header declares.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, byref, c_float, c_int, c_int64, c_size_t, c_void_p

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libosam.so")

OSAM_OK, OSAM_ERR_INVALID, OSAM_ERR_UNSUPPORTED, OSAM_ERR_CUDA, OSAM_ERR_TIMEOUT, OSAM_ERR_NOMEM = range(6)
EPI_STORE, EPI_BN_ACT, EPI_BIAS = 0, 1, 2
MAX_DEST = 4


class ConvGeom(ctypes.Structure):
    """osam_conv_geom — mirrors ConvGeom (reference src/conv.h:8-14)."""
    _fields_ = [(n, c_int) for n in ("N", "H", "W", "C", "K", "R", "S", "stride", "pad")]

    def P(self) -> int:
        return (self.H + 2 * self.pad - self.R) // self.stride + 1

    def Q(self) -> int:
        return (self.W + 2 * self.pad - self.S) // self.stride + 1


class Dest(ctypes.Structure):
    """osam_dest — mirrors Dest (reference src/bn.cuh:10-17)."""
    _fields_ = [("p", c_void_p), ("ctot", c_int), ("choff", c_int), ("c0", c_int), ("c1", c_int), ("up", c_int)]


class Epilogue(ctypes.Structure):
    _fields_ = [("kind", c_int), ("scale", c_void_p), ("shift", c_void_p), ("bias", c_void_p), ("res", c_void_p),
                ("act", c_int), ("round_z", c_int), ("n_dest", c_int), ("dest", Dest * MAX_DEST)]


class Tensor(ctypes.Structure):
    """osam_tensor — a device NHWC fp16 buffer owned by a model."""
    _fields_ = [("p", c_void_p), ("n", c_int), ("h", c_int), ("w", c_int), ("c", c_int)]


class Detections(ctypes.Structure):
    """osam_detections — the detect step's output buffers (device pointers)."""
    _fields_ = [(f, c_int) for f in ("batch", "anchors", "max_det", "packed", "proto_h", "proto_w")] + \
               [(f, c_void_p) for f in ("xyxy", "conf", "n_det", "keep", "box", "score", "coef_g", "masks")]


class OsamError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"osam error {code}: {msg}")
        self.code = code


class AugBatch(ctypes.Structure):
    """osam_aug_batch — device pointers of one training batch (≙ the reference's device BatchBuf)."""
    _fields_ = [(n, c_void_p) for n in ("hdr", "smp", "src", "inst", "img", "mask")]


class AugOut(ctypes.Structure):
    """osam_aug_out — ≙ AugOut + GtBatch (reference src/augment.cuh:11-17, src/loss.cuh:25-30)."""
    _fields_ = [("img", c_void_p), ("n_gt", c_void_p), ("box", c_void_p), ("mask", c_void_p), ("ignore", c_void_p),
                ("gt_inst", c_void_p), ("G", c_int), ("Hp", c_int), ("Wp", c_int)]


# symbol → (restype, argtypes); every entry point of include/osam.h
_SIGS = {
    "osam_conv_plan_create": (c_int, [POINTER(ConvGeom), c_int, POINTER(c_void_p)]),
    "osam_conv_plan_destroy": (c_int, [c_void_p]),
    "osam_conv_workspace_size": (c_size_t, [c_void_p]),
    "osam_conv_out_elems": (c_int64, [c_void_p]),
    "osam_conv_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_size_t, c_void_p]),
    "osam_conv_fwd_fused": (c_int, [c_void_p, c_void_p, c_void_p, POINTER(Epilogue), c_void_p, c_size_t, c_void_p]),
    "osam_conv_dgrad": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_size_t, c_void_p]),
    "osam_conv_wgrad": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_size_t, c_void_p]),
    "osam_convt_fwd_static_scratch": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p]),
    "osam_sppf_fwd": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "osam_sppf_bwd": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "osam_bn_workspace_size": (c_size_t, [c_int]),
    "osam_bn_eval_scale": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_void_p, c_void_p,
                                   c_void_p]),
    "osam_bn_forward_stats": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t,
                                      c_void_p]),
    "osam_bn_forward_apply": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                      POINTER(Dest), c_int, c_int, c_void_p]),
    "osam_bn_forward_train": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_float, c_float, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, POINTER(Dest),
                                      c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "osam_bn_backward": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p,
                                 POINTER(Dest), c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                 c_void_p, c_size_t, c_void_p]),
    "osam_chan_sum_workspace_size": (c_size_t, [c_int]),
    "osam_chan_sum": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "osam_add_bias": (c_int, [c_void_p, c_int64, c_int, c_void_p, c_void_p]),
    "osam_mask_loss_workspace_size": (c_size_t, [c_int, c_int]),
    "osam_mask_loss": (c_int, [POINTER(c_void_p), POINTER(c_int), c_void_p, c_int, c_int, c_int, c_int, c_int,
                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float,
                               c_void_p, POINTER(c_void_p), c_void_p, c_void_p, c_size_t, c_void_p]),
    "osam_det_loss_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "osam_det_loss": (c_int, [POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int), c_int, c_int, c_int, c_void_p,
                              c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_float, c_float, c_float,
                              POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_void_p, c_void_p,
                              c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "osam_seg_loss_items": (c_int, [c_void_p, c_float, c_float, c_float, c_void_p]),
    "osam_augment": (c_int, [POINTER(AugBatch), c_int, c_int, POINTER(AugOut), c_void_p]),
    "osam_decode": (c_int, [POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int), c_int, c_int, c_int, c_void_p,
                            c_void_p, c_void_p]),
    "osam_nms": (c_int, [c_void_p, c_void_p, c_int, c_int, c_float, c_float, c_int, c_int, POINTER(c_void_p),
                         POINTER(c_int), c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "osam_mask_assemble": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                   c_int, c_void_p, c_void_p]),
    "osam_model_create": (c_int, [c_int, c_int, c_int, POINTER(c_void_p)]),
    "osam_model_destroy": (c_int, [c_void_p]),
    "osam_model_set_param": (c_int, [c_void_p, ctypes.c_char_p, c_void_p, POINTER(c_int64), c_int]),
    "osam_model_load_fsow": (c_int, [c_void_p, ctypes.c_char_p]),
    "osam_model_sync_weights": (c_int, [c_void_p, c_void_p]),
    "osam_model_input": (c_int, [c_void_p, POINTER(Tensor)]),
    "osam_model_head": (c_int, [c_void_p, c_int, c_int, POINTER(Tensor)]),
    "osam_model_proto": (c_int, [c_void_p, POINTER(Tensor)]),
    "osam_model_act": (c_int, [c_void_p, ctypes.c_char_p, POINTER(Tensor)]),
    "osam_model_forward": (c_int, [c_void_p, c_int, c_void_p]),
    "osam_model_num_launches": (c_int, [c_void_p]),
    "osam_model_detect_init": (c_int, [c_void_p, c_float, c_float, c_int, c_int, c_int]),
    "osam_model_forward_detect": (c_int, [c_void_p, c_int, c_void_p]),
    "osam_model_detections": (c_int, [c_void_p, POINTER(Detections)]),
    "osam_model_forward_nodes": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "osam_model_node_info": (c_int, [c_void_p, c_int, ctypes.c_char_p, c_int, POINTER(c_int), POINTER(ConvGeom)]),
    "osam_model_train_init": (c_int, [c_void_p, c_void_p]),
    "osam_model_forward_train": (c_int, [c_void_p, c_float, c_void_p]),
    "osam_model_backward_nodes": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "osam_model_act_grad": (c_int, [c_void_p, ctypes.c_char_p, POINTER(Tensor)]),
    "osam_model_grad_arena": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_int64)]),
    "osam_model_node_grad_range": (c_int, [c_void_p, c_int, POINTER(c_int64), POINTER(c_int64)]),
    "osam_model_get_grad": (c_int, [c_void_p, ctypes.c_char_p, c_void_p, c_int64]),
    "osam_dp_unique_id": (c_int, [ctypes.c_char_p]),
    "osam_dp_create": (c_int, [c_void_p, c_int, c_int, ctypes.c_char_p, c_size_t, c_int, POINTER(c_void_p)]),
    "osam_dp_create_from_comm": (c_int, [c_void_p, c_void_p, c_size_t, POINTER(c_void_p)]),
    "osam_dp_num_buckets": (c_int, [c_void_p]),
    "osam_dp_bucket": (c_int, [c_void_p, c_int, POINTER(c_int), POINTER(c_int), POINTER(c_int64), POINTER(c_int64)]),
    "osam_dp_backward": (c_int, [c_void_p, c_void_p]),
    "osam_dp_wait": (c_int, [c_void_p, c_int]),
    "osam_dp_destroy": (c_int, [c_void_p]),
    "osam_device_error": (c_int, []),
    "osam_device_error_peek": (c_int, []),
    "osam_selftest_wait_timeout": (c_int, [ctypes.c_ulonglong, c_void_p]),
    "osam_last_error": (ctypes.c_char_p, []),
}

_lib = None


def header_symbols() -> list[str]:
    """Names of every function declared in include/osam.h (parsed from the header text)."""
    import re
    hdr = os.path.join(os.path.dirname(PKG), "include", "osam.h")
    with open(hdr) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(osam_\w+)\s*\(", text, re.M)))


def lib() -> ctypes.CDLL:
    """Load libosam.so (once).  Raises if it is missing or incomplete — there is no fallback path."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is missing: build it with `python -m objectsam_b200.build` "
                      "(the CUDA path has no fallback)")
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != OSAM_OK:
        raise OsamError(rc, lib().osam_last_error().decode(errors="replace"))


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def device_error() -> int:
    return lib().osam_device_error()
