"""Host-side mirror of the reference's Model (src/model.h:97-140) for inference, over the C ABI.

    m = Model(batch=64, imgsz=640)          # Model::build (graph + activation arena)
    m.load(tensors) / m.load_fsow(path)     # Params::load (PyTorch names, OIHW fp32)
    m.sync_weights()                        # fp16 KRSC copies + folded eval-mode BN
    m.input().copy_(images_nhwc_fp16)       # Model::input()->p
    m.forward()                             # Model::forward(false)
    m.head(kind, lvl), m.proto()            # raw head tensors (box / cls / coef, proto), NHWC fp16

Tensors returned by input()/head()/proto()/act() are torch CUDA views of the model's own buffers.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import Tensor, check, lib, stream_ptr


class _DeviceArray:
    """__cuda_array_interface__ wrapper so torch can view a buffer owned by the library."""

    def __init__(self, ptr: int, shape, owner, typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}
        self._owner = owner


class Model:
    BOX, CLS, COEF = 0, 1, 2

    def __init__(self, batch: int, imgsz: int, reg_max: int = 16):
        self.batch, self.imgsz, self.reg_max = batch, imgsz, reg_max
        self._m = ctypes.c_void_p()
        check(lib().osam_model_create(batch, imgsz, reg_max, ctypes.byref(self._m)))

    def close(self) -> None:
        if getattr(self, "_m", None):
            lib().osam_model_destroy(self._m)
            self._m = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------- parameters
    def load(self, tensors: dict) -> None:
        for name, arr in tensors.items():
            a = np.ascontiguousarray(np.asarray(arr, dtype=np.float32))
            shape = (ctypes.c_int64 * a.ndim)(*a.shape)
            check(lib().osam_model_set_param(self._m, name.encode(), a.ctypes.data, shape, a.ndim))

    def load_fsow(self, path: str) -> None:
        check(lib().osam_model_load_fsow(self._m, path.encode()))

    def sync_weights(self, stream=None) -> None:
        check(lib().osam_model_sync_weights(self._m, stream_ptr(stream)))

    # ------------------------------------------------------------- tensors
    def _view(self, t: Tensor):
        import torch
        return torch.as_tensor(_DeviceArray(t.p, (t.n, t.h, t.w, t.c), self), device="cuda")

    def input(self):
        t = Tensor()
        check(lib().osam_model_input(self._m, ctypes.byref(t)))
        return self._view(t)

    def head(self, kind: int, lvl: int):
        t = Tensor()
        check(lib().osam_model_head(self._m, kind, lvl, ctypes.byref(t)))
        return self._view(t)

    def proto(self):
        t = Tensor()
        check(lib().osam_model_proto(self._m, ctypes.byref(t)))
        return self._view(t)

    def act(self, name: str):
        t = Tensor()
        check(lib().osam_model_act(self._m, name.encode(), ctypes.byref(t)))
        return self._view(t)

    def tensor_info(self, which: str, kind: int = 0, lvl: int = 0) -> Tensor:
        t = Tensor()
        if which == "input":
            check(lib().osam_model_input(self._m, ctypes.byref(t)))
        elif which == "head":
            check(lib().osam_model_head(self._m, kind, lvl, ctypes.byref(t)))
        else:
            check(lib().osam_model_proto(self._m, ctypes.byref(t)))
        return t

    # ------------------------------------------------------------- execution
    def forward(self, use_graph: bool = False, stream=None) -> None:
        check(lib().osam_model_forward(self._m, int(use_graph), stream_ptr(stream)))

    # ------------------------------------------------------------- the detect step (forward + post-process)
    def detect_init(self, conf_th: float = 0.25, iou_th: float = 0.7, max_det: int = 300, forced: bool = False,
                    packed: bool = True) -> None:
        """Settings and output buffers of forward_detect (the post-process joins the forward's graph)."""
        check(lib().osam_model_detect_init(self._m, float(conf_th), float(iou_th), int(max_det), int(forced),
                                           int(packed)))

    def forward_detect(self, use_graph: bool = True, stream=None) -> None:
        """Forward + decode + NMS + masks as one step; decode and NMS overlap the proto branch."""
        check(lib().osam_model_forward_detect(self._m, int(use_graph), stream_ptr(stream)))

    def detections(self) -> dict:
        """The detect step's outputs as torch views of the model's buffers: xyxy, conf, n_det, keep, box,
        score, coef_g, masks (packed int32 words or u8), in the layouts of objectsam_b200.postproc."""
        import torch
        from ._lib import Detections
        d = Detections()
        check(lib().osam_model_detections(self._m, ctypes.byref(d)))
        B, A, M = d.batch, d.anchors, d.max_det
        pad = (M + 127) // 128 * 128
        hw = d.proto_h * d.proto_w

        def view(ptr, shape, typestr):
            return torch.as_tensor(_DeviceArray(ptr, shape, self, typestr), device="cuda")
        out = dict(xyxy=view(d.xyxy, (B, A, 4), "<f4"), conf=view(d.conf, (B, A), "<f4"),
                   n_det=view(d.n_det, (B,), "<i4"), keep=view(d.keep, (B, M), "<i4"),
                   box=view(d.box, (B, M, 4), "<f4"), score=view(d.score, (B, M), "<f4"),
                   coef_g=view(d.coef_g, (B, pad, 32), "<f2"))
        out["masks"] = view(d.masks, (B, M, (hw + 31) // 32), "<i4") if d.packed else \
            view(d.masks, (B, M, d.proto_h, d.proto_w), "|u1")
        return out

    @property
    def handle(self) -> int:
        return self._m.value

    def num_launches(self) -> int:
        return lib().osam_model_num_launches(self._m)

    def forward_nodes(self, first: int, count: int, stream=None) -> None:
        check(lib().osam_model_forward_nodes(self._m, first, count, stream_ptr(stream)))

    # ------------------------------------------------------------- training (Model::forward(true), backward)
    def train_init(self, stream=None) -> None:
        """Allocate gradients, z buffers and BN state (after sync_weights)."""
        check(lib().osam_model_train_init(self._m, stream_ptr(stream)))

    def forward_train(self, momentum: float = 0.03, stream=None) -> None:
        check(lib().osam_model_forward_train(self._m, float(momentum), stream_ptr(stream)))

    def backward_nodes(self, first: int, count: int, stream=None) -> None:
        """Backward of nodes [first, first + count), last node first."""
        check(lib().osam_model_backward_nodes(self._m, first, count, stream_ptr(stream)))

    def backward(self, stream=None) -> None:
        self.backward_nodes(0, self.num_launches(), stream)

    def act_grad(self, name: str):
        """Gradient buffer of an activation ("out.box0", "out.proto", …) as a torch NHWC fp16 view."""
        t = Tensor()
        check(lib().osam_model_act_grad(self._m, name.encode(), ctypes.byref(t)))
        return self._view(t)

    def grad_arena(self):
        """All parameter gradients (fp32, nodes in reverse order) as one torch view."""
        import torch
        p, n = ctypes.c_void_p(), ctypes.c_int64()
        check(lib().osam_model_grad_arena(self._m, ctypes.byref(p), ctypes.byref(n)))
        return torch.as_tensor(_DeviceArray(p.value, (n.value,), self, "<f4"), device="cuda")

    def node_grad_range(self, i: int) -> tuple[int, int]:
        off, n = ctypes.c_int64(), ctypes.c_int64()
        check(lib().osam_model_node_grad_range(self._m, i, ctypes.byref(off), ctypes.byref(n)))
        return off.value, n.value

    def get_grad(self, name: str, shape) -> np.ndarray:
        out = np.zeros(int(np.prod(shape)), np.float32)
        check(lib().osam_model_get_grad(self._m, name.encode(), out.ctypes.data, out.size))
        return out.reshape(shape)

    def nodes(self) -> list[dict]:
        """Per node: name, kind (0 conv+BN+SiLU, 1 head conv, 2 transposed conv, 3 SPPF pool), geometry,
        conv FLOPs (2·N·P·Q·K·C·R·S; the transposed conv counts H·W — the reference's formula,
        src/model.cpp:483) and minimum HBM bytes (input + weights + every destination write)."""
        from ._lib import ConvGeom
        out = []
        for i in range(self.num_launches()):
            buf = ctypes.create_string_buffer(128)
            kind = ctypes.c_int()
            g = ConvGeom()
            check(lib().osam_model_node_info(self._m, i, buf, 128, ctypes.byref(kind), ctypes.byref(g)))
            k = kind.value
            if k == 3:
                flops = 0.0
                nbytes = 2.0 * g.N * g.H * g.W * g.C * 4  # read slice 0, write slices 1..3
            else:
                pq = g.H * g.W if k == 2 else g.P() * g.Q()
                kout = 4 * g.K if k == 2 else g.K
                flops = 2.0 * g.N * pq * g.K * g.C * g.R * g.S
                nbytes = 2.0 * (g.N * g.H * g.W * g.C + kout * g.R * g.S * g.C / (4 if k == 2 else 1)
                                + g.N * pq * kout)
            out.append(dict(index=i, name=buf.value.decode(), kind=k, N=g.N, H=g.H, W=g.W, C=g.C, K=g.K, R=g.R,
                            S=g.S, stride=g.stride, flops=flops, bytes=nbytes))
        return out
