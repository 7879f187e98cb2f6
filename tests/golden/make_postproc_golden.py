"""Generates tests/golden/postproc_golden.npz by running the reference's own post-process code.

The reference's inference post-process lives in archive/tools/ref_detect.py (OrtDetector.detect).  It is
imported from the reference tree unchanged; its two external dependencies are replaced by stand-ins that
do no arithmetic of their own:
  - onnxruntime.InferenceSession → returns the seeded head tensors (o0 = [xywh | conf | coefs] × anchors,
    o1 = proto) prepared here, i.e. exactly what the exported network would emit;
  - cv2.resize → identity (the synthetic input is already S×S, so the letterbox is a no-op: r = 1).
Every case stores the inputs and the reference's outputs (score, box, grid).  Run in a checkout that
has the reference mounted:  python tests/golden/make_postproc_golden.py [reference_root]
"""
from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "postproc_golden.npz")


class _FakeSession:
    outputs = None

    def __init__(self, path, so=None, providers=None):
        self.S = _FakeSession.S

    def get_inputs(self):
        return [types.SimpleNamespace(shape=[1, 3, self.S, self.S], name="images")]

    def run(self, names, feeds):
        o0, o1 = _FakeSession.outputs
        return [o0[None], o1[None]]


def _install_stand_ins():
    ort = types.ModuleType("onnxruntime")
    ort.SessionOptions = lambda: types.SimpleNamespace(intra_op_num_threads=1)
    ort.InferenceSession = _FakeSession
    cv2 = types.ModuleType("cv2")
    cv2.INTER_LINEAR = 1

    def resize(img, size, interpolation=None):
        assert img.shape[1] == size[0] and img.shape[0] == size[1], "stand-in resize only handles identity"
        return img

    cv2.resize = resize
    sys.modules["onnxruntime"] = ort
    sys.modules["cv2"] = cv2


def _heads(rng, S, n_anchor_levels=((8,), (16,), (32,)), cluster=True):
    """Seeded exported heads: boxes clustered around a few centres so NMS has real overlaps."""
    A = sum((S // s) ** 2 for (s,) in n_anchor_levels)
    centres = rng.uniform(0.1 * S, 0.9 * S, (12, 2))
    which = rng.integers(0, len(centres), A)
    cxy = centres[which] + rng.normal(0, S * 0.03, (A, 2)) if cluster else rng.uniform(0, S, (A, 2))
    wh = rng.uniform(0.05 * S, 0.5 * S, (A, 2))
    conf = rng.uniform(0, 1, A)
    conf[rng.integers(0, A, A // 8)] = conf[rng.integers(0, A, A // 8)]  # exact ties
    coefs = rng.normal(0, 1, (A, 32))
    Pp = S // 4
    proto = rng.normal(0, 1, (32, Pp, Pp))
    # fp16-representable values so the fixture can store them as float16 without changing them
    o0 = np.concatenate([cxy.T, wh.T, conf[None], coefs.T], 0).astype(np.float16).astype(np.float32)
    return o0, proto.astype(np.float16).astype(np.float32)


def main(ref_root="/root/reference"):
    _install_stand_ins()
    path = os.path.join(ref_root, "archive", "tools", "ref_detect.py")
    spec = importlib.util.spec_from_file_location("ref_detect", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.Generator(np.random.PCG64(20261201))
    cases = []
    # (S, conf_th, nms_iou, mask_iou, area_min, max_det): the reference defaults and the BASELINE setting
    settings = [(256, 0.25, 0.7, 0.7, 24, 100), (256, 0.25, 0.7, 1.0, 0, 300), (320, 0.5, 0.5, 1.0, 0, 300),
                (192, 0.05, 0.7, 0.7, 24, 100)]
    out = {}
    for ci, (S, cth, nth, mth, amin, mdet) in enumerate(settings):
        o0, o1 = _heads(rng, S)
        _FakeSession.S = S
        _FakeSession.outputs = (o0, o1)
        det = mod.OrtDetector("stand-in.onnx", conf_th=cth, nms_iou=nth, mask_iou=mth, area_min=amin, max_det=mdet)
        res = det.detect(np.zeros((S, S, 3), np.uint8), full=False)
        out[f"c{ci}_o0"] = o0.astype(np.float16)
        out[f"c{ci}_o1"] = o1.astype(np.float16)
        out[f"c{ci}_cfg"] = np.array([S, cth, nth, mth, amin, mdet], np.float64)
        out[f"c{ci}_score"] = res["score"]
        out[f"c{ci}_box"] = res["box"]
        out[f"c{ci}_grid"] = np.packbits(res["grid"].astype(np.uint8), axis=-1)
        out[f"c{ci}_grid_shape"] = np.array(res["grid"].shape, np.int64)
        cases.append((S, len(res["score"])))
    out["n_cases"] = np.array(len(settings))
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, cases)


if __name__ == "__main__":
    main(*sys.argv[1:])
