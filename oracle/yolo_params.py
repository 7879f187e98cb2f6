"""Parameter table of YOLOv8s-seg nc=1 (ObjectSAM) and a seeded weight generator (test infrastructure).

Names and PyTorch shapes follow the reference's Params registration (src/model.cpp:95-166, :176-275):
  conv+BN layer  <name>.conv.weight (K,C,k,k), <name>.bn.{weight,bias,running_mean,running_var} (K)
  head 1×1 conv  <name>.weight (K,C,1,1), <name>.bias (K)
  proto upsample model.22.proto.upsample.weight (128,128,2,2), .bias (128)
"""
from __future__ import annotations

import numpy as np

REG_MAX = 16
HEAD_BOX = max(16, 128 // 4, 4 * REG_MAX)   # c2 = 64 (src/model.cpp:226-229)
HEAD_CLS = 128                             # c3 = max(ch0, min(nc, 100)) = 128
HEAD_COEF = 32
NM = 32                                    # mask coefficients / proto channels


def conv_layers():
    """Yields (kind, name, C_in, C_out, k) for every parameterised layer in registration order.
    kind ∈ {"convbn", "head", "convt"}."""
    L = []

    def cb(name, c, k_out, k):
        L.append(("convbn", name, c, k_out, k))

    def c2f(name, c1, c2, n):
        c = c2 // 2
        cb(f"{name}.cv1", c1, 2 * c, 1)
        for j in range(n):
            cb(f"{name}.m.{j}.cv1", c, c, 3)
            cb(f"{name}.m.{j}.cv2", c, c, 3)
        cb(f"{name}.cv2", (2 + n) * c, c2, 1)

    cb("model.0", 3, 32, 3)
    cb("model.1", 32, 64, 3)
    c2f("model.2", 64, 64, 1)
    cb("model.3", 64, 128, 3)
    c2f("model.4", 128, 128, 2)
    cb("model.5", 128, 256, 3)
    c2f("model.6", 256, 256, 2)
    cb("model.7", 256, 512, 3)
    c2f("model.8", 512, 512, 1)
    cb("model.9.cv1", 512, 256, 1)
    cb("model.9.cv2", 1024, 512, 1)
    c2f("model.12", 768, 256, 1)
    c2f("model.15", 384, 128, 1)
    cb("model.16", 128, 128, 3)
    c2f("model.18", 384, 256, 1)
    cb("model.19", 256, 256, 3)
    c2f("model.21", 768, 512, 1)
    for l, ch in enumerate((128, 256, 512)):
        for br, width, kout in (("cv2", HEAD_BOX, 4 * REG_MAX), ("cv3", HEAD_CLS, 1), ("cv4", HEAD_COEF, NM)):
            cb(f"model.22.{br}.{l}.0", ch, width, 3)
            cb(f"model.22.{br}.{l}.1", width, width, 3)
            L.append(("head", f"model.22.{br}.{l}.2", width, kout, 1))
    cb("model.22.proto.cv1", 128, 128, 3)
    L.append(("convt", "model.22.proto.upsample", 128, 128, 2))
    cb("model.22.proto.cv2", 128, 128, 3)
    cb("model.22.proto.cv3", 128, NM, 1)
    return L


def param_shapes():
    shapes = {}
    for kind, name, c, k, ks in conv_layers():
        if kind == "convbn":
            shapes[f"{name}.conv.weight"] = (k, c, ks, ks)
            for p in ("weight", "bias", "running_mean", "running_var"):
                shapes[f"{name}.bn.{p}"] = (k,)
        elif kind == "head":
            shapes[f"{name}.weight"] = (k, c, 1, 1)
            shapes[f"{name}.bias"] = (k,)
        else:
            shapes[f"{name}.weight"] = (c, k, 2, 2)
            shapes[f"{name}.bias"] = (k,)
    return shapes


def make_weights(seed: int = 0, random_bn: bool = False, gain: float = 1.0) -> dict:
    """Seeded weights: He-normal convs (std gain·√(2/fan_in); gain 1 = BASELINE config 1), BN γ=1 β=0 μ=0
    σ²=1 unless random_bn, head/upsample biases U(-0.1, 0.1).  numpy PCG64 → identical on every machine.
    Parity tests use gain ≈ 1.2 so activations stay O(1) through the 70 convs (SiLU loses variance that
    ReLU-calibrated He init does not restore)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name, shape in param_shapes().items():
        if name.endswith("conv.weight") or (name.endswith(".weight") and len(shape) == 4):
            if "upsample" in name:
                fan_in = shape[0] * shape[2] * shape[3]
            else:
                fan_in = shape[1] * shape[2] * shape[3]
            out[name] = (rng.standard_normal(shape) * (gain * np.sqrt(2.0 / fan_in))).astype(np.float32)
        elif name.endswith(".bias") and not name.endswith("bn.bias"):
            out[name] = rng.uniform(-0.1, 0.1, shape).astype(np.float32)
        elif name.endswith("bn.weight"):
            out[name] = (rng.uniform(0.5, 1.5, shape) if random_bn else np.ones(shape)).astype(np.float32)
        elif name.endswith("bn.bias"):
            out[name] = (rng.uniform(-0.2, 0.2, shape) if random_bn else np.zeros(shape)).astype(np.float32)
        elif name.endswith("running_mean"):
            out[name] = (rng.normal(0, 0.1, shape) if random_bn else np.zeros(shape)).astype(np.float32)
        elif name.endswith("running_var"):
            out[name] = (rng.uniform(0.5, 1.5, shape) if random_bn else np.ones(shape)).astype(np.float32)
        else:
            raise KeyError(name)
    return out


def make_images(n: int, size: int, seed: int = 0) -> np.ndarray:
    """Seeded synthetic input batch, NHWC fp32 U[0,1] (BASELINE configs 1/2)."""
    rng = np.random.Generator(np.random.PCG64(seed + 1000003))
    return rng.random((n, size, size, 3), dtype=np.float32)


def n_params() -> int:
    return int(sum(np.prod(s) for n, s in param_shapes().items() if "running" not in n))
