"""PyTorch CPU restatement of the YOLOv8s-seg nc=1 forward pass (test infrastructure — the checker).

Follows the reference's network (src/model.cpp:168-275) and its operator semantics:
  Conv+BN+SiLU    a = silu(scale·z + shift) [+ res], scale = γ/√(var+eps), shift = β − μ·scale
                  (eval mode: bn_eval_scale src/bn.cu:277-284; apply src/bn.cu:204-238 — the residual
                  is added AFTER the activation, :216-220), eps = 1e-3 (src/model.h:95)
  C2f             cv1 → split; n × Bottleneck(3×3, 3×3, +x if shortcut); concat; cv2 (src/model.cpp:134-151)
  SPPF            cv1; three chained 5×5/s1/p2 max-pools; concat; cv2 (src/model.cpp:203-214, src/misc.cu:32-46)
  neck            upsample ×2 nearest + concat (the reference's DestList routing, src/model.cpp:187-224)
  Segment head    per level box/cls/coef branches: Conv3×3, Conv3×3, Conv2d1×1+bias (src/model.cpp:226-253);
                  proto: Conv3×3 → ConvTranspose 2×2/s2 + bias → Conv3×3 → Conv1×1 (src/model.cpp:254-275)

With emulate_fp16=True the tensors are rounded to fp16 where the reference's fp16 build stores them:
input image, weights (w_act), every conv output z (before BN), every activation, head outputs.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import yolo_params as P

BN_EPS = 1e-3


class YoloSegRef:
    def __init__(self, weights: dict, emulate_fp16: bool = True, dtype=torch.float32, device="cpu",
                 calibrate: bool = False, train: bool = False):
        self.fp16 = emulate_fp16
        self.calibrate = calibrate
        self.train = train  # BN on batch statistics, autograd on (reference Model::forward(true), src/bn.cu:112-202)
        self.dtype = dtype
        self.device = device
        self.w = {}
        for k, v in weights.items():
            t = torch.from_numpy(np.asarray(v, dtype=np.float32)).to(device)
            if self.fp16 and (k.endswith("conv.weight") or (t.ndim == 4)):
                t = t.half().float()
            self.w[k] = t.to(dtype)
            if train and not k.endswith(("running_mean", "running_var")):
                self.w[k].requires_grad_(True)
        self.acts = {}

    # -------------------------------------------------------------- helpers
    def _r(self, t):
        """Round to the reference's storage precision (fp16) when emulating it."""
        return t.half().to(self.dtype) if self.fp16 else t

    def conv_bn(self, x, name, k, s, res=None, keep=None):
        w = self.w[f"{name}.conv.weight"]
        z = self._r(F.conv2d(x, w, stride=s, padding=k // 2))
        if self.calibrate:  # running stats ← this batch's per-channel statistics (like a trained net)
            self.w[f"{name}.bn.running_mean"] = z.mean((0, 2, 3))
            self.w[f"{name}.bn.running_var"] = z.var((0, 2, 3), unbiased=False)
        g, b = self.w[f"{name}.bn.weight"], self.w[f"{name}.bn.bias"]
        if self.train:  # batch statistics, biased variance (the normalisation the reference's stats pass feeds)
            mu, var = z.mean((0, 2, 3)), z.var((0, 2, 3), unbiased=False)
            scale = g * torch.rsqrt(var + BN_EPS)
            shift = b - mu * scale
        else:
            rm, rv = self.w[f"{name}.bn.running_mean"], self.w[f"{name}.bn.running_var"]
            scale = (g.float() * torch.rsqrt(rv.float() + BN_EPS)).to(self.dtype)
            shift = (b.float() - rm.float() * scale.float()).to(self.dtype)
        y = z * scale.view(1, -1, 1, 1) + shift.view(1, -1, 1, 1)
        y = y * torch.sigmoid(y)
        if res is not None:
            y = y + res
        y = self._r(y)
        if keep is not None:
            self.acts[keep] = y
        return y

    def c2f(self, x, name, c2, n, shortcut):
        c = c2 // 2
        y = self.conv_bn(x, f"{name}.cv1", 1, 1)
        parts = [y[:, :c], y[:, c:]]
        b = parts[-1]
        for j in range(n):
            t = self.conv_bn(b, f"{name}.m.{j}.cv1", 3, 1)
            b = self.conv_bn(t, f"{name}.m.{j}.cv2", 3, 1, res=b if shortcut else None)
            parts.append(b)
        return self.conv_bn(torch.cat(parts, 1), f"{name}.cv2", 1, 1)

    def head_conv(self, x, name):
        z = self._r(F.conv2d(x, self.w[f"{name}.weight"]))
        return self._r(z + self.w[f"{name}.bias"].view(1, -1, 1, 1))

    @staticmethod
    def _pool5(x):
        return F.max_pool2d(x, 5, 1, 2)

    @staticmethod
    def _up(x):
        return F.interpolate(x, scale_factor=2, mode="nearest")

    # -------------------------------------------------------------- network
    def forward(self, img_nhwc) -> dict:
        """img_nhwc: (N, S, S, 3) float array/tensor in [0,1].  Returns NCHW tensors:
        box[l] (N,64,H,W), cls[l] (N,1,H,W), coef[l] (N,32,H,W), proto (N,32,S/4,S/4).
        In training mode the graph is kept for autograd (the parameters in self.w require grad)."""
        with torch.set_grad_enabled(self.train):
            return self._forward(img_nhwc)

    def _forward(self, img_nhwc) -> dict:
        x = torch.as_tensor(np.asarray(img_nhwc), dtype=torch.float32).to(self.device)
        x = self._r(x.to(self.dtype).permute(0, 3, 1, 2).contiguous())
        self.acts = {}
        a0 = self.conv_bn(x, "model.0", 3, 2, keep="a0")
        a1 = self.conv_bn(a0, "model.1", 3, 2, keep="a1")
        a2 = self.c2f(a1, "model.2", 64, 1, True)
        a3 = self.conv_bn(a2, "model.3", 3, 2, keep="a3")
        a4 = self.c2f(a3, "model.4", 128, 2, True)
        a5 = self.conv_bn(a4, "model.5", 3, 2, keep="a5")
        a6 = self.c2f(a5, "model.6", 256, 2, True)
        a7 = self.conv_bn(a6, "model.7", 3, 2, keep="a7")
        a8 = self.c2f(a7, "model.8", 512, 1, True)
        s0 = self.conv_bn(a8, "model.9.cv1", 1, 1)
        s1 = self._pool5(s0)
        s2 = self._pool5(s1)
        s3 = self._pool5(s2)
        a9 = self.conv_bn(torch.cat([s0, s1, s2, s3], 1), "model.9.cv2", 1, 1, keep="a9")
        a12 = self.c2f(torch.cat([self._up(a9), a6], 1), "model.12", 256, 1, False)
        p3 = self.c2f(torch.cat([self._up(a12), a4], 1), "model.15", 128, 1, False)
        a16 = self.conv_bn(p3, "model.16", 3, 2)
        p4 = self.c2f(torch.cat([a16, a12], 1), "model.18", 256, 1, False)
        a19 = self.conv_bn(p4, "model.19", 3, 2)
        p5 = self.c2f(torch.cat([a19, a9], 1), "model.21", 512, 1, False)
        self.acts.update(a2=a2, a4=a4, a6=a6, a8=a8, a12=a12, p3=p3, p4=p4, p5=p5)
        out = {"box": [], "cls": [], "coef": []}
        for l, feat in enumerate((p3, p4, p5)):
            for br, key in (("cv2", "box"), ("cv3", "cls"), ("cv4", "coef")):
                t = self.conv_bn(feat, f"model.22.{br}.{l}.0", 3, 1)
                t = self.conv_bn(t, f"model.22.{br}.{l}.1", 3, 1)
                out[key].append(self.head_conv(t, f"model.22.{br}.{l}.2"))
        pr = self.conv_bn(p3, "model.22.proto.cv1", 3, 1)
        up = self._r(F.conv_transpose2d(pr, self.w["model.22.proto.upsample.weight"], stride=2))
        up = self._r(up + self.w["model.22.proto.upsample.bias"].view(1, -1, 1, 1))
        pr = self.conv_bn(up, "model.22.proto.cv2", 3, 1)
        out["proto"] = self.conv_bn(pr, "model.22.proto.cv3", 1, 1)
        return out


def calibrated_weights(seed: int = 0, size: int = 128, n: int = 2) -> dict:
    """Seeded test weights whose BN running statistics are set from a calibration batch, so every layer
    sees normalised inputs and the activations stay O(1) through the network (random He-init weights with
    identity BN shrink or blow up with depth).  γ ~ U(0.5, 1.5), β ~ U(-0.2, 0.2)."""
    w = P.make_weights(seed, random_bn=True)
    m = YoloSegRef(w, emulate_fp16=False, calibrate=True)
    m.forward(P.make_images(n, size, seed + 7))
    out = dict(w)
    for k, v in m.w.items():
        if "running" in k:
            out[k] = v.detach().cpu().numpy().astype(np.float32)
    return out


def forward_flops(size: int = 640) -> float:
    """Conv FLOPs of one image (2·P·Q·K·C·R·S, the reference's formula src/model.cpp:483; convT uses H·W)."""
    tot = 0.0
    grids = {}
    S = size
    # spatial output size of each layer, from the topology
    def hw(name):
        if name.startswith("model.0"):
            return S // 2
        if name.startswith("model.1") and not name.startswith(("model.12", "model.15", "model.16", "model.18", "model.19")):
            return S // 4
        if name.startswith("model.2."):
            return S // 4
        if name.startswith(("model.3", "model.4")):
            return S // 8
        if name.startswith(("model.5", "model.6")):
            return S // 16
        if name.startswith(("model.7", "model.8", "model.9")):
            return S // 32
        if name.startswith("model.12"):
            return S // 16
        if name.startswith("model.15"):
            return S // 8
        if name.startswith(("model.16", "model.18")):
            return S // 16
        if name.startswith(("model.19", "model.21")):
            return S // 32
        if name.startswith("model.22.proto.cv1") or name.startswith("model.22.proto.upsample"):
            return S // 8
        if name.startswith("model.22.proto"):
            return S // 4
        lvl = int(name.split(".")[3])
        return S // (8 << lvl)
    for kind, name, c, k, ks in P.conv_layers():
        h = hw(name)
        grids[name] = h
        tot += 2.0 * h * h * k * c * ks * ks
    return tot
