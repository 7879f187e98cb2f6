"""Training pass of the whole network (reference Model::forward(true) + Model::backward, src/model.cpp:383-470)
through the C ABI: batch-statistics BN forward, then the backward of every node from given head gradients,
against torch autograd of the CPU restatement in training mode (oracle/yolo_ref.py, fp16 storage emulated).

Tolerances, against fp64 autograd: a head's max error ≤ 2× the error that the reference's fp16 storage
points alone cause (the fp32 restatement with fp16 rounding where the reference stores fp16) + 1e-2·max;
each parameter gradient's relL2 = ‖ours − ref‖/‖ref‖ ≤ max(2× that of the fp16-storage restatement, 1e-2).
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from objectsam_b200.model import Model
from oracle import fsow, yolo_params, yolo_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TRAIN = os.path.join(ROOT, "oracle", "_ref", "ref_train")


def _setup(N, S, seed):
    w = yolo_ref.calibrated_weights(seed, S)
    imgs = yolo_params.make_images(N, S, seed + 1)
    m = Model(N, S)
    m.load(w)
    m.sync_weights()
    m.train_init()
    m.input().copy_(torch.from_numpy(imgs).half())
    return m, w, imgs


def _head_grads(m, S, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    grads = {}
    names = [f"out.{k}{l}" for k in ("box", "cls", "coef") for l in range(3)] + ["out.proto"]
    for n in names:
        t = m.act_grad(n)
        r = (torch.randn(t.shape, generator=g) * 0.05).half()
        t.copy_(r.to(DEV))
        grads[n] = r.float()
    return grads


def _oracle(w, imgs, G, fp16):
    """Outputs and parameter gradients of the CPU restatement in training mode: fp64 exact, or fp32 with the
    reference's fp16 storage points emulated."""
    ref = yolo_ref.YoloSegRef(w, emulate_fp16=fp16, dtype=torch.float32 if fp16 else torch.float64, train=True)
    out = ref.forward(imgs)
    d = torch.float32 if fp16 else torch.float64
    loss = sum((out[k][l] * G[f"out.{k}{l}"].to(d).permute(0, 3, 1, 2)).sum() for k in ("box", "cls", "coef")
               for l in range(3))
    loss = loss + (out["proto"] * G["out.proto"].to(d).permute(0, 3, 1, 2)).sum()
    loss.backward()
    grads = {n: t.grad.double().numpy() for n, t in ref.w.items() if t.grad is not None}
    return {k: ([t.detach().double() for t in v] if isinstance(v, list) else v.detach().double())
            for k, v in out.items()}, grads


@pytest.mark.parametrize("N,S", [(2, 256)])
def test_train_pass_matches_autograd(cuda_lib, N, S):
    """Against fp64 autograd; the allowed error is twice what the reference's fp16 storage alone causes
    (the same network in fp32 with fp16 rounding at the reference's storage points), or 1e-2."""
    m, w, imgs = _setup(N, S, 3)
    m.forward_train(0.03)
    G = _head_grads(m, S, 9)
    m.backward()
    torch.cuda.synchronize()
    o64, g64 = _oracle(w, imgs, G, fp16=False)
    o16, g16 = _oracle(w, imgs, G, fp16=True)
    for key, kind in (("box", 0), ("cls", 1), ("coef", 2)):
        for l in range(3):
            y = m.head(kind, l).double().cpu().permute(0, 3, 1, 2)
            r, r16 = o64[key][l], o16[key][l]
            e, e16 = (y - r).abs().max().item(), (r16 - r).abs().max().item()
            assert e <= 2 * e16 + 1e-2 * r.abs().max().item(), f"{key}{l}: max err {e:.3e} (fp16 storage {e16:.3e})"
    worst, checked = [], 0
    for name, want in g64.items():
        got = m.get_grad(name, want.shape).astype(np.float64)
        nrm = np.linalg.norm(want) + 1e-30
        rel, rel16 = np.linalg.norm(got - want) / nrm, np.linalg.norm(g16[name] - want) / nrm
        worst.append((rel, rel16, name))
        checked += 1
        assert rel <= max(2 * rel16, 1e-2), f"{name}: relL2 {rel:.3e} (fp16 storage {rel16:.3e})"
    assert checked > 150, f"only {checked} parameter gradients compared"
    worst.sort(reverse=True)
    print(f"{checked} parameter gradients; worst relL2 {worst[0][0]:.3e} ({worst[0][2]}, fp16 storage "
          f"{worst[0][1]:.3e})")


def test_train_backward_in_buckets_equals_whole(cuda_lib):
    """Backward run as consecutive node ranges (last first, as the data-parallel buckets run it) gives the
    gradients of one whole backward (up to the order of the weight gradients' fp32 atomics)."""
    m, w, imgs = _setup(2, 128, 5)
    m.forward_train(0.0)
    _head_grads(m, 128, 4)
    m.backward()
    whole = m.grad_arena().clone()
    n = m.num_launches()
    cuts = [n, 50, 31, 7, 0]
    for hi, lo in zip(cuts, cuts[1:]):
        m.backward_nodes(lo, hi - lo)
    torch.cuda.synchronize()
    again = m.grad_arena()
    assert torch.norm(again - whole) <= 1e-5 * torch.norm(whole)


@pytest.mark.skipif(not os.path.exists(REF_TRAIN), reason="oracle/_ref/ref_train not built (make -C oracle)")
def test_train_pass_matches_reference_cudnn(cuda_lib):
    """The same weights, images and head gradients through the reference's own training pass (its cuDNN fp16
    build: Model::forward(true) + backward); both are measured against fp64 autograd and this build's error
    may be at most twice the reference's (or 1e-2) on every head and every parameter gradient.  The cuDNN
    build tunes its algorithms at start-up and some of them accumulate in a run-dependent order, so its own
    error moves between runs (model.2.m.0.cv2.bn.bias: relL2 5.3e-2 … 6.7e-2 on identical inputs, while
    this build's is the same every run); a gradient also passes when it is within twice the error that the
    reference's fp16 storage points alone cause (the fp32 restatement rounding where the reference stores
    fp16), the run-independent form of the same bound."""
    N, S = 2, 256
    m, w, imgs = _setup(N, S, 3)
    m.forward_train(0.03)
    G = _head_grads(m, S, 9)
    m.backward()
    torch.cuda.synchronize()
    ins = {"images": imgs.astype(np.float32)}
    ins.update({f"grad.{k}": v.numpy() for k, v in G.items()})
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "w.fsow"), w)
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_TRAIN, os.path.join(td, "w.fsow"), os.path.join(td, "in.fsow"), os.path.join(td, "o.fsow")],
                       check=True, timeout=600)
        ref = fsow.load(os.path.join(td, "o.fsow"))
    o64, g64 = _oracle(w, imgs, G, fp16=False)
    _, g16 = _oracle(w, imgs, G, fp16=True)
    for key, kind in (("box", 0), ("cls", 1), ("coef", 2)):
        for l in range(3):
            y = m.head(kind, l).double().cpu().permute(0, 3, 1, 2)
            rr = torch.from_numpy(ref[f"out.{key}{l}"]).double().permute(0, 3, 1, 2)
            r = o64[key][l]
            e, eref = (y - r).abs().max().item(), (rr - r).abs().max().item()
            assert e <= 2 * eref + 1e-2 * r.abs().max().item(), f"{key}{l}: max err {e:.3e}, reference {eref:.3e}"
    worst = []
    for name, want in g64.items():
        got = m.get_grad(name, want.shape).astype(np.float64)
        theirs = ref["grad." + name].astype(np.float64)
        nrm = np.linalg.norm(want) + 1e-30
        rel, rref = np.linalg.norm(got - want) / nrm, np.linalg.norm(theirs - want) / nrm
        r16 = np.linalg.norm(g16[name] - want) / nrm
        worst.append((rel / max(rref, 1e-12), rel, rref, name))
        assert rel <= max(2 * rref, 2 * r16, 1e-2), \
            f"{name}: relL2 {rel:.3e}, reference {rref:.3e}, fp16 storage {r16:.3e}"
    worst.sort(reverse=True)
    print(f"{len(worst)} gradients; largest ratio to the reference's error {worst[0][0]:.2f} ({worst[0][3]}: "
          f"{worst[0][1]:.3e} vs {worst[0][2]:.3e})")
