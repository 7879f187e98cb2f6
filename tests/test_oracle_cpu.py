"""CPU tests of the oracle (the checker) against the golden vectors and known answers."""
import os

import numpy as np
import pytest
import torch

from oracle import fsow, postproc_ref, yolo_params, yolo_ref

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _golden_cases():
    z = np.load(os.path.join(GOLDEN, "postproc_golden.npz"))
    for ci in range(int(z["n_cases"])):
        yield ci, {k[len(f"c{ci}_"):]: z[k] for k in z.files if k.startswith(f"c{ci}_")}


@pytest.mark.parametrize("ci", range(4))
def test_postproc_oracle_matches_reference_ref_detect(ci):
    """The numpy restatement reproduces archive/tools/ref_detect.py exactly (scores, boxes, masks)."""
    case = dict(_golden_cases())[ci]
    o0 = case["o0"].astype(np.float32)
    o1 = case["o1"].astype(np.float32)
    S, cth, nth, mth, amin, mdet = case["cfg"]
    xywh, conf, coefs = o0[:4].T, o0[4], o0[5:].T
    det = postproc_ref.detect_one(xywh, conf, coefs, o1, int(S), conf_th=cth, nms_iou=nth, max_det=int(mdet),
                                  area_min=int(amin), mask_iou=mth)
    sel = det["sel"]
    np.testing.assert_array_equal(det["score"][sel], case["score"])
    np.testing.assert_array_equal(det["box"][sel], case["box"])
    grid = np.unpackbits(case["grid"], axis=-1)[..., : int(case["grid_shape"][-1])].astype(bool)
    np.testing.assert_array_equal(det["masks"][sel], grid.reshape(tuple(case["grid_shape"])))


def test_nms_known_answer():
    """Hand-checked case: strict '>' at the threshold, union>0 guard, stable tie order, max_det."""
    boxes = np.array([[0, 0, 10, 10], [0, 0, 10, 10], [5, 0, 15, 10], [100, 100, 100, 110], [0, 0, 10, 7]],
                     np.float32)
    # 0 kept; 1 identical (IoU 1) suppressed; 2 IoU 50/150 kept; 3 zero-area box kept (union > 0 guard);
    # 4 IoU with 0 = 70/100 rounds to exactly float32(0.7) and the test is strict '>', so it is kept.
    assert np.float32(np.float32(70) / np.float32(100)) == np.float32(0.7)
    assert postproc_ref.greedy_nms(boxes, 0.7, 10) == [0, 2, 3, 4]
    assert postproc_ref.greedy_nms(boxes, 0.7, 2) == [0, 2]
    conf = np.array([0.5, 0.9, 0.5, 0.2, 0.9], np.float32)
    assert list(postproc_ref.nms_order(conf, 0.25)) == [1, 4, 0, 2]


@pytest.mark.parametrize("thr", [0.7, 0.5, 1 / 3, 0.45, 0.0, 1e-7, 0.999, -0.25])
def test_exact_iou_threshold_identity(thr):
    """The GPU NMS decides float32(inter / union) > thr without dividing: inter > union·m in double, m the
    midpoint between thr and the next float up, ties going up when thr's last bit is 1.  Same answers as
    the float32 division on random, near-threshold and small-integer (exact-fraction) operands."""
    import struct
    rng = np.random.Generator(np.random.PCG64(0))
    t = np.float32(thr)
    nx = np.nextafter(t, np.float32(np.inf))
    mid = (float(t) + float(nx)) * 0.5
    odd = struct.unpack("<I", struct.pack("<f", t))[0] & 1
    u = (rng.random(100000) * 1e5 + 1e-3).astype(np.float32)
    inter = (u.astype(np.float64) * float(t) * (1 + rng.integers(-40, 40, 100000) * 6e-8)).astype(np.float32)
    a, b = rng.integers(1, 200, 50000).astype(np.float32), rng.integers(1, 200, 50000).astype(np.float32)
    inter, u = np.concatenate([np.abs(inter), np.minimum(a, b)]), np.concatenate([u, np.maximum(a, b)])
    ref = (inter / u).astype(np.float32) > t
    p = u.astype(np.float64) * mid
    got = (inter.astype(np.float64) > p) | ((inter.astype(np.float64) == p) & bool(odd))
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("kind", ["mixed", "grid", "dense", "sparse"])
def test_greedy_nms_vec_matches_scalar(kind):
    """The vectorised greedy NMS (used to check the GPU on thousands of candidates) keeps exactly the
    boxes of the scalar restatement of ref_detect's loop."""
    boxes = postproc_ref.stress_boxes(kind, 400, 5)
    for thr, md in ((0.5, 300), (0.7, 40), (1 / 3, 1000)):
        assert postproc_ref.greedy_nms_vec(boxes, thr, md) == postproc_ref.greedy_nms(boxes, thr, md)


def test_dfl_decode_known_answer():
    """A one-hot DFL distribution decodes to its bin; anchors are cell centres × stride."""
    N, H, W = 1, 2, 2
    box = [np.full((N, 64, H * 2 ** (2 - l), W * 2 ** (2 - l)), -30.0, np.float32) for l in range(3)]
    for b in box:
        b[:, 0 * 16 + 3] = 30.0   # left  = 3
        b[:, 1 * 16 + 1] = 30.0   # top   = 1
        b[:, 2 * 16 + 4] = 30.0   # right = 4
        b[:, 3 * 16 + 2] = 30.0   # bottom= 2
    cls = [np.zeros((N, 1) + b.shape[2:], np.float32) for b in box]
    coef = [np.zeros((N, 32) + b.shape[2:], np.float32) for b in box]
    xywh, conf, _ = postproc_ref.decode(box, cls, coef)
    # first anchor of level 0: cell (0,0) → anchor (0.5, 0.5); x1=-2.5 y1=-0.5 x2=4.5 y2=2.5 → ×8
    np.testing.assert_allclose(xywh[0, 0], [8 * 1.0, 8 * 1.0, 8 * 7.0, 8 * 3.0], atol=1e-4)
    np.testing.assert_allclose(conf, 0.5)


def test_fsow_roundtrip(tmp_path):
    t = {"a.weight": np.arange(24, dtype=np.float32).reshape(2, 3, 4), "b": np.array([1, 2], np.int32),
         "m": np.array([[1, 0]], np.uint8), "s": np.float32(3.5).reshape(())}
    p = str(tmp_path / "x.fsow")
    fsow.save(p, t)
    r = fsow.load(p)
    assert set(r) == set(t)
    for k in t:
        np.testing.assert_array_equal(r[k], t[k])
        assert r[k].dtype == np.asarray(t[k]).dtype
    with open(p, "r+b") as f:
        f.write(b"XXXX")
    with pytest.raises(ValueError):
        fsow.load(p)


def test_param_table_matches_yolov8s_seg():
    shapes = yolo_params.param_shapes()
    assert yolo_params.n_params() == 11790467  # 11.8 M (docs/SPEC.md:18-23)
    assert shapes["model.22.cv2.0.2.weight"] == (64, 64, 1, 1)  # 4·reg_max box channels
    assert shapes["model.22.proto.upsample.weight"] == (128, 128, 2, 2)
    assert shapes["model.9.cv2.conv.weight"] == (512, 1024, 1, 1)
    assert len([l for l in yolo_params.conv_layers()]) == 76  # 70 reference conv nodes + 6 unfused head convs


def test_forward_flops_match_survey():
    assert abs(yolo_ref.forward_flops(640) / 1e9 - 39.92) < 0.01
    assert abs(yolo_ref.forward_flops(1024) / 1e9 - 102.18) < 0.01


def _network_golden_cases():
    z = np.load(os.path.join(GOLDEN, "network_golden.npz"))
    for ci in range(int(z["n_cases"])):
        seed, n, s = (int(v) for v in z[f"c{ci}_cfg"])
        yield ci, seed, n, s, {k[len(f"c{ci}_"):]: z[k] for k in z.files if k.startswith(f"c{ci}_fp")}


@pytest.mark.parametrize("ci", range(2))
def test_network_oracle_matches_reference_cudnn_golden(ci):
    """Pins the network restatement (oracle/yolo_ref.py) to the reference itself on CPU: the committed
    outputs of the reference's own cuDNN build (tests/golden/make_network_golden.py runs
    oracle/_ref/ref_forward_fp32 / _fp16, built from its sources) on BN-calibrated weights and seeded
    images.  fp32 against the reference's fp32 parity build: relL2 <= 1e-3 per head tensor, the
    reference's own parity bar (tests/parity.cpp:23-29).  The fp16-storage emulation against its fp16
    production build: two fp16 evaluations of a 60-conv chain that round at the same points still drift
    apart by accumulation order, so both are measured against the float64 network and the emulation's
    relL2 error may be at most 1.5x the reference fp16 build's own (plus 1e-3)."""
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    _, seed, n, s, gold = dict((c[0], c) for c in _network_golden_cases())[ci]
    w = yolo_ref.calibrated_weights(seed, 128)
    imgs = yolo_params.make_images(n, s, seed + 100)

    def heads(emulate, dtype=torch.float32):
        o = yolo_ref.YoloSegRef(w, emulate_fp16=emulate, dtype=dtype).forward(imgs)
        d = {f"out.{k}{l}": o[k][l] for k in ("box", "cls", "coef") for l in range(3)}
        d["out.proto"] = o["proto"]
        return {k: t.double().permute(0, 2, 3, 1).numpy() for k, t in d.items()}

    def rel(a, b):
        return np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-30)

    o32, o16, o64 = heads(False), heads(True), heads(False, torch.float64)
    for name, y in o32.items():
        r = gold[f"fp32_{name}"].astype(np.float64)
        assert y.shape == r.shape, f"fp32 {name}: shape {y.shape} vs {r.shape}"
        assert rel(y, r) <= 1e-3, f"fp32 {name}: relL2 {rel(y, r):.2e} > 1e-3"
        r16 = gold[f"fp16_{name}"].astype(np.float64)
        e_ours, e_ref = rel(o16[name], o64[name]), rel(r16, o64[name])
        assert e_ours <= 1.5 * e_ref + 1e-3, f"fp16 {name}: relL2 vs fp64 {e_ours:.2e}, reference {e_ref:.2e}"


def test_oracle_forward_shapes_and_fp16_emulation_close_to_fp64():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    w = yolo_params.make_weights(1, random_bn=True)
    img = yolo_params.make_images(1, 128, 1)
    o16 = yolo_ref.YoloSegRef(w, emulate_fp16=True).forward(img)
    o64 = yolo_ref.YoloSegRef(w, emulate_fp16=False, dtype=torch.float64).forward(img)
    assert tuple(o16["proto"].shape) == (1, 32, 32, 32)
    assert [tuple(t.shape) for t in o16["box"]] == [(1, 64, 16, 16), (1, 64, 8, 8), (1, 64, 4, 4)]
    for k in ("box", "cls", "coef"):
        for a, b in zip(o16[k], o64[k]):
            scale = b.abs().max().item()
            assert (a.double() - b).abs().max().item() <= 2e-2 * scale + 1e-3


# ---------------------------------------------------------------- training BN + SiLU restatement (oracle/bn_ref.py)
@pytest.mark.parametrize("act,res", [(1, 1), (1, 0), (0, 0)])
def test_bn_oracle_matches_torch_autograd(act, res):
    """One conv+BN+SiLU node in training mode, two destinations (a concat slice and a 2× upsample of a channel
    subset): the restatement's statistics, running-statistics update and backward (dz, dγ, dβ, residual
    gradient) against torch batch_norm + SiLU autograd in fp64.  Tolerance 1e-4 relative to each tensor's
    max: the restatement does its elementwise math in fp32 and rounds dz to fp16, as the reference does."""
    from oracle import bn_ref
    r = np.random.default_rng(3)
    N, H, W, C, mom, eps = 2, 6, 5, 16, 0.03, 1e-3
    f16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)
    z = f16(1.5 + r.standard_normal((N, H, W, C)))
    gamma, beta = r.uniform(0.5, 1.5, C).astype(np.float32), r.uniform(-0.5, 0.5, C).astype(np.float32)
    rm0, rv0 = r.uniform(1, 2, C).astype(np.float32), r.uniform(0.5, 2, C).astype(np.float32)
    resv = f16(r.uniform(-1, 1, z.shape)) if res else None
    dests = [(32, 8, 0, 16, 1), (8, 0, 8, 16, 2)]
    grads = [f16(r.standard_normal((N, H * up, W * up, ct)) * 0.1) for ct, _, _, _, up in dests]

    st = bn_ref.bn_forward_stats(z, gamma, beta, rm0, rv0, mom, eps)
    bw = bn_ref.bn_backward(z, st["mean"], st["istd"], st["scale"], st["shift"],
                            [(g, choff, c0, c1, up) for g, (_, choff, c0, c1, up) in zip(grads, dests)], act,
                            res_grad=np.zeros_like(z) if res else None)

    d = torch.float64
    zt = torch.tensor(z, dtype=d, requires_grad=True)
    gt, bt = torch.tensor(gamma, dtype=d, requires_grad=True), torch.tensor(beta, dtype=d, requires_grad=True)
    rm, rv = torch.tensor(rm0, dtype=d), torch.tensor(rv0, dtype=d)
    y = torch.nn.functional.batch_norm(zt.permute(0, 3, 1, 2), rm, rv, gt, bt, training=True, momentum=mom,
                                       eps=eps).permute(0, 2, 3, 1)
    a = torch.nn.functional.silu(y) if act else y
    rt = torch.tensor(resv, dtype=d, requires_grad=True) if res else None
    if res:
        a = a + rt
    loss = 0
    for g, (ct, choff, c0, c1, up) in zip(grads, dests):
        s = a[..., c0:c1]
        if up == 2:
            s = s.repeat_interleave(2, 1).repeat_interleave(2, 2)
        loss = loss + (s * torch.tensor(g[..., choff:choff + c1 - c0], dtype=d)).sum()
    loss.backward()

    def close(x, ref, tol=1e-4):
        ref = np.asarray(ref, np.float64)
        assert np.abs(np.asarray(x, np.float64) - ref).max() <= tol * (np.abs(ref).max() + 1e-12)

    close(st["mean"], zt.detach().mean((0, 1, 2)).numpy(), 1e-6)
    close(st["istd"], 1 / np.sqrt(zt.detach().var((0, 1, 2), unbiased=False).numpy() + eps), 1e-6)
    close(st["run_mean"], rm.numpy(), 1e-6)
    close(st["run_var"], rv.numpy(), 1e-6)
    close(bw["dz"], zt.grad.numpy(), 2e-3)  # dz is rounded to fp16
    close(bw["gw_gamma"], gt.grad.numpy())
    close(bw["gw_beta"], bt.grad.numpy())
    if res:
        close(bw["res_grad"], rt.grad.numpy(), 1e-3)


def test_chan_sum_and_add_bias_oracle():
    from oracle import bn_ref
    x = np.arange(12, dtype=np.float32).reshape(4, 3)
    assert np.array_equal(bn_ref.chan_sum(x), np.array([18, 22, 26], np.float32))
    assert np.array_equal(bn_ref.chan_sum(x, np.ones(3, np.float32), True), np.array([19, 23, 27], np.float32))
    y = bn_ref.add_bias(np.full((2, 3), 2048, np.float32), np.array([0.5, 1.0, 1.5], np.float32))
    # fp16 spacing at 2048 is 2: 2048.5 → 2048, 2049 ties to even → 2048, 2049.5 → 2050
    assert np.array_equal(y, np.array([[2048, 2048, 2050]] * 2, np.float32))


def test_mask_loss_oracle_matches_torch_autograd():
    """The mask-loss restatement against torch autograd of Σ_pos Σ_crop BCE-with-logits(coef·proto, bit)·inv
    (fp64): loss, and its gradients ·gk for proto and the positives' coefficients."""
    from oracle import mask_loss_ref
    r = np.random.default_rng(5)
    B, S, G = 1, 128, 3
    Hp = Wp = S // 4
    lv = [(S // 8, S // 8), (S // 16, S // 16), (S // 32, S // 32)]
    A = sum(h * w for h, w in lv)
    coef = [r.uniform(-1, 1, (B, h, w, 32)).astype(np.float32) for h, w in lv]
    proto = r.uniform(-1, 1, (B, Hp, Wp, 32)).astype(np.float32)
    box = np.array([[[10, 12, 90, 70], [40, 40, 127, 120], [3, 50, 30, 126]]], np.float32)
    bits = (r.random((B, G, Hp * Wp)) < 0.4).astype(np.uint32)
    words = (bits.reshape(B, G, -1, 32) << np.arange(32, dtype=np.uint32)).sum(-1, dtype=np.uint64).astype(np.uint32)
    words = words.view(np.int32)
    sel = np.array([5, 77, 300, A - 1])
    pos = np.zeros((B, A), np.int32)
    pos[0, :4] = sel
    agt = np.full((B, A), -1, np.int32)
    agt[0, sel] = [0, 1, 2, 1]
    npos = np.array([4], np.int32)
    fg, scale, gain = 4.0, 8.0, 7.5
    dp, dc, loss = mask_loss_ref.mask_loss(coef, proto, npos, pos, agt, box, words, fg, scale, S, gain)

    pt = torch.tensor(proto, dtype=torch.float64, requires_grad=True)
    cts = [torch.tensor(c, dtype=torch.float64, requires_grad=True) for c in coef]
    tot = 0
    for i, a in enumerate(sel):
        j = agt[0, a]
        x1, y1, x2, y2 = (box[0, j] / S).astype(np.float64)
        inv = 1 / (Hp * Wp * (x2 - x1) * (y2 - y1))
        px = torch.arange(Wp, dtype=torch.float64)
        py = torch.arange(Hp, dtype=torch.float64)
        m = ((px[None, :] >= x1 * Wp) & (px[None, :] < x2 * Wp) & (py[:, None] >= y1 * Hp) & (py[:, None] < y2 * Hp))
        l, h, w = mask_loss_ref.anchor_of(lv, int(a))
        z = pt[0] @ cts[l][0, h, w]
        y = torch.tensor(bits[0, j].reshape(Hp, Wp), dtype=torch.float64)
        bce = torch.nn.functional.binary_cross_entropy_with_logits(z, y, reduction="none")
        tot = tot + (bce * m).sum() * inv
    tot.backward()
    gk = gain * B / fg * scale
    assert abs(loss - tot.item()) <= 2e-6 * abs(tot.item())  # inv in fp32 in the restatement
    assert np.abs(dp - pt.grad.numpy() * gk).max() <= 1e-5 * np.abs(dp).max()
    for a in sel:
        l, h, w = mask_loss_ref.anchor_of(lv, int(a))
        want = cts[l].grad[0, h, w].numpy() * gk
        assert np.abs(dc[(0, int(a))] - want).max() <= 1e-5 * np.abs(want).max()


@pytest.mark.parametrize("ties", [False, True])
def test_sppf_oracle_matches_torch_autograd(ties):
    """The SPPF restatement (forward chain and first-max backward) against torch max_pool2d autograd; with
    ties (values from a handful of integers) torch's CPU max-pool also takes the first maximum of the window
    in row-major order, so the routing must agree exactly."""
    from oracle import sppf_ref
    r = np.random.default_rng(2)
    N, H, W, c = 2, 9, 11, 8
    x = (r.integers(-2, 3, (N, H, W, c)) if ties else r.standard_normal((N, H, W, c))).astype(np.float32)
    cat = np.zeros((N, H, W, 4 * c), np.float32)
    cat[..., :c] = x
    for k in range(1, 4):
        cat[..., k * c:(k + 1) * c] = sppf_ref.pool5_fwd(cat[..., (k - 1) * c:k * c])
    dcat = (r.integers(-8, 9, (N, H, W, 4 * c)) / 8).astype(np.float32)  # exact in fp16 and in fp32 sums
    got = sppf_ref.sppf_bwd(cat, dcat, c)
    xt = torch.tensor(x, dtype=torch.float64).permute(0, 3, 1, 2).requires_grad_(True)
    s1 = torch.nn.functional.max_pool2d(xt, 5, 1, 2)
    s2 = torch.nn.functional.max_pool2d(s1, 5, 1, 2)
    s3 = torch.nn.functional.max_pool2d(s2, 5, 1, 2)
    assert np.array_equal(s3.detach().permute(0, 2, 3, 1).numpy(), cat[..., 3 * c:])
    g = lambda k: torch.tensor(dcat[..., k * c:(k + 1) * c], dtype=torch.float64).permute(0, 3, 1, 2)
    ((s1 * g(1)).sum() + (s2 * g(2)).sum() + (s3 * g(3)).sum()).backward()
    want = dcat[..., :c] + xt.grad.permute(0, 2, 3, 1).numpy()
    assert np.array_equal(got[..., :c], want.astype(np.float16).astype(np.float32))
    assert np.array_equal(got[..., c:], dcat[..., c:])
