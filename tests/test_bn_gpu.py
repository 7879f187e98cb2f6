"""Training-mode BatchNorm + SiLU, bias add and bias gradient on the GPU (through the C ABI), against the CPU
restatement (oracle/bn_ref.py) on the same inputs and, when oracle/_ref/ref_bn is built, against the
reference's own kernels (src/bn.cu, src/misc.cu) run on the same GPU.

Each pass is checked on its own inputs: the apply and backward passes get this build's statistics, so a
mismatch points at one kernel.  Tolerances (written per check below):
  statistics     |Δ| ≤ 1e-5·(|ref| + 1)          (fp32 per-thread sums vs fp64; rsqrt.approx ≈ 2 ulp)
  fp16 outputs   |Δ| ≤ 1e-3·|ref| + 1e-3·max|ref|  (one fp16 rounding, ≈ 2^-10 relative)
  dz             |Δ| ≤ 2e-3·|ref| + 2e-3·max|ref|  (MUFU σ, cancellation in g − mean(g) − x̂·mean(g·x̂))
  dγ, dβ         |Δ| ≤ 1e-4·Σ|term| per channel    (fp32 partial sums over the batch)
Channels of a destination outside its slice must be untouched (bit-exact).
"""
import os
import subprocess
import tempfile

import numpy as np
import pytest
import torch

from objectsam_b200 import bn
from objectsam_b200.conv import DestSpec
from oracle import bn_ref, fsow

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BN = os.path.join(ROOT, "oracle", "_ref", "ref_bn")

# (N, H, W, C, act, res, dests [(ctot, choff, c0, c1, up)], accum, res_accum, z mean)
CASES = [
    (2, 16, 16, 64, 1, 0, [(64, 0, 0, 64, 1)], 0, 0, 0.0),
    (2, 20, 12, 32, 1, 1, [(96, 32, 0, 32, 1), (32, 0, 0, 32, 1)], 0, 0, 3.0),        # concat slice + residual
    (1, 8, 8, 128, 1, 0, [(256, 128, 0, 128, 2), (64, 0, 64, 128, 1)], 0, 0, -2.0),   # upsample + channel split
    (2, 10, 10, 224, 1, 0, [(64, 0, 0, 64, 1), (128, 0, 64, 192, 1), (32, 0, 192, 224, 1)], 0, 0, 0.5),  # head
    (3, 5, 5, 512, 1, 1, [(512, 0, 0, 512, 1)], 1, 1, 1.0),                           # 20²-level channels
    (4, 80, 80, 64, 1, 1, [(128, 64, 0, 64, 1), (64, 0, 0, 64, 1)], 1, 1, 0.25),       # M = 25600
    (2, 6, 6, 8, 0, 0, [(8, 0, 0, 8, 1)], 0, 0, 0.0),                                 # C = 8, no activation
    (1, 2, 1, 16, 1, 0, [(16, 0, 0, 16, 1)], 0, 0, 0.0),                              # M = 2
]
IDS = [f"{c[0]}x{c[1]}x{c[2]}x{c[3]}-d{len(c[6])}-act{c[4]}-res{c[5]}-acc{c[7]}" for c in CASES]
MOM, EPS = 0.03, 1e-3  # YOLOv8 BN (reference src/model.h ModelCfg bn_momentum / bn_eps)


def fp16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def make_case(case, seed):
    N, H, W, C, act, res, dests, accum, res_accum, zm = case
    r = np.random.default_rng(seed)
    d = {"z": fp16(zm + r.standard_normal((N, H, W, C)) * r.uniform(0.5, 2.0, C)),
         "gamma": r.uniform(0.5, 1.5, C).astype(np.float32), "beta": r.uniform(-0.5, 0.5, C).astype(np.float32),
         "run_mean": (zm + r.uniform(-0.2, 0.2, C)).astype(np.float32),
         "run_var": r.uniform(0.5, 2.0, C).astype(np.float32),
         "gw_gamma0": r.standard_normal(C).astype(np.float32), "gw_beta0": r.standard_normal(C).astype(np.float32)}
    if res:
        d["res"] = fp16(r.uniform(-1, 1, (N, H, W, C)))
        d["res_grad0"] = fp16(r.standard_normal((N, H, W, C)) * 0.1)
    for k, (ctot, choff, c0, c1, up) in enumerate(dests):
        d[f"dest{k}"] = fp16(r.uniform(-4, 4, (N, H * up, W * up, ctot)))
        d[f"grad{k}"] = fp16(r.standard_normal((N, H * up, W * up, ctot)) * 0.1)
    return d


def t16(a):
    return torch.from_numpy(np.ascontiguousarray(a)).half().to(DEV)


def t32(a):
    return torch.from_numpy(np.ascontiguousarray(a)).float().to(DEV)


def run_ours(case, d, fused=True):
    """The node through bn_forward_train (fused = True) or bn_forward_stats + bn_forward_apply, then the
    backward."""
    N, H, W, C, act, res, dests, accum, res_accum, zm = case
    z = t16(d["z"])
    gamma, beta, rm, rv = t32(d["gamma"]), t32(d["beta"]), t32(d["run_mean"]), t32(d["run_var"])
    mean, istd, scale, shift = (torch.empty(C, device=DEV) for _ in range(4))
    outs = [t16(d[f"dest{k}"]) for k in range(len(dests))]
    specs = [DestSpec(o, choff, c0, c1, up) for o, (_, choff, c0, c1, up) in zip(outs, dests)]
    if fused:
        bn.bn_forward_train(z, gamma, beta, rm, rv, MOM, EPS, mean, istd, scale, shift,
                            t16(d["res"]) if res else None, specs, bool(act))
    else:
        bn.bn_forward_stats(z, gamma, beta, rm, rv, MOM, EPS, mean, istd, scale, shift)
        bn.bn_forward_apply(z, scale, shift, t16(d["res"]) if res else None, specs, bool(act))
    grads = [t16(d[f"grad{k}"]) for k in range(len(dests))]
    dz = torch.empty_like(z)
    gwg, gwb = t32(d["gw_gamma0"]), t32(d["gw_beta0"])
    rg = t16(d["res_grad0"]) if res else None
    bn.bn_backward(z, mean, istd, scale, shift,
                   [DestSpec(g, choff, c0, c1, up) for g, (_, choff, c0, c1, up) in zip(grads, dests)], bool(act),
                   dz, gwg, gwb, bool(accum), rg, bool(res_accum))
    torch.cuda.synchronize()
    o = {k: v.cpu().numpy() for k, v in (("mean", mean), ("istd", istd), ("scale", scale), ("shift", shift),
                                          ("run_mean", rm), ("run_var", rv), ("gw_gamma", gwg), ("gw_beta", gwb))}
    o["dz"] = dz.float().cpu().numpy()
    for k, t in enumerate(outs):
        o[f"dest{k}"] = t.float().cpu().numpy()
    if res:
        o["res_grad"] = rg.float().cpu().numpy()
    return o


def close_stats(a, b, what):
    err = np.abs(a - b)
    lim = 1e-5 * (np.abs(b) + 1)
    assert (err <= lim).all(), f"{what}: max err {err.max():.3e}"


def close_f16(a, b, what, rel=1e-3):
    err = np.abs(a - b)
    lim = rel * np.abs(b) + rel * (np.abs(b).max() + 1e-6)
    assert (err <= lim).all(), f"{what}: {(err > lim).sum()} out of tolerance, max err {err.max():.3e}"


def check_dests_untouched(case, d, o):
    C = case[3]
    for k, (ctot, choff, c0, c1, up) in enumerate(case[6]):
        keep = np.ones(ctot, bool)
        keep[choff:choff + c1 - c0] = False
        assert np.array_equal(o[f"dest{k}"][..., keep], d[f"dest{k}"][..., keep]), f"dest{k}: other channels changed"


@pytest.mark.parametrize("case", CASES, ids=IDS)
@pytest.mark.parametrize("fused", [True, False], ids=["forward_train", "stats+apply"])
def test_bn_train_node_matches_oracle(cuda_lib, case, fused):
    N, H, W, C, act, res, dests, accum, res_accum, zm = case
    d = make_case(case, 7)
    o = run_ours(case, d, fused)
    st = bn_ref.bn_forward_stats(d["z"], d["gamma"], d["beta"], d["run_mean"], d["run_var"], MOM, EPS)
    for k in ("mean", "istd", "scale", "shift", "run_mean", "run_var"):
        close_stats(o[k], st[k], k)
    # apply on this build's scale/shift
    bufs = [d[f"dest{k}"].copy() for k in range(len(dests))]
    bn_ref.bn_forward_apply(d["z"], o["scale"], o["shift"], d.get("res"),
                            [(b, choff, c0, c1, up) for b, (_, choff, c0, c1, up) in zip(bufs, dests)], bool(act))
    for k, b in enumerate(bufs):
        close_f16(o[f"dest{k}"], b, f"dest{k}")
    check_dests_untouched(case, d, o)
    # backward on this build's statistics
    bw = bn_ref.bn_backward(d["z"], o["mean"], o["istd"], o["scale"], o["shift"],
                            [(d[f"grad{k}"], choff, c0, c1, up) for k, (_, choff, c0, c1, up) in enumerate(dests)],
                            bool(act), d["gw_gamma0"], d["gw_beta0"], bool(accum), d.get("res_grad0"), bool(res_accum))
    close_f16(o["dz"], bw["dz"], "dz", rel=2e-3)
    dA = bn_ref.gather_grad([(d[f"grad{k}"], choff, c0, c1, up) for k, (_, choff, c0, c1, up) in enumerate(dests)],
                            d["z"].shape)
    xh_max = (np.abs(d["z"] - o["mean"]) * o["istd"]).reshape(-1, C).max(0)
    tot = np.abs(dA).reshape(-1, C).sum(0) * 1.2 * (1 + xh_max)  # ≥ Σ|g|, Σ|g·x̂| (|silu'| < 1.1)
    for k in ("gw_gamma", "gw_beta"):
        base = np.abs(d[k + "0"]) if accum else 0
        assert (np.abs(o[k] - bw[k]) <= 1e-4 * (tot + base) + 1e-6).all(), f"{k}: max err {np.abs(o[k] - bw[k]).max():.3e}"
    if res:
        close_f16(o["res_grad"], bw["res_grad"], "res_grad")


@pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")
def test_bn_train_node_matches_reference_kernels(cuda_lib):
    """The whole node (stats → apply → backward) against the reference's own bn.cu on identical inputs."""
    ins, datas = {}, []
    for i, case in enumerate(CASES):
        N, H, W, C, act, res, dests, accum, res_accum, zm = case
        d = make_case(case, 100 + i)
        datas.append(d)
        meta = [0, N, H, W, C, act, res, len(dests), accum, res_accum] + [v for dd in dests for v in dd]
        ins[f"c{i}.meta"] = np.array(meta, np.int32)
        ins[f"c{i}.f"] = np.array([MOM, EPS], np.float32)
        for k, v in d.items():
            ins[f"c{i}.{k}"] = v
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        ref = fsow.load(os.path.join(td, "out.fsow"))
    for i, case in enumerate(CASES):
        o = run_ours(case, datas[i])
        p = f"c{i}."
        for k in ("mean", "istd", "scale", "shift", "run_mean", "run_var"):
            close_stats(o[k], ref[p + k], f"case {i} {k}")
        for k in range(len(case[6])):
            close_f16(o[f"dest{k}"], ref[p + f"dest{k}"], f"case {i} dest{k}", rel=2e-3)
        close_f16(o["dz"], ref[p + "dz"], f"case {i} dz", rel=5e-3)
        for k in ("gw_gamma", "gw_beta"):
            r = ref[p + k]
            assert np.abs(o[k] - r).max() <= 1e-3 * (np.abs(r).max() + 1), f"case {i} {k}"
        if case[5]:
            close_f16(o["res_grad"], ref[p + "res_grad"], f"case {i} res_grad")


def test_bn_workspace_returns_zeroed(cuda_lib):
    case = CASES[1]
    d = make_case(case, 3)
    C = case[3]
    ws = torch.zeros(int(cuda_lib.osam_bn_workspace_size(C)), dtype=torch.uint8, device=DEV)
    z = t16(d["z"])
    args = [t32(d[k]) for k in ("gamma", "beta", "run_mean", "run_var")]
    outs = [torch.empty(C, device=DEV) for _ in range(4)]
    first = None
    for _ in range(3):  # momentum 0: running statistics unchanged, so every call must give the same result
        bn.bn_forward_stats(z, *args, 0.0, EPS, *outs, ws=ws)
        torch.cuda.synchronize()
        assert int(ws.count_nonzero()) == 0, "workspace not returned zeroed"
        if first is None:
            first = [o.clone() for o in outs]
        for a, b in zip(first, outs):
            assert torch.equal(a, b)
    # bn_forward_train and the backward
    dests = case[6]
    bufs = [t16(d[f"dest{k}"]) for k in range(len(dests))]
    specs = [DestSpec(o, choff, c0, c1, up) for o, (_, choff, c0, c1, up) in zip(bufs, dests)]
    grads = [DestSpec(t16(d[f"grad{k}"]), choff, c0, c1, up) for k, (_, choff, c0, c1, up) in enumerate(dests)]
    dz = torch.empty_like(z)
    gg, gb = torch.zeros(C, device=DEV), torch.zeros(C, device=DEV)
    for _ in range(3):
        bn.bn_forward_train(z, *args, 0.0, EPS, *outs, t16(d["res"]), specs, True, ws=ws)
        bn.bn_backward(z, *outs, grads, True, dz, gg, gb, ws=ws)
        torch.cuda.synchronize()
        # the fp64 accumulators and the counter are zeroed again; the backward leaves its per-channel means
        # (2·C fp32) in the scratch at the end of the workspace (rewritten before every read)
        nz = torch.nonzero(ws).flatten()
        assert nz.numel() == 0 or int(nz.min()) >= ws.numel() - 8 * C - 256, "accumulators not returned zeroed"
        for a, b in zip(first, outs):
            close_stats(b.cpu().numpy(), a.cpu().numpy(), "fused statistics")


def test_bn_train_node_in_cuda_graph(cuda_lib):
    """forward_train → backward captured once and replayed: same results as eager (no allocation, no host
    sync)."""
    case = CASES[2]
    N, H, W, C, act, res, dests, accum, res_accum, zm = case
    d = make_case(case, 5)
    eager = run_ours(case, d)
    z = t16(d["z"])
    gamma, beta, rm, rv = t32(d["gamma"]), t32(d["beta"]), t32(d["run_mean"]), t32(d["run_var"])
    mean, istd, scale, shift = (torch.empty(C, device=DEV) for _ in range(4))
    outs = [t16(d[f"dest{k}"]) for k in range(len(dests))]
    grads = [t16(d[f"grad{k}"]) for k in range(len(dests))]
    dz = torch.empty_like(z)
    gwg, gwb = torch.zeros(C, device=DEV), torch.zeros(C, device=DEV)
    s = torch.cuda.Stream()
    ws = torch.zeros(int(cuda_lib.osam_bn_workspace_size(C)), dtype=torch.uint8, device=DEV)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        bn.bn_forward_train(z, gamma, beta, rm, rv, MOM, EPS, mean, istd, scale, shift, None,
                            [DestSpec(o, choff, c0, c1, up) for o, (_, choff, c0, c1, up) in zip(outs, dests)],
                            bool(act), ws=ws, stream=s)
        bn.bn_backward(z, mean, istd, scale, shift,
                       [DestSpec(t, choff, c0, c1, up) for t, (_, choff, c0, c1, up) in zip(grads, dests)],
                       bool(act), dz, gwg, gwb, False, ws=ws, stream=s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(dz.float().cpu(), torch.from_numpy(eager["dz"]))
    for k in range(len(dests)):
        assert torch.equal(outs[k].float().cpu(), torch.from_numpy(eager[f"dest{k}"]))
    assert torch.equal(gwg.cpu(), torch.from_numpy(eager["gw_gamma"]))
    del g


CHAN_CASES = [(1, 1), (300, 1), (25600, 1), (777, 3), (4096, 32), (25600, 64), (1000, 224), (50, 512), (9, 2048)]


@pytest.mark.parametrize("M,C", CHAN_CASES)
@pytest.mark.parametrize("accum", [0, 1])
def test_chan_sum(cuda_lib, M, C, accum):
    r = np.random.default_rng(M * 7 + C)
    x = fp16(r.standard_normal((M, C)))
    out0 = r.standard_normal(C).astype(np.float32)
    out = t32(out0)
    bn.chan_sum(t16(x), out, bool(accum))
    torch.cuda.synchronize()
    ref = bn_ref.chan_sum(x, out0, bool(accum))
    lim = 1e-5 * (np.abs(x).sum(0) + np.abs(out0) * accum) + 1e-6  # |Δ| ≤ 1e-5·Σ|x| (fp32 partial sums)
    assert (np.abs(out.cpu().numpy() - ref) <= lim).all()


@pytest.mark.parametrize("M,C", [(1, 1), (1000, 1), (6400, 64), (999, 3), (128, 224)])
def test_add_bias(cuda_lib, M, C):
    r = np.random.default_rng(M + C)
    y0 = fp16(r.uniform(-3, 3, (M, C)))
    b = r.uniform(-1, 1, C).astype(np.float32)
    y = t16(y0)
    bn.add_bias(y, t32(b))
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), bn_ref.add_bias(y0, b)), "fp32 add + one fp16 rounding is exact"


def test_bn_eval_scale(cuda_lib):
    r = np.random.default_rng(1)
    C = 200
    g, b, m = (r.uniform(-1, 1, C).astype(np.float32) for _ in range(3))
    v = r.uniform(0.1, 3, C).astype(np.float32)
    sc, sh = torch.empty(C, device=DEV), torch.empty(C, device=DEV)
    bn.bn_eval_scale(t32(g), t32(b), t32(m), t32(v), EPS, sc, sh)
    rsc, rsh = bn_ref.bn_eval_scale(g, b, m, v, EPS)
    close_stats(sc.cpu().numpy(), rsc, "scale")
    close_stats(sh.cpu().numpy(), rsh, "shift")


@pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")
def test_chan_sum_and_add_bias_match_reference_kernels(cuda_lib):
    ins, cases = {}, [(1, 25600, 1, 0), (1, 4096, 64, 1), (2, 999, 3, 0), (2, 6400, 64, 0)]
    r = np.random.default_rng(9)
    for i, (op, M, C, accum) in enumerate(cases):
        if op == 1:
            ins[f"c{i}.meta"] = np.array([1, M, C, accum], np.int32)
            ins[f"c{i}.x"] = fp16(r.standard_normal((M, C)))
            ins[f"c{i}.out0"] = r.standard_normal(C).astype(np.float32)
        else:
            ins[f"c{i}.meta"] = np.array([2, M, C], np.int32)
            ins[f"c{i}.y"] = fp16(r.uniform(-3, 3, (M, C)))
            ins[f"c{i}.bias"] = r.uniform(-1, 1, C).astype(np.float32)
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        ref = fsow.load(os.path.join(td, "out.fsow"))
    for i, (op, M, C, accum) in enumerate(cases):
        if op == 1:
            out = t32(ins[f"c{i}.out0"])
            bn.chan_sum(t16(ins[f"c{i}.x"]), out, bool(accum))
            lim = 1e-5 * (np.abs(ins[f"c{i}.x"]).sum(0) + np.abs(ins[f"c{i}.out0"])) + 1e-6
            assert (np.abs(out.cpu().numpy() - ref[f"c{i}.out"]) <= lim).all()
        else:
            y = t16(ins[f"c{i}.y"])
            bn.add_bias(y, t32(ins[f"c{i}.bias"]))
            assert np.array_equal(y.float().cpu().numpy(), ref[f"c{i}.y"].reshape(M, C))


@pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")
def test_stem_wgrad_matches_reference_kernel(cuda_lib):
    """The stem's weight gradient (3×3/s2/p1, C = 3 → K = 32) against the reference's own WMMA kernel
    wgrad_rgb_s2 (src/misc.cu:193-273) on identical inputs; both accumulate in fp32 and round to fp16."""
    from objectsam_b200.conv import ConvGeom, ConvOp
    N, H, W, K = 2, 256, 384, 32
    r = np.random.default_rng(21)
    x = fp16(r.uniform(0, 1, (N, H, W, 3)))
    dz = fp16(r.uniform(-1, 1, (N, H // 2, W // 2, K)))
    ins = {"c0.meta": np.array([3, N, H, W, K], np.int32), "c0.x": x, "c0.dz": dz}
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        ref = fsow.load(os.path.join(td, "out.fsow"))
    assert ref["c0.ran"][0] == 1.0, "the reference declined the shape"
    op = ConvOp().init(ConvGeom(N, H, W, 3, K, 3, 3, 2, 1))
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    dw = torch.empty(K, 3, 3, 3, dtype=torch.half, device=DEV)
    op.wgrad(t16(x), t16(dz), dw, ws=ws)
    torch.cuda.synchronize()
    close_f16(dw.float().cpu().numpy(), ref["c0.dw"], "stem dw", rel=2e-3)


@pytest.mark.skipif(not os.path.exists(REF_BN), reason="oracle/_ref/ref_bn not built (make -C oracle)")
def test_sppf_bwd_matches_reference_kernel(cuda_lib):
    """SPPF backward against the reference's own sppf_pool_bwd (src/misc.cu:155-166): its fp32 atomics add in
    any order, so one fp16 rounding step of difference is allowed."""
    from objectsam_b200.conv import sppf_pool_bwd, sppf_pool_fwd
    N, H, W, c = 2, 20, 20, 128
    r = np.random.default_rng(31)
    cat = torch.zeros(N, H, W, 4 * c, dtype=torch.half, device=DEV)
    cat[..., :c] = t16(r.standard_normal((N, H, W, c)))
    sppf_pool_fwd(cat, N, H, W, c)
    dcat = t16(fp16(r.standard_normal((N, H, W, 4 * c)) * 0.5))
    ins = {"c0.meta": np.array([4, N, H, W, c], np.int32), "c0.cat": cat.float().cpu().numpy(),
           "c0.dcat": dcat.float().cpu().numpy()}
    with tempfile.TemporaryDirectory() as td:
        fsow.save(os.path.join(td, "in.fsow"), ins)
        subprocess.run([REF_BN, os.path.join(td, "in.fsow"), os.path.join(td, "out.fsow")], check=True, timeout=300)
        ref = fsow.load(os.path.join(td, "out.fsow"))
    sppf_pool_bwd(cat, dcat, N, H, W, c)
    torch.cuda.synchronize()
    close_f16(dcat.float().cpu().numpy(), ref["c0.dcat"], "sppf dcat", rel=1e-3)
