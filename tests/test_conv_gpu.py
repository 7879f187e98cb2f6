"""Parity of the sm_100a conv kernels (through the C ABI) with a plain PyTorch fp32 reference of the same op.

Tolerance: fp16 outputs of an fp32-accumulated conv differ from the fp32 reference by the fp16 rounding
of the output (≤ 2^-11 relative) plus accumulation-order noise, so every element must satisfy
|y − ref| ≤ 2e-3·|ref| + 2e-3·max|ref|.
"""
import pytest
import torch
import torch.nn.functional as F

from objectsam_b200.conv import EPI_BIAS, EPI_BN_ACT, ConvGeom, ConvOp, DestSpec, sppf_pool_bwd, sppf_pool_fwd
from objectsam_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda"


def ref_conv(x, w, stride, pad):
    """NHWC fp16 x, KRSC fp16 w → NHWC fp32 conv (TF32 off)."""
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    y = F.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(0, 3, 1, 2), stride=stride, padding=pad)
    return y.permute(0, 2, 3, 1)


def assert_close(y, ref, rel=2e-3):
    y = y.float()
    scale = ref.abs().max().item() + 1e-6
    err = (y - ref).abs()
    bound = rel * ref.abs() + rel * scale
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance; max err {err.max().item():.3e} (scale {scale:.3e})"


def rand_conv(N, H, W, C, K, R, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.rand(N, H, W, C, generator=g) * 2 - 1).half().to(DEV)
    w = (torch.randn(K, R, R, C, generator=g) * (2.0 / (C * R * R)) ** 0.5).half().to(DEV)
    return x, w


# (N, H, W, C, K, R, stride): every kernel family — 3×3 s1/s2, 1×1, BK 32/64, BN 16..256, multi-N-tile, stem
SHAPES = [
    (2, 16, 16, 32, 32, 3, 1),
    (2, 20, 20, 64, 64, 3, 1),
    (3, 40, 40, 128, 128, 3, 1),
    (2, 20, 20, 256, 224, 3, 1),
    (1, 24, 36, 64, 256, 3, 1),
    (2, 16, 16, 32, 64, 3, 2),
    (2, 40, 40, 128, 256, 3, 2),
    (1, 20, 20, 256, 512, 3, 2),
    (2, 16, 16, 96, 64, 1, 1),
    (2, 20, 20, 128, 1, 1, 1),
    (2, 10, 10, 512, 512, 1, 1),
    (1, 7, 9, 64, 32, 1, 1),
    (2, 64, 64, 3, 32, 3, 2),
    (2, 128, 256, 3, 32, 3, 2),
    (1, 70, 90, 3, 32, 3, 2),
    (2, 40, 36, 3, 16, 3, 1),
    (1, 80, 80, 64, 64, 3, 1),
    (3, 33, 17, 64, 128, 3, 1),
]


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_fwd_matches_torch(cuda_lib, shape):
    N, H, W, C, K, R, s = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=sum(shape))
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, R // 2))
    y = torch.empty(op.out_shape(), dtype=torch.half, device=DEV)
    op.fwd(x, w, y)
    torch.cuda.synchronize()
    assert_close(y, ref_conv(x, w, s, R // 2))


# The forms of the tensor-map kernel, each forced for every size: single CTAs with one A box per tap
# ("tap"), CTA pairs with 2-SM UMMAs (M = 256 over two SMs, each staging its tile and half of the weight
# rows: "pair"), column-shifted input windows for 3×3/s1/p1 ("w3", 128-pixel tiles, ragged grids
# zero-filled), both at once ("w3pair"), the window form with all nine weight taps resident for the narrow
# layers ("w3res") and with them always streamed ("w3stream"), and the stride-2 window form streamed,
# resident and paired ("s2win", "s2winres", "s2winpair").  3×3 s1/s2 and 1×1, BK 32/64, BN 32..256,
# several N tiles, odd tile counts (the last pair's second tile is empty), every epilogue store form.
FORMS = {"tap": {"OSAM_FPROP_PAIR": "0", "OSAM_FPROP_W3": "0"},
         "pair": {"OSAM_FPROP_PAIR": "1", "OSAM_FPROP_W3": "0"},
         "w3": {"OSAM_FPROP_PAIR": "0", "OSAM_FPROP_W3": "1"},
         "w3pair": {"OSAM_FPROP_PAIR": "1", "OSAM_FPROP_W3": "1"},
         "w3stream": {"OSAM_FPROP_PAIR": "0", "OSAM_FPROP_W3": "1", "OSAM_FPROP_W3R": "0"},
         "w3res": {"OSAM_FPROP_PAIR": "1", "OSAM_FPROP_W3": "1", "OSAM_FPROP_W3R": "1"},
         "s2win": {"OSAM_FPROP_PAIR": "0", "OSAM_FPROP_W3S2": "1", "OSAM_FPROP_W3R": "0"},
         "s2winres": {"OSAM_FPROP_PAIR": "0", "OSAM_FPROP_W3S2": "1", "OSAM_FPROP_W3R": "1"},
         "s2winpair": {"OSAM_FPROP_PAIR": "1", "OSAM_FPROP_W3S2": "1", "OSAM_FPROP_W3R": "0"}}
FORM_SHAPES = [
    (3, 40, 40, 128, 128, 3, 1),
    (2, 20, 20, 64, 64, 3, 1),
    (3, 33, 17, 64, 128, 3, 1),
    (2, 20, 20, 64, 384, 3, 1),
    (2, 20, 20, 256, 224, 3, 1),
    (1, 24, 36, 64, 256, 3, 1),
    (2, 32, 48, 32, 32, 3, 1),
    (1, 50, 70, 64, 64, 3, 1),
    (2, 16, 16, 32, 64, 3, 2),
    (2, 40, 40, 128, 256, 3, 2),
    (1, 20, 20, 256, 512, 3, 2),
    (2, 64, 32, 64, 128, 3, 2),   # stride-2 window form: 32 × 16 output, exact 16 × 8 tiles
    (3, 36, 20, 32, 64, 3, 2),    # ragged stride-2 windows (18 × 10 output)
    (2, 16, 16, 96, 64, 1, 1),
    (1, 7, 9, 64, 64, 1, 1),
    (3, 30, 30, 64, 384, 1, 1),
    (2, 10, 10, 512, 512, 1, 1),
    (8, 8, 8, 64, 64, 3, 1),      # window form: 8 × 8 × 2-image tiles
    (4, 20, 20, 32, 64, 3, 1),    # window form: 8 × 4 × 4-image tiles, ragged rows
    (6, 40, 40, 128, 128, 3, 1),
    (5, 12, 20, 64, 128, 3, 1),   # odd batch: the last tile's second image is zero fill
    (2, 80, 80, 64, 64, 3, 1),    # window form on 16 × 8 tiles (the network's 80² 64 → 64 layers)
    (1, 34, 20, 32, 32, 3, 1),    # 16 × 8 tiles, ragged rows and columns, BK 32
    (3, 32, 24, 32, 32, 3, 1),    # 16 × 8 tiles, BK 32, several images
    (1, 48, 24, 64, 32, 3, 1),    # 16 × 8 tiles, BN 32 over 64 channels
]


def set_form(monkeypatch, form):
    for k, v in FORMS[form].items():
        monkeypatch.setenv(k, v)


@pytest.mark.parametrize("form", list(FORMS))
@pytest.mark.parametrize("shape", FORM_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_fwd_forms(cuda_lib, monkeypatch, shape, form):
    set_form(monkeypatch, form)
    N, H, W, C, K, R, s = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=sum(shape) + 5)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, R // 2))
    y = torch.full(op.out_shape(), 3.0, dtype=torch.half, device=DEV)
    op.fwd(x, w, y)
    assert_close(y, ref_conv(x, w, s, R // 2))
    y0 = (torch.rand(op.out_shape(), device=DEV) - 0.5).half()  # beta = 1: the per-element epilogue
    y = y0.clone()
    op.fwd(x, w, y, beta=1.0)
    assert_close(y, ref_conv(x, w, s, R // 2) + y0.float())


@pytest.mark.parametrize("form", list(FORMS))
@pytest.mark.parametrize("nhw", [(3, 24, 40), (4, 8, 8)], ids=lambda s: "x".join(map(str, s)))
def test_fused_residual_dests_forms(cuda_lib, monkeypatch, form, nhw):
    """The multi-destination BN + SiLU + residual epilogue (TMA stores) with every kernel form (the 8 × 8
    grid takes two-image window tiles)."""
    set_form(monkeypatch, form)
    N, H, W = nhw
    C, K = 64, 128
    x, w = rand_conv(N, H, W, C, K, 3, seed=13)
    g = torch.Generator(device="cpu").manual_seed(9)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    res = (torch.rand(N, H, W, K, generator=g) - 0.5).half().to(DEV)
    out = torch.zeros(N, H, W, K, dtype=torch.half, device=DEV)
    cat = torch.zeros(N, H, W, 3 * 64, dtype=torch.half, device=DEV)
    up = torch.zeros(N, 2 * H, 2 * W, 96, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    op.fwd_fused(x, w, [DestSpec(out), DestSpec(cat, choff=64, c0=64, c1=128), DestSpec(up, choff=32, c0=0, c1=64, up=2)],
                 kind=EPI_BN_ACT, scale=scale, shift=shift, res=res)
    a = F.silu(ref_conv(x, w, 1, 1).half().float() * scale + shift) + res.float()
    assert_close(out, a)
    assert_close(cat[..., 64:128], a[..., 64:128])
    assert cat[..., :64].abs().max().item() == 0 and cat[..., 128:].abs().max().item() == 0
    assert_close(up[..., 32:96], a[..., 0:64].repeat_interleave(2, dim=1).repeat_interleave(2, dim=2))
    assert up[..., :32].abs().max().item() == 0


@pytest.mark.parametrize("form", list(FORMS))
@pytest.mark.parametrize("shape", [(2, 20, 20, 64, 64), (1, 33, 40, 128, 128), (2, 16, 24, 256, 128)],
                         ids=lambda s: "x".join(map(str, s)))
def test_conv_dgrad_forms(cuda_lib, monkeypatch, shape, form):
    """Stride-1 3×3 input gradients run as forward convs over dz: every kernel form."""
    set_form(monkeypatch, form)
    N, H, W, C, K = shape
    x, w = rand_conv(N, H, W, C, K, 3, seed=sum(shape))
    g = torch.Generator(device="cpu").manual_seed(2)
    dz = (torch.rand(N, H, W, K, generator=g) * 2 - 1).half().to(DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=DEV)
    dx = torch.full((N, H, W, C), 3.0, dtype=torch.half, device=DEV)
    op.dgrad(dz, w, dx, ws=ws)
    torch.cuda.synchronize()
    assert_close(dx, ref_dgrad(dz, w, (N, H, W, C), 1, 1))


# Larger stride-1 grids at the network's sizes: full and ragged, BN 32..256, 3×3 and 5×5.
LARGE_SHAPES = [
    (2, 160, 160, 32, 32, 3),
    (2, 80, 80, 64, 64, 3),
    (2, 40, 40, 128, 128, 3),
    (1, 80, 80, 128, 224, 3),
    (2, 48, 48, 256, 256, 3),
    (1, 50, 70, 64, 64, 3),
    (1, 33, 100, 32, 128, 3),
    (1, 64, 64, 64, 64, 5),
    (1, 24, 16, 128, 128, 3),
    (1, 40, 24, 64, 224, 3),
]


@pytest.mark.parametrize("shape", LARGE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_large_s1_matches_torch(cuda_lib, shape):
    N, H, W, C, K, R = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=sum(shape) + 1)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, 1, R // 2))
    y = torch.full(op.out_shape(), 7.0, dtype=torch.half, device=DEV)
    op.fwd(x, w, y)
    torch.cuda.synchronize()
    assert_close(y, ref_conv(x, w, 1, R // 2))


def test_fused_residual_dests_large(cuda_lib):
    """C2f epilogue at a multi-tile size: BN + SiLU + residual to a full buffer, a concat slice and a 2×
    upsampled slice (each destination on 32-channel boundaries, so the TMA-store epilogue runs)."""
    N, H, W, C, K = 2, 64, 64, 64, 128
    x, w = rand_conv(N, H, W, C, K, 3, seed=12)
    g = torch.Generator(device="cpu").manual_seed(5)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    res = (torch.rand(N, H, W, K, generator=g) - 0.5).half().to(DEV)
    out = torch.zeros(N, H, W, K, dtype=torch.half, device=DEV)
    cat = torch.zeros(N, H, W, 3 * 64, dtype=torch.half, device=DEV)
    up = torch.zeros(N, 2 * H, 2 * W, 96, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    op.fwd_fused(x, w, [DestSpec(out), DestSpec(cat, choff=64, c0=64, c1=128), DestSpec(up, choff=32, c0=0, c1=64, up=2)],
                 kind=EPI_BN_ACT, scale=scale, shift=shift, res=res)
    a = F.silu(ref_conv(x, w, 1, 1) * scale + shift) + res.float()
    assert_close(out, a)
    assert_close(cat[..., 64:128], a[..., 64:128])
    assert cat[..., :64].abs().max().item() == 0 and cat[..., 128:].abs().max().item() == 0
    assert_close(up[..., 32:96], a[..., 0:64].repeat_interleave(2, dim=1).repeat_interleave(2, dim=2))
    assert up[..., :32].abs().max().item() == 0


# Narrow 3×3 convs (32 input channels, grids ≥ 64 wide) served from one shared input window per tile:
# odd heights, ragged widths, K 32 and 64, a few rows only (the window wraps rows within a tile).
WIN_SHAPES = [
    (2, 7, 70, 32, 32),
    (1, 33, 97, 32, 64),
    (2, 40, 64, 32, 64),
    (2, 24, 100, 32, 32),
    (1, 200, 64, 32, 32),
    (3, 5, 130, 32, 64),
]


@pytest.mark.parametrize("shape", WIN_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_window_matches_torch(cuda_lib, shape):
    N, H, W, C, K = shape
    x, w = rand_conv(N, H, W, C, K, 3, seed=sum(shape) + 2)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    y = torch.full(op.out_shape(), 7.0, dtype=torch.half, device=DEV)
    op.fwd(x, w, y)
    torch.cuda.synchronize()
    assert_close(y, ref_conv(x, w, 1, 1))


def test_conv_window_fused_residual_dests(cuda_lib):
    """Bottleneck-style narrow conv: BN + SiLU + residual to a full buffer, a concat slice and a 2×
    upsampled slice."""
    N, H, W, C, K = 2, 48, 76, 32, 64
    x, w = rand_conv(N, H, W, C, K, 3, seed=13)
    g = torch.Generator(device="cpu").manual_seed(6)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    res = (torch.rand(N, H, W, K, generator=g) - 0.5).half().to(DEV)
    out = torch.zeros(N, H, W, K, dtype=torch.half, device=DEV)
    cat = torch.zeros(N, H, W, 128, dtype=torch.half, device=DEV)
    up = torch.zeros(N, 2 * H, 2 * W, 64, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    op.fwd_fused(x, w, [DestSpec(out), DestSpec(cat, choff=64, c0=0, c1=64), DestSpec(up, choff=32, c0=32, c1=64, up=2)],
                 kind=EPI_BN_ACT, scale=scale, shift=shift, res=res)
    a = F.silu(ref_conv(x, w, 1, 1) * scale + shift) + res.float()
    assert_close(out, a)
    assert_close(cat[..., 64:], a)
    assert cat[..., :64].abs().max().item() == 0
    assert_close(up[..., 32:64], a[..., 32:64].repeat_interleave(2, dim=1).repeat_interleave(2, dim=2))
    assert up[..., :32].abs().max().item() == 0


def test_conv_fwd_beta_accumulates(cuda_lib):
    x, w = rand_conv(2, 16, 16, 64, 64, 3, seed=7)
    op = ConvOp().init(ConvGeom(2, 16, 16, 64, 64, 3, 3, 1, 1))
    y0 = (torch.rand(2, 16, 16, 64, device=DEV) - 0.5).half()
    y = y0.clone()
    op.fwd(x, w, y, beta=1.0)
    assert_close(y, ref_conv(x, w, 1, 1) + y0.float())


def test_fused_bn_silu_residual_dests(cuda_lib):
    """C2f-style epilogue: a = silu(scale·z + shift) + res → full buffer, a concat slice, and an upsampled slice."""
    N, H, W, C, K = 2, 20, 20, 64, 128
    x, w = rand_conv(N, H, W, C, K, 3, seed=11)
    g = torch.Generator(device="cpu").manual_seed(3)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    res = (torch.rand(N, H, W, K, generator=g) - 0.5).half().to(DEV)
    out = torch.zeros(N, H, W, K, dtype=torch.half, device=DEV)
    cat = torch.zeros(N, H, W, 3 * 64, dtype=torch.half, device=DEV)
    up = torch.zeros(N, 2 * H, 2 * W, 96, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    op.fwd_fused(x, w, [DestSpec(out), DestSpec(cat, choff=64, c0=64, c1=128), DestSpec(up, choff=32, c0=0, c1=64, up=2)],
                 kind=EPI_BN_ACT, scale=scale, shift=shift, res=res)
    z = ref_conv(x, w, 1, 1).half().float()  # the reference stores z in fp16 before BN (round_z)
    a = F.silu(z * scale + shift) + res.float()
    assert_close(out, a)
    assert_close(cat[..., 64:128], a[..., 64:128])
    assert cat[..., :64].abs().max().item() == 0 and cat[..., 128:].abs().max().item() == 0
    a_up = a[..., 0:64].repeat_interleave(2, dim=1).repeat_interleave(2, dim=2)
    assert_close(up[..., 32:96], a_up)
    assert up[..., :32].abs().max().item() == 0


def test_fused_1x1_k512_upsample_dest(cuda_lib):
    """SPPF.cv2-style node: 1×1 1024→512 with BN+SiLU to an upsampled concat slice and a plain slice."""
    N, H, W, C, K = 2, 10, 10, 1024, 512
    x, w = rand_conv(N, H, W, C, K, 1, seed=21)
    g = torch.Generator(device="cpu").manual_seed(4)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    cat_up = torch.zeros(N, 2 * H, 2 * W, 768, dtype=torch.half, device=DEV)
    cat = torch.zeros(N, H, W, 768, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 1, 1, 1, 0))
    op.fwd_fused(x, w, [DestSpec(cat_up, up=2), DestSpec(cat, choff=256)], kind=EPI_BN_ACT, scale=scale, shift=shift)
    a = F.silu(ref_conv(x, w, 1, 0).half().float() * scale + shift)
    assert_close(cat[..., 256:], a)
    assert_close(cat_up[..., :512], a.repeat_interleave(2, dim=1).repeat_interleave(2, dim=2))
    assert cat[..., :256].abs().max().item() == 0 and cat_up[..., 512:].abs().max().item() == 0


@pytest.mark.parametrize("shape", [(2, 64, 64, 3, 32, 3, 2), (2, 128, 256, 3, 32, 3, 2), (3, 256, 128, 3, 32, 3, 2),
                                   (1, 70, 90, 3, 32, 3, 2), (2, 40, 36, 3, 16, 3, 1)],
                         ids=lambda s: "x".join(map(str, s)))
def test_fused_stem_bn_silu(cuda_lib, shape):
    """The C = 3 stem with its folded-BN + SiLU epilogue (model.0)."""
    N, H, W, C, K, R, s = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=31)
    g = torch.Generator(device="cpu").manual_seed(6)
    scale = (torch.rand(K, generator=g) + 0.5).to(DEV)
    shift = (torch.rand(K, generator=g) - 0.5).to(DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, R // 2))
    y = torch.empty(op.out_shape(), dtype=torch.half, device=DEV)
    op.fwd_fused(x, w, [DestSpec(y)], kind=EPI_BN_ACT, scale=scale, shift=shift, round_z=False)
    assert_close(y, F.silu(ref_conv(x, w, s, R // 2) * scale + shift))


def test_fused_bias_head_k1(cuda_lib):
    """Head 1×1 conv with bias and a single output channel (cls head, reference src/model.cpp:251)."""
    N, H, W, C = 2, 40, 40, 128
    x, w = rand_conv(N, H, W, C, 1, 1, seed=5)
    bias = torch.tensor([0.25], device=DEV)
    y = torch.empty(N, H, W, 1, dtype=torch.half, device=DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, 1, 1, 1, 1, 0))
    op.fwd_fused(x, w, [DestSpec(y)], kind=EPI_BIAS, bias=bias)
    assert_close(y, ref_conv(x, w, 1, 0).half().float() + 0.25)


def test_conv_transpose_2x2(cuda_lib):
    """proto.upsample: ConvTranspose2d(128→128, k=2, s=2) with weights in the reference's (C_in, R, S, C_out)."""
    N, H, W, C, K = 2, 20, 20, 128, 128
    g = torch.Generator(device="cpu").manual_seed(9)
    x = (torch.rand(N, H, W, C, generator=g) * 2 - 1).half().to(DEV)
    w_pt = (torch.randn(C, K, 2, 2, generator=g) * 0.1).half()  # PyTorch ConvTranspose2d weight
    w = w_pt.permute(0, 2, 3, 1).contiguous().to(DEV)            # (C_in, kh, kw, C_out)
    bias = (torch.rand(K, generator=g) - 0.5).to(DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 2, 2, 2, 0), transposed=True)
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    y = torch.empty(op.out_shape(), dtype=torch.half, device=DEV)
    op.fwd(x, w, y, ws=ws)
    ref = F.conv_transpose2d(x.float().permute(0, 3, 1, 2), w_pt.float().to(DEV), stride=2).permute(0, 2, 3, 1)
    assert_close(y, ref)
    y2 = torch.empty_like(y)
    op.fwd_fused(x, w, [DestSpec(y2)], kind=EPI_BIAS, bias=bias, ws=ws)
    assert_close(y2, ref.half().float() + bias)


CONVT_SHAPES = [(2, 20, 20, 128, 128), (1, 80, 80, 128, 128), (3, 9, 13, 64, 32)]


@pytest.mark.parametrize("shape", CONVT_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_conv_transpose_2x2_dgrad_wgrad(cuda_lib, shape, beta):
    """Input and weight gradients of ConvTranspose2d(k = s = 2) (reference ConvOp::dgrad/wgrad on its transposed
    descriptor, src/conv.cpp:351-353, :362-364) against torch autograd in fp32, weights in (C_in, R, S, C_out)."""
    N, H, W, C, K = shape
    g = torch.Generator(device="cpu").manual_seed(sum(shape))
    x = (torch.rand(N, H, W, C, generator=g) * 2 - 1).half().to(DEV)
    w_pt = (torch.randn(C, K, 2, 2, generator=g) * 0.1).half()
    w = w_pt.permute(0, 2, 3, 1).contiguous().to(DEV)
    dy = (torch.rand(N, 2 * H, 2 * W, K, generator=g) * 2 - 1).half().to(DEV)
    dx0 = (torch.rand(N, H, W, C, generator=g) - 0.5).half().to(DEV)
    dw0 = (torch.rand(C, 2, 2, K, generator=g) - 0.5).half().to(DEV)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 2, 2, 2, 0), transposed=True)
    ws = torch.empty(max(op.workspace_size(), 256), dtype=torch.uint8, device=DEV)
    dx, dw = dx0.clone(), dw0.clone()
    op.dgrad(dy, w, dx, ws=ws, beta=beta)
    op.wgrad(x, dy, dw, ws=ws, beta=beta)
    torch.cuda.synchronize()
    xt = x.float().permute(0, 3, 1, 2).requires_grad_(True)
    wt = w_pt.float().to(DEV).requires_grad_(True)
    F.conv_transpose2d(xt, wt, stride=2).backward(dy.float().permute(0, 3, 1, 2))
    assert_close(dx, xt.grad.permute(0, 2, 3, 1) + beta * dx0.float())
    assert_close(dw, wt.grad.permute(0, 2, 3, 1) + beta * dw0.float())


SPPF_BWD_SHAPES = [(3, 20, 20, 256, False), (2, 9, 11, 64, False), (2, 20, 20, 64, True), (1, 40, 40, 32, False),
                   (1, 40, 40, 32, True)]


@pytest.mark.parametrize("shape", SPPF_BWD_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_sppf_bwd_matches_oracle_bit_exact(cuda_lib, shape):
    """SPPF backward against the restatement (same fp32 summation order: bit-exact), ties included."""
    import numpy as np
    from oracle import sppf_ref
    N, H, W, c, ties = shape
    r = np.random.default_rng(H * W + c)
    x = r.integers(-2, 3, (N, H, W, c)) if ties else r.standard_normal((N, H, W, c))
    cat = torch.zeros(N, H, W, 4 * c, dtype=torch.half, device=DEV)
    cat[..., :c] = torch.from_numpy(x.astype(np.float32)).half().to(DEV)
    sppf_pool_fwd(cat, N, H, W, c)
    dcat = torch.from_numpy((r.standard_normal((N, H, W, 4 * c)) * 0.5).astype(np.float32)).half().to(DEV)
    want = sppf_ref.sppf_bwd(cat.float().cpu().numpy(), dcat.float().cpu().numpy(), c)
    sppf_pool_bwd(cat, dcat, N, H, W, c)
    torch.cuda.synchronize()
    assert np.array_equal(dcat.float().cpu().numpy(), want)


def test_sppf_pool_exact(cuda_lib):
    N, H, W, c = 3, 20, 20, 256
    cat = torch.zeros(N, H, W, 4 * c, dtype=torch.half, device=DEV)
    cat[..., :c] = torch.randn(N, H, W, c, device=DEV).half()
    sppf_pool_fwd(cat, N, H, W, c)
    x = cat[..., :c].permute(0, 3, 1, 2).float()
    for k in range(1, 4):
        x = F.max_pool2d(x, 5, 1, 2)
        assert torch.equal(cat[..., k * c:(k + 1) * c].float(), x.permute(0, 2, 3, 1))


def test_invalid_geometry_is_an_error(cuda_lib):
    from objectsam_b200 import OsamError
    with pytest.raises(OsamError):
        ConvOp().init(ConvGeom(1, 16, 16, 48, 32, 3, 3, 1, 1))  # C % 32 != 0 and R·S·C > 32


def ref_dgrad(dz, w, x_shape, stride, pad):
    """NHWC fp16 dz, KRSC w → NHWC fp32 input gradient of conv2d (TF32 off)."""
    torch.backends.cudnn.allow_tf32 = False
    N, H, W, C = x_shape
    dx = torch.nn.grad.conv2d_input((N, C, H, W), w.float().permute(0, 3, 1, 2), dz.float().permute(0, 3, 1, 2),
                                    stride=stride, padding=pad)
    return dx.permute(0, 2, 3, 1)


# (N, H, W, C, K, R, stride): the network's dgrad shapes — 3×3 s1 and s2, 1×1, narrow and wide, ragged
DGRAD_SHAPES = [
    (2, 16, 16, 32, 32, 3, 1),
    (2, 20, 20, 64, 128, 3, 1),
    (1, 40, 24, 128, 64, 3, 1),
    (2, 10, 10, 256, 256, 3, 1),
    (2, 16, 16, 96, 64, 1, 1),
    (1, 20, 20, 512, 256, 1, 1),
    (2, 32, 32, 32, 64, 3, 2),
    (2, 40, 40, 128, 256, 3, 2),
    (1, 20, 28, 256, 512, 3, 2),
    (1, 80, 80, 64, 128, 3, 2),
    (2, 20, 20, 192, 128, 1, 1),   # GEMM N 192 and 96 (the C2f output convs' input gradients)
    (3, 17, 9, 96, 64, 1, 1),
    (1, 30, 22, 96, 32, 3, 1),
]


@pytest.mark.parametrize("shape", DGRAD_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_dgrad_matches_torch(cuda_lib, shape):
    N, H, W, C, K, R, s = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=sum(shape) + 3)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, R // 2))
    P, Q = op.geom().P(), op.geom().Q()
    g = torch.Generator(device="cpu").manual_seed(9)
    dz = (torch.rand(N, P, Q, K, generator=g) * 2 - 1).half().to(DEV)
    ws = torch.empty(max(op.workspace_size(), 1), dtype=torch.uint8, device=DEV)
    dx = torch.full((N, H, W, C), 3.0, dtype=torch.half, device=DEV)
    op.dgrad(dz, w, dx, ws=ws)
    torch.cuda.synchronize()
    assert_close(dx, ref_dgrad(dz, w, (N, H, W, C), s, R // 2))


@pytest.mark.parametrize("stride,R,C,K", [(1, 3, 64, 64), (2, 3, 64, 64), (1, 1, 96, 64), (1, 1, 192, 128),
                                          (1, 3, 128, 256), (2, 3, 32, 64), (1, 1, 64, 32)])
def test_conv_dgrad_beta_accumulates(cuda_lib, stride, R, C, K):
    """beta = 1 adds the gradient to dx (the reference's dgrad_accum for inputs with several consumers):
    the coalesced epilogue reads the old rows through its stage, for 3×3 / 1×1, both strides, GEMM N 96/192."""
    N, H, W = 2, 24, 24
    x, w = rand_conv(N, H, W, C, K, R, seed=17)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, stride, R // 2))
    P, Q = op.geom().P(), op.geom().Q()
    g = torch.Generator(device="cpu").manual_seed(10)
    dz = (torch.rand(N, P, Q, K, generator=g) - 0.5).half().to(DEV)
    dx0 = (torch.rand(N, H, W, C, generator=g) - 0.5).half().to(DEV)
    dx = dx0.clone()
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    op.dgrad(dz, w, dx, ws=ws, beta=1.0)
    torch.cuda.synchronize()
    assert_close(dx, ref_dgrad(dz, w, (N, H, W, C), stride, R // 2) + dx0.float())


def ref_wgrad(x, dz, w_shape, stride, pad):
    """NHWC fp16 x and dz → KRSC fp32 weight gradient of conv2d (TF32 off)."""
    torch.backends.cudnn.allow_tf32 = False
    K, R, S, C = w_shape
    dw = torch.nn.grad.conv2d_weight(x.float().permute(0, 3, 1, 2), (K, C, R, S), dz.float().permute(0, 3, 1, 2),
                                     stride=stride, padding=pad)
    return dw.permute(0, 2, 3, 1)


@pytest.mark.parametrize("shape", DGRAD_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv_wgrad_matches_torch(cuda_lib, shape):
    N, H, W, C, K, R, s = shape
    x, w = rand_conv(N, H, W, C, K, R, seed=sum(shape) + 4)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, R, R, s, R // 2))
    P, Q = op.geom().P(), op.geom().Q()
    g = torch.Generator(device="cpu").manual_seed(11)
    dz = (torch.rand(N, P, Q, K, generator=g) * 2 - 1).half().to(DEV)
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    dw = torch.full((K, R, R, C), 5.0, dtype=torch.half, device=DEV)
    op.wgrad(x, dz, dw, ws=ws)
    torch.cuda.synchronize()
    assert_close(dw, ref_wgrad(x, dz, (K, R, R, C), s, R // 2))


# small-C input convs (R·S·C ≤ 32): the RGB stem and odd sizes, both strides, K = 32 and 64
STEM_WGRAD_SHAPES = [(2, 64, 64, 3, 32, 2), (1, 640, 640, 3, 32, 2), (3, 30, 46, 3, 64, 2), (2, 33, 17, 3, 32, 1),
                     (1, 9, 7, 2, 32, 2)]


@pytest.mark.parametrize("shape", STEM_WGRAD_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_conv_wgrad_small_c_matches_torch(cuda_lib, shape, beta):
    N, H, W, C, K, s = shape
    x, _ = rand_conv(N, H, W, C, K, 3, seed=sum(shape) + 9)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, s, 1))
    P, Q = op.geom().P(), op.geom().Q()
    g = torch.Generator(device="cpu").manual_seed(13)
    dz = (torch.rand(N, P, Q, K, generator=g) * 2 - 1).half().to(DEV)
    dw0 = (torch.rand(K, 3, 3, C, generator=g) - 0.5).half().to(DEV)
    dw = dw0.clone()
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    op.wgrad(x, dz, dw, ws=ws, beta=beta)
    torch.cuda.synchronize()
    assert_close(dw, ref_wgrad(x, dz, (K, 3, 3, C), s, 1) + beta * dw0.float())


def test_conv_wgrad_beta_accumulates(cuda_lib):
    N, H, W, C, K = 2, 24, 24, 64, 128
    x, w = rand_conv(N, H, W, C, K, 3, seed=19)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, 1, 1))
    g = torch.Generator(device="cpu").manual_seed(12)
    dz = (torch.rand(N, H, W, K, generator=g) - 0.5).half().to(DEV)
    dw0 = (torch.rand(K, 3, 3, C, generator=g) - 0.5).half().to(DEV)
    dw = dw0.clone()
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    op.wgrad(x, dz, dw, ws=ws, beta=1.0)
    torch.cuda.synchronize()
    assert_close(dw, ref_wgrad(x, dz, (K, 3, 3, C), 1, 1) + dw0.float())


# window form of the weight gradient (3×3, pad 1, C ∈ {32, 64}; stride 1, or 2 on even sizes): both channel
# blocks, every dz block width (32, 64, 128 — and K split over two CTAs), ragged tiles, odd batches, runs of
# many tiles per CTA; the per-tap form (OSAM_WGRAD_WIN=0) on the same inputs must agree too
WGRAD_WIN_SHAPES = [(2, 20, 20, 32, 32, 1), (3, 40, 24, 64, 64, 1), (1, 13, 11, 32, 128, 1), (2, 17, 9, 64, 32, 1),
                    (2, 32, 32, 32, 64, 2), (3, 24, 40, 64, 128, 2), (1, 18, 14, 32, 32, 2), (4, 160, 160, 32, 32, 1),
                    (2, 320, 320, 32, 64, 2), (5, 80, 80, 64, 64, 1)]


@pytest.mark.parametrize("shape", WGRAD_WIN_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("beta", [0.0, 1.0])
def test_conv_wgrad_window_form_matches_torch(cuda_lib, monkeypatch, shape, beta):
    N, H, W, C, K, s = shape
    x, _ = rand_conv(N, H, W, C, K, 3, seed=sum(shape) + 21)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 3, 3, s, 1))
    P, Q = op.geom().P(), op.geom().Q()
    g = torch.Generator(device="cpu").manual_seed(15)
    dz = (torch.rand(N, P, Q, K, generator=g) * 2 - 1).half().to(DEV)
    dw0 = (torch.rand(K, 3, 3, C, generator=g) - 0.5).half().to(DEV)
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    ref = ref_wgrad(x, dz, (K, 3, 3, C), s, 1) + beta * dw0.float()
    for form in ("1", "0"):  # window form, then the per-tap form
        monkeypatch.setenv("OSAM_WGRAD_WIN", form)
        dw = dw0.clone()
        op.wgrad(x, dz, dw, ws=ws, beta=beta)
        torch.cuda.synchronize()
        assert_close(dw, ref)
    assert _lib.device_error() == 0
