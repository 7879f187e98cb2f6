"""osam_convt_fwd_static_scratch: the transposed-conv forward that allocates nothing.

Callers that cannot allocate device memory or provide a workspace (a plugin host that owns the device
budget and only hands out a stream; a loop that must never reach cudaMalloc, which can synchronise the
device) use this entry point; its weight-relayout scratch is a fixed 256 KiB device array inside the
library.  Checked through the C ABI against the workspace path (osam_conv_fwd with a caller workspace)
and against torch's fp32 conv_transpose2d, on two calls in a row with different inputs, with the conv
tests' tolerance.  This file sorts last so a
run that stops at the first failure has already run every other test; it also passes alone.
"""
import pytest
import torch

from objectsam_b200 import _lib
from objectsam_b200.conv import ConvGeom, ConvOp

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _assert_close(y, ref, rel=2e-3):
    y, ref = y.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    bad = ((y - ref).abs() > rel * ref.abs() + rel * scale).sum().item()
    assert bad == 0, f"{bad} elements differ beyond tolerance"


def test_static_scratch_matches_workspace_path_twice(cuda_lib):
    N, H, W, C, K = 2, 20, 20, 128, 128  # the model's proto upsample shape (128 → 128, k = s = 2)
    op = ConvOp().init(ConvGeom(N, H, W, C, K, 2, 2, 2, 0), transposed=True)
    ws = torch.empty(op.workspace_size(), dtype=torch.uint8, device=DEV)
    stream = _lib.stream_ptr()
    for call in range(2):
        g = torch.Generator(device="cpu").manual_seed(1000 + call)
        x = (torch.rand(N, H, W, C, generator=g) * 2 - 1).half().to(DEV)
        w = (torch.randn(C, 2, 2, K, generator=g) * 0.1).half().to(DEV)
        y_ref = torch.empty(op.out_shape(), dtype=torch.half, device=DEV)
        op.fwd(x, w, y_ref, ws=ws)
        y = torch.full(op.out_shape(), float("nan"), dtype=torch.half, device=DEV)
        rc = _lib.lib().osam_convt_fwd_static_scratch(op._plan, x.data_ptr(), w.data_ptr(), y.data_ptr(), 0.0,
                                                      stream)
        _lib.check(rc)
        torch.cuda.synchronize()
        assert not torch.isnan(y).any()
        _assert_close(y, y_ref)
        # and against torch's fp32 transposed conv of the same fp16 operands (weights (C_in, R, S, C_out))
        y32 = torch.nn.functional.conv_transpose2d(x.float().permute(0, 3, 1, 2), w.float().permute(0, 3, 1, 2),
                                                   stride=2).permute(0, 2, 3, 1)
        _assert_close(y, y32)
    assert _lib.device_error() == 0


def test_static_scratch_rejects_oversize_plans(cuda_lib):
    op = ConvOp().init(ConvGeom(1, 4, 4, 512, 128, 2, 2, 2, 0), transposed=True)  # 512 KiB of weights
    x = torch.zeros(1, 4, 4, 512, dtype=torch.half, device=DEV)
    w = torch.zeros(512, 2, 2, 128, dtype=torch.half, device=DEV)
    y = torch.zeros(1, 8, 8, 128, dtype=torch.half, device=DEV)
    rc = _lib.lib().osam_convt_fwd_static_scratch(op._plan, x.data_ptr(), w.data_ptr(), y.data_ptr(), 0.0,
                                                  _lib.stream_ptr())
    assert rc == _lib.OSAM_ERR_INVALID
    assert b"static array holds" in _lib.lib().osam_last_error()
    plain = ConvOp().init(ConvGeom(1, 8, 8, 32, 32, 3, 3, 1, 1))
    rc = _lib.lib().osam_convt_fwd_static_scratch(plain._plan, x.data_ptr(), w.data_ptr(), y.data_ptr(), 0.0,
                                                  _lib.stream_ptr())
    assert rc == _lib.OSAM_ERR_INVALID
