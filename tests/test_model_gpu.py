"""spa_rms_norm (the integrated decoder's norm in one launch) against a plain PyTorch fp32
reference of the same formula."""

import pytest
import torch

import attention_b200 as spa
from attention_b200.decoder import rms_norm

pytestmark = pytest.mark.gpu


def _ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 512), (3, 7, 128), (5, 1000), (1, 4096)])
def test_rms_norm_matches_fp32_reference(dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = (torch.randn(shape, device="cuda", generator=g) * 3).to(dtype)
    w = (torch.rand(shape[-1], device="cuda", generator=g) + 0.5).to(dtype)
    y = rms_norm(x, w, 1e-5)
    assert y.dtype == dtype and y.shape == x.shape
    r = _ref(x, w, 1e-5)
    # fp32: 1e-5 absolute + relative; 16-bit: one rounding of the output (2^-8 relative)
    atol, rtol = (1e-5, 1e-5) if dtype == torch.float32 else (1e-3, 8e-3)
    assert ((y.float() - r).abs() <= atol + rtol * r.abs()).all()
    assert spa.device_error_flags() == 0


def test_rms_norm_zero_rows_and_validation():
    x = torch.empty(0, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    assert rms_norm(x, w, 1e-5).shape == (0, 64)
    with pytest.raises(ValueError):
        rms_norm(torch.ones(2, 64), torch.ones(64), 1e-5)
