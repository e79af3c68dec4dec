"""The FMA-pipe exponential of the prefill softmax (exp2_poly) against exp2 in float64.

Bound: relative error <= 1e-4 on [-125, 126] (the cubic's minimax error is 7.5e-5,
plus fp32 rounding of the reduction and Horner steps); x below -125 returns 2^-125."""

import pytest
import torch

from attention_b200 import _lib
from attention_b200._util import stream_ptr

pytestmark = pytest.mark.gpu


def _exp2_poly(x: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    _lib.check(_lib.lib.spa_debug_exp2_poly(x.data_ptr(), y.data_ptr(), x.numel(), stream_ptr(x.device)),
               "spa_debug_exp2_poly")
    torch.cuda.synchronize()
    return y


def test_exp2_poly_relative_error():
    dev = torch.device("cuda")
    grid = torch.linspace(-125.0, 126.0, 2_000_001, dtype=torch.float32, device=dev)
    # every fp32 value of the reduced argument near 0 and the rounding ties at +-1/2
    fine = torch.linspace(-1.0, 1.0, 1_000_001, dtype=torch.float32, device=dev)
    ties = torch.arange(-124, 125, dtype=torch.float32, device=dev) + 0.5  # +-124.5 stay in range
    x = torch.cat([grid, fine, ties, -ties])
    y = _exp2_poly(x).double()
    ref = torch.exp2(x.double())
    rel = ((y - ref).abs() / ref).max().item()
    assert rel <= 1e-4, rel


def test_exp2_poly_clamps_below_range():
    x = torch.tensor([-125.5, -126.0, -200.0, -1e30, float("-inf")], device="cuda")
    y = _exp2_poly(x)
    assert torch.all(y > 0) and torch.all(y <= 2.0 ** -124.5)


def test_exp2_poly_rejects_null():
    with pytest.raises(ValueError):
        _lib.check(_lib.lib.spa_debug_exp2_poly(None, None, 4, None), "spa_debug_exp2_poly")
