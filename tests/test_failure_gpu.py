"""Failure detection on the GPU without a fault: a bounded wait that nothing completes
gives up within its limit, the host reads the timeout bit from the device error word, and
the context stays usable (a decode right after it is still correct)."""

import time

import pytest
import torch

import attention_b200 as spa
import oracle
from attention_b200 import _lib
from attention_b200._util import stream_ptr

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    assert spa.device_error_flags() == 0
    t0 = time.perf_counter()
    _lib.check(_lib.lib.spa_debug_wait_timeout(2_000_000, stream_ptr(torch.device("cuda"))),
               "spa_debug_wait_timeout")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert spa.device_error_flags() == 1  # SPA_DEVERR_WAIT_TIMEOUT; reading clears it
    assert spa.device_error_flags() == 0
    # the context is intact: a decode after the timeout matches the oracle
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(2, 4, 64, generator=gen)
    k = torch.randn(2, 4, 512, 64, generator=gen)
    v = torch.randn(2, 4, 512, 64, generator=gen)
    out = spa.paged_decode_attention(q.cuda(), k.cuda(), v.cuda())
    ref = oracle.reference_attention(q, k, v)
    assert ((out.double().cpu() - ref).abs() <= 1e-5).all()
    assert spa.device_error_flags() == 0


def test_wait_limit_is_validated():
    with pytest.raises(ValueError):
        _lib.check(_lib.lib.spa_debug_wait_timeout(0, None), "spa_debug_wait_timeout")
