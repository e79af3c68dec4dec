"""spa_copy (kernel copy for small transfers to and from mapped pinned host memory) and
spa_host_device_pointer, the two pieces of the zero-copy session step."""



import pytest
import torch

from attention_b200 import _lib
from attention_b200._util import stream_ptr

pytestmark = pytest.mark.gpu


def _copy(dst_ptr: int, src_ptr: int, n: int) -> None:
    _lib.check(_lib.lib.spa_copy(dst_ptr, src_ptr, n, stream_ptr(torch.device("cuda", 0))), "spa_copy")


@pytest.mark.parametrize("n", [16, 4096, 32896, 33, 1_000_003])
def test_copy_device_to_pinned_host(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda", generator=g)
    dst = torch.zeros(n, dtype=torch.uint8).pin_memory()
    _copy(_lib.host_device_pointer(dst.data_ptr()), src.data_ptr(), n)
    torch.cuda.synchronize()
    assert torch.equal(dst, src.cpu())


@pytest.mark.parametrize("offset", [0, 1, 8])
def test_copy_pinned_host_to_device_unaligned(offset):
    n = 5000
    src = torch.arange(n + offset, dtype=torch.int32).to(torch.uint8).pin_memory()
    dst = torch.zeros(n + 16, dtype=torch.uint8, device="cuda")
    _copy(dst.data_ptr() + 3, _lib.host_device_pointer(src.data_ptr()) + offset, n)
    torch.cuda.synchronize()
    assert torch.equal(dst[3:3 + n].cpu(), src[offset:offset + n])
    assert int(dst[:3].sum()) == 0 and int(dst[3 + n:].sum()) == 0


def test_copy_zero_bytes_and_validation():
    x = torch.zeros(16, dtype=torch.uint8, device="cuda")
    _copy(x.data_ptr(), x.data_ptr(), 0)
    with pytest.raises(ValueError):
        _copy(0, x.data_ptr(), 16)


def test_host_device_pointer_rejects_pageable_memory():
    pageable = torch.zeros(64, dtype=torch.uint8)
    with pytest.raises(ValueError):
        _lib.host_device_pointer(pageable.data_ptr())
    pinned = torch.zeros(64, dtype=torch.uint8).pin_memory()
    assert _lib.host_device_pointer(pinned.data_ptr()) != 0
    # the call left no error behind for the next launch
    y = torch.ones(4, device="cuda") * 2
    assert float(y.sum()) == 8.0

