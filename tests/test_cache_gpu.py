"""KV append and the promotion table on the GPU (bit-exact against the oracle)."""

import numpy as np
import pytest
import torch

import attention_b200 as spa
import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert spa.device_error_flags() == 0


def test_kv_append_then_decode():
    gen = torch.Generator().manual_seed(0)
    b, hkv, page, d = 3, 2, 128, 64
    k_pool = torch.randn(12, hkv, page, d, generator=gen).to(torch.bfloat16)
    v_pool = torch.randn(12, hkv, page, d, generator=gen).to(torch.bfloat16)
    table = torch.randperm(12, generator=gen)[:12].view(b, 4).to(torch.int32)
    pos = torch.tensor([0, 130, 511], dtype=torch.int32)
    kn = torch.randn(b, hkv, d, generator=gen).to(torch.bfloat16)
    vn = torch.randn(b, hkv, d, generator=gen).to(torch.bfloat16)
    kd, vd = k_pool.to(DEV), v_pool.to(DEV)
    spa.kv_append(kd, vd, table.to(DEV), kn.to(DEV), vn.to(DEV), pos.to(DEV))
    for i in range(b):
        p = int(pos[i])
        k_pool[table[i, p // page], :, p % page] = kn[i]
        v_pool[table[i, p // page], :, p % page] = vn[i]
    assert torch.equal(kd.cpu(), k_pool) and torch.equal(vd.cpu(), v_pool)


def test_promotion_table_many_steps_bit_exact():
    rng = np.random.default_rng(0)
    rows, slots, ttl, m = 6, 16, 5, 4
    cache = spa.PromotionCache(rows, slots=slots, ttl=ttl, device=DEV)
    pages = np.full((rows, slots), -1, np.int32)
    last = np.zeros((rows, slots), np.int32)
    for step in range(300):
        # a drifting hot set with repeats, -1 holes and duplicates
        sel = rng.integers(0, 40, size=(rows, m)) + (step // 25)
        sel[rng.random((rows, m)) < 0.05] = -1
        if step % 7 == 0:
            sel[:, 1] = sel[:, 0]
        cache.update(torch.from_numpy(sel).to(DEV), step)
        oracle.promotion_update(pages, last, sel, step, ttl)
        assert np.array_equal(cache.pages.cpu().numpy(), pages), step
        assert np.array_equal(cache.last_hit.cpu().numpy(), last), step
