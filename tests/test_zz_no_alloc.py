"""The allocation-free decode entry point (spa_paged_decode_noalloc) against the
workspace entry point (spa_paged_decode), through the C ABI.

It serves callers that cannot allocate device memory or pass a workspace: the
split-K partials live in a fixed scratch array inside the library.  Two calls in a
row with different inputs check that the shared scratch carries nothing from one
call into the next.  Tolerance: bf16 outputs within 2e-2 absolute + 1e-2 relative.
This file is collected last so a failure here never hides the other tests."""

import ctypes

import pytest
import torch

from attention_b200 import _lib
from attention_b200.paged_attention import pool_layout

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed: int):
    # few (sequence, kv head) pairs: the decode splits each pair widely and keeps the
    # split partials in scratch memory (the path that needs the scratch array)
    gen = torch.Generator().manual_seed(seed)
    b, hq, hkv, d, page, pages = 2, 8, 2, 128, 256, 24
    k_pool = (torch.randn(b * pages, hkv, page, d, generator=gen) * 0.5).to(torch.bfloat16)
    v_pool = (torch.randn(b * pages, hkv, page, d, generator=gen) * 0.5).to(torch.bfloat16)
    table = torch.randperm(b * pages, generator=gen).view(b, pages).to(torch.int32)
    q = (torch.randn(b, hq, d, generator=gen) * 0.5).to(torch.bfloat16)
    sel = torch.stack([torch.randperm(pages - 1, generator=gen)[:8] for _ in range(b)])
    ctx = torch.full((b,), pages * page - 7, dtype=torch.int32)
    t = {n: x.to(DEV) for n, x in dict(k=k_pool, v=v_pool, table=table, q=q, sel=sel, ctx=ctx).items()}
    t.update(b=b, hq=hq, hkv=hkv, d=d, window=256, m=8, max_cand=256 + 8 * page)
    return t


def _call(x, noalloc: bool) -> torch.Tensor:
    out = torch.empty_like(x["q"])
    layout = pool_layout(x["k"], x["v"], x["table"])
    stream = torch.cuda.current_stream().cuda_stream
    args = (x["q"].data_ptr(), _lib.SPA_BF16, x["b"], x["hq"], x["hkv"], x["d"], ctypes.byref(layout),
            x["ctx"].data_ptr(), x["window"], x["sel"].data_ptr(), x["m"], x["max_cand"], x["d"] ** -0.5,
            out.data_ptr())
    if noalloc:
        rc = _lib.lib.spa_paged_decode_noalloc(*args, stream)
    else:
        need = _lib.lib.spa_decode_workspace_size(x["b"], x["hq"], x["hkv"], x["d"], x["max_cand"])
        ws = torch.zeros(max(need, 1), dtype=torch.uint8, device=DEV)
        rc = _lib.lib.spa_paged_decode(*args, ws.data_ptr(), need, stream)
    assert rc == _lib.SPA_OK, rc
    torch.cuda.synchronize()
    return out


def test_noalloc_matches_workspace_entry_point_twice():
    first, second = _inputs(1), _inputs(2)
    # the request really uses split-K scratch
    assert _lib.lib.spa_decode_workspace_size(2, 8, 2, 128, first["max_cand"]) > 0
    for x in (first, second):
        ref = _call(x, noalloc=False).double()
        got = _call(x, noalloc=True).double()
        assert torch.isfinite(got).all()
        assert ((got - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()
    assert _lib.device_error_flags() == 0


def test_noalloc_rejects_requests_beyond_the_scratch():
    # 1 sequence, 16 q heads on 1 kv head, head_dim 256 and a long context need
    # more split-K scratch than the fixed array holds
    need = _lib.lib.spa_decode_workspace_size(1, 16, 1, 256, 1 << 17)
    assert need > (4 << 20)
    q = torch.zeros(1, 16, 256, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(1, 1, 64, 256, dtype=torch.bfloat16, device=DEV)
    layout = _lib.KvLayout(k.data_ptr(), k.data_ptr(), 64, 64, 64, 64, None, 0, 64)
    ctx = torch.full((1,), 64, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    rc = _lib.lib.spa_paged_decode_noalloc(q.data_ptr(), _lib.SPA_BF16, 1, 16, 1, 256, ctypes.byref(layout),
                                           ctx.data_ptr(), 0, None, 0, 1 << 17, 256 ** -0.5, out.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SPA_ERR_WORKSPACE
