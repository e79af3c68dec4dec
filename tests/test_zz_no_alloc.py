"""The allocation-free decode entry point (spa_paged_decode_noalloc) through the C ABI.

It serves callers that cannot allocate device memory or pass a workspace at the point
where they decode -- a serving engine that owns all of HBM through its own pool, a
plugin interface with no workspace argument: the split-K partials live in a fixed
scratch array inside the library.  The outputs are checked against the oracle and
against the workspace entry point (spa_paged_decode), on two calls in a row with
different inputs, which shows that the shared scratch carries nothing from one call
into the next.  Tolerances: bf16 within 2e-2 absolute + 1e-2 relative, fp32 within
1e-5 absolute.  This file is collected last so a failure here never hides the other
tests."""

import ctypes

import pytest
import torch

import oracle
from attention_b200 import _lib
from attention_b200.paged_attention import pool_layout

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH = 4 << 20  # SPA_DECODE_STATIC_SCRATCH_BYTES


def _inputs(seed: int, dtype):
    # few (sequence, kv head) pairs: the decode splits each pair widely and keeps the
    # split partials in scratch memory (the path that needs the scratch array)
    gen = torch.Generator().manual_seed(seed)
    b, hq, hkv, d, page, pages = 2, 8, 2, 128, 256, 24
    k_pool = (torch.randn(b * pages, hkv, page, d, generator=gen) * 0.5).to(dtype)
    v_pool = (torch.randn(b * pages, hkv, page, d, generator=gen) * 0.5).to(dtype)
    table = torch.randperm(b * pages, generator=gen).view(b, pages).to(torch.int32)
    q = (torch.randn(b, hq, d, generator=gen) * 0.5).to(dtype)
    sel = torch.stack([torch.randperm(pages - 1, generator=gen)[:8] for _ in range(b)])
    ctx = [pages * page - 7] * b
    cpu = dict(k=k_pool, v=v_pool, table=table, q=q, sel=sel)
    t = {n: x.to(DEV) for n, x in cpu.items()}
    t["ctx"] = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    t.update(b=b, hq=hq, hkv=hkv, d=d, window=256, m=8, max_cand=256 + 8 * page, page=page, pages=pages,
             cpu=cpu, ctx_list=ctx, dtype=dtype)
    return t


def _oracle(x) -> torch.Tensor:
    c = x["cpu"]
    k = oracle.paged_to_contiguous(c["k"], c["table"], x["pages"] * x["page"])
    v = oracle.paged_to_contiguous(c["v"], c["table"], x["pages"] * x["page"])
    return oracle.gather_decode(c["q"], k, v, c["sel"], local_window=x["window"], block_size=x["page"],
                                context_lens=x["ctx_list"])


def _call(x, noalloc: bool) -> torch.Tensor:
    out = torch.empty_like(x["q"])
    layout = pool_layout(x["k"], x["v"], x["table"])
    stream = torch.cuda.current_stream().cuda_stream
    code = _lib.SPA_BF16 if x["dtype"] == torch.bfloat16 else _lib.SPA_F32
    args = (x["q"].data_ptr(), code, x["b"], x["hq"], x["hkv"], x["d"], ctypes.byref(layout),
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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_oracle_and_workspace_entry_point_twice(dtype):
    first, second = _inputs(1, dtype), _inputs(2, dtype)
    # the request really keeps split-K partials in the scratch array: it needs scratch,
    # fits in it, and (bf16) its splits are merged through global partials, not on chip
    # in a cluster; the fp32 kernel always merges through global partials
    need = _lib.lib.spa_decode_workspace_size(2, 8, 2, 128, first["max_cand"])
    assert 0 < need <= SCRATCH
    nsplit, on_chip = _lib.decode_plan(2, 8, 2, first["max_cand"])
    assert nsplit > 1
    if dtype == torch.bfloat16:
        assert not on_chip
    for x in (first, second):
        ref = _oracle(x)
        got = _call(x, noalloc=True).double().cpu()
        ws = _call(x, noalloc=False).double().cpu()
        assert torch.isfinite(got).all()
        if dtype == torch.bfloat16:
            assert ((got - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()
        else:
            assert (got - ref).abs().max().item() <= 1e-5
        assert ((got - ws).abs() <= 2e-2 + 1e-2 * ws.abs()).all()
    assert _lib.device_error_flags() == 0


def test_noalloc_rejects_requests_beyond_the_scratch():
    # the split plan (and so the scratch a request needs) depends on the device's SM
    # count: grow the batch until the request exceeds the fixed array
    hq, hkv, d, cand = 16, 1, 256, 1 << 17
    batch = next((b for b in range(1, 257) if _lib.lib.spa_decode_workspace_size(b, hq, hkv, d, cand) > SCRATCH),
                 None)
    if batch is None:
        pytest.skip("no request of this shape exceeds the scratch on this device")
    q = torch.zeros(batch, hq, d, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(1, hkv, 64, d, dtype=torch.bfloat16, device=DEV)
    layout = _lib.KvLayout(k.data_ptr(), k.data_ptr(), 64, 0, 64, 64, None, 0, 64)
    ctx = torch.full((batch,), 64, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    rc = _lib.lib.spa_paged_decode_noalloc(q.data_ptr(), _lib.SPA_BF16, batch, hq, hkv, d, ctypes.byref(layout),
                                           ctx.data_ptr(), 0, None, 0, cand, d ** -0.5, out.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.SPA_ERR_WORKSPACE
    assert _lib.device_error_flags() == 0
