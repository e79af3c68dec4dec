"""Split-K paged decode on the GPU against the CPU oracle.

Tolerances (written here, from the path's contract): fp32 outputs within 1e-5
absolute; fp16/bf16 outputs within 2e-2 absolute + 1e-2 relative."""

import numpy as np
import pytest
import torch

import attention_b200 as spa
import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def assert_close(out: torch.Tensor, ref: torch.Tensor, dtype) -> None:
    atol, rtol = (1e-5, 0.0) if dtype == torch.float32 else (2e-2, 1e-2)
    o = out.detach().double().cpu()
    r = ref.double().cpu()
    assert torch.isfinite(o).all()
    err = (o - r).abs()
    bound = atol + rtol * r.abs()
    assert (err <= bound).all(), f"max err {err.max().item():.3e}"


def _rand(shape, dtype, gen, scale=1.0):
    return (torch.randn(shape, generator=gen) * scale).to(dtype)


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert spa.device_error_flags() == 0


# ---------------------------------------------------------------- configuration 1
def test_cfg1_sparse_decode_matches_reference(golden_dir):
    fx = dict(np.load(golden_dir / "cfg1_sparse_decode.npz"))
    from attention_b200 import workloads

    inp = workloads.cpu_sparse_decode_inputs()
    k, v, q = inp["keys"].to(DEV), inp["values"].to(DEV), inp["query"].to(DEV)
    page, win, m = inp["page_size"], inp["local_window"], inp["top_m"]
    summ = spa.page_summaries(k, block_size=page, local_window=win)
    ref_summ, _ = oracle.summaries_fp64(inp["keys"], page, 31)
    assert torch.equal(summ.cpu(), ref_summ)  # bit-exact
    sel = spa.select_blocks(q, summ, m, scale=64 ** -0.5)
    assert torch.equal(sel.cpu(), torch.from_numpy(fx["selected"]))
    out = spa.paged_gather_decode_attention(q, k, v, sel, local_window=win, block_size=page)
    assert_close(out, torch.from_numpy(fx["out"]), torch.float32)
    assert_close(out, torch.from_numpy(fx["dense_masked"]), torch.float32)


# ---------------------------------------------------------------- dense, contiguous [B,H,L,D]
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("heads", [(4, 4), (32, 8), (8, 1)])
@pytest.mark.parametrize("dim", [16, 64, 128])
def test_dense_contiguous(dtype, heads, dim):
    hq, hkv = heads
    gen = torch.Generator().manual_seed(hq * 100 + dim)
    for length in (1, 63, 640, 1283):
        q = _rand((3, hq, dim), dtype, gen)
        k = _rand((3, hkv, length, dim), dtype, gen)
        v = _rand((3, hkv, length, dim), dtype, gen)
        out = spa.paged_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV))
        assert out.dtype == dtype and out.shape == q.shape
        assert_close(out, oracle.dense_decode(q, k, v, [length] * 3), dtype)


def test_dense_golden(golden_dir):
    fx = dict(np.load(golden_dir / "dense_small.npz"))
    b, h, length, d = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    q = torch.randn(b, h, d)
    k = torch.randn(b, h, length, d)
    v = torch.randn_like(k)
    out = spa.paged_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV))
    assert_close(out, torch.from_numpy(fx["out"]), torch.float32)


# ---------------------------------------------------------------- dense, page pool
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("page", [64, 128, 256, 16])
def test_dense_page_pool_ragged(dtype, page):
    gen = torch.Generator().manual_seed(page)
    b, hq, hkv, d = 4, 16, 4, 128
    ctx = [1, page * 3 + 17, 5 * page, 2 * page - 1]
    max_pages = 6
    n_pool = 40
    k_pool = _rand((n_pool, hkv, page, d), dtype, gen, 0.5)
    v_pool = _rand((n_pool, hkv, page, d), dtype, gen, 0.5)
    table = torch.randperm(n_pool, generator=gen)[: b * max_pages].view(b, max_pages).to(torch.int32)
    q = _rand((b, hq, d), dtype, gen, 0.5)
    lens = torch.tensor(ctx, dtype=torch.int32)
    out = spa.paged_decode_attention(q.to(DEV), k_pool.to(DEV), v_pool.to(DEV), page_table=table.to(DEV),
                                     context_lens=lens.to(DEV))
    kc = oracle.paged_to_contiguous(k_pool, table, max_pages * page)
    vc = oracle.paged_to_contiguous(v_pool, table, max_pages * page)
    assert_close(out, oracle.dense_decode(q, kc, vc, ctx), dtype)
    # sliding-window form: only the last W tokens
    w = page + 5
    out = spa.paged_decode_attention(q.to(DEV), k_pool.to(DEV), v_pool.to(DEV), page_table=table.to(DEV),
                                     context_lens=lens.to(DEV), local_window=w)
    assert_close(out, oracle.dense_decode(q, kc, vc, ctx, local_window=w), dtype)


# ---------------------------------------------------------------- gather decode
def test_gather_golden(golden_dir):
    fx = dict(np.load(golden_dir / "gather_small.npz"))
    b, h, length, d, page, win, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    q = torch.randn(b, h, d)
    k = torch.randn(b, h, length, d)
    v = torch.randn_like(k)
    sel = torch.from_numpy(fx["selected"])
    out = spa.paged_gather_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), sel.to(DEV), local_window=win,
                                            block_size=page)
    assert_close(out, torch.from_numpy(fx["out"]), torch.float32)
    # the device router reproduces the reference's selection on these inputs
    summ = spa.page_summaries(k.to(DEV), block_size=page, local_window=win)
    assert torch.equal(spa.select_blocks(q.to(DEV), summ, m).cpu(), sel)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dim", [64, 128])
def test_gather_contiguous_gqa(dtype, dim):
    gen = torch.Generator().manual_seed(dim)
    b, hq, hkv, page, win, n_pages = 3, 32, 8, 256, 256, 9
    length = win + n_pages * page
    q = _rand((b, hq, dim), dtype, gen, 0.5)
    k = _rand((b, hkv, length, dim), dtype, gen, 0.5)
    v = _rand((b, hkv, length, dim), dtype, gen, 0.5)
    for m in (1, 4, 8):
        sel = torch.stack([torch.randperm(n_pages, generator=gen)[:m] for _ in range(b)])
        out = spa.paged_gather_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), sel.to(DEV), local_window=win,
                                                block_size=page)
        ref = oracle.gather_decode(q, k, v, sel, local_window=win, block_size=page)
        assert_close(out, ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gather_page_pool_misaligned_window(dtype):
    """Context not a multiple of the page, window not a multiple of the chunk, empty (-1) slots."""
    gen = torch.Generator().manual_seed(11)
    b, hq, hkv, d, page = 3, 8, 2, 128, 128
    ctx = [5 * page + 77, 3 * page + 1, 7 * page]
    win = 100
    max_pages = 8
    k_pool = _rand((30, hkv, page, d), dtype, gen, 0.5)
    v_pool = _rand((30, hkv, page, d), dtype, gen, 0.5)
    table = torch.randperm(30, generator=gen)[: b * max_pages].view(b, max_pages).to(torch.int32)
    q = _rand((b, hq, d), dtype, gen, 0.5)
    sel = torch.tensor([[0, 3, -1], [2, -1, 0], [4, 1, 5]], dtype=torch.int64)
    lens = torch.tensor(ctx, dtype=torch.int32)
    out = spa.paged_gather_decode_attention(q.to(DEV), k_pool.to(DEV), v_pool.to(DEV), sel.to(DEV),
                                            local_window=win, block_size=page, page_table=table.to(DEV),
                                            context_lens=lens.to(DEV))
    kc = oracle.paged_to_contiguous(k_pool, table, max_pages * page)
    vc = oracle.paged_to_contiguous(v_pool, table, max_pages * page)
    ref = oracle.gather_decode(q, kc, vc, sel, local_window=win, block_size=page, context_lens=ctx)
    assert_close(out, ref, dtype)


def test_gather_stale_nan_rows_do_not_leak():
    """Pool rows outside the candidate set hold NaN; the output must stay finite and exact."""
    gen = torch.Generator().manual_seed(5)
    b, hq, hkv, d, page = 2, 8, 2, 128, 128
    k_pool = _rand((8, hkv, page, d), torch.bfloat16, gen, 0.5)
    v_pool = _rand((8, hkv, page, d), torch.bfloat16, gen, 0.5)
    table = torch.arange(8, dtype=torch.int32).view(b, 4)
    ctx = [3 * page + 10, 2 * page + 100]
    for i, c in enumerate(ctx):  # poison everything past the context
        for t in range(c, 4 * page):
            k_pool[table[i, t // page], :, t % page] = float("nan")
            v_pool[table[i, t // page], :, t % page] = float("nan")
    q = _rand((b, hq, d), torch.bfloat16, gen, 0.5)
    sel = torch.tensor([[0, 1], [1, 0]])
    out = spa.paged_gather_decode_attention(q.to(DEV), k_pool.to(DEV), v_pool.to(DEV), sel.to(DEV), local_window=70,
                                            block_size=page, page_table=table.to(DEV),
                                            context_lens=torch.tensor(ctx, dtype=torch.int32).to(DEV))
    kc = oracle.paged_to_contiguous(k_pool, table, 4 * page)
    vc = oracle.paged_to_contiguous(v_pool, table, 4 * page)
    ref = oracle.gather_decode(q, kc, vc, sel, local_window=70, block_size=page, context_lens=ctx)
    assert_close(out, ref, torch.bfloat16)


# ---------------------------------------------------------------- full-size dense decode (32k)
def test_dense_decode_32k_full_size():
    from attention_b200 import workloads

    cfg = workloads.DenseDecodeConfig()
    wl = workloads.dense_decode_workload(cfg, seed=1)
    out = spa.paged_decode_attention(wl["query"], wl["k_pool"], wl["v_pool"], page_table=wl["page_table"],
                                     context_lens=wl["context_lens"])
    for b in (0, cfg.batch - 1):
        tab = wl["page_table"][b : b + 1].cpu()
        kc = oracle.paged_to_contiguous(wl["k_pool"][tab[0].long()].cpu(), torch.arange(cfg.pages_per_seq)[None],
                                        cfg.context)
        vc = oracle.paged_to_contiguous(wl["v_pool"][tab[0].long()].cpu(), torch.arange(cfg.pages_per_seq)[None],
                                        cfg.context)
        ref = oracle.dense_decode(wl["query"][b : b + 1].cpu(), kc, vc, [cfg.context])
        assert_close(out[b : b + 1], ref, torch.bfloat16)


# ---------------------------------------------------------------- span gather decode
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dim,span", [(64, 3), (128, 3), (128, 70), (16, 5)])
def test_span_gather_contiguous(dtype, dim, span):
    """Reference layout: spans at arbitrary token starts (unaligned, overlapping the window)."""
    gen = torch.Generator().manual_seed(dim + span)
    b, hq, hkv, length, win = 3, 8, 4, 1500, 64
    q = _rand((b, hq, dim), dtype, gen, 0.5)
    k = _rand((b, hkv, length, dim), dtype, gen, 0.5)
    v = _rand((b, hkv, length, dim), dtype, gen, 0.5)
    starts = torch.tensor([[5, 700, 63, 1499], [0, -1, 1436, 900], [128, 129, 64, 1000]], dtype=torch.int64)
    out = spa.span_gather_decode_attention(q.to(DEV), k.to(DEV), v.to(DEV), starts.to(DEV), local_window=win,
                                           span_width=span)
    assert_close(out, oracle.span_decode(q, k, v, starts, local_window=win, span_width=span), dtype)


def test_span_gather_page_pool():
    gen = torch.Generator().manual_seed(77)
    b, hq, hkv, d, page = 2, 16, 4, 128, 128
    ctx = [6 * page + 30, 4 * page]
    k_pool = _rand((20, hkv, page, d), torch.bfloat16, gen, 0.5)
    v_pool = _rand((20, hkv, page, d), torch.bfloat16, gen, 0.5)
    table = torch.randperm(20, generator=gen)[:14].view(b, 7).to(torch.int32)
    q = _rand((b, hq, d), torch.bfloat16, gen, 0.5)
    # spans crossing page boundaries
    starts = torch.tensor([[120, 250, 600], [0, 383, -1]], dtype=torch.int64)
    out = spa.span_gather_decode_attention(q.to(DEV), k_pool.to(DEV), v_pool.to(DEV), starts.to(DEV),
                                           local_window=100, span_width=40, page_table=table.to(DEV),
                                           context_lens=torch.tensor(ctx, dtype=torch.int32).to(DEV))
    kc = oracle.paged_to_contiguous(k_pool, table, 7 * page)
    vc = oracle.paged_to_contiguous(v_pool, table, 7 * page)
    ref = oracle.span_decode(q, kc, vc, starts, local_window=100, span_width=40, context_lens=ctx)
    assert_close(out, ref, torch.bfloat16)


def test_span_gather_pinned_to_reference(golden_dir):
    """fp32 span decode against the reference's build_candidate_indices +
    candidate_attention (span width 3), within the fp32 tolerance."""
    import importlib
    import sys

    import numpy as np

    sys.path.insert(0, str(golden_dir))
    ri = importlib.import_module("router_inputs")
    fx = dict(np.load(golden_dir / "span_gather.npz"))
    inp = ri.span_inputs(int(fx["seed"]))
    c = ri.SPAN
    out = spa.span_gather_decode_attention(inp["query"].to(DEV), inp["keys"].to(DEV), inp["values"].to(DEV),
                                           inp["centers"].to(DEV), local_window=c["local_window"],
                                           span_width=c["span_width"])
    ref = torch.from_numpy(fx["out"]).double()
    assert (out.double().cpu() - ref).abs().max().item() <= 1e-5
