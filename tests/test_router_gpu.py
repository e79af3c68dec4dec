"""Summaries and router kernels: bit-exact against the oracle (scores and indices)."""

import pytest
import torch

import attention_b200 as spa
import oracle
from attention_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert spa.device_error_flags() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("heads,dim", [((32, 8), 128), ((8, 8), 64), ((12, 4), 96)])
def test_summaries_and_scores_bit_exact(dtype, heads, dim):
    hq, hkv = heads
    gen = torch.Generator().manual_seed(dim + hq)
    b, page, n_pages, win = 3, 64, 21, 64
    k = (torch.randn(b, hkv, n_pages * page + win, dim, generator=gen) * 0.5).to(dtype)
    q = (torch.randn(b, hq, dim, generator=gen) * 0.5).to(dtype)
    summ, sup = spa.page_summaries(k.to(DEV), block_size=page, local_window=win, superblock=4)
    ref, sums = oracle.summaries_fp64(k, page, n_pages)
    assert torch.equal(summ.cpu(), ref)
    assert torch.equal(sup.cpu(), oracle.super_summaries(sums, 4, page))
    scale = dim ** -0.5
    for m in (1, 5, n_pages):
        sel, scores = spa.select_blocks(q.to(DEV), summ, m, scale=scale, return_scores=True)
        ref_scores = oracle.router_scores(q, ref, scale)
        assert torch.equal(scores.cpu(), ref_scores)  # fp64, bit for bit
        assert torch.equal(sel.cpu(), oracle.topm(ref_scores, m))


@pytest.mark.parametrize("heads,dim,n_pages", [((8, 8), 64, 130), ((32, 8), 128, 200), ((16, 16), 64, 150),
                                               ((8, 8), 64, 65)])
def test_single_level_router_many_pages(heads, dim, n_pages):
    """Single-level routing with more candidates than warps in the cluster (several per
    warp: the prefetching scoring loop when kv heads <= 8), scores bit-exact."""
    hq, hkv = heads
    gen = torch.Generator().manual_seed(n_pages + hq)
    b, page = 2, 16
    k = (torch.randn(b, hkv, n_pages * page, dim, generator=gen) * 0.5).to(torch.bfloat16)
    q = (torch.randn(b, hq, dim, generator=gen) * 0.5).to(torch.bfloat16)
    summ, _ = spa.page_summaries(k.to(DEV), block_size=page, superblock=4)
    ref, _ = oracle.summaries_fp64(k, page, n_pages)
    assert torch.equal(summ.cpu(), ref)
    for m in (1, 8, 33):
        sel, scores = spa.select_blocks(q.to(DEV), summ, m, scale=dim ** -0.5, return_scores=True)
        ref_scores = oracle.router_scores(q, ref, dim ** -0.5)
        assert torch.equal(scores.cpu(), ref_scores)
        assert torch.equal(sel.cpu(), oracle.topm(ref_scores, m))


def test_exact_ties_resolve_to_lower_page():
    gen = torch.Generator().manual_seed(4)
    b, h, d, page = 2, 4, 64, 32
    base = torch.randn(b, h, page, d, generator=gen)
    # pages 1, 4, 6 identical (identical summaries -> identical scores); page 2 a different copy
    pages = [torch.randn(b, h, page, d, generator=gen) for _ in range(8)]
    for i in (1, 4, 6):
        pages[i] = base
    k = torch.cat(pages, dim=2)
    q = torch.randn(b, h, d, generator=gen)
    summ = spa.page_summaries(k.to(DEV), block_size=page)
    scores = oracle.router_scores(q, oracle.summaries_fp64(k, page, 8)[0])
    assert scores[0, 1] == scores[0, 4] == scores[0, 6]
    for m in range(1, 9):
        sel = spa.select_blocks(q.to(DEV), summ, m)
        assert torch.equal(sel.cpu(), oracle.topm(scores, m))
    order = spa.select_blocks(q.to(DEV), summ, 8)[0].tolist()
    tied = [p for p in order if p in (1, 4, 6)]
    assert tied == [1, 4, 6]


@pytest.mark.parametrize("n_pages,superblock,top_super",
                         [(100, 16, 4), (511, 16, 4), (37, 8, 2), (64, 16, 4), (600, 2, 32), (800, 4, 40)])
def test_tree_router_matches_oracle(n_pages, superblock, top_super):
    gen = torch.Generator().manual_seed(n_pages)
    b, hq, hkv, d, page = 2, 32, 8, 128, 16
    k = (torch.randn(b, hkv, n_pages * page, d, generator=gen) * 0.5).to(torch.bfloat16)
    q = (torch.randn(b, hq, d, generator=gen) * 0.5).to(torch.bfloat16)
    summ, sup = spa.page_summaries(k.to(DEV), block_size=page, superblock=superblock)
    ref_summ, sums = oracle.summaries_fp64(k, page, n_pages)
    ref_sup = oracle.super_summaries(sums, superblock, page)
    for m in (2, 4, 8):
        got = spa.select_blocks_tree(q.to(DEV), sup, summ, superblock=superblock, top_super=top_super,
                                     top_blocks=m, scale=d ** -0.5)
        exp = oracle.select_blocks_tree(q, ref_sup, ref_summ, superblock=superblock, top_super=top_super,
                                        top_blocks=m, scale=d ** -0.5)
        assert torch.equal(got.cpu(), exp)


@pytest.mark.parametrize("m", [2, 4, 8])
def test_sparse_decode_128k_full_size(m):
    """The full tree-routed configuration (B4, 32/8 heads, D128, P256, 512 pages, W256):
    summaries and selection bit-exact, output within bf16 tolerance on every head."""
    cfg = workloads.SparseDecodeConfig(top_m=m)
    wl = workloads.sparse_decode_workload(cfg, groups=1, seed=3)
    k_pool, v_pool, table = wl["k_pool"], wl["v_pool"], wl["page_table"][0]
    q = wl["query"][0]
    summ, sup = spa.page_summaries(k_pool, block_size=cfg.page_size, n_pages=cfg.routable_pages, page_table=table,
                                   superblock=cfg.superblock)
    # bit-exact summaries on a sample of (b, page) against the oracle
    for b, g in ((0, 0), (1, 77), (3, cfg.routable_pages - 1)):
        keys = k_pool[table[b, g].long()].cpu().unsqueeze(0)  # [1, Hkv, P, D] = one page
        ref, _ = oracle.summaries_fp64(keys, cfg.page_size, 1)  # [1, Hkv, 1, D]
        assert torch.equal(summ[b, :, g].cpu(), ref[0, :, 0])
    sel = spa.select_blocks_tree(q, sup, summ, superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=m,
                                 scale=cfg.head_dim ** -0.5)
    exp = oracle.select_blocks_tree(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                    top_super=cfg.top_super, top_blocks=m, scale=cfg.head_dim ** -0.5)
    assert torch.equal(sel.cpu(), exp)
    # the reference's own arithmetic order (einsum, mean over heads, topk) picks the same pages
    ein = oracle.select_blocks_tree_einsum(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                           top_super=cfg.top_super, top_blocks=m)
    assert torch.equal(sel.cpu(), ein)
    out = spa.paged_gather_decode_attention(q, k_pool, v_pool, sel, local_window=cfg.local_window,
                                            block_size=cfg.page_size, page_table=table,
                                            context_lens=wl["context_lens"])
    selc = sel.cpu()
    for b in range(cfg.batch):
        toks = oracle.candidate_tokens(cfg.context, cfg.local_window, selc[b].tolist(), cfg.page_size)
        pages = sorted({t // cfg.page_size for t in toks})
        kp = k_pool[table[b, pages].long()].cpu()
        vp = v_pool[table[b, pages].long()].cpu()
        remap = {p: i for i, p in enumerate(pages)}
        idx = torch.tensor([remap[t // cfg.page_size] * cfg.page_size + t % cfg.page_size for t in toks])
        kc = kp.permute(1, 0, 2, 3).reshape(cfg.kv_heads, -1, cfg.head_dim)[:, idx][None]
        vc = vp.permute(1, 0, 2, 3).reshape(cfg.kv_heads, -1, cfg.head_dim)[:, idx][None]
        ref = oracle.reference_attention(q[b : b + 1].cpu(), kc, vc)
        o = out[b : b + 1].double().cpu()
        assert ((o - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()


def _router_inputs():
    import importlib
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    return importlib.import_module("router_inputs")


@pytest.mark.parametrize("tag", ["needles", "plain"])
def test_tree_router_pinned_to_reference_cfg3(golden_dir, tag):
    """spa_router_tree_topm returns exactly the reference's select_blocks composed over
    superblocks then pages (fixture made by the reference's functions) at the 128k
    shape: 511 pages, 32/8 heads, D128, m = 2, 4, 8, with the step's scale and without."""
    import numpy as np

    ri = _router_inputs()
    fx = dict(np.load(golden_dir / "router_cfg3.npz"))
    batch, needles = fx[f"{tag}_shape"].tolist()
    inp = ri.router_cfg3_inputs(int(fx[f"{tag}_seed"]), batch, needles)
    c = ri.CFG3
    q, sup, summ = (inp[k].to(DEV) for k in ("query", "supers", "summaries"))
    for m in (2, 4, 8):
        ref = torch.from_numpy(fx[f"{tag}_m{m}_f32"])
        for scale in (1.0, c["head_dim"] ** -0.5):
            got = spa.select_blocks_tree(q, sup, summ, superblock=c["superblock"], top_super=c["top_super"],
                                         top_blocks=m, scale=scale)
            assert torch.equal(got.cpu(), ref), (m, scale)


def test_router_pinned_to_reference_cfg5(golden_dir):
    import numpy as np

    ri = _router_inputs()
    fx = dict(np.load(golden_dir / "router_cfg5.npz"))
    inp = ri.router_cfg5_inputs(int(fx["seed"]), int(fx["batch"]))
    ref = torch.from_numpy(fx["m8_f32"])
    for scale in (1.0, ri.CFG5["head_dim"] ** -0.5):
        got = spa.select_blocks(inp["query"].to(DEV), inp["summaries"].to(DEV), 8, scale=scale)
        assert torch.equal(got.cpu(), ref)


def test_tree_router_reference_order_bench_workload():
    """Every batch row of the bench's 128k workload (16 independent batches of 4 rows
    in one pool): the kernel's selection equals the reference's einsum/mean/topk order."""
    cfg = workloads.SparseDecodeConfig(top_m=8)
    groups = 16
    wl = workloads.sparse_decode_workload(cfg, groups=groups, seed=0)
    scale = cfg.head_dim ** -0.5
    for gi in range(groups):
        table = wl["page_table"][gi]
        summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=table, superblock=cfg.superblock)
        q = wl["query"][gi]
        for m in (2, 4, 8):
            got = spa.select_blocks_tree(q, sup, summ, superblock=cfg.superblock, top_super=cfg.top_super,
                                         top_blocks=m, scale=scale)
            ref = oracle.select_blocks_tree_einsum(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                                   top_super=cfg.top_super, top_blocks=m)
            assert torch.equal(got.cpu(), ref), (gi, m)


# ---------------------------------------------------------------- periodic causal router
def test_periodic_router_golden(golden_dir):
    import numpy as np

    fx = dict(np.load(golden_dir / "periodic_router.npz"))
    b, h, ctx, d, page, stride, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    q = torch.randn(b, h, ctx, d)
    k = torch.randn_like(q)
    out = spa.periodic_router(q.to(DEV), k.to(DEV), block_size=page, router_stride=stride, top_blocks=m)
    assert torch.equal(out.cpu(), torch.from_numpy(fx["selected"]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [
    (2, 3, 4096, 64, 256, 128, 4),   # tiled kernel, top-4 lists
    (1, 2, 832, 96, 64, 64, 8),      # 13 updates (partial tile of 8), head_dim not a multiple of 32
    (1, 2, 2048, 128, 64, 128, 20),  # top_m > 16: the untiled kernel; early updates padded with -1
    (1, 1, 1024, 32, 128, 32, 1),    # updates before the first complete block: all -1
])
def test_periodic_router_matches_oracle(dtype, shape):
    gen = torch.Generator().manual_seed(11)
    b, h, s, d, page, stride, m = shape
    q = (torch.randn(b, h, s, d, generator=gen) * 0.5).to(dtype)
    k = (torch.randn(b, h, s, d, generator=gen) * 0.5).to(dtype)
    out = spa.periodic_router(q.to(DEV), k.to(DEV), block_size=page, router_stride=stride, top_blocks=m)
    ref = oracle.periodic_router(q, k, block_size=page, router_stride=stride, top_blocks=m)
    assert torch.equal(out.cpu(), ref)
