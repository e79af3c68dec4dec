"""The fused step (router -> gather decode, chained on the device) equals the two
separate calls bit for bit, and the oracle within tolerance."""

import numpy as np
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


@pytest.mark.parametrize("m", [2, 4, 8])
def test_tree_step_equals_separate_calls(m):
    cfg = workloads.SparseDecodeConfig(top_m=m, pages_per_seq=64)
    wl = workloads.sparse_decode_workload(cfg, groups=2, seed=m)
    for g in range(2):
        table, q = wl["page_table"][g], wl["query"][g]
        summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=table, superblock=cfg.superblock)
        scale = cfg.head_dim ** -0.5
        out, sel = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                          superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=m,
                                          local_window=cfg.local_window, block_size=cfg.page_size, router_scale=scale,
                                          page_table=table, context_lens=wl["context_lens"])
        sel2 = spa.select_blocks_tree(q, sup, summ, superblock=cfg.superblock, top_super=cfg.top_super,
                                      top_blocks=m, scale=scale)
        out2 = spa.paged_gather_decode_attention(q, wl["k_pool"], wl["v_pool"], sel2, local_window=cfg.local_window,
                                                 block_size=cfg.page_size, page_table=table,
                                                 context_lens=wl["context_lens"])
        assert torch.equal(sel, sel2)
        assert torch.equal(out, out2)
        exp = oracle.select_blocks_tree(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                        top_super=cfg.top_super, top_blocks=m, scale=scale)
        assert torch.equal(sel.cpu(), exp)


def test_single_level_step_on_reference_layout(golden_dir):
    fx = dict(np.load(golden_dir / "gather_small.npz"))
    b, h, length, d, page, win, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    q = torch.randn(b, h, d)
    k = torch.randn(b, h, length, d)
    v = torch.randn_like(k)
    kd, vd = k.to(DEV), v.to(DEV)
    summ = spa.page_summaries(kd, block_size=page, local_window=win)
    out, sel = spa.sparse_decode_step(q.to(DEV), kd, vd, summ, top_blocks=m, local_window=win, block_size=page)
    assert torch.equal(sel.cpu(), torch.from_numpy(fx["selected"]))
    ref = torch.from_numpy(fx["out"]).double()
    assert ((out.double().cpu() - ref).abs() <= 1e-5).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_step_head_dim_64(dtype):
    gen = torch.Generator().manual_seed(9)
    b, hq, hkv, d, page, win, n_pages = 2, 16, 4, 64, 128, 128, 20
    length = win + n_pages * page
    q = (torch.randn(b, hq, d, generator=gen) * 0.5).to(dtype)
    k = (torch.randn(b, hkv, length, d, generator=gen) * 0.5).to(dtype)
    v = (torch.randn(b, hkv, length, d, generator=gen) * 0.5).to(dtype)
    kd, vd = k.to(DEV), v.to(DEV)
    summ = spa.page_summaries(kd, block_size=page, local_window=win)
    out, sel = spa.sparse_decode_step(q.to(DEV), kd, vd, summ, top_blocks=3, local_window=win, block_size=page,
                                      router_scale=d ** -0.5)
    ref_summ, _ = oracle.summaries_fp64(k, page, n_pages)
    exp_sel = oracle.select_blocks(q, ref_summ, 3, scale=d ** -0.5)
    assert torch.equal(sel.cpu(), exp_sel)
    ref = oracle.gather_decode(q, k, v, exp_sel, local_window=win, block_size=page)
    o = out.double().cpu()
    assert ((o - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()


def test_session_replays_match_direct_steps():
    """SparseDecodeSession (native session: the step's kernels read the query from pinned
    host memory, a copy kernel returns output and page ids) returns the same outputs and
    page ids as sparse_decode_step, for consecutive steps with different queries (both host
    buffers of the double buffering are checked)."""
    cfg = workloads.SparseDecodeConfig(top_m=4)
    wl = workloads.sparse_decode_workload(cfg, groups=3, seed=9)
    table = wl["page_table"][0]
    summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                   page_table=table, superblock=cfg.superblock)
    kw = dict(top_blocks=cfg.top_m, local_window=cfg.local_window, block_size=cfg.page_size,
              super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super,
              router_scale=cfg.head_dim ** -0.5, page_table=table, context_lens=wl["context_lens"])
    sess = spa.SparseDecodeSession(wl["k_pool"], wl["v_pool"], summ, q_heads=cfg.q_heads, **kw)
    queries = [wl["query"][g] for g in range(3)]
    results = []
    for q in queries:
        out, sel = sess.step(q.cpu())
        results.append((out, sel))
        torch.cuda.synchronize()
        results[-1] = (out.clone(), sel.clone())
    for q, (out, sel) in zip(queries, results):
        ref_out, ref_sel = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **kw)
        assert torch.equal(out, ref_out.cpu()) and torch.equal(sel, ref_sel.cpu())
    # two steps in flight before one synchronisation: each keeps its own host buffers
    o1, s1 = sess.step(queries[1].cpu())
    o2, s2 = sess.step(queries[2].cpu())
    torch.cuda.synchronize()
    assert torch.equal(o1, results[1][0]) and torch.equal(s1, results[1][1])
    assert torch.equal(o2, results[2][0]) and torch.equal(s2, results[2][1])
    sess.close()
    sess.close()  # idempotent


@pytest.mark.parametrize("io_mode", [0, 1, 2, 3])
def test_session_transfer_modes_agree(io_mode):
    """Every way the session moves the query in and the results out over PCIe (kernels read
    host memory, copy kernel in, router copy, direct host writes) returns the direct step's
    output and page ids."""
    cfg = workloads.SparseDecodeConfig(top_m=4)
    wl = workloads.sparse_decode_workload(cfg, groups=2, seed=11)
    table = wl["page_table"][1]
    summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                   page_table=table, superblock=cfg.superblock)
    kw = dict(top_blocks=cfg.top_m, local_window=cfg.local_window, block_size=cfg.page_size,
              super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super,
              router_scale=cfg.head_dim ** -0.5, page_table=table, context_lens=wl["context_lens"])
    sess = spa.SparseDecodeSession(wl["k_pool"], wl["v_pool"], summ, q_heads=cfg.q_heads, io_mode=io_mode, **kw)
    for g in (1, 0):
        q = wl["query"][g]
        out, sel = sess.step(q.cpu())
        torch.cuda.synchronize()
        ref_out, ref_sel = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **kw)
        assert torch.equal(out, ref_out.cpu()) and torch.equal(sel, ref_sel.cpu())
    sess.close()


def test_session_rejects_unknown_transfer_mode():
    cfg = workloads.SparseDecodeConfig(top_m=4)
    wl = workloads.sparse_decode_workload(cfg, groups=1, seed=12)
    table = wl["page_table"][0]
    summ = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                              page_table=table)
    with pytest.raises(ValueError):
        spa.SparseDecodeSession(wl["k_pool"], wl["v_pool"], summ, q_heads=cfg.q_heads, top_blocks=cfg.top_m,
                                local_window=cfg.local_window, block_size=cfg.page_size, page_table=table,
                                context_lens=wl["context_lens"], io_mode=7)


def test_step_argument_cache_follows_the_tensors():
    """Repeated calls reuse the prepared arguments; in-place updates of the summaries are
    seen (the cache borrows the caller's tensors, it copies nothing); a new pool with the
    same shapes gets its own entry; fresh views of the same storage reuse the entry;
    non-fp32 summaries are converted per call; wrong outputs are refused before any launch."""
    from attention_b200 import step as step_mod

    cfg = workloads.SparseDecodeConfig(top_m=4, pages_per_seq=64)
    wl = workloads.sparse_decode_workload(cfg, groups=2, seed=41)
    table, q, ctx = wl["page_table"][0], wl["query"][0], wl["context_lens"]
    summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                   page_table=table, superblock=cfg.superblock)
    kw = dict(super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
              local_window=cfg.local_window, block_size=cfg.page_size, router_scale=cfg.head_dim ** -0.5,
              page_table=table, context_lens=ctx)
    step_mod._STEP_CACHE.clear()
    step_mod._STEP_META.clear()
    o1, s1 = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **kw)
    o2, s2 = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **kw)
    assert len(step_mod._STEP_CACHE) == 1 and len(step_mod._STEP_META) == 1
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    # a fresh view of the same table each call: same prepared arguments
    for _ in range(3):
        o4, s4 = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **{**kw, "page_table": wl["page_table"][0]})
        assert torch.equal(o4, o1) and torch.equal(s4, s1)
    assert len(step_mod._STEP_META) == 1
    # the other group's table (another storage address): its own entry and its own pages
    summ_b, sup_b = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=wl["page_table"][1], superblock=cfg.superblock)
    _, s5 = spa.sparse_decode_step(wl["query"][1], wl["k_pool"], wl["v_pool"], summ_b,
                                   **{**kw, "page_table": wl["page_table"][1], "super_summaries": sup_b})
    assert len(step_mod._STEP_META) == 2
    exp_b = oracle.select_blocks_tree(wl["query"][1].cpu(), sup_b.cpu(), summ_b.cpu(), superblock=cfg.superblock,
                                      top_super=cfg.top_super, top_blocks=cfg.top_m, scale=cfg.head_dim ** -0.5)
    assert torch.equal(s5.cpu(), exp_b)
    with pytest.raises(ValueError):
        spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, out=torch.empty_like(q)[:-1], **kw)
    with pytest.raises(ValueError):
        spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ,
                               selected=torch.empty(q.size(0), cfg.top_m, dtype=torch.int32, device=q.device), **kw)
    # boost a page that was not selected: the next call must pick it
    row = 0
    cand = [g for g in range(cfg.routable_pages) if g not in s1[row].tolist()
            and (g // cfg.superblock) in s1[row].div(cfg.superblock, rounding_mode="floor").tolist()][0]
    summ[row, :, cand] += 10 * q[row].float().view(cfg.kv_heads, -1, cfg.head_dim).mean(1)
    _, s3 = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, **kw)
    assert cand in s3[row].tolist()
    exp = oracle.select_blocks_tree(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                    top_super=cfg.top_super, top_blocks=cfg.top_m, scale=cfg.head_dim ** -0.5)
    assert torch.equal(s3.cpu(), exp)
    # bf16 summaries: converted per call, never cached
    n_before = len(step_mod._STEP_CACHE), len(step_mod._STEP_META)
    spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ.to(torch.bfloat16), **kw)
    assert (len(step_mod._STEP_CACHE), len(step_mod._STEP_META)) == n_before


@pytest.mark.parametrize("top_m", [2, 8])
def test_host_buffer_step_matches_device_step(top_m):
    """The per-call step with pinned host buffers (copy kernel in, results written into host
    memory by the step) equals the device-buffer step bit for bit, on two batches in a row;
    pageable host memory is refused before any launch."""
    cfg = workloads.SparseDecodeConfig(top_m=top_m, pages_per_seq=128)
    wl = workloads.sparse_decode_workload(cfg, groups=2, seed=43)
    kw = dict(superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
              local_window=cfg.local_window, block_size=cfg.page_size, router_scale=cfg.head_dim ** -0.5,
              context_lens=wl["context_lens"])
    outs = []
    for g in range(2):
        table = wl["page_table"][g]
        summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=table, superblock=cfg.superblock)
        q = wl["query"][g]
        o_dev, s_dev = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                              page_table=table, **kw)
        q_host = q.cpu().pin_memory()
        o_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
        s_host = torch.full((cfg.batch, top_m), -7, dtype=torch.int64).pin_memory()
        r_out, r_sel = spa.sparse_decode_step(q_host, wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                              page_table=table, out=o_host, selected=s_host, **kw)
        assert r_out is o_host and r_sel is s_host
        outs.append((o_dev, s_dev, o_host, s_host))
        if g == 0:
            with pytest.raises(ValueError):
                spa.sparse_decode_step(q.cpu(), wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                       page_table=table, **kw)
    torch.cuda.synchronize()
    for o_dev, s_dev, o_host, s_host in outs:
        assert torch.equal(s_host, s_dev.cpu())
        assert torch.equal(o_host, o_dev.cpu())
    assert spa.device_error_flags() == 0
