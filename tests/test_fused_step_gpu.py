"""The single-launch step (every decode cluster routes its sequence itself) against the
chained router + decode launches and the oracle: the same pages bit for bit, the same
outputs bit for bit (same split plan and merge order), and the oracle within the bf16
tolerance (2e-2 absolute + 1e-2 relative).  Also the (sequence, kv head) shard entry
point: every shard selects the full step's pages, and the shards' outputs assemble into
the full output within the same tolerance."""

import pytest
import torch

import attention_b200 as spa
import oracle
from attention_b200 import workloads
from attention_b200.sharding import DecodeShard

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    spa.set_step_fusion(True)
    yield
    spa.set_step_fusion(True)
    assert spa.device_error_flags() == 0


def _both(fn):
    """(fused result, chained result) of one step call."""
    spa.set_step_fusion(True)
    a = fn()
    torch.cuda.synchronize()
    spa.set_step_fusion(False)
    b = fn()
    torch.cuda.synchronize()
    spa.set_step_fusion(True)
    return a, b


def _close(out, ref):
    o = out.double().cpu()
    return bool(((o - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all())


@pytest.mark.parametrize("m", [2, 4, 8])
def test_fused_tree_step_full_size(m):
    """The 128k configuration (B4, 32/8 heads, D128, P256, 512 pages, W256, two-level
    router): fused == chained exactly, pages == the oracle's."""
    cfg = workloads.SparseDecodeConfig(top_m=m)
    wl = workloads.sparse_decode_workload(cfg, groups=2, seed=20 + m)
    scale = cfg.head_dim ** -0.5
    for g in range(2):
        table, q = wl["page_table"][g], wl["query"][g]
        summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=table, superblock=cfg.superblock)

        def step():
            return spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                          superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=m,
                                          local_window=cfg.local_window, block_size=cfg.page_size,
                                          router_scale=scale, page_table=table, context_lens=wl["context_lens"])

        (out_f, sel_f), (out_c, sel_c) = _both(step)
        assert torch.equal(sel_f, sel_c)
        assert torch.equal(out_f, out_c)
        exp = oracle.select_blocks_tree(q.cpu(), sup.cpu(), summ.cpu(), superblock=cfg.superblock,
                                        top_super=cfg.top_super, top_blocks=m, scale=scale)
        assert torch.equal(sel_f.cpu(), exp)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d,tree", [(32, 8, 128, True), (8, 8, 64, False), (16, 1, 128, True),
                                           (12, 4, 64, True), (64, 4, 128, False), (8, 2, 64, False)])
def test_fused_step_shapes_against_oracle(dtype, hq, hkv, d, tree):
    """GQA groups 1..16, head_dim 64/128, one and two levels, a partial last superblock,
    ragged contexts whose local window overlaps the last routable page."""
    gen = torch.Generator().manual_seed(hq * 7 + d + hkv)
    b, page, n_pages, win, m, sb = 3, 64, 45, 96, 5, 8
    max_ctx = n_pages * page + win
    ctx = [max_ctx, max_ctx - 37, max_ctx - win + 1]
    n_phys = b * (max_ctx // page + 1)
    k_pool = (torch.randn(n_phys, hkv, page, d, generator=gen) * 0.5).to(dtype)
    v_pool = (torch.randn(n_phys, hkv, page, d, generator=gen) * 0.5).to(dtype)
    table = torch.randperm(n_phys, generator=gen).view(b, -1).to(torch.int32)
    q = (torch.randn(b, hq, d, generator=gen) * 0.5).to(dtype)
    kd, vd, td = k_pool.to(DEV), v_pool.to(DEV), table.to(DEV)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=DEV)
    summ, sup = spa.page_summaries(kd, block_size=page, n_pages=n_pages, page_table=td, superblock=sb)
    scale = d ** -0.5
    kw = dict(super_summaries=sup, superblock=sb, top_super=3) if tree else {}

    def step():
        return spa.sparse_decode_step(q.to(DEV), kd, vd, summ, top_blocks=m, local_window=win, block_size=page,
                                      router_scale=scale, page_table=td, context_lens=ctx_d, **kw)

    (out_f, sel_f), (out_c, sel_c) = _both(step)
    assert torch.equal(sel_f, sel_c)
    assert torch.equal(out_f, out_c)
    if tree:
        exp = oracle.select_blocks_tree(q, sup.cpu(), summ.cpu(), superblock=sb, top_super=3, top_blocks=m,
                                        scale=scale)
    else:
        exp = oracle.select_blocks(q, summ.cpu(), m, scale=scale)
    assert torch.equal(sel_f.cpu(), exp)
    kc = oracle.paged_to_contiguous(k_pool, table, max_ctx)
    vc = oracle.paged_to_contiguous(v_pool, table, max_ctx)
    ref = oracle.gather_decode(q, kc, vc, exp, local_window=win, block_size=page, context_lens=ctx)
    assert _close(out_f, ref)


def test_fused_step_decoder_shape():
    """The integrated decoder's step: B1, 8 heads (MHA), D64, pages of 128, 129 routable
    pages, 128-token window, top-8, one level."""
    gen = torch.Generator().manual_seed(5)
    b, h, d, page, n_pages, win, m = 1, 8, 64, 128, 129, 128, 8
    ctx = n_pages * page + win
    k = (torch.randn(b, h, ctx, d, generator=gen) * 0.5).to(torch.bfloat16)
    v = (torch.randn(b, h, ctx, d, generator=gen) * 0.5).to(torch.bfloat16)
    q = (torch.randn(b, h, d, generator=gen) * 0.5).to(torch.bfloat16)
    k_pool = k.view(b, h, ctx // page, page, d).permute(0, 2, 1, 3, 4).reshape(-1, h, page, d).contiguous()
    v_pool = v.view(b, h, ctx // page, page, d).permute(0, 2, 1, 3, 4).reshape(-1, h, page, d).contiguous()
    table = torch.arange(ctx // page, dtype=torch.int32).view(1, -1)
    kd, vd, td = k_pool.to(DEV), v_pool.to(DEV), table.to(DEV)
    ctx_d = torch.tensor([ctx], dtype=torch.int32, device=DEV)
    summ = spa.page_summaries(kd, block_size=page, n_pages=n_pages, page_table=td)

    def step():
        return spa.sparse_decode_step(q.to(DEV), kd, vd, summ, top_blocks=m, local_window=win, block_size=page,
                                      router_scale=d ** -0.5, page_table=td, context_lens=ctx_d)

    (out_f, sel_f), (out_c, sel_c) = _both(step)
    assert torch.equal(sel_f, sel_c) and torch.equal(out_f, out_c)
    ref_summ, _ = oracle.summaries_fp64(k, page, n_pages)
    exp = oracle.select_blocks(q, ref_summ, m, scale=d ** -0.5)
    assert torch.equal(sel_f.cpu(), exp)
    assert _close(out_f, oracle.gather_decode(q, k, v, exp, local_window=win, block_size=page))


@pytest.mark.parametrize("world,m,pages", [(2, 4, 128), (4, 4, 128), (8, 4, 128), (2, 8, 512), (8, 2, 512)])
def test_kv_head_shards_assemble_the_full_step(world, m, pages):
    """The 128k batch split into (sequence, kv head) shards as on `world` GPUs, run here
    one shard after another: each shard's pages equal the full step's for its
    sequences, and the assembled outputs match the full step within tolerance.  (Two
    sequences per shard at m = 8: fewer pairs than the decode's cluster plan wants, so the
    one-launch step takes clusters of 8 splits anyway.)"""
    cfg = workloads.SparseDecodeConfig(top_m=m, pages_per_seq=pages)
    wl = workloads.sparse_decode_workload(cfg, groups=1, seed=31)
    table, q, ctx = wl["page_table"][0], wl["query"][0], wl["context_lens"]
    summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                   page_table=table, superblock=cfg.superblock)
    kw = dict(super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
              local_window=cfg.local_window, block_size=cfg.page_size, router_scale=cfg.head_dim ** -0.5)
    full_out, full_sel = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, page_table=table,
                                                context_lens=ctx, **kw)
    assembled = torch.empty_like(full_out)
    for rank in range(world):
        sh = DecodeShard(cfg.batch, cfg.q_heads, cfg.kv_heads, world, rank)
        rows, kv = sh.rows, sh.kv
        tab = table[rows]
        phys = tab.reshape(-1).long()
        kp = wl["k_pool"][phys][:, kv].contiguous()
        vp = wl["v_pool"][phys][:, kv].contiguous()
        local_tab = torch.arange(phys.numel(), dtype=torch.int32, device=DEV).view(tab.shape)
        sk = dict(kw, super_summaries=sup[rows].contiguous())
        out, sel = spa.sparse_decode_step(q[rows].contiguous(), kp, vp, summ[rows].contiguous(), page_table=local_tab,
                                          context_lens=ctx[rows].contiguous(),
                                          kv_head_range=(kv.start, kv.stop - kv.start), **sk)
        assert torch.equal(sel, full_sel[rows])
        assembled[rows, sh.q_heads] = out
    ref = full_out.double().cpu()
    assert ((assembled.double().cpu() - ref).abs() <= 2e-2 + 1e-2 * ref.abs()).all()
