"""Promotion refresh gate and gated routers on the GPU against the oracle restatement.

The gate's batch means are compared with the reference's RefreshHead and drift distance
(tests/golden/refresh_gate.npz) within 1e-5; decisions are compared at thresholds far from
the computed means; selections are bit-exact."""

import numpy as np
import pytest
import torch

import attention_b200 as spa
import oracle
from oracle.refresh_gate import GateSim, drift_distance

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert spa.device_error_flags() == 0


def _primed(gate, cached_state=None):
    """A gate with a promoted selection and a given cached state (decisions then depend
    on the policy, not on the first-step rule)."""
    gate.flags[1] = 1
    if cached_state is not None:
        gate.cached_state.copy_(cached_state)
    return gate


@pytest.mark.parametrize("mode", ["drift", "learned"])
def test_gate_scores_match_reference_fixture(golden_dir, mode):
    fx = dict(np.load(golden_dir / "refresh_gate.npz"))
    b, w = fx["shape"].tolist()
    head = {k: torch.from_numpy(fx[k]) for k in ("w1", "b1", "w2", "b2")}
    for case in range(fx["state"].shape[0]):
        state = torch.from_numpy(fx["state"][case]).to(DEV)
        cached = torch.from_numpy(fx["cached"][case]).to(DEV)
        ref = float((fx["drift"] if mode == "drift" else fx["prob"])[case].mean())
        for thr, expect in ((ref - 0.01, True), (ref + 0.01, False)):
            gate = _primed(spa.RefreshGate(mode, b, width=w, threshold=thr, head=head), cached)
            gate.decide(state=state)
            assert abs(gate.score.item() - ref) <= 1e-5
            assert gate.refreshed == expect
            # a refresh caches the current state; a closed gate keeps the old one
            assert torch.equal(gate.cached_state, state if expect else cached)


@pytest.mark.parametrize("batch,width", [(3, 6), (40, 100), (4, 4096), (1, 4099), (5, 4096)])
def test_drift_gate_shapes(batch, width):
    """Drift scores and the refresh copy at widths and batches that take every path of the
    gate kernel: 16-byte and element loads, several warps per row or several rows per
    warp, a refresh copy with and without 16-byte accesses and with a partial last round."""
    gen = torch.Generator().manual_seed(batch * 10007 + width)
    state = torch.randn(batch, width, generator=gen)
    cached = state + 0.3 * torch.randn(batch, width, generator=gen)
    ref = float(drift_distance(state, cached).mean())
    for thr, expect in ((ref - 0.01, True), (ref + 0.01, False)):
        gate = _primed(spa.RefreshGate("drift", batch, width=width, threshold=thr), cached.to(DEV))
        gate.decide(state=state.to(DEV))
        assert abs(gate.score.item() - ref) <= 1e-5
        assert gate.refreshed == expect
        assert torch.equal(gate.cached_state.cpu(), state if expect else cached)


def test_first_step_always_routes():
    gate = spa.RefreshGate("drift", 2, width=16, threshold=10.0)
    gate.decide(state=torch.zeros(2, 16, device=DEV))
    assert gate.refreshed


def test_ttl_and_signature_decisions():
    gate = _primed(spa.RefreshGate("ttl", 3, ttl=4))
    step_dev = torch.zeros(1, dtype=torch.int32, device=DEV)
    for t in range(10):
        gate.decide(step=t)
        assert gate.refreshed == (t % 4 == 0)
        step_dev.fill_(t)
        gate.decide(step=step_dev)
        assert gate.refreshed == (t % 4 == 0)
    sig_gate = _primed(spa.RefreshGate("signature", 2, sig_len=3))
    sig_gate.cached_signature.copy_(torch.tensor([[1, 2, 3], [4, 5, 6]]))
    same = torch.tensor([[1, 2, 3], [4, 5, 6]], device=DEV)
    sig_gate.decide(signature=same)
    assert not sig_gate.refreshed
    changed = torch.tensor([[1, 2, 3], [4, 5, 7]], device=DEV)
    sig_gate.decide(signature=changed)
    assert sig_gate.refreshed and torch.equal(sig_gate.cached_signature, changed)


def test_gated_router_sequence_matches_oracle():
    """Drift-gated single-level router over 12 steps whose query jumps at steps 4 and 8:
    the selection used each step equals the oracle's promotion-reuse loop, and steps with a
    closed gate use no summary (they run on NaN summaries)."""
    gen = torch.Generator().manual_seed(11)
    b, hq, hkv, d, n_pages, m = 2, 8, 2, 64, 40, 5
    summ = torch.randn(b, hkv, n_pages, d, generator=gen)
    poisoned = torch.full_like(summ, float("nan")).to(DEV)
    summ_dev = summ.to(DEV)
    gate = spa.RefreshGate("drift", b, width=hq * d, threshold=0.05)
    sim = GateSim("drift", threshold=0.05)
    q = torch.randn(b, hq, d, generator=gen)
    refreshes = []
    for t in range(12):
        if t in (4, 8):
            q = torch.randn(b, hq, d, generator=gen)
        qt = (q + 0.01 * torch.randn(b, hq, d, generator=gen)).to(torch.bfloat16)
        state = qt.float().reshape(b, -1)
        fresh = oracle.select_blocks(qt, summ, m)
        if sim.cached_state is not None:  # the decision is far from the threshold
            assert abs(float(drift_distance(state, sim.cached_state).mean()) - 0.05) > 1e-3
        used, refresh = sim.step(fresh, state=state)
        gate.decide(state=state.to(DEV))
        sel = spa.select_blocks(qt.to(DEV), summ_dev if refresh else poisoned, m, gate=gate)
        assert gate.refreshed == refresh
        assert torch.equal(sel.cpu(), used)
        refreshes.append(refresh)
    assert refreshes == [t in (0, 4, 8) for t in range(12)]


def test_gated_tree_step_reuses_promoted_pages():
    """sparse_decode_step with a TTL gate: routed steps equal the ungated step; reused
    steps attend over the promoted pages (equal to the gather decode over them)."""
    from attention_b200 import workloads

    cfg = workloads.SparseDecodeConfig(top_m=4)
    wl = workloads.sparse_decode_workload(cfg, groups=3, seed=5)
    k_pool, v_pool, lens = wl["k_pool"], wl["v_pool"], wl["context_lens"]
    table = wl["page_table"][0]
    summ, sup = spa.page_summaries(k_pool, block_size=cfg.page_size, n_pages=cfg.routable_pages, page_table=table,
                                   superblock=cfg.superblock)
    kw = dict(top_blocks=cfg.top_m, local_window=cfg.local_window, block_size=cfg.page_size,
              super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super,
              router_scale=cfg.head_dim ** -0.5, page_table=table, context_lens=lens)
    gate = spa.RefreshGate("ttl", cfg.batch, ttl=2)
    promoted = None
    for t in range(3):
        q = wl["query"][t]
        gate.decide(step=t)
        out, sel = spa.sparse_decode_step(q, k_pool, v_pool, summ, gate=gate, **kw)
        ref_out, ref_sel = spa.sparse_decode_step(q, k_pool, v_pool, summ, **kw)
        if t % 2 == 0:
            assert torch.equal(sel, ref_sel) and torch.equal(out, ref_out)
            promoted = ref_sel.clone()
        else:
            assert torch.equal(sel, promoted)
            exp = spa.paged_gather_decode_attention(q, k_pool, v_pool, promoted, local_window=cfg.local_window,
                                                    block_size=cfg.page_size, page_table=table, context_lens=lens)
            assert torch.equal(out, exp)


def test_gated_session_matches_gated_steps():
    """SparseDecodeSession built with a gate: after each gate decision on the same stream,
    the session's step returns what sparse_decode_step with an identical gate returns."""
    from attention_b200 import workloads

    cfg = workloads.SparseDecodeConfig(top_m=4)
    wl = workloads.sparse_decode_workload(cfg, groups=4, seed=6)
    k_pool, v_pool, lens = wl["k_pool"], wl["v_pool"], wl["context_lens"]
    table = wl["page_table"][0]
    summ, sup = spa.page_summaries(k_pool, block_size=cfg.page_size, n_pages=cfg.routable_pages, page_table=table,
                                   superblock=cfg.superblock)
    kw = dict(top_blocks=cfg.top_m, local_window=cfg.local_window, block_size=cfg.page_size,
              super_summaries=sup, superblock=cfg.superblock, top_super=cfg.top_super,
              router_scale=cfg.head_dim ** -0.5, page_table=table, context_lens=lens)
    g_sess = spa.RefreshGate("ttl", cfg.batch, ttl=2)
    g_ref = spa.RefreshGate("ttl", cfg.batch, ttl=2)
    sess = spa.SparseDecodeSession(k_pool, v_pool, summ, q_heads=cfg.q_heads, gate=g_sess, **kw)
    g_sess.reset()  # the session's set-up step routed once; start both gates from scratch
    for t in range(4):
        q = wl["query"][t]
        g_sess.decide(step=t)
        out, sel = sess.step(q.cpu())
        torch.cuda.synchronize()
        g_ref.decide(step=t)
        ref_out, ref_sel = spa.sparse_decode_step(q, k_pool, v_pool, summ, gate=g_ref, **kw)
        assert torch.equal(sel, ref_sel.cpu()) and torch.equal(out, ref_out.cpu()), t
    sess.close()
