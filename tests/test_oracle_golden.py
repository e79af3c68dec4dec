"""The oracle against the fixtures produced by the reference's own functions."""

import numpy as np
import torch

import oracle


def _load(golden_dir, name):
    return dict(np.load(golden_dir / name))


def _check_sums(fx, **tensors):
    for key, t in tensors.items():
        assert abs(t.double().sum().item() - float(fx[key])) < 1e-6 * max(1.0, abs(float(fx[key]))), key


def test_cfg1_selection_and_output(golden_dir):
    fx = _load(golden_dir, "cfg1_sparse_decode.npz")
    b, h, length, d, page, win, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    keys = torch.randn(b, h, length, d)
    values = torch.randn(b, h, length, d)
    query = torch.randn(b, h, d)
    _check_sums(fx, k_sum=keys, v_sum=values, q_sum=query)
    n_pages = (length - win) // page
    summ, _ = oracle.summaries_fp64(keys, page, n_pages)
    # fp64-accumulated means agree with the reference's fp32 .mean(3) to fp32 rounding
    assert torch.allclose(summ, torch.from_numpy(fx["summaries"]), atol=1e-6, rtol=0)
    sel = oracle.select_blocks(query, summ, m, scale=d ** -0.5)
    assert torch.equal(sel, torch.from_numpy(fx["selected"]))
    out = oracle.gather_decode(query, keys, values, sel, local_window=win, block_size=page)
    assert (out - torch.from_numpy(fx["out"]).double()).abs().max().item() <= 1e-5
    assert (out - torch.from_numpy(fx["dense_masked"]).double()).abs().max().item() <= 1e-5
    # the dense masked form of the oracle agrees with its gather form
    allowed = torch.zeros(b, length, dtype=torch.bool)
    for t in oracle.candidate_tokens(length, win, sel[0].tolist(), page):
        allowed[0, t] = True
    dm = oracle.masked_dense_attention(query, keys, values, allowed)
    assert (dm - out).abs().max().item() <= 1e-12


def test_gather_small(golden_dir):
    fx = _load(golden_dir, "gather_small.npz")
    b, h, length, d, page, win, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    query = torch.randn(b, h, d)
    keys = torch.randn(b, h, length, d)
    values = torch.randn_like(keys)
    _check_sums(fx, k_sum=keys, v_sum=values, q_sum=query)
    summ, _ = oracle.summaries_fp64(keys, page, (length - win) // page)
    sel = oracle.select_blocks(query, summ, m)
    assert torch.equal(sel, torch.from_numpy(fx["selected"]))
    ck, cv = oracle.make_candidates(keys, values, sel, win, page)
    out = oracle.reference_attention(query, ck, cv)
    assert (out - torch.from_numpy(fx["out"]).double()).abs().max().item() <= 1e-5
    out2 = oracle.gather_decode(query, keys, values, sel, local_window=win, block_size=page)
    assert (out2 - out).abs().max().item() <= 1e-12


def test_dense_small(golden_dir):
    fx = _load(golden_dir, "dense_small.npz")
    b, h, length, d = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    query = torch.randn(b, h, d)
    keys = torch.randn(b, h, length, d)
    values = torch.randn_like(keys)
    _check_sums(fx, k_sum=keys, v_sum=values, q_sum=query)
    out = oracle.dense_decode(query, keys, values, [length] * b)
    assert (out - torch.from_numpy(fx["out"]).double()).abs().max().item() <= 1e-5


def test_prefill_small(golden_dir):
    fx = _load(golden_dir, "prefill_small.npz")
    b, h, s, d, w = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    query = torch.randn(b, h, s, d)
    keys = torch.randn_like(query)
    values = torch.randn_like(query)
    _check_sums(fx, k_sum=keys, v_sum=values, q_sum=query)
    ref = torch.from_numpy(fx["out"]).double()
    assert (oracle.local_reference(query, keys, values, w) - ref).abs().max().item() <= 1e-5
    for chunk in (64, 100, 300):
        out = oracle.local_reference_chunked(query, keys, values, w, chunk=chunk)
        assert (out - ref).abs().max().item() <= 1e-5


def test_prefill_chunked_halo_equals_full():
    torch.manual_seed(3)
    q, k, v = (torch.randn(1, 2, 96, 8) for _ in range(3))
    full = oracle.local_reference(q, k, v, 40)
    halo = 40
    part = oracle.local_reference_chunked(q[:, :, 50:], k[:, :, 50:], v[:, :, 50:], 40, chunk=17,
                                          k_halo=k[:, :, 50 - halo:50], v_halo=v[:, :, 50 - halo:50])
    assert (part - full[:, :, 50:]).abs().max().item() <= 1e-12


def test_periodic_router(golden_dir):
    fx = _load(golden_dir, "periodic_router.npz")
    b, h, ctx, d, page, stride, m = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    query = torch.randn(b, h, ctx, d)
    keys = torch.randn_like(query)
    _check_sums(fx, k_sum=keys, q_sum=query)
    sel = oracle.periodic_router(query, keys, block_size=page, router_stride=stride, top_blocks=m)
    assert torch.equal(sel, torch.from_numpy(fx["selected"]))


def test_topm_ties_go_to_lower_index():
    scores = torch.tensor([[1.0, 3.0, 3.0, 3.0, 0.0, 3.0]], dtype=torch.float64)
    assert oracle.topm(scores, 2).tolist() == [[1, 2]]
    assert oracle.topm(scores, 4).tolist() == [[1, 2, 3, 5]]
    ids = torch.tensor([[9, 4, 7, 2, 5, 1]])
    # page ids, not positions, break ties
    assert oracle.topm(scores, 3, ids).tolist() == [[1, 2, 4]]


def test_router_scores_match_einsum_mean():
    torch.manual_seed(1)
    q = torch.randn(2, 8, 64)
    s = torch.randn(2, 2, 17, 64)
    got = oracle.router_scores(q, s, scale=0.125)
    exp = torch.einsum("bhd,bhgd->bhg", q.double(), oracle.expand_kv(s.double(), 8)).mean(1) * 0.125
    assert got.dtype == torch.float32
    assert torch.allclose(got.double(), exp, atol=1e-5, rtol=1e-5)


def test_tree_router_is_two_select_levels():
    torch.manual_seed(2)
    keys = torch.randn(2, 2, 40 * 16, 32)
    q = torch.randn(2, 4, 32)
    summ, sums = oracle.summaries_fp64(keys, 16, 37)
    sup = oracle.super_summaries(sums, 8, 16)
    assert sup.shape == (2, 2, 5, 32)
    # last superblock holds 37 - 32 = 5 pages; its mean is the mean of their tokens
    assert torch.allclose(sup[:, :, 4], keys[:, :, 32 * 16:37 * 16].double().mean(2).float(), atol=1e-6)
    sel = oracle.select_blocks_tree(q, sup, summ, superblock=8, top_super=2, top_blocks=3)
    chosen = oracle.select_blocks(q, sup, 2)
    scores = oracle.router_scores(q, summ)
    for b in range(2):
        allowed = [g for s in chosen[b].tolist() for g in range(s * 8, min(s * 8 + 8, 37))]
        best = sorted(allowed, key=lambda g: (-scores[b, g].item(), g))[:3]
        assert sel[b].tolist() == best


def test_refresh_gate_restatement(golden_dir):
    """Drift distance and learned refresh probability restated from the reference
    (evaluate_promotion_ttl.py:130, train_refresh_head.py:24-31)."""
    from oracle.refresh_gate import drift_distance, refresh_probability

    fx = _load(golden_dir, "refresh_gate.npz")
    head = (fx["w1"], fx["b1"], fx["w2"], fx["b2"])
    for case in range(fx["state"].shape[0]):
        s, c = torch.from_numpy(fx["state"][case]), torch.from_numpy(fx["cached"][case])
        assert torch.allclose(drift_distance(s, c), torch.from_numpy(fx["drift"][case]), atol=1e-6, rtol=0)
        assert torch.allclose(refresh_probability(s, c, *head), torch.from_numpy(fx["prob"][case]), atol=1e-6, rtol=0)


def test_gate_sim_policies():
    from oracle.refresh_gate import GateSim

    fresh = [torch.tensor([[i, i + 1]]) for i in range(10)]
    ttl = GateSim("ttl", ttl=4)
    used = [ttl.step(fresh[t], step=t) for t in range(10)]
    assert [r for _, r in used] == [t % 4 == 0 for t in range(10)]
    assert torch.equal(used[5][0], fresh[4])
    sig = GateSim("signature")
    sigs = [torch.tensor([[1, 2, 3]])] * 3 + [torch.tensor([[1, 2, 4]])] * 2
    assert [sig.step(fresh[t], signature=sigs[t])[1] for t in range(5)] == [True, False, False, True, False]
