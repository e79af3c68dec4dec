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


# ---------------------------------------------------------------- router pins at the benchmark shapes
def _router_inputs():
    import importlib
    import sys

    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parent / "golden"))
    return importlib.import_module("router_inputs")


def _check_inputs(fx, prefix, inputs):
    for key, val in _router_inputs().checksums(inputs).items():
        exp = float(fx[prefix + key])
        assert abs(val - exp) <= 1e-9 * max(1.0, abs(exp)), key


def test_router_cfg3_tree_pinned(golden_dir):
    """The canonical router (oracle.select_blocks_tree, the CUDA kernels' arithmetic) and
    the reference-order restatement give exactly the reference's own select_blocks,
    composed over superblocks then pages, at the 128k shape (511 pages, 32/8 heads,
    D128), with and without needle pages, for m = 2, 4, 8."""
    ri = _router_inputs()
    fx = _load(golden_dir, "router_cfg3.npz")
    c = ri.CFG3
    for tag in ("needles", "plain"):
        batch, needles = fx[f"{tag}_shape"].tolist()
        inp = ri.router_cfg3_inputs(int(fx[f"{tag}_seed"]), batch, needles)
        _check_inputs(fx, f"{tag}_", inp)
        for m in (2, 4, 8):
            ref = torch.from_numpy(fx[f"{tag}_m{m}_f32"])
            assert torch.equal(ref, torch.from_numpy(fx[f"{tag}_m{m}_f64"]))
            for scale in (1.0, c["head_dim"] ** -0.5):
                got = oracle.select_blocks_tree(inp["query"], inp["supers"], inp["summaries"],
                                                superblock=c["superblock"], top_super=c["top_super"], top_blocks=m,
                                                scale=scale)
                assert torch.equal(got, ref), (tag, m, scale)
            einsum = oracle.select_blocks_tree_einsum(inp["query"], inp["supers"], inp["summaries"],
                                                      superblock=c["superblock"], top_super=c["top_super"],
                                                      top_blocks=m)
            assert torch.equal(einsum, ref)


def test_router_cfg5_pinned(golden_dir):
    ri = _router_inputs()
    fx = _load(golden_dir, "router_cfg5.npz")
    inp = ri.router_cfg5_inputs(int(fx["seed"]), int(fx["batch"]))
    _check_inputs(fx, "", inp)
    ref = torch.from_numpy(fx["m8_f32"])
    assert torch.equal(ref, torch.from_numpy(fx["m8_f64"]))
    for scale in (1.0, ri.CFG5["head_dim"] ** -0.5):
        assert torch.equal(oracle.select_blocks(inp["query"], inp["summaries"], 8, scale=scale), ref)
    assert torch.equal(oracle.select_blocks_einsum(inp["query"], inp["summaries"], 8), ref)


def test_span_gather_pinned(golden_dir):
    """The span index map and attention restated in the oracle equal the reference's
    build_candidate_indices + candidate_attention (span width 3)."""
    ri = _router_inputs()
    fx = _load(golden_dir, "span_gather.npz")
    inp = ri.span_inputs(int(fx["seed"]))
    _check_inputs(fx, "", inp)
    c = ri.SPAN
    idx = oracle.span_candidate_indices(inp["centers"], c["context"], c["local_window"], c["span_width"])
    assert torch.equal(idx, torch.from_numpy(fx["indices"]))
    ref = torch.from_numpy(fx["out"]).double()
    out = oracle.span_candidate_attention(inp["query"], inp["keys"], inp["values"], idx)
    assert (out - ref).abs().max().item() <= 1e-5
    # the per-sequence token-list form (span_tokens) used by the GPU tests gives the same
    out2 = oracle.span_decode(inp["query"], inp["keys"], inp["values"], inp["centers"],
                              local_window=c["local_window"], span_width=c["span_width"])
    assert (out2 - ref).abs().max().item() <= 1e-5


def test_reference_decode_step_composition():
    """The reference arm's timed CPU step (reference-order router, make_candidates, fp32
    attention) on a reduced tree-routed shape agrees with the canonical oracle: the same
    pages, the fp64 gather decode within the fp32 tolerance."""
    gen = torch.Generator().manual_seed(5)
    b, hq, hkv, d, page, n_pages, win, sb = 2, 8, 2, 32, 16, 37, 16, 8
    ctx = n_pages * page + win
    keys = torch.randn(b, hkv, ctx, d, generator=gen)
    values = torch.randn(b, hkv, ctx, d, generator=gen)
    q = torch.randn(b, hq, d, generator=gen)
    summ, sums = oracle.summaries_fp64(keys, page, n_pages)
    sup = oracle.super_summaries(sums, sb, page)
    for m in (2, 4, 8):
        sel, out = oracle.reference_decode_step(q, keys, values, sup, summ, superblock=sb, top_super=2,
                                                top_blocks=m, local_window=win, block_size=page)
        assert torch.equal(sel, oracle.select_blocks_tree(q, sup, summ, superblock=sb, top_super=2, top_blocks=m))
        ref = oracle.gather_decode(q, keys, values, sel, local_window=win, block_size=page)
        assert out.dtype == torch.float32
        assert (out.double() - ref).abs().max().item() <= 1e-5
