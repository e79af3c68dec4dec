"""Generates tests/golden/*.npz by running the reference's own PyTorch functions.

Run where the reference checkout is importable (it is not needed anywhere else):

    python tests/golden/make_golden.py /path/to/divagr18-attention

Every fixture stores the seed and shapes that regenerate its inputs with
torch.manual_seed + torch.randn on CPU (the reference's own draw order), input
checksums to prove the regeneration, and the reference's outputs:

* cfg1_sparse_decode  -- batch 1, 8 heads, head_dim 64, fp32, 4096 tokens in 32
  pages of 128, seed 0, draws K, V, q; select_blocks top-4 over the 31 historical
  pages, make_candidates + reference_attention over 640 tokens, and the dense
  masked attention over the same token set.
* gather_small        -- seed 7 (reference main() order q, K, V): select_blocks,
  make_candidates + reference_attention, paged_candidates equality.
* dense_small         -- seed 7: reference_attention over the whole buffer.
* prefill_small       -- seed 7: local_reference (masked causal window).
* periodic_router     -- seed 7: periodic_router indices with -1 padding.
* refresh_gate        -- seed 7: the reference's RefreshHead (train_refresh_head.py) on
  three (state, cached state) sets of growing drift, its sigmoid probabilities, and the
  drift distance 1 - cosine_similarity of evaluate_promotion_ttl.py:130.
* router_cfg3         -- the tree-routed 128k router shape (router_inputs.py): the
  reference's select_blocks run twice, the way hierarchical_retrieval composes its
  stages (benchmark_decode_attention.py:58-67): top-4 superblocks from the superblock
  summaries, then top-m (m = 2, 4, 8) among those superblocks' page summaries.  With
  needles (batch 4, seed 11) and without (batch 16, seed 12), each in fp32 and fp64.
* router_cfg5         -- the integrated decoder's router shape (8 heads, head_dim 64,
  129 pages): select_blocks top-8, batch 32, seed 13, fp32 and fp64.
* span_gather         -- seed 14: build_candidate_indices (benchmark_decode_attention.py:86-90,
  span width 3) + candidate_attention, the reference's PyTorch form of the
  span_gather_decode_attention index map (triton_paged_attention.py:187-193).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "experiments"))
    import triton_local_prefill as tlp  # noqa: E402
    import triton_paged_attention as tpa  # noqa: E402
    import triton_paged_decode_benchmark as tpd  # noqa: E402
    import triton_paged_gather_decode_benchmark as tpg  # noqa: E402
    import triton_prefill_router_overhead as tpr  # noqa: E402

    # ---- configuration 1
    torch.manual_seed(0)
    b, h, length, d, page, win, m = 1, 8, 4096, 64, 128, 128, 4
    keys = torch.randn(b, h, length, d)
    values = torch.randn(b, h, length, d)
    query = torch.randn(b, h, d)
    hist = length - win
    summaries = keys[:, :, :hist].view(b, h, hist // page, page, d).mean(3).contiguous()
    sel = tpg.select_blocks(query, summaries, m)
    ck, cv = tpg.make_candidates(keys, values, sel, win, page)
    out = tpa.reference_attention(query, ck, cv)
    allowed = torch.zeros(b, length, dtype=torch.bool)
    allowed[:, hist:] = True
    for bb in range(b):
        for p in sel[bb].tolist():
            allowed[bb, p * page:(p + 1) * page] = True
    scores = torch.einsum("bhd,bhld->bhl", query, keys) / d ** 0.5
    dense_masked = torch.einsum("bhl,bhld->bhd", scores.masked_fill(~allowed[:, None], float("-inf")).softmax(-1),
                                values)
    np.savez(HERE / "cfg1_sparse_decode.npz", seed=0, shape=np.array([b, h, length, d, page, win, m]),
             k_sum=keys.double().sum().item(), v_sum=values.double().sum().item(), q_sum=query.double().sum().item(),
             selected=sel.numpy(), out=out.numpy(), dense_masked=dense_masked.numpy(),
             summaries=summaries.numpy())

    # ---- gather (reference main() draw order: q, K, V)
    torch.manual_seed(7)
    b, h, length, d, page, win, m = 2, 4, 2048, 32, 256, 256, 3
    query = torch.randn(b, h, d)
    keys = torch.randn(b, h, length, d)
    values = torch.randn_like(keys)
    hist = length - win
    summaries = keys[:, :, :hist].view(b, h, hist // page, page, d).mean(3).contiguous()
    sel = tpg.select_blocks(query, summaries, m)
    ck, cv = tpg.make_candidates(keys, values, sel, win, page)
    out = tpa.reference_attention(query, ck, cv)
    pk, pv = tpd.paged_candidates(query, keys, values, summaries, local_window=win, block_size=page, top_blocks=m)
    assert torch.equal(pk, ck) and torch.equal(pv, cv)
    np.savez(HERE / "gather_small.npz", seed=7, shape=np.array([b, h, length, d, page, win, m]),
             k_sum=keys.double().sum().item(), v_sum=values.double().sum().item(), q_sum=query.double().sum().item(),
             selected=sel.numpy(), out=out.numpy())

    # ---- dense candidate buffer
    torch.manual_seed(7)
    b, h, length, d = 2, 4, 1280, 16
    query = torch.randn(b, h, d)
    keys = torch.randn(b, h, length, d)
    values = torch.randn_like(keys)
    out = tpa.reference_attention(query, keys, values)
    np.savez(HERE / "dense_small.npz", seed=7, shape=np.array([b, h, length, d]),
             k_sum=keys.double().sum().item(), v_sum=values.double().sum().item(), q_sum=query.double().sum().item(),
             out=out.numpy())

    # ---- prefill
    torch.manual_seed(7)
    b, h, s, d, w = 1, 2, 300, 16, 64
    query = torch.randn(b, h, s, d)
    keys = torch.randn_like(query)
    values = torch.randn_like(query)
    out = tlp.local_reference(query, keys, values, w)
    np.savez(HERE / "prefill_small.npz", seed=7, shape=np.array([b, h, s, d, w]),
             k_sum=keys.double().sum().item(), v_sum=values.double().sum().item(), q_sum=query.double().sum().item(),
             out=out.numpy())

    # ---- periodic causal router
    torch.manual_seed(7)
    b, h, ctx, d, page, stride, m = 1, 2, 1024, 16, 128, 128, 3
    query = torch.randn(b, h, ctx, d)
    keys = torch.randn_like(query)
    sel = tpr.periodic_router(query, keys, block_size=page, router_stride=stride, top_blocks=m)
    np.savez(HERE / "periodic_router.npz", seed=7, shape=np.array([b, h, ctx, d, page, stride, m]),
             k_sum=keys.double().sum().item(), q_sum=query.double().sum().item(), selected=sel.numpy())

    # ---- promotion refresh gates
    import train_refresh_head as trh  # noqa: E402

    torch.manual_seed(7)
    b, w = 8, 64
    head = trh.RefreshHead(w)
    states, cached, probs, drifts = [], [], [], []
    with torch.no_grad():
        for noise in (0.05, 0.3, 1.5):
            x = torch.randn(b, w)
            y = x + noise * torch.randn(b, w)
            states.append(x)
            cached.append(y)
            probs.append(torch.sigmoid(head(x, y)))
            drifts.append(1.0 - torch.nn.functional.cosine_similarity(x, y, dim=-1))
    np.savez(HERE / "refresh_gate.npz", seed=7, shape=np.array([b, w]),
             w1=head.network[0].weight.detach().numpy(), b1=head.network[0].bias.detach().numpy(),
             w2=head.network[2].weight.detach().numpy(), b2=head.network[2].bias.detach().numpy(),
             state=torch.stack(states).numpy(), cached=torch.stack(cached).numpy(),
             prob=torch.stack(probs).numpy(), drift=torch.stack(drifts).numpy())
    # ---- router at the tree-routed 128k shape and the decoder shape
    import benchmark_decode_attention as bda  # noqa: E402

    sys.path.insert(0, str(HERE))
    import router_inputs as ri  # noqa: E402

    def ref_tree(inp, top_super, m, dt):
        q, sup, summ = inp["query"], inp["supers"], inp["summaries"]
        grp = q.size(1) // sup.size(1)
        chosen = tpg.select_blocks(q.to(dt), sup.to(dt).repeat_interleave(grp, 1), top_super)
        sb, n_pages, rows = ri.CFG3["superblock"], summ.size(2), []
        for bb in range(q.size(0)):
            ids = []
            for sblk in chosen[bb].tolist():
                ids.extend(range(sblk * sb, min((sblk + 1) * sb, n_pages)))
            ids = torch.tensor(ids)
            pick = tpg.select_blocks(q[bb : bb + 1].to(dt), summ[bb : bb + 1, :, ids].to(dt).repeat_interleave(grp, 1),
                                     m)[0]
            rows.append(ids[pick])
        return chosen, torch.stack(rows)

    fx = {}
    for tag, seed, batch, needles in (("needles", 11, 4, 8), ("plain", 12, 16, 0)):
        inp = ri.router_cfg3_inputs(seed, batch, needles)
        fx[f"{tag}_seed"] = seed
        fx[f"{tag}_shape"] = np.array([batch, needles])
        for key, val in ri.checksums(inp).items():
            fx[f"{tag}_{key}"] = val
        for m in (2, 4, 8):
            for dt, name in ((torch.float32, "f32"), (torch.float64, "f64")):
                chosen, sel = ref_tree(inp, ri.CFG3["top_super"], m, dt)
                fx[f"{tag}_m{m}_{name}"] = sel.numpy()
                fx[f"{tag}_super_{name}"] = chosen.numpy()
    np.savez(HERE / "router_cfg3.npz", **fx)

    inp = ri.router_cfg5_inputs(13, 32)
    grp = inp["query"].size(1) // inp["summaries"].size(1)
    fx = {"seed": 13, "batch": 32, **ri.checksums(inp)}
    for dt, name in ((torch.float32, "f32"), (torch.float64, "f64")):
        fx[f"m8_{name}"] = tpg.select_blocks(inp["query"].to(dt),
                                             inp["summaries"].to(dt).repeat_interleave(grp, 1), 8).numpy()
    np.savez(HERE / "router_cfg5.npz", **fx)

    # ---- span gather: the reference's PyTorch candidate path with span width 3
    inp = ri.span_inputs(14)
    c = ri.SPAN
    cfg = bda.Config(context=c["context"], local_window=c["local_window"], block_size=64, top_blocks=1,
                     top_tokens=c["centers"], batch_size=c["batch"], heads=c["heads"], head_dim=c["head_dim"],
                     iterations=1, warmup=0, seed=14, device="cpu")
    idx = bda.build_candidate_indices(inp["centers"], cfg, torch.device("cpu"))
    out = bda.candidate_attention(inp["query"], inp["keys"], inp["values"], idx)
    np.savez(HERE / "span_gather.npz", seed=14, indices=idx.numpy(), out=out.numpy(), **ri.checksums(inp))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of a divagr18/attention checkout>")
    main(sys.argv[1])
