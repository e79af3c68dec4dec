"""Seeded CPU inputs of the router and span fixtures.

Shared by make_golden.py (which runs the reference's functions on them) and the
tests (which regenerate them from the seed, check the stored checksums, and run the
oracle or the CUDA kernels on them).  torch.manual_seed + CPU draws only, so the
inputs are the same on every machine with the same torch build.

* router_cfg3_inputs -- the tree-routed 128k shape: 32 query heads / 8 kv heads,
  head_dim 128, bf16 query ~ N(0,1)*0.5, 511 routable pages of 256 tokens, fp64 page
  sums distributed as the sum of 256 keys ~ N(0,1)*0.5, optionally 8 needle pages per
  (row, kv head) whose keys are shifted by 2*0.5*q_hat (q_hat the normalised mean of
  that kv head's query heads); summaries = fp32(sum / 256), superblocks of 16 pages =
  fp32(sequential fp64 sum of page sums / (pages * 256)).
* router_cfg5_inputs -- the integrated decoder's router shape: 8 heads (MHA),
  head_dim 64, 129 routable pages of 128 tokens, single level.
* span_inputs -- contiguous K/V [B, H, L, D] fp32 and span centers for
  span_gather_decode_attention with span width 3 (the record width of the reference's
  build_candidate_indices).
"""

from __future__ import annotations

import torch

CFG3 = dict(q_heads=32, kv_heads=8, head_dim=128, page_size=256, n_pages=511, superblock=16, top_super=4)
CFG5 = dict(q_heads=8, kv_heads=8, head_dim=64, page_size=128, n_pages=129)
SPAN = dict(batch=2, heads=4, context=2048, head_dim=64, local_window=128, span_width=3, centers=16)


def _supers(sums64: torch.Tensor, superblock: int, page_size: int) -> torch.Tensor:
    b, h, g, d = sums64.shape
    n_super = -(-g // superblock)
    out = torch.empty(b, h, n_super, d, dtype=torch.float32)
    for s in range(n_super):
        g0, g1 = s * superblock, min((s + 1) * superblock, g)
        acc = torch.zeros(b, h, d, dtype=torch.float64)
        for gg in range(g0, g1):
            acc = acc + sums64[:, :, gg]
        out[:, :, s] = (acc / (float(g1 - g0) * float(page_size))).to(torch.float32)
    return out


def router_cfg3_inputs(seed: int, batch: int, needles: int) -> dict:
    c = CFG3
    torch.manual_seed(seed)
    hq, hkv, d, p, g = c["q_heads"], c["kv_heads"], c["head_dim"], c["page_size"], c["n_pages"]
    q = (torch.randn(batch, hq, d) * 0.5).to(torch.bfloat16)
    sums64 = torch.randn(batch, hkv, g, d, dtype=torch.float64) * (0.5 * p ** 0.5)
    if needles:
        qf = q.float().view(batch, hkv, hq // hkv, d).mean(2)
        q_hat = (qf / qf.norm(dim=-1, keepdim=True)).double()
        for b in range(batch):
            for h in range(hkv):
                pages = torch.randperm(g)[:needles]
                sums64[b, h, pages] += p * (2 * 0.5) * q_hat[b, h]
    summaries = (sums64 / p).to(torch.float32)
    supers = _supers(sums64, c["superblock"], p)
    return {"query": q, "summaries": summaries, "supers": supers}


def router_cfg5_inputs(seed: int, batch: int) -> dict:
    c = CFG5
    torch.manual_seed(seed)
    q = torch.randn(batch, c["q_heads"], c["head_dim"]).to(torch.bfloat16)
    summaries = (torch.randn(batch, c["kv_heads"], c["n_pages"], c["head_dim"], dtype=torch.float64)
                 / c["page_size"] ** 0.5).to(torch.float32)
    return {"query": q, "summaries": summaries}


def span_inputs(seed: int) -> dict:
    c = SPAN
    torch.manual_seed(seed)
    b, h, ctx, d = c["batch"], c["heads"], c["context"], c["head_dim"]
    query = torch.randn(b, h, d)
    keys = torch.randn(b, h, ctx, d)
    values = torch.randn_like(keys)
    hist = ctx - c["local_window"]
    centers = torch.randint(0, hist - c["span_width"] + 1, (b, c["centers"]))
    return {"query": query, "keys": keys, "values": values, "centers": centers}


def checksums(tensors: dict) -> dict:
    return {k + "_sum": float(v.double().sum().item()) for k, v in tensors.items()}
