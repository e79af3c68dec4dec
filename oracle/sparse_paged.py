"""CPU restatement of the reference's sparse paged-attention path (torch CPU, fp64).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function cites the
reference code it restates (paths inside divagr18/attention).

Router arithmetic follows one canonical order, identical to the CUDA kernels', so
scores -- and therefore selections, ties included -- are bit-identical:
  page sum    fp64, sequential over tokens      summary = fp32(sum / P)
  super sum   fp64, sequential over page sums   super   = fp32(sum / (n_pages_in_super * P))
  qg[kvh]     fp32, sequential over that kv head's q heads
  dot_kvh     fp32: lane l (of 32) accumulates d = l, l+32, ... (separate multiply,
              add), then an xor butterfly over lanes with offsets 16, 8, 4, 2, 1
  score       fp32, sequential over kv heads, then / Hq, then * fp32(scale)
Ranking: descending score, ties to the lower page index (a stable sort).  The
reference's torch.topk leaves tie order unspecified; on the seeded inputs the
two agree (tests/test_oracle_golden.py).
"""

from __future__ import annotations

import numpy as np
import torch

__all__ = [
    "summaries_fp64", "super_summaries", "router_scores", "topm", "select_blocks", "select_blocks_tree",
    "expand_kv", "reference_attention", "make_candidates", "candidate_tokens", "gather_decode",
    "dense_decode", "paged_to_contiguous", "local_reference", "local_reference_chunked", "promotion_update",
    "masked_dense_attention", "periodic_router", "span_tokens", "span_decode", "select_blocks_einsum",
    "select_blocks_tree_einsum", "span_candidate_indices", "span_candidate_attention", "reference_decode_step",
]


# ------------------------------------------------------------------ summaries
def summaries_fp64(keys: torch.Tensor, block_size: int, n_pages: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Page means of contiguous keys [B, H, L, D] for pages g < n_pages.

    Restates keys[:, :, :hist].view(B, H, hist/P, P, D).mean(3)
    (triton_paged_gather_decode_benchmark.py:61) in the canonical fp64 order.
    Returns (fp32 summaries [B, H, n_pages, D], fp64 page sums)."""
    b, h, _, d = keys.shape
    k = keys[:, :, : n_pages * block_size].to(torch.float64).reshape(b, h, n_pages, block_size, d)
    acc = torch.zeros(b, h, n_pages, d, dtype=torch.float64)
    for t in range(block_size):
        acc = acc + k[:, :, :, t]
    return (acc / float(block_size)).to(torch.float32), acc


def super_summaries(sums64: torch.Tensor, superblock: int, page_size: int) -> torch.Tensor:
    """Superblock means from fp64 page sums [B, H, G, D] (pages in order)."""
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


# ------------------------------------------------------------------ router
def router_scores(query: torch.Tensor, summaries: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """fp32 scores [B, G] = scale * mean_h q[b,h] . summary[b, h // group, g].

    Restates einsum("bhd,bhgd->bhg", q, summaries).mean(dim=1)
    (triton_paged_gather_decode_benchmark.py:17) with GQA grouping, in the
    canonical fp32 order documented at the top of this module."""
    f32 = torch.float32
    b, hq, d = query.shape
    hkv, g = summaries.size(1), summaries.size(2)
    group = hq // hkv
    qd = query.to(f32).reshape(b, hkv, group, d)
    qg = torch.zeros(b, hkv, d, dtype=f32)
    for j in range(group):
        qg = qg + qd[:, :, j]
    lanes = 32
    dpad = -(-d // lanes) * lanes
    qgp = torch.zeros(b, hkv, dpad, dtype=f32)
    qgp[..., :d] = qg
    sp = torch.zeros(b, hkv, g, dpad, dtype=f32)
    sp[..., :d] = summaries.to(f32)
    qgp = qgp.reshape(b, hkv, 1, dpad // lanes, lanes)
    sp = sp.reshape(b, hkv, g, dpad // lanes, lanes)
    part = torch.zeros(b, hkv, g, lanes, dtype=f32)
    for kk in range(dpad // lanes):
        part = part + qgp[:, :, :, kk] * sp[:, :, :, kk]
    idx = torch.arange(lanes)
    for off in (16, 8, 4, 2, 1):
        part = part + part[..., idx ^ off]
    dots = part[..., 0]  # [B, Hkv, G]
    total = torch.zeros(b, g, dtype=f32)
    for kvh in range(hkv):
        total = total + dots[:, kvh]
    return (total / torch.tensor(float(hq), dtype=f32)) * torch.tensor(scale, dtype=f32)


def topm(scores: torch.Tensor, m: int, index: torch.Tensor | None = None) -> torch.Tensor:
    """Top-m per row by descending score, ties to the lower index; int64 [B, m].

    ``index`` (same shape as scores) gives the page id of each column; rows are
    first ordered by page id so a stable descending sort breaks ties low."""
    if index is None:
        index = torch.arange(scores.size(1)).expand_as(scores)
    order = torch.argsort(index, dim=1, stable=True)
    s = torch.gather(scores, 1, order)
    ix = torch.gather(index, 1, order)
    pick = torch.sort(s, dim=1, descending=True, stable=True).indices[:, :m]
    return torch.gather(ix, 1, pick).to(torch.int64)


def select_blocks(query: torch.Tensor, summaries: torch.Tensor, top_blocks: int, scale: float = 1.0) -> torch.Tensor:
    """Restates select_blocks (triton_paged_gather_decode_benchmark.py:16-17)."""
    return topm(router_scores(query, summaries, scale), top_blocks)


def select_blocks_tree(query: torch.Tensor, supers: torch.Tensor, summaries: torch.Tensor, *, superblock: int,
                       top_super: int, top_blocks: int, scale: float = 1.0) -> torch.Tensor:
    """Two levels of select_blocks: top_super superblocks, then top_blocks pages
    among the pages of those superblocks (block -> finer-unit hierarchy of
    hierarchical_retrieval, benchmark_decode_attention.py:58-67, one level up)."""
    n_pages = summaries.size(2)
    chosen = topm(router_scores(query, supers, scale), top_super)
    page_scores = router_scores(query, summaries, scale)
    out = []
    for b in range(query.size(0)):
        ids = []
        for s in chosen[b].tolist():
            ids.extend(range(s * superblock, min((s + 1) * superblock, n_pages)))
        ids_t = torch.tensor(ids, dtype=torch.int64)
        out.append(topm(page_scores[b, ids_t][None], top_blocks, ids_t[None])[0])
    return torch.stack(out)


def select_blocks_einsum(query: torch.Tensor, summaries: torch.Tensor, top_blocks: int,
                         dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """The reference's own router expression in the reference's arithmetic order:
    einsum("bhd,bhgd->bhg").mean(dim=1).topk(m).indices
    (triton_paged_gather_decode_benchmark.py:16-17), evaluated in ``dtype``, with the
    kv-head summaries repeated over their query heads for GQA.  Unlike select_blocks
    above it does not follow the CUDA kernels' canonical order: it is the yardstick the
    canonical order is compared with (ties follow torch.topk)."""
    q = query.to(dtype)
    s = expand_kv(summaries.to(dtype), query.size(1))
    return torch.einsum("bhd,bhgd->bhg", q, s).mean(dim=1).topk(top_blocks, dim=-1).indices.contiguous()


def select_blocks_tree_einsum(query: torch.Tensor, supers: torch.Tensor, summaries: torch.Tensor, *, superblock: int,
                              top_super: int, top_blocks: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Two levels of select_blocks_einsum, the way hierarchical_retrieval composes its
    stages (benchmark_decode_attention.py:58-67): level 1 picks top_super superblocks
    from the superblock summaries; level 2 runs the same expression over the gathered
    summaries of those superblocks' pages (superblock order, pages ascending) and maps
    the winners back to page ids."""
    n_pages = summaries.size(2)
    chosen = select_blocks_einsum(query, supers, top_super, dtype)
    out = []
    for b in range(query.size(0)):
        ids = []
        for s in chosen[b].tolist():
            ids.extend(range(s * superblock, min((s + 1) * superblock, n_pages)))
        ids_t = torch.tensor(ids, dtype=torch.int64)
        pick = select_blocks_einsum(query[b : b + 1], summaries[b : b + 1, :, ids_t], top_blocks, dtype)[0]
        out.append(ids_t[pick])
    return torch.stack(out)


# ------------------------------------------------------------------ attention
def expand_kv(t: torch.Tensor, q_heads: int) -> torch.Tensor:
    """[B, Hkv, L, D] -> [B, Hq, L, D]: q head h reads kv head h // (Hq / Hkv)."""
    return t.repeat_interleave(q_heads // t.size(1), dim=1)


def reference_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                        dtype: torch.dtype = torch.float64) -> torch.Tensor:
    """softmax(q . K^T * D^-1/2) V in ``dtype`` (fp64 unless asked; triton_paged_attention.py:227-231),
    GQA-expanded."""
    q = query.to(dtype)
    k = expand_kv(keys.to(dtype), q.size(1))
    v = expand_kv(values.to(dtype), q.size(1))
    scores = torch.einsum("bhd,bhld->bhl", q, k) * q.size(-1) ** -0.5
    return torch.einsum("bhl,bhld->bhd", scores.softmax(dim=-1), v)


def make_candidates(keys: torch.Tensor, values: torch.Tensor, selected: torch.Tensor, local_window: int,
                    block_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Local window followed by the selected pages, contiguous [B, H, W + m*P, D].

    Restates make_candidates (triton_paged_gather_decode_benchmark.py:20-28)."""
    b, h, length, d = keys.shape
    hist = length - local_window
    n_pages = hist // block_size
    pk = keys[:, :, : n_pages * block_size].reshape(b, h, n_pages, block_size, d).permute(0, 2, 1, 3, 4)
    pv = values[:, :, : n_pages * block_size].reshape(b, h, n_pages, block_size, d).permute(0, 2, 1, 3, 4)
    bi = torch.arange(b).unsqueeze(1)
    sk = pk[bi, selected].permute(0, 2, 1, 3, 4).flatten(2, 3)
    sv = pv[bi, selected].permute(0, 2, 1, 3, 4).flatten(2, 3)
    return torch.cat((keys[:, :, hist:], sk), dim=2), torch.cat((values[:, :, hist:], sv), dim=2)


def reference_decode_step(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, supers: torch.Tensor,
                          summaries: torch.Tensor, *, superblock: int, top_super: int, top_blocks: int,
                          local_window: int, block_size: int,
                          dtype: torch.dtype = torch.float32) -> tuple[torch.Tensor, torch.Tensor]:
    """One tree-routed sparse decode step the way the reference's PyTorch path computes
    it, in ``dtype`` on contiguous K/V [B, Hkv, L, D]: the router expression of
    select_blocks at two levels (select_blocks_tree_einsum), candidate assembly
    (make_candidates, triton_paged_gather_decode_benchmark.py:20-28) and softmax attention
    (reference_attention, triton_paged_attention.py:227-231; the timed unit of
    triton_paged_gather_decode_benchmark.py:71).  Returns (selected [B, m], out [B, Hq, D]).
    This is the reference arm's timed CPU path."""
    sel = select_blocks_tree_einsum(query, supers, summaries, superblock=superblock, top_super=top_super,
                                    top_blocks=top_blocks, dtype=dtype)
    ck, cv = make_candidates(keys, values, sel, local_window, block_size)
    return sel, reference_attention(query, ck, cv, dtype=dtype)


def candidate_tokens(ctx: int, local_window: int, selected_row: list[int], block_size: int) -> list[int]:
    """Token ids attended by the gather kernel for one sequence: the last
    local_window tokens, then each selected page (negative ids skipped); candidate
    order of triton_paged_attention.py:111-122."""
    toks = list(range(max(0, ctx - local_window), ctx))
    for p in selected_row:
        if p < 0:
            continue
        toks.extend(t for t in range(p * block_size, (p + 1) * block_size) if t < ctx)
    return toks


def span_tokens(ctx: int, local_window: int, starts_row: list[int], span_width: int) -> list[int]:
    """Token ids attended by the span kernel for one sequence: the last local_window
    tokens, then span_width tokens from each start (candidate c >= W reads
    centers[(c-W)//span] + (c-W)%span, triton_paged_attention.py:187-193); negative
    starts skipped, tokens at or past the context dropped."""
    toks = list(range(max(0, ctx - local_window), ctx))
    for c in starts_row:
        if c < 0:
            continue
        toks.extend(t for t in range(c, c + span_width) if t < ctx)
    return toks


def span_decode(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, starts: torch.Tensor, *,
                local_window: int, span_width: int, context_lens: list[int] | None = None) -> torch.Tensor:
    """Attention over span_tokens per sequence; keys/values contiguous [B, Hkv, L, D]."""
    out = []
    for i in range(query.size(0)):
        ctx = context_lens[i] if context_lens is not None else keys.size(2)
        toks = torch.tensor(span_tokens(ctx, local_window, starts[i].tolist(), span_width), dtype=torch.int64)
        out.append(reference_attention(query[i : i + 1], keys[i : i + 1, :, toks], values[i : i + 1, :, toks]))
    return torch.cat(out)


def span_candidate_indices(centers: torch.Tensor, context: int, local_window: int, span_width: int) -> torch.Tensor:
    """Token indices [B, W + k*span]: the last local_window tokens, then span_width
    tokens from each center, clamped to the last historical token.  Restates
    build_candidate_indices (benchmark_decode_attention.py:86-90), whose record width
    is fixed at 3, for any span width; the span kernel's index map
    (triton_paged_attention.py:187-193) is the same for centers <= hist - span_width."""
    hist = context - local_window
    promoted = (centers.to(torch.int64).unsqueeze(-1) + torch.arange(span_width)).clamp_max(hist - 1).flatten(1)
    local = torch.arange(hist, context).expand(centers.size(0), -1)
    return torch.cat((local, promoted), dim=1)


def span_candidate_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                             indices: torch.Tensor) -> torch.Tensor:
    """exact_attention over the gathered candidate tokens, fp64 (candidate_attention and
    exact_attention, benchmark_decode_attention.py:39-49), GQA-expanded."""
    idx = indices.to(torch.int64)[:, None, :, None].expand(-1, keys.size(1), -1, keys.size(-1))
    return reference_attention(query, keys.gather(2, idx), values.gather(2, idx))


def gather_decode(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, selected: torch.Tensor, *,
                  local_window: int, block_size: int, context_lens: list[int] | None = None) -> torch.Tensor:
    """Attention over candidate_tokens per sequence; keys/values contiguous [B, Hkv, L, D]."""
    b = query.size(0)
    out = []
    for i in range(b):
        ctx = context_lens[i] if context_lens is not None else keys.size(2)
        toks = torch.tensor(candidate_tokens(ctx, local_window, selected[i].tolist(), block_size), dtype=torch.int64)
        out.append(reference_attention(query[i : i + 1], keys[i : i + 1, :, toks], values[i : i + 1, :, toks]))
    return torch.cat(out)


def dense_decode(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, context_lens: list[int],
                 local_window: int = 0) -> torch.Tensor:
    """Attention of q over tokens [lo, ctx) of each sequence (lo = ctx - W when W > 0)."""
    out = []
    for i in range(query.size(0)):
        ctx = context_lens[i]
        lo = max(0, ctx - local_window) if local_window > 0 else 0
        out.append(reference_attention(query[i : i + 1], keys[i : i + 1, :, lo:ctx], values[i : i + 1, :, lo:ctx]))
    return torch.cat(out)


def masked_dense_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                           allowed: torch.Tensor) -> torch.Tensor:
    """Dense attention over all L tokens with a [B, L] token mask (fp64); the
    masked-attention form of CausalAttention (train_tiny_transformer.py:145-172)."""
    q = query.to(torch.float64)
    k = expand_kv(keys.to(torch.float64), q.size(1))
    v = expand_kv(values.to(torch.float64), q.size(1))
    scores = torch.einsum("bhd,bhld->bhl", q, k) * q.size(-1) ** -0.5
    scores = scores.masked_fill(~allowed[:, None, :], float("-inf"))
    return torch.einsum("bhl,bhld->bhd", scores.softmax(dim=-1), v)


def paged_to_contiguous(pool: torch.Tensor, page_table: torch.Tensor, length: int) -> torch.Tensor:
    """Pool [N, Hkv, P, D] + table [B, pages] -> contiguous [B, Hkv, length, D]."""
    n, hkv, p, d = pool.shape
    b = page_table.size(0)
    n_pages = -(-length // p)
    tab = page_table[:, :n_pages].to(torch.int64)
    g = pool[tab.reshape(-1)].reshape(b, n_pages, hkv, p, d).permute(0, 2, 1, 3, 4).reshape(b, hkv, n_pages * p, d)
    return g[:, :, :length]


# ------------------------------------------------------------------ prefill
def local_reference(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, window: int) -> torch.Tensor:
    """Dense masked causal-window attention, fp64 (triton_local_prefill.py:84-89)."""
    q, k, v = (t.to(torch.float64) for t in (query, keys, values))
    s = q.size(2)
    pos = torch.arange(s)
    allowed = (pos[:, None] >= pos[None, :]) & (pos[:, None] - pos[None, :] < window)
    scores = torch.einsum("bhid,bhjd->bhij", q, k) * q.size(-1) ** -0.5
    return torch.einsum("bhij,bhjd->bhid", scores.masked_fill(~allowed, float("-inf")).softmax(dim=-1), v)


def local_reference_chunked(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, window: int, *,
                            chunk: int = 256, k_halo: torch.Tensor | None = None,
                            v_halo: torch.Tensor | None = None, dtype=torch.float64) -> torch.Tensor:
    """local_reference per query chunk with its window-1 key halo (no S x S matrix).

    With k_halo/v_halo [B, H, halo, D], query i sees keys of [halo ; keys] at
    positions i+halo-window+1 .. i+halo."""
    halo = 0 if k_halo is None else k_halo.size(2)
    kk = keys if k_halo is None else torch.cat((k_halo, keys), dim=2)
    vv = values if v_halo is None else torch.cat((v_halo, values), dim=2)
    q, k, v = (t.to(dtype) for t in (query, kk, vv))
    s = query.size(2)
    out = torch.empty(query.shape, dtype=dtype)
    scale = query.size(-1) ** -0.5
    for i0 in range(0, s, chunk):
        i1 = min(s, i0 + chunk)
        c0 = max(0, i0 + halo - window + 1)
        c1 = i1 + halo
        qc = q[:, :, i0:i1]
        sc = torch.einsum("bhid,bhjd->bhij", qc, k[:, :, c0:c1]) * scale
        qi = torch.arange(i0, i1)[:, None] + halo
        kj = torch.arange(c0, c1)[None, :]
        allowed = (kj <= qi) & (qi - kj < window)
        out[:, :, i0:i1] = torch.einsum("bhij,bhjd->bhid", sc.masked_fill(~allowed, float("-inf")).softmax(-1),
                                        v[:, :, c0:c1])
    return out


# ------------------------------------------------------------------ promotion table
def promotion_update(pages: np.ndarray, last_hit: np.ndarray, selected: np.ndarray, step: int, ttl: int) -> None:
    """In-place update of int32 tables [rows, slots] with selections [rows, m].

    Policy (fixed TTL as in evaluate_promotion_ttl.py:134-135, applied per page):
    hits refresh last_hit; entries idle >= ttl steps are freed; each new page
    takes the lowest free slot, else evicts the smallest (last_hit, page id)."""
    rows, slots = pages.shape
    for r in range(rows):
        pg, lh = pages[r], last_hit[r]
        sel = [int(x) for x in selected[r]]
        for pid in sel:
            if pid < 0:
                continue
            lh[pg == pid] = step
        for i in range(slots):
            if pg[i] >= 0 and step - lh[i] >= ttl:
                pg[i] = -1
        for pid in sel:
            if pid < 0 or pid > 0x7FFFFFFF or (pg == pid).any():
                continue
            free = np.nonzero(pg < 0)[0]
            if free.size:
                slot = int(free[0])
            else:
                slot = min(range(slots), key=lambda i: (int(lh[i]), int(pg[i])))
            pg[slot] = pid
            lh[slot] = step


# ------------------------------------------------------------------ periodic prefill router
def periodic_router(query: torch.Tensor, keys: torch.Tensor, *, block_size: int, router_stride: int,
                    top_blocks: int) -> torch.Tensor:
    """Causal routing every router_stride tokens; unfilled slots are -1.

    Restates periodic_router (triton_prefill_router_overhead.py:16-34) with the
    canonical fp64 scores and lower-index ties."""
    b, h, ctx, d = query.shape
    n_blocks = ctx // block_size
    summ, _ = summaries_fp64(keys, block_size, n_blocks)
    upd = list(range(router_stride - 1, ctx, router_stride))
    out = torch.full((b, h, len(upd), top_blocks), -1, dtype=torch.int64)
    for u, pos in enumerate(upd):
        avail = sum(1 for g in range(n_blocks) if g * block_size + block_size - 1 <= pos)
        cnt = min(top_blocks, avail)
        if not cnt:
            continue
        for hh in range(h):
            sc = router_scores(query[:, hh : hh + 1, pos], summ[:, hh : hh + 1, :avail])
            out[:, hh, u, :cnt] = topm(sc, cnt)
    return out

