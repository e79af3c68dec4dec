"""Page summaries and the page router (single level and superblock -> page tree).

Reference entry points:
* ``select_blocks(query, summaries, top_blocks)`` --
  experiments/triton_paged_gather_decode_benchmark.py:16-17 (also
  triton_promotion_cache_benchmark.py:16-17): einsum("bhd,bhgd->bhg").mean(1).topk(m).
* page summaries -- keys[:, :, :hist].view(B,H,hist/P,P,D).mean(3)
  (triton_paged_gather_decode_benchmark.py:61).
* ``paged_candidates`` -- triton_paged_decode_benchmark.py:16-36 (route, then
  assemble local window + selected pages into a contiguous buffer).

Scores are computed in fp32 (the precision of the reference's einsum) in one fixed
order and ties resolve to the lower page index, so the selection is deterministic
and reproducible bit-for-bit.
With grouped-query attention the q heads of one kv head score that kv head's
summary.  ``scale`` multiplies the mean score (1/sqrt(D) gives the
q.mean(K_page)/sqrt(D) form; the reference's select_blocks uses 1).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._util import as_int32, dtype_code, require_cuda, stream_ptr
from .paged_attention import contiguous_layout, pool_layout


def page_summaries(keys: torch.Tensor, *, block_size: int, n_pages: int | None = None,
                   local_window: int | None = None, page_table: torch.Tensor | None = None,
                   superblock: int | None = None):
    """Mean-key summaries of the routable pages, fp32 ``[B, Hkv, n_pages, D]``.

    ``keys`` is the reference's contiguous ``[B, H, L, D]`` (then n_pages defaults
    to (L - local_window) // block_size) or a page pool ``[num_pages, Hkv, P, D]``
    with ``page_table`` (then n_pages is required).  With ``superblock``, also
    returns superblock summaries ``[B, Hkv, ceil(n_pages/superblock), D]``."""
    require_cuda(keys, page_table)
    if page_table is None:
        b, h, length, d = keys.shape
        if n_pages is None:
            n_pages = (length - (local_window or 0)) // block_size
        if n_pages <= 0 or n_pages * block_size > length:
            raise ValueError("unsupported head dimension or page layout")
        layout = contiguous_layout(keys, keys, block_size)
    else:
        if n_pages is None:
            raise ValueError("n_pages is required with page_table")
        table = as_int32(page_table).contiguous()
        if keys.size(2) != block_size:
            raise ValueError("block_size must equal the pool's page size")
        if table.dim() != 2 or n_pages > table.size(1):
            raise ValueError("page_table must be [batch, pages] with at least n_pages columns")
        b, h, d = table.size(0), keys.size(1), keys.size(3)
        layout = pool_layout(keys, keys, table)
    if not keys.is_contiguous():
        raise ValueError("contiguous CUDA tensors are required")
    dev = keys.device
    summ = torch.empty(b, h, n_pages, d, dtype=torch.float32, device=dev)
    sup = sums = None
    if superblock:
        n_super = -(-n_pages // superblock)
        sup = torch.empty(b, h, n_super, d, dtype=torch.float32, device=dev)
        sums = torch.empty(b, h, n_pages, d, dtype=torch.float64, device=dev)
    rc = _lib.lib.spa_summaries_build(ctypes.byref(layout), b, h, d, dtype_code(keys), n_pages, summ.data_ptr(),
                                      superblock or 0, sup.data_ptr() if sup is not None else None,
                                      sums.data_ptr() if sums is not None else None, stream_ptr(dev))
    _lib.check(rc, "spa_summaries_build")
    return (summ, sup) if superblock else summ


def _router_args(query: torch.Tensor, summaries: torch.Tensor):
    require_cuda(query, summaries)
    if query.dim() != 3 or summaries.dim() != 4 or summaries.size(0) != query.size(0):
        raise ValueError("query must be [B, H, D] and summaries [B, Hkv, pages, D]")
    if summaries.size(3) != query.size(2) or query.size(1) % summaries.size(1):
        raise ValueError("query must be [B, H, D] and summaries [B, Hkv, pages, D]")
    q = query.contiguous()
    s = summaries.float().contiguous()
    return q, s


def select_blocks(query: torch.Tensor, summaries: torch.Tensor, top_blocks: int, *, scale: float = 1.0,
                  return_scores: bool = False, gate=None):
    """Top ``top_blocks`` pages per batch row, int64 ``[B, m]`` by descending score
    (ties to the lower page index).  With ``gate`` (a ``RefreshGate`` whose ``decide``
    ran for this step) a closed gate reuses the promoted pages without routing."""
    q, s = _router_args(query, summaries)
    b, hq, d = q.shape
    hkv, n_pages = s.size(1), s.size(2)
    if not 0 < top_blocks <= n_pages:
        raise ValueError("top_blocks must be in [1, pages]")
    out = torch.empty(b, top_blocks, dtype=torch.int64, device=q.device)
    if gate is not None:
        if return_scores:
            raise ValueError("return_scores is not available with a refresh gate")
        promoted = gate.promoted_for(b, top_blocks)
        rc = _lib.lib.spa_router_topm_gated(q.data_ptr(), dtype_code(q), b, hq, hkv, d, s.data_ptr(), n_pages,
                                            float(scale), top_blocks, out.data_ptr(), gate.flags.data_ptr(),
                                            promoted.data_ptr(), stream_ptr(q.device))
        _lib.check(rc, "spa_router_topm_gated")
        return out
    scores = torch.empty(b, n_pages, dtype=torch.float32, device=q.device) if return_scores else None
    rc = _lib.lib.spa_router_topm(q.data_ptr(), dtype_code(q), b, hq, hkv, d, s.data_ptr(), n_pages, float(scale),
                                  top_blocks, out.data_ptr(), scores.data_ptr() if scores is not None else None,
                                  stream_ptr(q.device))
    _lib.check(rc, "spa_router_topm")
    return (out, scores) if return_scores else out


def select_blocks_tree(query: torch.Tensor, super_summaries: torch.Tensor, summaries: torch.Tensor, *,
                       superblock: int, top_super: int, top_blocks: int, scale: float = 1.0,
                       gate=None) -> torch.Tensor:
    """Two-level router: top ``top_super`` superblocks, then the top ``top_blocks``
    pages inside them.  int64 ``[B, m]`` by descending page score.  ``gate`` as in
    ``select_blocks``."""
    q, s = _router_args(query, summaries)
    _, sup = _router_args(query, super_summaries)
    b, hq, d = q.shape
    hkv, n_pages, n_super = s.size(1), s.size(2), sup.size(2)
    if sup.size(1) != hkv or n_super != -(-n_pages // superblock):
        raise ValueError("super_summaries must be [B, Hkv, ceil(pages/superblock), D]")
    out = torch.empty(b, top_blocks, dtype=torch.int64, device=q.device)
    if gate is not None:
        promoted = gate.promoted_for(b, top_blocks)
        rc = _lib.lib.spa_router_tree_topm_gated(q.data_ptr(), dtype_code(q), b, hq, hkv, d, sup.data_ptr(), n_super,
                                                 s.data_ptr(), n_pages, superblock, top_super, float(scale),
                                                 top_blocks, out.data_ptr(), gate.flags.data_ptr(),
                                                 promoted.data_ptr(), stream_ptr(q.device))
        _lib.check(rc, "spa_router_tree_topm_gated")
        return out
    rc = _lib.lib.spa_router_tree_topm(q.data_ptr(), dtype_code(q), b, hq, hkv, d, sup.data_ptr(), n_super,
                                       s.data_ptr(), n_pages, superblock, top_super, float(scale), top_blocks,
                                       out.data_ptr(), stream_ptr(q.device))
    _lib.check(rc, "spa_router_tree_topm")
    return out


def periodic_router(query: torch.Tensor, keys: torch.Tensor, *, block_size: int, router_stride: int,
                    top_blocks: int) -> torch.Tensor:
    """Causal routing every ``router_stride`` tokens of a prefill; int64 [B, H, U, m]
    with -1 in unfilled slots (reference: triton_prefill_router_overhead.py:16-34).
    One batched kernel over all update positions replaces the per-update top-k loop."""
    require_cuda(query, keys)
    if query.dim() != 4 or keys.shape != query.shape:
        raise ValueError("query and keys must be [B, H, S, D]")
    b, h, s, d = query.shape
    if s % block_size or s % router_stride:
        raise ValueError("context must divide evenly into block-size and router-stride")
    summ = page_summaries(keys.contiguous(), block_size=block_size, n_pages=s // block_size)
    q = query.contiguous()
    out = torch.empty(b, h, s // router_stride, top_blocks, dtype=torch.int64, device=q.device)
    rc = _lib.lib.spa_periodic_router(q.data_ptr(), dtype_code(q), b, h, s, d, summ.data_ptr(), summ.size(2),
                                      block_size, router_stride, top_blocks, out.data_ptr(), stream_ptr(q.device))
    _lib.check(rc, "spa_periodic_router")
    return out
