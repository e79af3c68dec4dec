"""Paged decode attention: drop-in for the reference's fused decode entry points.

``paged_decode_attention``, ``paged_gather_decode_attention`` and
``span_gather_decode_attention`` keep the call signatures, argument meaning and
ValueError messages of experiments/triton_paged_attention.py:56-81, :139-168 and
:210-224.  Keyword-only
extensions (defaults reproduce the reference):

* ``page_table`` / ``context_lens``: K/V given as a shared page pool
  ``[num_pages, Hkv, P, D]`` addressed through ``page_table[B, pages]`` (int32)
  instead of a contiguous ``[B, H, L, D]`` buffer;
* grouped-query attention when ``keys.size(1)`` divides ``query.size(1)``;
* head_dim up to 256, dtypes float32 / float16 / bfloat16.

Both run the split-K sm_100a kernel of libspa_b200.so on the caller's stream.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._util import (as_int32, as_int64, const_i32, dtype_code, require_contiguous, require_cuda, stream_ptr,
                    workspace)


def contiguous_layout(keys: torch.Tensor, values: torch.Tensor, page_size: int) -> _lib.KvLayout:
    """Layout of the reference's contiguous K/V ``[B, H, L, D]`` with pages of ``page_size``
    consecutive tokens (no page table: page g of a sequence is tokens [g*P, (g+1)*P))."""
    b, h, length, d = keys.shape
    return _lib.KvLayout(keys.data_ptr(), values.data_ptr(), b * h * length, h * length, page_size, length, None,
                         0, page_size)


def pool_layout(k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: torch.Tensor) -> _lib.KvLayout:
    """Layout of a shared page pool ``[num_pages, Hkv, P, D]`` with ``page_table[B, max_pages]``."""
    n, hkv, p, d = k_pool.shape
    return _lib.KvLayout(k_pool.data_ptr(), v_pool.data_ptr(), n * hkv * p, 0, hkv * p, p, page_table.data_ptr(),
                         page_table.size(1), p)


def _check_heads(query: torch.Tensor, kv_heads: int) -> None:
    if kv_heads <= 0 or query.size(1) % kv_heads:
        raise ValueError("incompatible Q/K/V shapes")


def _decode(query, kv_layout, kv_heads, context_lens, local_window, selected, top_m, max_candidates,
            keepalive) -> torch.Tensor:
    batch, q_heads, head_dim = query.shape
    out = torch.empty_like(query)
    dev = query.device
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_candidates)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    # the dense form is spa_paged_decode; the selected-pages form its named gather entry point
    fn, name = ((_lib.lib.spa_paged_decode, "spa_paged_decode") if selected is None
                else (_lib.lib.spa_paged_gather_decode, "spa_paged_gather_decode"))
    rc = fn(query.data_ptr(), dtype_code(query), batch, q_heads, kv_heads, head_dim, ctypes.byref(kv_layout),
            context_lens.data_ptr(), local_window, selected.data_ptr() if selected is not None else None, top_m,
            max_candidates, head_dim ** -0.5, out.data_ptr(), ws.data_ptr() if ws is not None else None, ws_bytes,
            stream_ptr(dev))
    _lib.check(rc, name)
    del keepalive
    return out


def paged_decode_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, *,
                           page_table: torch.Tensor | None = None, context_lens: torch.Tensor | None = None,
                           local_window: int = 0) -> torch.Tensor:
    """Fused attention for q=[B,H,D] over K/V=[B,H,L,D] (reference: triton_paged_attention.py:56).

    With ``page_table``, K/V are a page pool ``[num_pages, Hkv, P, D]`` and the
    candidates of sequence b are its first ``context_lens[b]`` tokens (the last
    ``local_window`` of them when local_window > 0)."""
    if not (query.is_cuda and keys.is_cuda and values.is_cuda):
        raise ValueError("CUDA tensors are required")
    if not (query.is_contiguous() and keys.is_contiguous() and values.is_contiguous()):
        raise ValueError("contiguous candidate pages are required")
    if query.dim() != 3 or keys.dim() != 4 or values.shape != keys.shape or keys.dtype != query.dtype:
        raise ValueError("incompatible Q/K/V shapes")
    batch, heads, head_dim = query.shape
    if keys.size(3) != head_dim:
        raise ValueError("incompatible Q/K/V shapes")
    _check_heads(query, keys.size(1))
    if head_dim > 256:
        raise ValueError("head_dim <= 256 is supported")
    if local_window < 0:
        raise ValueError("local_window must be >= 0")
    if page_table is None:
        if keys.size(0) != batch:
            raise ValueError("incompatible Q/K/V shapes")
        length = keys.size(2)
        layout = contiguous_layout(keys, values, length)
        lens = const_i32(query.device, batch, length)
        max_cand = length if local_window <= 0 else min(length, local_window)
        return _decode(query, layout, keys.size(1), lens, local_window, None, 0, max_cand, None)
    if context_lens is None:
        raise ValueError("context_lens is required with page_table")
    require_cuda(page_table, context_lens)
    table = as_int32(page_table).contiguous()
    lens = as_int32(context_lens).contiguous()
    if table.dim() != 2 or table.size(0) != batch or lens.shape != (batch,):
        raise ValueError("page_table must be [batch, pages] and context_lens [batch]")
    layout = pool_layout(keys, values, table)
    max_cand = table.size(1) * keys.size(2)
    if local_window > 0:
        max_cand = min(max_cand, local_window)
    return _decode(query, layout, keys.size(1), lens, local_window, None, 0, max_cand, (table, lens))


def paged_gather_decode_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                                  selected_blocks: torch.Tensor, *, local_window: int, block_size: int,
                                  page_table: torch.Tensor | None = None,
                                  context_lens: torch.Tensor | None = None) -> torch.Tensor:
    """Fused page gather + attention (reference: triton_paged_attention.py:139).

    Candidates of sequence b: its last ``local_window`` tokens, then the pages
    ``selected_blocks[b, :]`` of ``block_size`` tokens, under one softmax.  A
    negative page id marks an empty slot and contributes nothing."""
    batch, heads, head_dim = query.shape
    if selected_blocks.dim() != 2 or selected_blocks.shape[0] != batch or not selected_blocks.is_contiguous():
        raise ValueError("selected_blocks must be contiguous [batch, top_blocks]")
    if not (query.is_contiguous() and keys.is_contiguous() and values.is_contiguous()):
        raise ValueError("contiguous CUDA tensors are required")
    if not (query.is_cuda and keys.is_cuda and values.is_cuda and selected_blocks.is_cuda):
        raise ValueError("contiguous CUDA tensors are required")
    if keys.dim() != 4 or values.shape != keys.shape or keys.size(3) != head_dim or keys.dtype != query.dtype:
        raise ValueError("incompatible Q/K/V shapes")
    _check_heads(query, keys.size(1))
    if local_window < 0 or block_size <= 0:
        raise ValueError("unsupported head dimension or page layout")
    sel = as_int64(selected_blocks).contiguous()
    top_m = sel.size(1)
    if top_m == 0:
        raise ValueError("selected_blocks must be contiguous [batch, top_blocks]")
    max_cand = local_window + top_m * block_size
    if page_table is None:
        if keys.size(0) != batch:
            raise ValueError("incompatible Q/K/V shapes")
        length = keys.size(2)
        if head_dim > 256 or (length - local_window) % block_size or local_window > length:
            raise ValueError("unsupported head dimension or page layout")
        layout = contiguous_layout(keys, values, block_size)
        lens = const_i32(query.device, batch, length)
        return _decode(query, layout, keys.size(1), lens, local_window, sel, top_m, max_cand, (sel,))
    if context_lens is None:
        raise ValueError("context_lens is required with page_table")
    if keys.size(2) != block_size or head_dim > 256:
        raise ValueError("unsupported head dimension or page layout")
    table = as_int32(page_table).contiguous()
    lens = as_int32(context_lens).contiguous()
    if table.dim() != 2 or table.size(0) != batch or lens.shape != (batch,):
        raise ValueError("page_table must be [batch, pages] and context_lens [batch]")
    layout = pool_layout(keys, values, table)
    return _decode(query, layout, keys.size(1), lens, local_window, sel, top_m, max_cand, (sel, table, lens))


def span_gather_decode_attention(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, centers: torch.Tensor,
                                 *, local_window: int, span_width: int, page_table: torch.Tensor | None = None,
                                 context_lens: torch.Tensor | None = None) -> torch.Tensor:
    """Local window plus short spans (reference: triton_paged_attention.py:210).

    Candidates of sequence b: its last ``local_window`` tokens, then for every
    ``centers[b, j]`` the ``span_width`` tokens starting there, under one softmax.
    Negative centers are empty slots; span tokens at or past the context are dropped."""
    batch, heads, head_dim = query.shape
    if not (query.is_contiguous() and keys.is_contiguous() and values.is_contiguous() and centers.is_contiguous()):
        raise ValueError("contiguous CUDA tensors are required")
    if not (query.is_cuda and keys.is_cuda and values.is_cuda and centers.is_cuda):
        raise ValueError("contiguous CUDA tensors are required")
    if centers.dim() != 2 or centers.shape[0] != batch or head_dim > 256:
        raise ValueError("invalid centers or head dimension")
    if keys.dim() != 4 or values.shape != keys.shape or keys.size(3) != head_dim or keys.dtype != query.dtype:
        raise ValueError("incompatible Q/K/V shapes")
    _check_heads(query, keys.size(1))
    if local_window < 0 or span_width <= 0:
        raise ValueError("invalid centers or head dimension")
    starts = as_int64(centers).contiguous()
    n_spans = starts.size(1)
    if page_table is None:
        if keys.size(0) != batch:
            raise ValueError("incompatible Q/K/V shapes")
        length = keys.size(2)
        layout = contiguous_layout(keys, values, length)
        lens = const_i32(query.device, batch, length)
        keep = (starts, lens)
    else:
        if context_lens is None:
            raise ValueError("context_lens is required with page_table")
        table = as_int32(page_table).contiguous()
        lens = as_int32(context_lens).contiguous()
        layout = pool_layout(keys, values, table)
        keep = (starts, table, lens)
    kv_heads = keys.size(1)
    out = torch.empty_like(query)
    dev = query.device
    max_cand = local_window + n_spans * (span_width + 128)
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, heads, kv_heads, head_dim, max_cand)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    rc = _lib.lib.spa_span_gather_decode(query.data_ptr(), dtype_code(query), batch, heads, kv_heads, head_dim,
                                         ctypes.byref(layout), lens.data_ptr(), local_window, starts.data_ptr(),
                                         n_spans, span_width, head_dim ** -0.5, out.data_ptr(),
                                         ws.data_ptr() if ws is not None else None, ws_bytes, stream_ptr(dev))
    _lib.check(rc, "spa_span_gather_decode")
    del keep
    return out
