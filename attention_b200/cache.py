"""Paged KV cache (shared page pool + page table), KV append and the promotion cache.

* ``PagedKVCache``: K and V pools ``[num_pages, Hkv, P, D]``; one (page, kv head)
  tile of P*D elements is contiguous, so a page is one TMA box column.  The
  reference keeps contiguous ``[B, H, L, D]`` tensors and overwrites their tail
  (experiments/triton_kvcache_transformer_decode.py:51-55); here a new token is
  written in place at its (page, offset) with ``kv_append``.
* ``PromotionCache``: per-row table of ``slots`` hot pages with a fixed TTL,
  updated in place on the device every decode step (reference policy:
  evaluate_promotion_ttl.py:134-135, reuse at triton_promotion_cache_benchmark.py:53-60).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._util import as_int32, as_int64, dtype_code, stream_ptr
from .paged_attention import pool_layout


class PagedKVCache:
    def __init__(self, num_pages: int, kv_heads: int, page_size: int, head_dim: int, *, batch: int,
                 max_pages_per_seq: int, dtype=torch.bfloat16, device="cuda"):
        self.k = torch.zeros(num_pages, kv_heads, page_size, head_dim, dtype=dtype, device=device)
        self.v = torch.zeros_like(self.k)
        self.page_table = torch.full((batch, max_pages_per_seq), -1, dtype=torch.int32, device=device)
        self.context_lens = torch.zeros(batch, dtype=torch.int32, device=device)
        self.page_size = page_size

    @property
    def layout(self) -> _lib.KvLayout:
        return pool_layout(self.k, self.v, self.page_table)


def kv_append(k_pool: torch.Tensor, v_pool: torch.Tensor, page_table: torch.Tensor, k_new: torch.Tensor,
              v_new: torch.Tensor, positions: torch.Tensor) -> None:
    """Writes ``k_new``/``v_new`` ``[B, Hkv, D]`` at token ``positions[b]`` of each sequence."""
    if not (k_pool.is_cuda and k_new.is_cuda and positions.is_cuda):
        raise ValueError("CUDA tensors are required")
    if k_new.shape != v_new.shape or k_new.dim() != 3 or k_new.size(1) != k_pool.size(1):
        raise ValueError("k_new/v_new must be [B, Hkv, D]")
    if k_new.dtype != k_pool.dtype or k_new.size(2) != k_pool.size(3):
        raise ValueError("k_new/v_new must match the pool's dtype and head_dim")
    table = as_int32(page_table).contiguous()
    pos = as_int32(positions).contiguous()
    kn, vn = k_new.contiguous(), v_new.contiguous()
    layout = pool_layout(k_pool, v_pool, table)
    rc = _lib.lib.spa_kv_append(ctypes.byref(layout), dtype_code(k_pool), kn.size(0), kn.size(1), kn.size(2),
                                kn.data_ptr(), vn.data_ptr(), pos.data_ptr(), stream_ptr(k_pool.device))
    _lib.check(rc, "spa_kv_append")


class PromotionCache:
    """Device table of promoted (hot) pages: ``pages[rows, slots]`` (int32, -1 free)
    and ``last_hit[rows, slots]`` (int32 decode step)."""

    def __init__(self, rows: int, slots: int = 64, ttl: int = 32, device="cuda"):
        self.pages = torch.full((rows, slots), -1, dtype=torch.int32, device=device)
        self.last_hit = torch.zeros((rows, slots), dtype=torch.int32, device=device)
        self.rows, self.slots, self.ttl = rows, slots, ttl

    def update(self, selected: torch.Tensor, step) -> None:
        """Applies one step's selections ``[rows, m]`` (int64 or int32 page ids).  ``step``
        is an int, or a device int32 tensor of one element read by the kernel (graph replay)."""
        sel = as_int64(selected).contiguous()
        if sel.dim() != 2 or sel.size(0) != self.rows or not sel.is_cuda:
            raise ValueError("selected must be a CUDA tensor [rows, m]")
        if isinstance(step, torch.Tensor):
            if step.dtype != torch.int32 or not step.is_cuda or step.numel() != 1:
                raise ValueError("a device step must be a one-element int32 CUDA tensor")
            step_val, step_ptr = 0, step.data_ptr()
        else:
            step_val, step_ptr = int(step), None
        rc = _lib.lib.spa_promotion_update(self.pages.data_ptr(), self.last_hit.data_ptr(), self.rows, self.slots,
                                           sel.data_ptr(), sel.size(1), step_val, step_ptr, self.ttl,
                                           stream_ptr(self.pages.device))
        _lib.check(rc, "spa_promotion_update")
