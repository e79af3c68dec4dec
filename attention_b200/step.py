"""One routed sparse decode step as a single call: router, then fused page-gather decode.

Reference: the timed unit of experiments/triton_paged_gather_decode_benchmark.py:69
(and triton_promotion_cache_benchmark.py:59),
``paged_gather_decode_attention(q, K, V, select_blocks(q, summaries, m), local_window=W, block_size=P)``.
Here the router and the decode are chained kernels on the device: the decode grid
starts while the router runs and streams the local window before it reads the
selected page ids.  Returns ``(out, selected)``; both equal what
``select_blocks[_tree]`` followed by ``paged_gather_decode_attention`` return.
With ``gate`` (a ``RefreshGate``), a step whose gate is closed reuses the promoted
pages and the router reads no summaries (promotion reuse,
triton_promotion_cache_benchmark.py:53-60).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._util import as_int32, const_i32, dtype_code, stream_ptr, workspace
from .paged_attention import contiguous_layout, pool_layout


def sparse_decode_step(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, summaries: torch.Tensor, *,
                       top_blocks: int, local_window: int, block_size: int,
                       super_summaries: torch.Tensor | None = None, superblock: int = 0, top_super: int = 0,
                       router_scale: float = 1.0, page_table: torch.Tensor | None = None,
                       context_lens: torch.Tensor | None = None, out: torch.Tensor | None = None,
                       selected: torch.Tensor | None = None, gate=None):
    if not (query.is_cuda and keys.is_cuda and values.is_cuda and summaries.is_cuda):
        raise ValueError("CUDA tensors are required")
    if not (query.is_contiguous() and keys.is_contiguous() and values.is_contiguous()):
        raise ValueError("contiguous CUDA tensors are required")
    batch, q_heads, head_dim = query.shape
    kv_heads = keys.size(1)
    if keys.dim() != 4 or values.shape != keys.shape or keys.size(3) != head_dim or q_heads % kv_heads:
        raise ValueError("incompatible Q/K/V shapes")
    summ = summaries.float().contiguous()
    if summ.dim() != 4 or summ.shape[:2] != (batch, kv_heads) or summ.size(3) != head_dim:
        raise ValueError("summaries must be [B, Hkv, pages, D]")
    sup = None
    if super_summaries is not None:
        sup = super_summaries.float().contiguous()
        if sup.shape[:2] != (batch, kv_heads) or sup.size(2) != -(-summ.size(2) // superblock):
            raise ValueError("super_summaries must be [B, Hkv, ceil(pages/superblock), D]")
    dev = query.device
    if page_table is None:
        length = keys.size(2)
        if (length - local_window) % block_size or local_window > length:
            raise ValueError("unsupported head dimension or page layout")
        layout = contiguous_layout(keys, values, block_size)
        lens = const_i32(dev, batch, length)
    else:
        if context_lens is None or keys.size(2) != block_size:
            raise ValueError("page pool needs context_lens and block_size == page size")
        table = as_int32(page_table).contiguous()
        lens = as_int32(context_lens).contiguous()
        layout = pool_layout(keys, values, table)
    if out is None:
        out = torch.empty_like(query)
    if selected is None:
        selected = torch.empty(batch, top_blocks, dtype=torch.int64, device=dev)
    max_cand = local_window + top_blocks * block_size
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_cand)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    args = (query.data_ptr(), dtype_code(query), batch, q_heads, kv_heads, head_dim, ctypes.byref(layout),
            lens.data_ptr(), local_window, sup.data_ptr() if sup is not None else None,
            sup.size(2) if sup is not None else 0, summ.data_ptr(), summ.size(2), superblock, top_super, top_blocks,
            float(router_scale), head_dim ** -0.5, selected.data_ptr(), out.data_ptr(),
            ws.data_ptr() if ws is not None else None, ws_bytes)
    if gate is not None:
        promoted = gate.promoted_for(batch, top_blocks)
        rc = _lib.lib.spa_sparse_decode_step_gated(*args, gate.flags.data_ptr(), promoted.data_ptr(), stream_ptr(dev))
        _lib.check(rc, "spa_sparse_decode_step_gated")
    else:
        rc = _lib.lib.spa_sparse_decode_step(*args, stream_ptr(dev))
        _lib.check(rc, "spa_sparse_decode_step")
    return out, selected
