"""Causal sliding-window local prefill: drop-in for
experiments/triton_local_prefill.py:61-81 ``local_causal_prefill(query, keys, values, window)``.

q/k/v/out are ``[B, H, S, D]``; query i attends keys [i-window+1, i].  bf16/fp16
with head_dim 64 or 128 run the tcgen05/TMEM tensor-core kernel; other dtypes and
head dims run a CUDA-core kernel.  Keyword-only extension for sequence-parallel
chunks: ``k_halo``/``v_halo`` ``[B, H, halo, D]`` hold the keys that precede the
chunk (the previous rank's last tokens).
"""

from __future__ import annotations

import torch

from . import _lib
from ._util import dtype_code, stream_ptr


def local_causal_prefill(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, window: int, *,
                         k_halo: torch.Tensor | None = None, v_halo: torch.Tensor | None = None,
                         out: torch.Tensor | None = None, rows: tuple[int, int] | None = None) -> torch.Tensor:
    """``rows=(begin, end)`` computes only those query rows of ``out`` (the rest of
    ``out`` is left as it was), so halo-free rows can overlap the halo exchange."""
    if not (query.is_cuda and query.is_contiguous() and keys.is_contiguous() and values.is_contiguous()):
        raise ValueError("contiguous CUDA tensors are required")
    if not (keys.is_cuda and values.is_cuda):
        raise ValueError("contiguous CUDA tensors are required")
    if query.dim() != 4 or keys.shape != query.shape or values.shape != query.shape or query.size(3) > 256:
        raise ValueError("unsupported Q/K/V shape")
    if keys.dtype != query.dtype or values.dtype != query.dtype:
        raise ValueError("unsupported Q/K/V shape")
    if window <= 0:
        raise ValueError("window must be positive")
    batch, heads, seq, dim = query.shape
    halo = 0
    if k_halo is not None or v_halo is not None:
        if k_halo is None or v_halo is None or k_halo.shape != v_halo.shape:
            raise ValueError("k_halo and v_halo must be given together with equal shapes")
        if k_halo.dim() != 4 or k_halo.shape[:2] != query.shape[:2] or k_halo.size(3) != dim:
            raise ValueError("halo must be [B, H, halo, D]")
        if not (k_halo.is_cuda and k_halo.is_contiguous() and v_halo.is_contiguous()):
            raise ValueError("contiguous CUDA tensors are required")
        if k_halo.dtype != query.dtype or v_halo.dtype != query.dtype:
            raise ValueError("unsupported Q/K/V shape")
        halo = k_halo.size(2)
    if out is None:
        out = torch.empty_like(query)
    elif out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous():
        raise ValueError("out must match query")
    r0, r1 = rows if rows is not None else (0, seq)
    if not 0 <= r0 < r1 <= seq:
        raise ValueError("rows must satisfy 0 <= begin < end <= seq_len")
    rc = _lib.lib.spa_local_prefill(query.data_ptr(), keys.data_ptr(), values.data_ptr(), dtype_code(query), batch,
                                    heads, seq, dim, window,
                                    k_halo.data_ptr() if halo else None, v_halo.data_ptr() if halo else None, halo,
                                    r0, r1, out.data_ptr(), stream_ptr(query.device))
    _lib.check(rc, "spa_local_prefill")
    return out
