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
    if not query.is_cuda:
        raise ValueError("CUDA tensors are required")
    return _launch_step(query.data_ptr(), query, keys, values, summaries, top_blocks=top_blocks,
                        local_window=local_window, block_size=block_size, super_summaries=super_summaries,
                        superblock=superblock, top_super=top_super, router_scale=router_scale,
                        page_table=page_table, context_lens=context_lens, out=out, selected=selected, gate=gate)


def _launch_step(query_ptr: int, query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                 summaries: torch.Tensor, *, top_blocks: int, local_window: int, block_size: int,
                 super_summaries: torch.Tensor | None, superblock: int, top_super: int, router_scale: float,
                 page_table: torch.Tensor | None, context_lens: torch.Tensor | None, out: torch.Tensor | None,
                 selected: torch.Tensor | None, gate):
    """Validates and launches one step; the kernels read the query at ``query_ptr`` (device
    memory, or mapped pinned host memory), shaped and typed like ``query``."""
    if not (keys.is_cuda and values.is_cuda and summaries.is_cuda):
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
    dev = keys.device
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
        out = torch.empty(query.shape, dtype=query.dtype, device=dev)
    if selected is None:
        selected = torch.empty(batch, top_blocks, dtype=torch.int64, device=dev)
    max_cand = local_window + top_blocks * block_size
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_cand)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    args = (query_ptr, dtype_code(query), batch, q_heads, kv_heads, head_dim, ctypes.byref(layout),
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


class SparseDecodeSession:
    """One prepared sparse decode step for a fixed pool, page table and summaries.

    The query lives in a pinned host buffer that the step's kernels read directly over
    PCIe (mapped host memory, no copy-engine transfer); right after the decode, a copy
    kernel (``spa_copy``, launched as the decode's programmatic dependent) writes the
    output and page ids into a pinned host buffer.  The whole step is captured once as a
    CUDA graph; ``step(query)`` writes the host query and replays, so a decode step costs
    one graph launch on the host.  The host buffers are double-buffered: step i reuses
    the buffers of step i-2 after waiting for its completion, so the host can prepare one
    step ahead of the device.  The returned tensors are filled when the step's work
    completes (``torch.cuda.synchronize()``)."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor, summaries: torch.Tensor, *, q_heads: int,
                 top_blocks: int, local_window: int, block_size: int, batch: int | None = None,
                 super_summaries: torch.Tensor | None = None, superblock: int = 0, top_super: int = 0,
                 router_scale: float = 1.0, page_table: torch.Tensor | None = None,
                 context_lens: torch.Tensor | None = None, gate=None):
        dev = keys.device
        batch = batch if batch is not None else summaries.size(0)
        shape = (batch, q_heads, keys.size(3))
        # output and page ids share one buffer (page ids at a 16-byte aligned offset), so one
        # copy returns both
        n_out = batch * q_heads * keys.size(3) * keys.element_size()
        off = -(-n_out // 16) * 16
        nbytes = -(-(off + batch * top_blocks * 8) // 16) * 16

        def views(buf):
            return (buf[:n_out].view(keys.dtype).view(shape),
                    buf[off:off + batch * top_blocks * 8].view(torch.int64).view(batch, top_blocks))

        self.host_query = [torch.zeros(shape, dtype=keys.dtype).pin_memory() for _ in range(2)]
        self._host_buf = [torch.zeros(nbytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self.host_out, self.host_selected = zip(*(views(b) for b in self._host_buf))
        # device addresses of the pinned buffers, read and written by the kernels
        self._q_dev = [_lib.host_device_pointer(t.data_ptr()) for t in self.host_query]
        self._out_dev = [_lib.host_device_pointer(b.data_ptr()) for b in self._host_buf]
        self._q_like = torch.empty(shape, dtype=keys.dtype, device=dev)  # shape and dtype of the query
        self._buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self._out, self._sel = views(self._buf)
        self._done = [torch.cuda.Event(), torch.cuda.Event()]
        self._n = 0
        kw = dict(top_blocks=top_blocks, local_window=local_window, block_size=block_size,
                  super_summaries=super_summaries, superblock=superblock, top_super=top_super,
                  router_scale=router_scale, page_table=page_table, context_lens=context_lens,
                  out=self._out, selected=self._sel, gate=gate)

        def body(k):
            _launch_step(self._q_dev[k], self._q_like, keys, values, summaries, **kw)
            _lib.check(_lib.lib.spa_copy(self._out_dev[k], self._buf.data_ptr(), nbytes, stream_ptr(dev)),
                       "spa_copy")

        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up on the capture stream (workspace, descriptors)
            body(0)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self._graphs = []
        for k in range(2):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                body(k)
            self._graphs.append(g)
        for e in self._done:
            e.record()
        self._keep = (keys, values, summaries, super_summaries, page_table, context_lens, gate)

    def step(self, query: torch.Tensor | None = None):
        """Runs one step; returns (host_out, host_selected) of this step, filled when the
        step completes.  Without ``query``, the step reads the query already in
        ``host_query[i % 2]``."""
        k = self._n & 1
        self._done[k].synchronize()  # step i-2 used these host buffers
        if query is not None:
            self.host_query[k].copy_(query)
        self._graphs[k].replay()
        self._done[k].record()
        self._n += 1
        return self.host_out[k], self.host_selected[k]
