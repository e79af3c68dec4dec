"""One routed sparse decode step as a single call: router, then fused page-gather decode.

Reference: the timed unit of experiments/triton_paged_gather_decode_benchmark.py:69
(and triton_promotion_cache_benchmark.py:59),
``paged_gather_decode_attention(q, K, V, select_blocks(q, summaries, m), local_window=W, block_size=P)``.
Here, for the shapes the fused kernel serves (bf16/fp16, head_dim 64 or 128, at
most 8 kv heads, top_m <= 32, each (sequence, kv head) pair's splits merged in one
cluster), the step is ONE kernel launch: every decode cluster scores its sequence's
page summaries, selects the pages and streams them, while its local-window chunks
load.  Otherwise the router and the decode are chained kernels on the device: the
decode grid starts while the router runs and streams the local window before it
reads the selected page ids.  Returns ``(out, selected)``; both equal what
``select_blocks[_tree]`` followed by ``paged_gather_decode_attention`` return.
With ``gate`` (a ``RefreshGate``), a step whose gate is closed reuses the promoted
pages and the router reads no summaries (promotion reuse,
triton_promotion_cache_benchmark.py:53-60).
"""

from __future__ import annotations

import ctypes
import weakref

import torch

from . import _lib
from ._util import as_int32, const_i32, dtype_code, stream_ptr, workspace
from .paged_attention import contiguous_layout, pool_layout


def _prepare_step(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, summaries: torch.Tensor, *,
                  top_blocks: int, local_window: int, block_size: int, super_summaries: torch.Tensor | None,
                  superblock: int, top_super: int, page_table: torch.Tensor | None,
                  context_lens: torch.Tensor | None) -> dict:
    """Validates one step's inputs (``query`` gives the query's shape and dtype) and returns
    the C arguments with the tensors they borrow."""
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
    max_cand = local_window + top_blocks * block_size
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_cand)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    return dict(dev=dev, batch=batch, q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim, layout=layout,
                lens=lens, summ=summ, sup=sup, ws=ws, ws_bytes=ws_bytes, dtype=dtype_code(query))


# Prepared C arguments of recent step forms.  An entry is kept only when validation borrowed
# the caller's tensors as they are (fp32 summaries, int32 table and lengths: nothing
# converted, so nothing cached can go stale) and holds only integers (pointers, sizes) and
# the library's workspace, so it keeps none of the caller's memory alive.  Two keys lead to
# an entry:
# * the identity of the borrowed tensors (weak references: a hit needs the same live objects
#   at the same storage addresses) -- the cheap path for a caller that passes the same tensors;
# * their metadata (address, shape, strides, dtype), which determines every argument the
#   entry holds -- a caller that passes fresh views of the same storage (``table[g]``) hits
#   here, and a tensor freed and reallocated with other metadata cannot.
# Both keys also carry the query's shape and dtype, the step parameters and the stream.
_STEP_CACHE: dict = {}
_STEP_META: dict = {}
_STEP_CACHE_MAX = 32


def _meta(t):
    return None if t is None else (t.data_ptr(), t.shape, t.stride(), t.dtype)


def _remember(cache: dict, key, value) -> None:
    if len(cache) >= _STEP_CACHE_MAX:
        cache.pop(next(iter(cache)))
    cache[key] = value


def _prepared_step(query, keys, values, summaries, *, top_blocks, local_window, block_size, super_summaries,
                   superblock, top_super, page_table, context_lens, router_scale, stream, host_query=False):
    """The step's C arguments except the query, selection and output pointers:
    (head, tail, batch), from the cache when the same tensors (or tensors with the same
    storage and metadata) and parameters were prepared before."""
    held = (keys, values, summaries, super_summaries, page_table, context_lens)
    params = (query.shape, query.dtype, query.get_device(), top_blocks, local_window, block_size, superblock,
              top_super, float(router_scale), stream)
    key = (tuple(id(t) for t in held),) + params
    hit = _STEP_CACHE.get(key)
    if hit is not None:
        entry, refs, ptrs = hit
        if all((r is None and t is None) or (r is not None and r() is t and t.data_ptr() == ptr)
               for r, t, ptr in zip(refs, held, ptrs)):
            return entry
    mkey = tuple(_meta(t) for t in held) + params
    entry = _STEP_META.get(mkey)
    if entry is not None:
        # same storage and metadata as a prepared form (a caller passing fresh views): the
        # identity key stays that of the tensors first prepared
        return entry
    if not (query.is_cuda or host_query):
        raise ValueError("CUDA tensors are required")
    pr = _prepare_step(query, keys, values, summaries, top_blocks=top_blocks, local_window=local_window,
                       block_size=block_size, super_summaries=super_summaries, superblock=superblock,
                       top_super=top_super, page_table=page_table, context_lens=context_lens)
    sup, ws = pr["sup"], pr["ws"]
    head = (pr["dtype"], pr["batch"], pr["q_heads"], pr["kv_heads"], pr["head_dim"], ctypes.byref(pr["layout"]),
            pr["lens"].data_ptr(), local_window, sup.data_ptr() if sup is not None else None,
            sup.size(2) if sup is not None else 0, pr["summ"].data_ptr(), pr["summ"].size(2), superblock,
            top_super, top_blocks, float(router_scale), pr["head_dim"] ** -0.5)
    tail = (ws.data_ptr() if ws is not None else None, pr["ws_bytes"])
    entry = {"head": head, "tail": tail, "batch": pr["batch"], "ws": ws}
    borrowed = pr["summ"] is summaries and (super_summaries is None or sup is super_summaries) and (
        page_table is None or (pr["lens"] is context_lens and pr["layout"].page_table == page_table.data_ptr()
                               and page_table.dtype == torch.int32))
    if not borrowed:
        # converted copies: the arguments point into them, so the entry keeps them
        entry["keep"] = pr
        return entry
    _remember(_STEP_META, mkey, entry)
    refs = [weakref.ref(t) if t is not None else None for t in held]
    _remember(_STEP_CACHE, key, (entry, refs, [t.data_ptr() if t is not None else 0 for t in held]))
    return entry


def _check_outputs(query, out, selected, batch, top_blocks):
    if out is not None and (out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous()
                            or out.get_device() != query.get_device()):
        raise ValueError("out must be a contiguous CUDA tensor of the query's shape and dtype")
    if selected is not None and (selected.shape != (batch, top_blocks) or selected.dtype != torch.int64
                                 or not selected.is_contiguous() or selected.get_device() != query.get_device()):
        raise ValueError("selected must be a contiguous int64 CUDA tensor [batch, top_blocks]")


def set_step_fusion(enabled: bool) -> bool:
    """Process-wide: run qualifying steps as one launch (True, the default) or always as a
    router launch followed by a decode launch (False).  Returns the previous setting."""
    return bool(_lib.lib.spa_set_step_fusion(1 if enabled else 0))


def _sparse_decode_step_heads(query, keys, values, summaries, *, top_blocks, local_window, block_size,
                              super_summaries, superblock, top_super, router_scale, page_table, context_lens, out,
                              selected, kv_head_range):
    """The step over kv heads [begin, begin + count) of every sequence (one rank's shard):
    query and summaries hold every head, keys/values (and the output) those kv heads."""
    begin, count = (int(x) for x in kv_head_range)
    batch, q_heads, head_dim = query.shape
    kv_total = summaries.size(1)
    if not (query.is_cuda and keys.is_cuda and values.is_cuda and summaries.is_cuda):
        raise ValueError("CUDA tensors are required")
    if not (query.is_contiguous() and keys.is_contiguous() and values.is_contiguous()):
        raise ValueError("contiguous CUDA tensors are required")
    if q_heads % kv_total or begin < 0 or count <= 0 or begin + count > kv_total or keys.size(1) != count:
        raise ValueError("incompatible Q/K/V shapes")
    if keys.dim() != 4 or values.shape != keys.shape or keys.size(3) != head_dim:
        raise ValueError("incompatible Q/K/V shapes")
    group = q_heads // kv_total
    summ = summaries.float().contiguous()
    if summ.dim() != 4 or summ.size(0) != batch or summ.size(3) != head_dim:
        raise ValueError("summaries must be [B, Hkv, pages, D]")
    sup = None
    if super_summaries is not None:
        sup = super_summaries.float().contiguous()
        if sup.shape[:2] != (batch, kv_total) or sup.size(2) != -(-summ.size(2) // superblock):
            raise ValueError("super_summaries must be [B, Hkv, ceil(pages/superblock), D]")
    if page_table is None or context_lens is None or keys.size(2) != block_size:
        raise ValueError("page pool needs context_lens and block_size == page size")
    dev = keys.device
    table = as_int32(page_table).contiguous()
    lens = as_int32(context_lens).contiguous()
    layout = pool_layout(keys, values, table)
    max_cand = local_window + top_blocks * block_size
    ws_bytes = _lib.lib.spa_decode_workspace_size(batch, count * group, count, head_dim, max_cand)
    ws = workspace(dev, ws_bytes) if ws_bytes else None
    if out is not None and (out.shape != (batch, count * group, head_dim) or out.dtype != query.dtype
                            or not out.is_contiguous() or out.get_device() != query.get_device()):
        raise ValueError("out must be a contiguous CUDA tensor [batch, the shard's query heads, head_dim] "
                         "of the query's dtype")
    _check_outputs(query, None, selected, batch, top_blocks)
    if out is None:
        out = torch.empty(batch, count * group, head_dim, dtype=query.dtype, device=dev)
    if selected is None:
        selected = torch.empty(batch, top_blocks, dtype=torch.int64, device=dev)
    rc = _lib.lib.spa_sparse_decode_step_heads(
        query.data_ptr(), dtype_code(query), batch, q_heads, kv_total, head_dim, begin, count, ctypes.byref(layout),
        lens.data_ptr(), local_window, sup.data_ptr() if sup is not None else None,
        sup.size(2) if sup is not None else 0, summ.data_ptr(), summ.size(2), superblock, top_super, top_blocks,
        float(router_scale), head_dim ** -0.5, selected.data_ptr(), out.data_ptr(),
        ws.data_ptr() if ws is not None else None, ws_bytes, stream_ptr(dev))
    _lib.check(rc, "spa_sparse_decode_step_heads")
    return out, selected


def _sparse_decode_step_host(query, keys, values, summaries, *, top_blocks, local_window, block_size,
                             super_summaries, superblock, top_super, router_scale, page_table, context_lens, out,
                             selected):
    """The step with pinned host buffers (``spa_sparse_decode_step_host``): the query is read
    from host memory by a copy kernel, output and page ids are written into host memory by
    the step; they are complete when the caller's stream is."""
    if query.is_cuda or not query.is_contiguous() or not keys.is_cuda:
        raise ValueError("host query: a contiguous pinned CPU query with CUDA keys/values/summaries")
    dev_index = keys.get_device()
    stream = stream_ptr(dev_index)
    prep = _prepared_step(query, keys, values, summaries, top_blocks=top_blocks, local_window=local_window,
                          block_size=block_size, super_summaries=super_summaries, superblock=superblock,
                          top_super=top_super, page_table=page_table, context_lens=context_lens,
                          router_scale=router_scale, stream=stream, host_query=True)
    batch = prep["batch"]
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, pin_memory=True)
    elif out.is_cuda or out.shape != query.shape or out.dtype != query.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous pinned CPU tensor of the query's shape and dtype")
    if selected is None:
        selected = torch.empty(batch, top_blocks, dtype=torch.int64, pin_memory=True)
    elif (selected.is_cuda or selected.shape != (batch, top_blocks) or selected.dtype != torch.int64
          or not selected.is_contiguous()):
        raise ValueError("selected must be a contiguous pinned int64 CPU tensor [batch, top_blocks]")
    q_dev = prep.get("q_dev")
    if q_dev is None:  # device staging of the query and the page ids, kept with the prepared arguments
        q_dev = prep["q_dev"] = torch.empty(query.shape, dtype=query.dtype, device=keys.device)
        prep["sel_dev"] = torch.empty(batch, top_blocks, dtype=torch.int64, device=keys.device)
    rc = _lib.lib.spa_sparse_decode_step_host(query.data_ptr(), q_dev.data_ptr(), *prep["head"],
                                              prep["sel_dev"].data_ptr(), selected.data_ptr(), out.data_ptr(),
                                              *prep["tail"], stream)
    if rc == _lib.SPA_ERR_INVALID:
        raise ValueError("spa_sparse_decode_step_host: query, out and selected must be pinned host memory")
    _lib.check(rc, "spa_sparse_decode_step_host")
    return out, selected


def sparse_decode_step(query: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, summaries: torch.Tensor, *,
                       top_blocks: int, local_window: int, block_size: int,
                       super_summaries: torch.Tensor | None = None, superblock: int = 0, top_super: int = 0,
                       router_scale: float = 1.0, page_table: torch.Tensor | None = None,
                       context_lens: torch.Tensor | None = None, out: torch.Tensor | None = None,
                       selected: torch.Tensor | None = None, gate=None,
                       kv_head_range: tuple[int, int] | None = None, chained: bool = False):
    """``kv_head_range=(begin, count)``: one rank's (sequence, kv head) shard -- query and
    summaries hold every head of the sequences, keys/values only kv heads
    [begin, begin + count) of a page pool, and the output those kv heads' query heads.
    Every shard of a sequence selects the same pages.  ``chained``: the step's first
    kernel launches as a programmatic dependent of the kernel before it
    (``spa_sparse_decode_step_chained``; a model's decode step).

    A pinned CPU ``query`` (with pinned CPU ``out`` / ``selected``, allocated pinned when
    omitted) runs the step with host buffers (``spa_sparse_decode_step_host``): no copy
    engine, results on the host once the current stream has completed."""
    if not query.is_cuda:
        if gate is not None or kv_head_range is not None or chained:
            raise ValueError("CUDA tensors are required")
        return _sparse_decode_step_host(query, keys, values, summaries, top_blocks=top_blocks,
                                        local_window=local_window, block_size=block_size,
                                        super_summaries=super_summaries, superblock=superblock, top_super=top_super,
                                        router_scale=router_scale, page_table=page_table,
                                        context_lens=context_lens, out=out, selected=selected)
    if kv_head_range is not None:
        if gate is not None:
            raise ValueError("a refresh gate is not supported with kv_head_range")
        return _sparse_decode_step_heads(query, keys, values, summaries, top_blocks=top_blocks,
                                         local_window=local_window, block_size=block_size,
                                         super_summaries=super_summaries, superblock=superblock,
                                         top_super=top_super, router_scale=router_scale, page_table=page_table,
                                         context_lens=context_lens, out=out, selected=selected,
                                         kv_head_range=kv_head_range)
    if not query.is_contiguous():
        raise ValueError("contiguous CUDA tensors are required")
    stream = stream_ptr(query.get_device())
    prep = _prepared_step(query, keys, values, summaries, top_blocks=top_blocks, local_window=local_window,
                          block_size=block_size, super_summaries=super_summaries, superblock=superblock,
                          top_super=top_super, page_table=page_table, context_lens=context_lens,
                          router_scale=router_scale, stream=stream)
    _check_outputs(query, out, selected, prep["batch"], top_blocks)
    if out is None:
        out = torch.empty_like(query)
    if selected is None:
        selected = torch.empty(prep["batch"], top_blocks, dtype=torch.int64, device=query.device)
    args = (query.data_ptr(),) + prep["head"] + (selected.data_ptr(), out.data_ptr()) + prep["tail"]
    if gate is not None:
        promoted = gate.promoted_for(prep["batch"], top_blocks)
        rc = _lib.lib.spa_sparse_decode_step_gated(*args, gate.flags.data_ptr(), promoted.data_ptr(), stream)
        _lib.check(rc, "spa_sparse_decode_step_gated")
    else:
        fn = _lib.lib.spa_sparse_decode_step_chained if chained else _lib.lib.spa_sparse_decode_step
        rc = fn(*args, stream)
        _lib.check(rc, "spa_sparse_decode_step")
    return out, selected


class SparseDecodeSession:
    """One prepared sparse decode step for a fixed pool, page table and summaries.

    A native session object (``spa_session_*`` in the C ABI) holds every argument of the
    step and captures, per host-buffer slot, a CUDA graph of the fused step's two kernels:
    the router reads the query from a pinned host buffer over PCIe (mapped host memory, no
    copy-engine transfer) and leaves a device copy for the decode; the decode writes the
    output, and the router a copy of the page ids, into a pinned host buffer.  A step is
    one ctypes call: one graph launch and one event record on the host.  The
    host buffers are double-buffered: step i reuses the buffers of step i-2 after waiting
    for its completion, so the host can prepare one step ahead of the device.  The returned
    tensors are filled when the step's work completes (``torch.cuda.synchronize()``)."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor, summaries: torch.Tensor, *, q_heads: int,
                 top_blocks: int, local_window: int, block_size: int, batch: int | None = None,
                 super_summaries: torch.Tensor | None = None, superblock: int = 0, top_super: int = 0,
                 router_scale: float = 1.0, page_table: torch.Tensor | None = None,
                 context_lens: torch.Tensor | None = None, gate=None, io_mode: int | None = None):
        dev = keys.device
        batch = batch if batch is not None else summaries.size(0)
        shape = (batch, q_heads, keys.size(3))
        if io_mode is None:
            io_mode = _lib.SESSION_COPY_IN
        q_like = torch.empty(shape, dtype=keys.dtype, device=dev)  # shape and dtype of the query
        pr = _prepare_step(q_like, keys, values, summaries, top_blocks=top_blocks, local_window=local_window,
                           block_size=block_size, super_summaries=super_summaries, superblock=superblock,
                           top_super=top_super, page_table=page_table, context_lens=context_lens)
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
        self._buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        sup = pr["sup"]
        p = _lib.SessionParams()
        p.dtype, p.batch, p.q_heads, p.kv_heads, p.head_dim = (pr["dtype"], batch, q_heads, pr["kv_heads"],
                                                              pr["head_dim"])
        p.kv = pr["layout"]
        p.context_lens = pr["lens"].data_ptr()
        p.local_window = local_window
        p.super_summaries = sup.data_ptr() if sup is not None else None
        p.n_super = sup.size(2) if sup is not None else 0
        p.summaries, p.n_pages = pr["summ"].data_ptr(), pr["summ"].size(2)
        p.superblock, p.top_super, p.top_m = superblock, top_super, top_blocks
        p.router_scale, p.attn_scale = float(router_scale), pr["head_dim"] ** -0.5
        p.workspace = pr["ws"].data_ptr() if pr["ws"] is not None else None
        p.workspace_bytes = pr["ws_bytes"]
        if gate is not None:
            promoted = gate.promoted_for(batch, top_blocks)
            p.gate, p.promoted = gate.flags.data_ptr(), promoted.data_ptr()
        for k in range(2):
            p.query[k] = _lib.host_device_pointer(self.host_query[k].data_ptr())
            p.result_host[k] = _lib.host_device_pointer(self._host_buf[k].data_ptr())
        self._q_dev = torch.empty(shape, dtype=keys.dtype, device=dev)
        p.query_dev, p.query_bytes = self._q_dev.data_ptr(), n_out
        p.io_mode = int(io_mode)
        p.result_dev, p.result_sel_offset, p.result_bytes = self._buf.data_ptr(), off, nbytes
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib.spa_session_create(ctypes.byref(p), ctypes.byref(handle)), "spa_session_create")
        self._handle = handle
        self._params = p
        self._dev = dev
        self._n = 0
        self._keep = (keys, values, summaries, super_summaries, page_table, context_lens, gate, pr)

    def step(self, query: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None):
        """Runs one step; returns (host_out, host_selected) of this step, filled when the
        step completes.  Without ``query``, the step reads the query already in
        ``host_query[i % 2]``.  ``stream``: the CUDA stream to enqueue on (default: the
        current stream)."""
        k = self._n & 1
        _lib.check(_lib.lib.spa_session_wait(self._handle, k), "spa_session_wait")  # step i-2 is done
        if query is not None:
            self.host_query[k].copy_(query)
        st = (stream if stream is not None else torch.cuda.current_stream(self._dev)).cuda_stream
        _lib.check(_lib.lib.spa_session_step(self._handle, k, st), "spa_session_step")
        self._n += 1
        return self.host_out[k], self.host_selected[k]

    def close(self) -> None:
        """Releases the native session (waits for its steps)."""
        if getattr(self, "_handle", None):
            _lib.lib.spa_session_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
