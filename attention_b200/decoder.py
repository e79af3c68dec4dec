"""Integrated KV-cache decoder with sparse paged attention and a promotion cache.

The model follows the reference's tiny decoder block (train_tiny_transformer.py:134-190:
pre-norm attention and a 4x GELU MLP, learned token and position embeddings) with
RMSNorm in place of LayerNorm.  Its decode step is the reference's page_decode
(triton_kvcache_transformer_decode.py:47-66) re-built around the paged cache:

  per layer: RMSNorm -> QKV -> kv_append(new token into its page) -> router top-m over
  the routable pages (mean-key summaries) -> fused page-gather decode over the local
  window + selected pages -> output projection -> residual -> RMSNorm -> MLP -> residual;
  the promotion table of the layer is updated with the step's selection
  (fixed-TTL policy, evaluate_promotion_ttl.py:134-135).

The prompt is prefilled with the causal tensor-core prefill (window = prompt length,
i.e. full causal attention) and written into the page cache; its GEMMs (16k rows) run on
the library GEMM.  A decode step runs this library's kernels only: few-row linear layers
with the norms fused in front, routing + gather decode in one launch per layer, the
promotion table and the greedy argmax.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib
from ._util import dtype_code, stream_ptr
from .cache import PromotionCache, kv_append
from .paged_attention import paged_gather_decode_attention, pool_layout
from .prefill import local_causal_prefill
from .router import page_summaries
from .step import sparse_decode_step


@dataclass
class DecoderConfig:
    vocab: int = 4096
    d_model: int = 512
    heads: int = 8
    layers: int = 4
    mlp_mult: int = 4
    page_size: int = 128
    local_window: int = 128
    top_m: int = 8
    promo_slots: int = 64
    promo_ttl: int = 32
    max_context: int = 16384 + 256
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads

    @property
    def max_pages(self) -> int:
        return -(-self.max_context // self.page_size)


def init_weights(cfg: DecoderConfig, seed: int = 0) -> dict:
    """Seeded random init (CPU, fp32): N(0, 0.02) matrices, unit norms, zero biases."""
    g = torch.Generator().manual_seed(seed)
    d, v, f = cfg.d_model, cfg.vocab, cfg.mlp_mult * cfg.d_model

    def n(*shape):
        return torch.randn(*shape, generator=g) * 0.02

    w = {"emb": n(v, d), "pos": n(cfg.max_context, d), "norm_f": torch.ones(d), "head": n(v, d)}
    for i in range(cfg.layers):
        w[f"l{i}.norm1"] = torch.ones(d)
        w[f"l{i}.qkv.w"] = n(3 * d, d)
        w[f"l{i}.qkv.b"] = torch.zeros(3 * d)
        w[f"l{i}.out.w"] = n(d, d)
        w[f"l{i}.out.b"] = torch.zeros(d)
        w[f"l{i}.norm2"] = torch.ones(d)
        w[f"l{i}.fc1.w"] = n(f, d)
        w[f"l{i}.fc1.b"] = torch.zeros(f)
        w[f"l{i}.fc2.w"] = n(d, f)
        w[f"l{i}.fc2.b"] = torch.zeros(d)
    return w


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm over the last dimension in one library launch (``spa_rms_norm``):
    ``(x * rsqrt(mean(x^2) + eps)) * weight`` in fp32, returned in x's dtype."""
    if not (x.is_cuda and weight.is_cuda):
        raise ValueError("CUDA tensors are required")
    xc = x.contiguous()
    w = weight.to(x.dtype).contiguous()
    out = torch.empty_like(xc)
    dim = xc.size(-1)
    _lib.check(_lib.lib.spa_rms_norm(xc.data_ptr(), w.data_ptr(), out.data_ptr(), xc.numel() // dim, dim,
                                     float(eps), dtype_code(xc), stream_ptr(xc.device)), "spa_rms_norm")
    return out


def add_rms_norm(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor, eps: float, *,
                 x_out: torch.Tensor | None = None) -> torch.Tensor:
    """The residual add and the RMSNorm after it in one launch (``spa_add_rms_norm``):
    ``x_out = x + delta`` (rounded as the elementwise add rounds it), returns
    ``rms_norm(x_out, weight, eps)``.  ``x_out`` may be ``x`` (in place); by default it is x."""
    if not (x.is_cuda and delta.is_cuda and weight.is_cuda):
        raise ValueError("CUDA tensors are required")
    if delta.shape != x.shape or delta.dtype != x.dtype or not (x.is_contiguous() and delta.is_contiguous()):
        raise ValueError("x and delta must be contiguous tensors of one shape and dtype")
    x_out = x if x_out is None else x_out
    if x_out.shape != x.shape or x_out.dtype != x.dtype or not x_out.is_contiguous():
        raise ValueError("x_out must be a contiguous tensor like x")
    w = weight.to(x.dtype).contiguous()
    out = torch.empty_like(x)
    dim = x.size(-1)
    _lib.check(_lib.lib.spa_add_rms_norm(x.data_ptr(), delta.data_ptr(), w.data_ptr(), x_out.data_ptr(),
                                         out.data_ptr(), x.numel() // dim, dim, float(eps), dtype_code(x),
                                         stream_ptr(x.device)), "spa_add_rms_norm")
    return out


LINEAR_MAX_ROWS = 4


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *, gelu: bool = False,
           out: torch.Tensor | None = None, chained: bool = False) -> torch.Tensor:
    """``F.linear`` (then exact GELU when ``gelu``) for 1..4 rows in one launch
    (``spa_linear``): fp32 products and sums, rounded to x's dtype.  ``out`` may be an fp32
    tensor, which then holds the rounded values.  ``chained``: ``spa_linear_chained``, which
    streams the weight rows while the kernel enqueued before it still runs (the weights
    must not be that kernel's outputs)."""
    if not (x.is_cuda and weight.is_cuda and (bias is None or bias.is_cuda)):
        raise ValueError("CUDA tensors are required")
    if x.dim() != 2 or not 0 < x.size(0) <= LINEAR_MAX_ROWS:
        raise ValueError(f"x must be [rows, in_features] with 1..{LINEAR_MAX_ROWS} rows")
    n, k = weight.shape
    if x.size(1) != k or weight.dtype != x.dtype or (bias is not None and (bias.shape != (n,) or bias.dtype != x.dtype)):
        raise ValueError("x, weight and bias shapes or dtypes do not match")
    if not (x.is_contiguous() and weight.is_contiguous() and (bias is None or bias.is_contiguous())):
        raise ValueError("inputs must be contiguous")
    if out is None:
        out = torch.empty(x.size(0), n, dtype=x.dtype, device=x.device)
    elif out.shape != (x.size(0), n) or out.dtype not in (x.dtype, torch.float32) or not out.is_contiguous():
        raise ValueError("out must be a contiguous [rows, out_features] tensor of x's dtype or fp32")
    fn = _lib.lib.spa_linear_chained if chained else _lib.lib.spa_linear
    _lib.check(fn(x.data_ptr(), weight.data_ptr(), bias.data_ptr() if bias is not None else None, out.data_ptr(),
                  x.size(0), k, n, 1 if gelu else 0, 1 if out.dtype != x.dtype else 0, dtype_code(x),
                  stream_ptr(x.device)), "spa_linear")
    return out


def norm_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
                norm_weight: torch.Tensor, eps: float, delta: torch.Tensor | None = None,
                x_out: torch.Tensor | None = None, ids: torch.Tensor | None = None,
                positions: torch.Tensor | None = None, gelu: bool = False,
                out: torch.Tensor | None = None, append: tuple | None = None, chained: bool = False) -> torch.Tensor:
    """``linear(rms_norm(x (+ delta)), weight, bias)`` for 1..4 rows in one launch
    (``spa_norm_linear``); the normalised rows are bit-identical to ``add_rms_norm`` /
    ``rms_norm``.  With ``ids`` (int64) and ``positions`` (int32), ``x`` and ``delta`` are
    the token and position embedding tables and the rows are looked up as in
    ``embed_rms_norm``.  ``x_out`` (optional) receives the summed rows and must be a
    separate buffer from ``x`` and ``delta``.  ``append = (k_pool, v_pool, page_table,
    positions, k_col, v_col)`` also stores output columns ``[k_col, k_col + Hkv*D)`` and
    ``[v_col, ...)`` of row m as batch row m's new K and V, as ``kv_append`` would.
    ``chained``: ``spa_norm_linear_chained`` (see ``linear``)."""
    tensors = [x, weight, norm_weight] + [t for t in (bias, delta, x_out, ids, positions, out) if t is not None]
    if not all(t.is_cuda for t in tensors):
        raise ValueError("CUDA tensors are required")
    n, k = weight.shape
    embed = ids is not None
    if embed:
        if (positions is None or delta is None or ids.dtype != torch.int64 or positions.dtype != torch.int32
                or ids.dim() != 1 or ids.shape != positions.shape):
            raise ValueError("embedding mode needs delta and matching 1-d int64 ids / int32 positions")
        rows = ids.numel()
        if x.dim() != 2 or delta.dim() != 2 or delta.size(1) != k:
            raise ValueError("embedding tables must be [rows, in_features]")
    else:
        rows = x.size(0) if x.dim() == 2 else -1
        if delta is not None and delta.shape != x.shape:
            raise ValueError("delta must match x")
    if not 0 < rows <= LINEAR_MAX_ROWS or x.size(-1) != k or norm_weight.numel() != k:
        raise ValueError(f"x must be [rows, in_features] with 1..{LINEAR_MAX_ROWS} rows")
    if weight.dtype != x.dtype or (delta is not None and delta.dtype != x.dtype) or (
            bias is not None and (bias.shape != (n,) or bias.dtype != x.dtype)):
        raise ValueError("x, delta, weight and bias shapes or dtypes do not match")
    if not all(t.is_contiguous() for t in tensors):
        raise ValueError("inputs must be contiguous")
    if x_out is not None:
        if x_out.shape != (rows, k) or x_out.dtype != x.dtype:
            raise ValueError("x_out must be [rows, in_features] of x's dtype")
        if x_out.data_ptr() in (x.data_ptr(), delta.data_ptr() if delta is not None else -1):
            raise ValueError("x_out must not overlap x or delta")
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=x.device)
    elif out.shape != (rows, n) or out.dtype not in (x.dtype, torch.float32):
        raise ValueError("out must be a contiguous [rows, out_features] tensor of x's dtype or fp32")
    epi = None
    if append is not None:
        k_pool, v_pool, table, pos, k_col, v_col = append[:6]
        q_out = append[6] if len(append) > 6 else None
        width = k_pool.size(1) * k_pool.size(3)
        if (k_pool.dtype != x.dtype or v_pool.shape != k_pool.shape or pos.dtype != torch.int32
                or pos.numel() != rows or table.dtype != torch.int32 or not (table.is_contiguous() and pos.is_contiguous())
                or not 0 <= k_col <= n - width or not 0 <= v_col <= n - width):
            raise ValueError("append needs pools of x's dtype, an int32 page table and [rows] int32 positions")
        epi = _lib.KvAppendEpilogue(pool_layout(k_pool, v_pool, table), pos.data_ptr(), k_col, v_col,
                                    k_pool.size(1), k_pool.size(3))
        if q_out is not None:
            # the query columns [0, q_width) also go to their own contiguous [rows, ...] buffer
            if (not q_out.is_cuda or q_out.dtype != x.dtype or not q_out.is_contiguous() or q_out.dim() < 2
                    or q_out.size(0) != rows or out.dtype != x.dtype or not 0 < q_out[0].numel() <= n):
                raise ValueError("q_out must be a contiguous CUDA tensor [rows, ...] of x's dtype")
            epi.q_out, epi.q_col, epi.q_width = q_out.data_ptr(), 0, q_out[0].numel()
    nw = norm_weight.to(x.dtype).contiguous()
    pro = _lib.NormPrologue()
    pro.delta = delta.data_ptr() if delta is not None else None
    if embed:
        pro.ids, pro.id_limit = ids.data_ptr(), x.size(0)
        pro.delta_ids, pro.delta_limit = positions.data_ptr(), delta.size(0)
    pro.norm_weight = nw.data_ptr()
    pro.eps = float(eps)
    pro.x_out = x_out.data_ptr() if x_out is not None else None
    fn = _lib.lib.spa_norm_linear_chained if chained else _lib.lib.spa_norm_linear
    _lib.check(fn(x.data_ptr(), ctypes.byref(pro), weight.data_ptr(), bias.data_ptr() if bias is not None else None,
                  out.data_ptr(), rows, k, n, 1 if gelu else 0, 1 if out.dtype != x.dtype else 0, dtype_code(x),
                  ctypes.byref(epi) if epi is not None else None, stream_ptr(x.device)), "spa_norm_linear")
    return out


def argmax_advance(logits: torch.Tensor, token: torch.Tensor, counters: torch.Tensor | None = None, *,
                   log: torch.Tensor | None = None, positions: torch.Tensor | None = None) -> None:
    """``token[r] = logits[r].argmax()`` (torch.argmax's rules) and ``counters += 1`` in one
    launch (``spa_argmax_advance``); logits fp32 [rows, cols], token int64 [rows], counters int32.
    With ``log`` (int64 [length, rows]) and ``positions`` (int32 [rows], read before the
    counters advance; may be a view of them): also ``log[positions[r], r] = token[r]``
    (``spa_argmax_advance_log``)."""
    if not (logits.is_cuda and token.is_cuda and (counters is None or counters.is_cuda)):
        raise ValueError("CUDA tensors are required")
    if (logits.dtype != torch.float32 or logits.dim() != 2 or not logits.is_contiguous() or token.dtype != torch.int64
            or token.shape != (logits.size(0),) or not token.is_contiguous()):
        raise ValueError("logits must be contiguous fp32 [rows, cols] and token int64 [rows]")
    if counters is not None and (counters.dtype != torch.int32 or not counters.is_contiguous()):
        raise ValueError("counters must be a contiguous int32 tensor")
    cptr, cn = (counters.data_ptr(), counters.numel()) if counters is not None else (None, 0)
    if log is None:
        _lib.check(_lib.lib.spa_argmax_advance(logits.data_ptr(), logits.size(0), logits.size(1), token.data_ptr(),
                                               cptr, cn, stream_ptr(logits.device)), "spa_argmax_advance")
        return
    rows = logits.size(0)
    if (positions is None or not (log.is_cuda and positions.is_cuda) or log.dtype != torch.int64 or log.dim() != 2
            or log.size(1) != rows or not log.is_contiguous() or positions.dtype != torch.int32
            or positions.shape != (rows,) or not positions.is_contiguous()):
        raise ValueError("log must be a contiguous int64 CUDA tensor [length, rows] and positions int32 [rows]")
    _lib.check(_lib.lib.spa_argmax_advance_log(logits.data_ptr(), rows, logits.size(1), token.data_ptr(), cptr, cn,
                                               positions.data_ptr(), log.data_ptr(), log.size(0),
                                               stream_ptr(logits.device)), "spa_argmax_advance_log")


def embed_rms_norm(table: torch.Tensor, ids: torch.Tensor, pos_table: torch.Tensor, positions: torch.Tensor,
                   weight: torch.Tensor, eps: float, *, x_out: torch.Tensor) -> torch.Tensor:
    """Token + position embedding lookup and the first RMSNorm in one launch
    (``spa_embed_rms_norm``): ``x_out = table[ids] + pos_table[positions]`` (ids int64,
    positions int32), returns ``rms_norm(x_out, weight, eps)``."""
    for t in (table, ids, pos_table, positions, weight, x_out):
        if not t.is_cuda:
            raise ValueError("CUDA tensors are required")
    if ids.dtype != torch.int64 or positions.dtype != torch.int32 or ids.shape != positions.shape or ids.dim() != 1:
        raise ValueError("ids (int64) and positions (int32) must be matching 1-d tensors")
    if not (ids.is_contiguous() and positions.is_contiguous() and table.is_contiguous() and pos_table.is_contiguous()):
        raise ValueError("inputs must be contiguous")
    dim = table.size(-1)
    if pos_table.dtype != table.dtype or pos_table.size(-1) != dim:
        raise ValueError("the embedding tables must share dtype and width")
    if x_out.shape != (ids.numel(), dim) or x_out.dtype != table.dtype or not x_out.is_contiguous():
        raise ValueError("x_out must be a contiguous [rows, dim] tensor of the tables' dtype")
    w = weight.to(table.dtype).contiguous()
    out = torch.empty_like(x_out)
    _lib.check(_lib.lib.spa_embed_rms_norm(table.data_ptr(), table.size(0), ids.data_ptr(), pos_table.data_ptr(),
                                           pos_table.size(0), positions.data_ptr(), w.data_ptr(), x_out.data_ptr(),
                                           out.data_ptr(), ids.numel(), dim, float(eps), dtype_code(table),
                                           stream_ptr(table.device)), "spa_embed_rms_norm")
    return out


def persistent_step_supported(cfg: DecoderConfig, batch: int) -> bool:
    """Whether ``spa_decoder_step`` (the whole decode step as one launch) takes this shape."""
    return (1 <= batch <= 4 and 1 <= cfg.layers <= _lib.DECODER_MAX_LAYERS and cfg.head_dim in (32, 64, 128)
            and cfg.d_model <= 512 and cfg.d_model % 8 == 0 and cfg.mlp_mult * cfg.d_model % 8 == 0
            and cfg.vocab % 8 == 0 and cfg.top_m <= 32 and cfg.max_pages <= 4096 and cfg.promo_slots <= 512)


class SparseDecoder:
    """Batch of sequences decoded with paged KV caches (one pool per layer).

    Sequence b owns pages [b * max_pages, (b+1) * max_pages) of every layer's pool.

    ``engine``: "kernels" runs a decode step as a chain of the library's few-row kernels
    (one per linear layer, one routed decode per layer, the promotion update and the
    argmax), launched as programmatic dependents of one another; "persistent" as one
    cooperative kernel (``spa_decoder_step``) whose phases exchange data through global
    memory.  "auto" is "kernels": on B200 the chain's launch boundaries cost less than the
    one kernel's seven inter-SM exchanges per layer (122 against 130 us per step at the
    benchmark's shape)."""

    def __init__(self, cfg: DecoderConfig, weights: dict, batch: int, *, dtype=torch.bfloat16, device="cuda",
                 engine: str = "auto"):
        if engine not in ("auto", "persistent", "kernels"):
            raise ValueError("engine must be 'auto', 'persistent' or 'kernels'")
        if engine == "auto":
            engine = "kernels"
        elif engine == "persistent" and not persistent_step_supported(cfg, batch):
            raise ValueError("this decoder shape is outside the persistent step's limits")
        self.engine = engine
        self.cfg, self.batch, self.dtype, self.device = cfg, batch, dtype, torch.device(device)
        self.w = {k: t.to(device=self.device, dtype=dtype) for k, t in weights.items()}
        h, p, dh = cfg.heads, cfg.page_size, cfg.head_dim
        n_pool = batch * cfg.max_pages
        self.k_pool = [torch.zeros(n_pool, h, p, dh, dtype=dtype, device=self.device) for _ in range(cfg.layers)]
        self.v_pool = [torch.zeros_like(self.k_pool[0]) for _ in range(cfg.layers)]
        self.page_table = torch.arange(n_pool, dtype=torch.int32, device=self.device).view(batch, cfg.max_pages)
        self.ctx = 0
        self.summaries: list[torch.Tensor | None] = [None] * cfg.layers
        self._summary_store: dict[int, torch.Tensor] = {}
        self.n_routable = 0
        self.prompt_len = 0
        self.promotion = PromotionCache(cfg.layers * batch, slots=cfg.promo_slots, ttl=cfg.promo_ttl,
                                        device=self.device)
        self.step_index = 0

    # ---------------------------------------------------------------- helpers
    def _linear(self, x, name, *, gelu=False, chained=False):
        w, b = self.w[f"{name}.w"], self.w[f"{name}.b"]
        if x.dim() == 2 and x.size(0) <= LINEAR_MAX_ROWS:
            return linear(x, w, b, gelu=gelu, chained=chained)  # decode: a few rows, one launch
        y = F.linear(x, w, b)
        return F.gelu(y) if gelu else y

    def _mlp(self, x, i):
        h = rms_norm(x, self.w[f"l{i}.norm2"], self.cfg.eps)
        return self._linear(self._linear(h, f"l{i}.fc1", gelu=True), f"l{i}.fc2")

    def _routable_pages(self, ctx: int) -> int:
        return max(0, (ctx - self.cfg.local_window) // self.cfg.page_size)

    def _refresh_summaries(self, n: int):
        """Summaries of pages [0, n) of every layer (recomputed when n changes: a page becomes
        routable once all its tokens are older than the local window).  They live at a fixed
        address per layer, so a step graph captured for n pages reads current summaries
        whenever it is replayed, after a rewind included."""
        self.n_routable = n
        for i in range(self.cfg.layers):
            if n <= 0:
                self.summaries[i] = None
                continue
            fresh = page_summaries(self.k_pool[i], block_size=self.cfg.page_size, n_pages=n,
                                   page_table=self.page_table)
            store = self._summary_store.get(i)
            if store is None:
                store = torch.empty(self.batch * self.cfg.heads * self.cfg.max_pages * self.cfg.head_dim,
                                    dtype=fresh.dtype, device=self.device)
                self._summary_store[i] = store
            view = store[: fresh.numel()].view(fresh.shape)
            view.copy_(fresh)
            self.summaries[i] = view

    # ---------------------------------------------------------------- prefill
    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [B, S] -> logits of the last position [B, vocab]."""
        cfg = self.cfg
        b, s = tokens.shape
        if s % cfg.page_size:
            raise ValueError("the prompt length must be a multiple of the page size")
        h, dh, p = cfg.heads, cfg.head_dim, cfg.page_size
        pos = torch.arange(s, device=self.device)
        x = self.w["emb"][tokens] + self.w["pos"][pos]
        for i in range(cfg.layers):
            hid = rms_norm(x, self.w[f"l{i}.norm1"], cfg.eps)
            qkv = self._linear(hid, f"l{i}.qkv").view(b, s, 3, h, dh).permute(2, 0, 3, 1, 4)
            q, k, v = (t.contiguous() for t in qkv)
            att = local_causal_prefill(q, k, v, s)  # full causal over the prompt
            # pages of sequence j are contiguous in the pool: [n_pages, H, P, Dh]
            npg = s // p
            for j in range(b):
                base = j * cfg.max_pages
                self.k_pool[i][base:base + npg] = k[j].view(h, npg, p, dh).permute(1, 0, 2, 3)
                self.v_pool[i][base:base + npg] = v[j].view(h, npg, p, dh).permute(1, 0, 2, 3)
            x = x + self._linear(att.transpose(1, 2).reshape(b, s, cfg.d_model), f"l{i}.out")
            x = x + self._mlp(x, i)
        self.ctx = s
        self.prompt_len = s
        self._refresh_summaries(self._routable_pages(s + 1))
        return F.linear(rms_norm(x[:, -1], self.w["norm_f"], cfg.eps), self.w["head"]).float()

    # ---------------------------------------------------------------- decode
    def _state(self):
        """Persistent device state of the decode loop (so one captured step replays)."""
        if not hasattr(self, "_token"):
            b = self.batch
            self._token = torch.zeros(b, dtype=torch.int64, device=self.device)
            # position, context length and step counter in one buffer: one launch advances all
            self._counters = torch.zeros(2 * b + 1, dtype=torch.int32, device=self.device)
            self._position = self._counters[:b]
            self._ctx_len = self._counters[b:2 * b]
            self._step_dev = self._counters[2 * b:]
            self._logits = torch.zeros(b, self.cfg.vocab, dtype=torch.float32, device=self.device)
            # the residual stream, alternating between two buffers (a fused norm + linear
            # reads one while its first CTA writes the updated rows to the other)
            self._xa = torch.zeros(b, self.cfg.d_model, dtype=self.dtype, device=self.device)
            self._xb = torch.zeros_like(self._xa)
            self._sel_bufs: dict = {}  # [layers, B, m] selections, per m
            self._graphs: dict = {}
            # the token chosen at each position, written by the step's last kernel (graph
            # replays follow one another with no copy in between)
            self._token_log = torch.zeros(self.cfg.max_context, b, dtype=torch.int64, device=self.device)
            # the query rows of the current layer, stored by the QKV product's epilogue
            self._q = torch.zeros(b, self.cfg.heads, self.cfg.head_dim, dtype=self.dtype, device=self.device)
            # the promotion update runs on a branch forked after the last layer's selection
            self._side = torch.cuda.Stream(device=self.device)

    def _norm_linear(self, x, delta, norm, name, x_out, *, gelu=False, append=None, chained=False):
        """x_out = x + delta; returns the linear layer ``name`` of rms_norm(x_out): one
        launch for a batch of up to four rows (with the K/V append when given), else the
        norm and a library GEMM (the caller then appends)."""
        w, b = self.w[f"{name}.w"], self.w[f"{name}.b"]
        if self.batch <= LINEAR_MAX_ROWS:
            return norm_linear(x, w, b, norm_weight=self.w[norm], eps=self.cfg.eps, delta=delta, x_out=x_out,
                               gelu=gelu, append=append, chained=chained)
        return self._linear(add_rms_norm(x, delta, self.w[norm], self.cfg.eps, x_out=x_out), name, gelu=gelu)

    def _persistent_params(self, m: int):
        """spa_decoder_step arguments for ``n_routable`` routable pages (cached per page
        count: every pointer is a persistent buffer)."""
        cache = self.__dict__.setdefault("_ds_params", {})
        p = cache.get(self.n_routable)
        if p is not None:
            return p
        cfg, w = self.cfg, self.w
        p = _lib.DecoderStepParams()
        p.dtype, p.batch, p.d_model, p.heads = dtype_code(self._xa), self.batch, cfg.d_model, cfg.heads
        p.ffn, p.vocab, p.layers = cfg.mlp_mult * cfg.d_model, cfg.vocab, cfg.layers
        p.local_window, p.top_m, p.n_pages, p.max_pages = cfg.local_window, cfg.top_m, self.n_routable, cfg.max_pages
        p.eps = cfg.eps
        p.router_scale = p.attn_scale = 1.0 / math.sqrt(cfg.head_dim)
        p.emb, p.emb_rows = w["emb"].data_ptr(), w["emb"].size(0)
        p.pos_emb, p.pos_rows = w["pos"].data_ptr(), w["pos"].size(0)
        p.norm_f, p.head_w = w["norm_f"].data_ptr(), w["head"].data_ptr()
        for i in range(cfg.layers):
            ly = p.layer[i]
            for field, name in (("norm1", f"l{i}.norm1"), ("qkv_w", f"l{i}.qkv.w"), ("qkv_b", f"l{i}.qkv.b"),
                                ("out_w", f"l{i}.out.w"), ("out_b", f"l{i}.out.b"), ("norm2", f"l{i}.norm2"),
                                ("fc1_w", f"l{i}.fc1.w"), ("fc1_b", f"l{i}.fc1.b"), ("fc2_w", f"l{i}.fc2.w"),
                                ("fc2_b", f"l{i}.fc2.b")):
                setattr(ly, field, w[name].data_ptr())
            ly.k_pool, ly.v_pool = self.k_pool[i].data_ptr(), self.v_pool[i].data_ptr()
            ly.summaries = self.summaries[i].data_ptr() if self.summaries[i] is not None else None
        p.kv = pool_layout(self.k_pool[0], self.v_pool[0], self.page_table)
        p.token, p.counters, p.logits = self._token.data_ptr(), self._counters.data_ptr(), self._logits.data_ptr()
        p.token_log, p.log_len = self._token_log.data_ptr(), self._token_log.size(0)
        p.selected = self._sel_bufs[max(m, 1)].data_ptr()
        p.promo_pages, p.promo_last_hit = self.promotion.pages.data_ptr(), self.promotion.last_hit.data_ptr()
        p.promo_slots, p.promo_ttl = self.promotion.slots, self.promotion.ttl
        ws = getattr(self, "_ds_workspace", None)
        need = _lib.lib.spa_decoder_step_workspace_size(ctypes.byref(p))
        if need == 0:
            raise ValueError("this decoder shape is outside the persistent step's limits")
        if ws is None or ws.numel() < need:
            # zero-filled once: the step's exchange words carry a launch counter kept in it
            ws = self._ds_workspace = torch.zeros(need, dtype=torch.uint8, device=self.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        cache[self.n_routable] = p
        return p

    def _persistent_step_body(self):
        """One decode step as one launch of ``spa_decoder_step``; returns the [layers, B, m]
        selections (m >= 1; -1 when no page is routable)."""
        m = min(self.cfg.top_m, self.n_routable)
        if max(m, 1) not in self._sel_bufs:
            self._sel_bufs[max(m, 1)] = torch.full((self.cfg.layers, self.batch, max(m, 1)), -1, dtype=torch.int64,
                                                   device=self.device)
        p = self._persistent_params(m)
        _lib.check(_lib.lib.spa_decoder_step(ctypes.byref(p), stream_ptr(self.device)), "spa_decoder_step")
        return self._sel_bufs[max(m, 1)]

    def _step_body(self):
        """One decode step on the persistent state (no host synchronisation, capturable).
        Each RMSNorm runs fused into the linear layer after it, together with the residual
        add before it (the embedding lookup for the first); the rounding is that of the
        separate ops.  Every kernel of the step is launched as a programmatic dependent of
        the one before it: it starts while its predecessor runs (the linear layers stream
        their weight rows then) and reads its other inputs after the predecessor completes."""
        if self.engine == "persistent":
            return self._persistent_step_body()
        cfg = self.cfg
        b = self.batch
        h, dh = cfg.heads, cfg.head_dim
        x, spare = self._xa, self._xb
        fused = b <= LINEAR_MAX_ROWS  # norms, products and the K/V append in few-row kernels
        d = cfg.d_model

        def append(i):  # the QKV product's K and V columns go straight into layer i's pools, Q into its buffer
            return (self.k_pool[i], self.v_pool[i], self.page_table, self._position, d, 2 * d, self._q) if fused else None

        if fused:
            qkv = norm_linear(self.w["emb"], self.w["l0.qkv.w"], self.w["l0.qkv.b"], norm_weight=self.w["l0.norm1"],
                              eps=cfg.eps, delta=self.w["pos"], ids=self._token, positions=self._position, x_out=x,
                              append=append(0), chained=True)
        else:
            hid = embed_rms_norm(self.w["emb"], self._token, self.w["pos"], self._position, self.w["l0.norm1"],
                                 cfg.eps, x_out=x)
            qkv = self._linear(hid, "l0.qkv")
        scale = 1.0 / math.sqrt(dh)
        m = min(cfg.top_m, self.n_routable)
        if m > 0:
            sel_all = self._sel_bufs.get(m)
            if sel_all is None:
                sel_all = self._sel_bufs[m] = torch.empty(cfg.layers, b, m, dtype=torch.int64, device=self.device)
        selected = []
        mlp_out = None
        for i in range(cfg.layers):
            if i > 0:
                qkv = self._norm_linear(x, mlp_out, f"l{i}.norm1", f"l{i}.qkv", spare, append=append(i), chained=True)
                x, spare = spare, x
            qkv = qkv.view(b, 3, h, dh)
            q = self._q if fused else qkv[:, 0].contiguous()
            if not fused:
                kv_append(self.k_pool[i], self.v_pool[i], self.page_table, qkv[:, 1].contiguous(),
                          qkv[:, 2].contiguous(), self._position)
            if m > 0:
                # router and gather decode chained on the device (one library call)
                att, sel = sparse_decode_step(q, self.k_pool[i], self.v_pool[i], self.summaries[i], top_blocks=m,
                                              local_window=cfg.local_window, block_size=cfg.page_size,
                                              router_scale=scale, page_table=self.page_table,
                                              context_lens=self._ctx_len, selected=sel_all[i], chained=True)
            else:
                sel = torch.full((b, 1), -1, dtype=torch.int64, device=self.device)
                att = paged_gather_decode_attention(q, self.k_pool[i], self.v_pool[i], sel,
                                                    local_window=cfg.local_window, block_size=cfg.page_size,
                                                    page_table=self.page_table, context_lens=self._ctx_len)
            if i == cfg.layers - 1:
                # every layer's selection is written: the promotion update runs beside the rest
                # of the step (nothing after it reads the promotion table)
                main = torch.cuda.current_stream(self.device)
                self._side.wait_stream(main)
                with torch.cuda.stream(self._side):
                    sel_rows = (sel_all if m > 0 else torch.stack(selected + [sel])).reshape(cfg.layers * b, -1)
                    self.promotion.update(sel_rows, self._step_dev)
            o = self._linear(att.reshape(b, cfg.d_model), f"l{i}.out", chained=True)
            hid = self._norm_linear(x, o, f"l{i}.norm2", f"l{i}.fc1", spare, gelu=True, chained=True)
            x, spare = spare, x
            mlp_out = self._linear(hid, f"l{i}.fc2", chained=True)
            selected.append(sel)
        if m == 0:
            sel_all = torch.stack(selected)  # [layers, B, 1]
        if b <= LINEAR_MAX_ROWS:
            # fp32 logits of the rounded products
            norm_linear(x, self.w["head"], norm_weight=self.w["norm_f"], eps=cfg.eps, delta=mlp_out, out=self._logits,
                        chained=True)
        else:
            hf = add_rms_norm(x, mlp_out, self.w["norm_f"], cfg.eps, x_out=spare)
            self._logits.copy_(F.linear(hf, self.w["head"]))
        # the branch (promotion update) joins before the counters advance: it reads the step
        # counter
        torch.cuda.current_stream(self.device).wait_stream(self._side)
        # greedy token (also logged at its position), then position, context length and step
        # advance (one launch)
        argmax_advance(self._logits, self._token, self._counters, log=self._token_log, positions=self._position)
        return sel_all

    def _check_room(self, steps: int) -> None:
        if self.ctx + steps > self.cfg.max_context:
            raise ValueError(f"decoding {steps} more tokens from position {self.ctx} exceeds max_context "
                             f"{self.cfg.max_context}")

    def rewind(self, ctx: int) -> None:
        """Moves the decode position back to ``ctx`` (between the prompt length and the
        current position), as after rejected speculative tokens: later steps overwrite the
        K/V from there.  The promotion table and the step counter are kept."""
        if not getattr(self, "prompt_len", None) or not self.prompt_len <= ctx <= self.ctx:
            raise ValueError("rewind target must lie between the prompt length and the current position")
        self.ctx = ctx
        self._begin_step()

    def _begin_step(self):
        """Host bookkeeping before a step: refresh summaries when a page becomes routable."""
        n_routable = self._routable_pages(self.ctx + 1)
        if n_routable != self.n_routable:
            self._refresh_summaries(n_routable)  # its pages were all written by earlier steps

    @torch.no_grad()
    def decode_step(self, token: torch.Tensor):
        """token [B] at position ctx -> (logits [B, vocab] fp32, selected [layers, B, m])."""
        self._check_room(1)
        self._state()
        if self.step_index == 0 or self._position[0].item() != self.ctx:
            self._position.fill_(self.ctx)
            self._ctx_len.fill_(self.ctx + 1)
            self._step_dev.fill_(self.step_index)
        self._token.copy_(token)
        self._begin_step()
        sel = self._step_body()
        self.step_index += 1
        self.ctx += 1
        return self._logits.clone(), sel.clone()

    @torch.no_grad()
    def generate(self, token: torch.Tensor, steps: int, *, graphed: bool = True) -> torch.Tensor:
        """Greedy decode of ``steps`` tokens starting from ``token`` [B]; returns the
        tokens [steps, B].  With ``graphed`` every step is one CUDA-graph replay (a new
        graph is captured only when the number of routable pages changes)."""
        self._check_room(steps)
        self._state()
        self._token.copy_(token)
        self._position.fill_(self.ctx)
        self._ctx_len.fill_(self.ctx + 1)
        self._step_dev.fill_(self.step_index)
        first = self.ctx
        for t in range(steps):
            self._begin_step()
            if graphed:
                key = self.n_routable
                g = self._graphs.get(key)
                if g is None:
                    # capture on a side stream; the capture itself must not advance the state
                    saved = [x.clone() for x in (self._token, self._position, self._ctx_len, self._step_dev)]
                    pages, last = self.promotion.pages.clone(), self.promotion.last_hit.clone()
                    s = torch.cuda.Stream(device=self.device)
                    s.wait_stream(torch.cuda.current_stream(self.device))
                    with torch.cuda.stream(s):
                        self._step_body()  # warm-up (allocates workspaces outside the graph)
                    torch.cuda.current_stream(self.device).wait_stream(s)
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g):
                        self._step_body()
                    for dst, src in zip((self._token, self._position, self._ctx_len, self._step_dev), saved):
                        dst.copy_(src)
                    self.promotion.pages.copy_(pages)
                    self.promotion.last_hit.copy_(last)
                    self._graphs[key] = g
                g.replay()
            else:
                self._step_body()
            self.step_index += 1
            self.ctx += 1
        # the step at position p logged its token at row p
        return self._token_log[first:first + steps].clone()
