"""ctypes binding of ``libspa_b200.so`` (declared in include/spa_b200.h).

The library is the product path: there is no fallback.  Importing this module
without the built library raises immediately with the command that builds it.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("SPA_B200_LIB", _PKG / "libspa_b200.so"))

SPA_OK, SPA_ERR_INVALID, SPA_ERR_UNSUPPORTED, SPA_ERR_CUDA, SPA_ERR_WORKSPACE, SPA_ERR_TIMEOUT = range(6)
STATUS_NAMES = {
    SPA_ERR_INVALID: "invalid argument",
    SPA_ERR_UNSUPPORTED: "unsupported configuration",
    SPA_ERR_CUDA: "CUDA error",
    SPA_ERR_WORKSPACE: "workspace missing or too small",
    SPA_ERR_TIMEOUT: "bounded device wait gave up",
}
SPA_F32, SPA_F16, SPA_BF16 = 0, 1, 2


class KvLayout(ctypes.Structure):
    """Mirror of ``spa_kv_layout``."""

    _fields_ = [
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("total_rows", ctypes.c_int64),
        ("batch_stride_rows", ctypes.c_int64),
        ("page_stride_rows", ctypes.c_int64),
        ("head_stride_rows", ctypes.c_int64),
        ("page_table", ctypes.c_void_p),
        ("table_stride", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
    ]


_vp, _i, _i64, _d, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double, ctypes.c_size_t
_KV = ctypes.POINTER(KvLayout)

# name -> (restype, argtypes); keep in the order of include/spa_b200.h
class RefreshGateArgs(ctypes.Structure):
    """spa_refresh_gate_args (include/spa_b200.h)."""

    _fields_ = [("mode", ctypes.c_int), ("batch", ctypes.c_int), ("ttl", ctypes.c_int), ("step", ctypes.c_int),
                ("step_dev", ctypes.c_void_p), ("signature", ctypes.c_void_p), ("cached_signature", ctypes.c_void_p),
                ("sig_len", ctypes.c_int), ("state", ctypes.c_void_p), ("cached_state", ctypes.c_void_p),
                ("width", ctypes.c_int), ("w1", ctypes.c_void_p), ("b1", ctypes.c_void_p), ("w2", ctypes.c_void_p),
                ("b2", ctypes.c_void_p), ("hidden", ctypes.c_int), ("threshold", ctypes.c_float),
                ("gate", ctypes.c_void_p), ("score_out", ctypes.c_void_p)]


GATE_TTL, GATE_SIGNATURE, GATE_DRIFT, GATE_LEARNED = 0, 1, 2, 3


SESSION_DIRECT_IN, SESSION_COPY_IN, SESSION_ROUTER_IN_DIRECT_OUT, SESSION_COPY_IN_DIRECT_OUT = 0, 1, 2, 3


class NormPrologue(ctypes.Structure):
    """spa_norm_prologue (include/spa_b200.h)."""

    _fields_ = [("delta", ctypes.c_void_p), ("ids", ctypes.c_void_p), ("id_limit", ctypes.c_int64),
                ("delta_ids", ctypes.c_void_p), ("delta_limit", ctypes.c_int64), ("norm_weight", ctypes.c_void_p),
                ("eps", ctypes.c_double), ("x_out", ctypes.c_void_p)]


class KvAppendEpilogue(ctypes.Structure):
    """spa_kv_append_epilogue (include/spa_b200.h)."""

    _fields_ = [("kv", KvLayout), ("positions", ctypes.c_void_p), ("k_col", ctypes.c_int), ("v_col", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("q_out", ctypes.c_void_p),
                ("q_col", ctypes.c_int), ("q_width", ctypes.c_int)]


class SessionParams(ctypes.Structure):
    """spa_session_params (include/spa_b200.h)."""

    _fields_ = [("dtype", ctypes.c_int), ("batch", ctypes.c_int), ("q_heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("kv", KvLayout),
                ("context_lens", ctypes.c_void_p), ("local_window", ctypes.c_int),
                ("super_summaries", ctypes.c_void_p), ("n_super", ctypes.c_int), ("summaries", ctypes.c_void_p),
                ("n_pages", ctypes.c_int), ("superblock", ctypes.c_int), ("top_super", ctypes.c_int),
                ("top_m", ctypes.c_int), ("router_scale", ctypes.c_double), ("attn_scale", ctypes.c_double),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t), ("gate", ctypes.c_void_p),
                ("promoted", ctypes.c_void_p), ("io_mode", ctypes.c_int), ("query", ctypes.c_void_p * 2),
                ("query_dev", ctypes.c_void_p),
                ("query_bytes", ctypes.c_size_t), ("result_dev", ctypes.c_void_p),
                ("result_sel_offset", ctypes.c_size_t), ("result_bytes", ctypes.c_size_t),
                ("result_host", ctypes.c_void_p * 2)]

DECODER_MAX_LAYERS = 8


class DecoderLayer(ctypes.Structure):
    """spa_decoder_layer (include/spa_b200.h)."""

    _fields_ = [(name, ctypes.c_void_p) for name in ("norm1", "qkv_w", "qkv_b", "out_w", "out_b", "norm2", "fc1_w",
                                                     "fc1_b", "fc2_w", "fc2_b", "k_pool", "v_pool", "summaries")]


class DecoderStepParams(ctypes.Structure):
    """spa_decoder_step_params (include/spa_b200.h)."""

    _fields_ = [("dtype", ctypes.c_int), ("batch", ctypes.c_int), ("d_model", ctypes.c_int), ("heads", ctypes.c_int),
                ("ffn", ctypes.c_int), ("vocab", ctypes.c_int), ("layers", ctypes.c_int),
                ("local_window", ctypes.c_int), ("top_m", ctypes.c_int), ("n_pages", ctypes.c_int),
                ("max_pages", ctypes.c_int), ("eps", ctypes.c_double), ("router_scale", ctypes.c_double),
                ("attn_scale", ctypes.c_double), ("emb", ctypes.c_void_p), ("emb_rows", ctypes.c_int64),
                ("pos_emb", ctypes.c_void_p), ("pos_rows", ctypes.c_int64), ("norm_f", ctypes.c_void_p),
                ("head_w", ctypes.c_void_p), ("layer", DecoderLayer * DECODER_MAX_LAYERS), ("kv", KvLayout),
                ("token", ctypes.c_void_p), ("counters", ctypes.c_void_p), ("logits", ctypes.c_void_p),
                ("token_log", ctypes.c_void_p), ("log_len", ctypes.c_int), ("selected", ctypes.c_void_p),
                ("promo_pages", ctypes.c_void_p), ("promo_last_hit", ctypes.c_void_p),
                ("promo_slots", ctypes.c_int), ("promo_ttl", ctypes.c_int), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_size_t)]


PROTOTYPES = {
    "spa_version": (ctypes.c_char_p, []),
    "spa_device_error": (_i, [ctypes.POINTER(ctypes.c_uint32)]),
    "spa_last_error": (ctypes.c_char_p, []),
    "spa_copy": (_i, [_vp, _vp, _sz, _vp]),
    "spa_host_device_pointer": (_i, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "spa_session_create": (_i, [ctypes.POINTER(SessionParams), ctypes.POINTER(ctypes.c_void_p)]),
    "spa_session_wait": (_i, [_vp, _i]),
    "spa_session_step": (_i, [_vp, _i, _vp]),
    "spa_session_destroy": (_i, [_vp]),
    "spa_debug_wait_timeout": (_i, [ctypes.c_longlong, _vp]),
    "spa_summaries_build": (_i, [_KV, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp, _vp]),
    "spa_router_topm": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _d, _i, _vp, _vp, _vp]),
    "spa_router_tree_topm": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _i, _i, _d, _i, _vp, _vp]),
    "spa_router_topm_gated": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _d, _i, _vp, _vp, _vp, _vp]),
    "spa_router_tree_topm_gated": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _vp, _i, _i, _i, _d, _i, _vp, _vp, _vp,
                                        _vp]),
    "spa_refresh_gate": (_i, [ctypes.POINTER(RefreshGateArgs), _vp]),
    "spa_periodic_router": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _i, _i, _i, _i, _vp, _vp]),
    "spa_decode_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "spa_decode_plan": (_i, [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "spa_paged_decode": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _i, _d, _vp, _vp, _sz, _vp]),
    "spa_paged_gather_decode": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _i, _d, _vp, _vp, _sz, _vp]),
    "spa_span_gather_decode": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _i, _d, _vp, _vp, _sz, _vp]),
    "spa_sparse_decode_step": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _d, _d, _vp,
                                    _vp, _vp, _sz, _vp]),
    "spa_sparse_decode_step_chained": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _d,
                                            _d, _vp, _vp, _vp, _sz, _vp]),
    "spa_sparse_decode_step_host": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i,
                                         _d, _d, _vp, _vp, _vp, _vp, _sz, _vp]),
    "spa_sparse_decode_step_gated": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _vp, _i, _i, _i, _i, _d,
                                          _d, _vp, _vp, _vp, _sz, _vp, _vp, _vp]),
    "spa_sparse_decode_step_heads": (_i, [_vp, _i, _i, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _vp, _i, _i, _i,
                                          _i, _d, _d, _vp, _vp, _vp, _sz, _vp]),
    "spa_sparse_step_launches": (_i, [_i, _i, _i, _i, _i, _i, _i, _i, _i, ctypes.POINTER(_i)]),
    "spa_set_step_fusion": (_i, [_i]),
    "spa_set_prefill_sm_reserve": (_i, [_i]),
    "spa_paged_decode_noalloc": (_i, [_vp, _i, _i, _i, _i, _i, _KV, _vp, _i, _vp, _i, _i, _d, _vp, _vp]),
    "spa_kv_append": (_i, [_KV, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "spa_local_prefill": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "spa_promotion_update": (_i, [_vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _vp]),
    "spa_rms_norm": (_i, [_vp, _vp, _vp, _i, _i, _d, _i, _vp]),
    "spa_add_rms_norm": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _d, _i, _vp]),
    "spa_embed_rms_norm": (_i, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i, _i, _d, _i, _vp]),
    "spa_linear": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "spa_linear_chained": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "spa_argmax_advance": (_i, [_vp, _i, _i, _vp, _vp, _i, _vp]),
    "spa_argmax_advance_log": (_i, [_vp, _i, _i, _vp, _vp, _i, _vp, _vp, _i, _vp]),
    "spa_norm_linear": (_i, [_vp, ctypes.POINTER(NormPrologue), _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                             ctypes.POINTER(KvAppendEpilogue), _vp]),
    "spa_norm_linear_chained": (_i, [_vp, ctypes.POINTER(NormPrologue), _vp, _vp, _vp, _i, _i, _i, _i, _i, _i,
                             ctypes.POINTER(KvAppendEpilogue), _vp]),
    "spa_decoder_step_workspace_size": (_sz, [ctypes.POINTER(DecoderStepParams)]),
    "spa_decoder_step": (_i, [ctypes.POINTER(DecoderStepParams), _vp]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"attention_b200: CUDA library {LIB_PATH} is not built "
            "(run `python attention_b200/build.py`); there is no CPU fallback"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class SpaError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != SPA_OK:
        if rc == SPA_ERR_INVALID:
            raise ValueError(f"{what}: {STATUS_NAMES[rc]}")
        detail = lib.spa_last_error().decode() if rc == SPA_ERR_CUDA else ""
        raise SpaError(f"{what}: {STATUS_NAMES.get(rc, rc)} (status {rc})" + (f": {detail}" if detail else ""))


def device_error_flags() -> int:
    """Reads and clears the library's device error word (synchronises the device)."""
    v = ctypes.c_uint32(0)
    check(lib.spa_device_error(ctypes.byref(v)), "spa_device_error")
    return int(v.value)


def sparse_step_launches(dtype: int, batch: int, q_heads: int, kv_heads: int, head_dim: int, *, kv_head_count: int = 0,
                         local_window: int, page_size: int, top_m: int) -> int:
    """Kernels one sparse decode step of this shape launches (1 fused, else 2 or 3)."""
    n = ctypes.c_int()
    check(lib.spa_sparse_step_launches(dtype, batch, q_heads, kv_heads, head_dim, kv_head_count, local_window,
                                       page_size, top_m, ctypes.byref(n)), "spa_sparse_step_launches")
    return n.value


def decode_plan(batch: int, q_heads: int, kv_heads: int, max_candidates: int) -> tuple[int, bool]:
    """(splits per (sequence, kv head), merged on chip in a cluster) for the decode kernel."""
    ns, cl = _i(0), _i(0)
    check(lib.spa_decode_plan(batch, q_heads, kv_heads, max_candidates, ctypes.byref(ns), ctypes.byref(cl)),
          "spa_decode_plan")
    return int(ns.value), bool(cl.value)


def host_device_pointer(host_ptr: int) -> int:
    """Device address of pinned, mapped host memory at ``host_ptr`` (raises ValueError
    for memory that is not)."""
    d = ctypes.c_void_p()
    check(lib.spa_host_device_pointer(ctypes.c_void_p(host_ptr), ctypes.byref(d)), "spa_host_device_pointer")
    return int(d.value)
