"""attention_b200: B200-native (sm_100a) sparse paged-attention hot path.

Drop-in replacements for the reference's decode / prefill / router entry points
(divagr18/attention experiments/), running hand-written CUDA from the in-tree
``libspa_b200.so`` through its C ABI (include/spa_b200.h).
"""

from ._lib import LIB_PATH, SpaError, device_error_flags
from .cache import PagedKVCache, PromotionCache, kv_append
from .gate import RefreshGate
from .paged_attention import paged_decode_attention, paged_gather_decode_attention, span_gather_decode_attention
from .prefill import local_causal_prefill
from .router import page_summaries, periodic_router, select_blocks, select_blocks_tree
from .step import SparseDecodeSession, set_step_fusion, sparse_decode_step

__all__ = [
    "LIB_PATH",
    "SpaError",
    "device_error_flags",
    "PagedKVCache",
    "PromotionCache",
    "RefreshGate",
    "kv_append",
    "paged_decode_attention",
    "paged_gather_decode_attention",
    "span_gather_decode_attention",
    "local_causal_prefill",
    "page_summaries",
    "periodic_router",
    "select_blocks",
    "select_blocks_tree",
    "sparse_decode_step",
    "set_step_fusion",
    "SparseDecodeSession",
]
