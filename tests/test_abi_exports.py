"""The C-ABI library loads and exports every function include/spa_b200.h declares (no GPU needed)."""

import ctypes
import re

from conftest import ROOT


def _declared():
    text = (ROOT / "include" / "spa_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(spa_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for required in ("spa_paged_decode", "spa_router_topm", "spa_router_tree_topm", "spa_summaries_build",
                     "spa_kv_append", "spa_local_prefill", "spa_promotion_update"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from attention_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding types every declared entry point
    assert sorted(_lib.PROTOTYPES) == _declared()


def test_version_string():
    from attention_b200 import _lib

    assert b"sm_100a" in _lib.lib.spa_version()


def test_invalid_arguments_rejected_without_gpu():
    """Argument checks run before any CUDA call, so they work on a CPU-only host."""
    from attention_b200 import _lib

    assert _lib.lib.spa_paged_decode(None, 2, 1, 1, 1, 64, None, None, 0, None, 0, 0, 1.0, None, None, 0,
                                     None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_promotion_update(None, None, 1, 64, None, 8, 0, None, 32, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_local_prefill(None, None, None, 2, 1, 1, 1, 64, 1, None, None, 0, 0, 0, None,
                                      None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_decode_workspace_size(0, 1, 1, 64, 10) == 0
    # the gather form requires a selection
    assert _lib.lib.spa_paged_gather_decode(None, 2, 1, 1, 1, 64, None, None, 0, None, 4, 0, 1.0, None, None, 0,
                                            None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_rms_norm(None, None, None, 2, 0, 1e-5, 2, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_add_rms_norm(None, None, None, None, None, 2, 64, 1e-5, 2, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_add_rms_norm(None, None, None, None, None, 0, 64, 1e-5, 2, None) == _lib.SPA_OK
    assert _lib.lib.spa_embed_rms_norm(None, 16, None, None, 16, None, None, None, None, 2, 64, 1e-5, 2,
                                       None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_embed_rms_norm(None, 0, None, None, 0, None, None, None, None, 0, 64, 1e-5, 2,
                                       None) == _lib.SPA_OK
    assert _lib.lib.spa_linear(None, None, None, None, 5, 64, 64, 0, 0, 2, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_linear(None, None, None, None, 1, 64, 64, 2, 0, 2, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_linear(None, None, None, None, 1, 64, 64, 0, 0, 2, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_linear(None, None, None, None, 0, 64, 64, 0, 0, 2, None) == _lib.SPA_OK
    assert _lib.lib.spa_argmax_advance(None, 2, 16, None, None, 0, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_argmax_advance(None, 2, 16, None, None, 3, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_norm_linear(None, None, None, None, None, 1, 64, 64, 0, 0, 2, None,
                                    None) == _lib.SPA_ERR_INVALID
    pro = _lib.NormPrologue()  # no norm weight
    assert _lib.lib.spa_norm_linear(None, ctypes.byref(pro), None, None, None, 1, 64, 64, 0, 0, 2, None,
                                    None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_copy(None, None, 16, None) == _lib.SPA_ERR_INVALID
    assert _lib.lib.spa_session_create(None, None) == _lib.SPA_ERR_INVALID
