"""The Python entry points raise the reference's ValueErrors before touching a GPU."""

import pytest
import torch

import attention_b200 as spa


def test_decode_requires_cuda():
    q = torch.randn(2, 4, 16)
    k = torch.randn(2, 4, 64, 16)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        spa.paged_decode_attention(q, k, k)


def test_gather_requires_contiguous_selection():
    q = torch.randn(2, 4, 16)
    k = torch.randn(2, 4, 512, 16)
    sel = torch.zeros(4, 2, dtype=torch.int64)[::2]
    with pytest.raises(ValueError, match="selected_blocks must be contiguous"):
        spa.paged_gather_decode_attention(q, k, k, sel, local_window=256, block_size=128)


def test_gather_requires_cuda():
    q = torch.randn(2, 4, 16)
    k = torch.randn(2, 4, 512, 16)
    sel = torch.zeros(2, 2, dtype=torch.int64)
    with pytest.raises(ValueError, match="contiguous CUDA tensors are required"):
        spa.paged_gather_decode_attention(q, k, k, sel, local_window=256, block_size=128)


def test_prefill_requires_cuda():
    q = torch.randn(1, 2, 32, 16)
    with pytest.raises(ValueError, match="contiguous CUDA tensors are required"):
        spa.local_causal_prefill(q, q, q, 8)


def test_router_requires_cuda():
    q = torch.randn(1, 2, 16)
    s = torch.randn(1, 2, 5, 16)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        spa.select_blocks(q, s, 2)


def test_decoder_glue_requires_cuda():
    from attention_b200.decoder import add_rms_norm, embed_rms_norm, linear, norm_linear, rms_norm

    x = torch.randn(2, 64)
    w = torch.randn(32, 64)
    nw = torch.ones(64)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        rms_norm(x, nw, 1e-5)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        add_rms_norm(x, x, nw, 1e-5)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        embed_rms_norm(x, torch.zeros(2, dtype=torch.int64), x, torch.zeros(2, dtype=torch.int32), nw, 1e-5,
                       x_out=torch.empty(2, 64))
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        linear(x, w)
    with pytest.raises(ValueError, match="CUDA tensors are required"):
        norm_linear(x, w, norm_weight=nw, eps=1e-5)


def test_decoder_engine_choice_and_limits():
    from attention_b200.decoder import DecoderConfig, SparseDecoder, init_weights, persistent_step_supported

    cfg = DecoderConfig(vocab=64, d_model=64, heads=2, layers=1, max_context=512)
    assert persistent_step_supported(cfg, 1) and persistent_step_supported(cfg, 4)
    assert not persistent_step_supported(cfg, 5)  # batch above 4
    assert not persistent_step_supported(DecoderConfig(d_model=1024, heads=8), 1)  # d_model above 512
    assert not persistent_step_supported(DecoderConfig(d_model=512, heads=2), 1)  # head_dim 256
    w = init_weights(cfg)
    with pytest.raises(ValueError, match="engine must be"):
        SparseDecoder(cfg, w, 1, device="cpu", engine="fast")
    with pytest.raises(ValueError, match="outside the persistent step's limits"):
        SparseDecoder(cfg, w, 5, device="cpu", engine="persistent")


def test_decoder_step_abi_rejects_bad_shapes_without_a_gpu():
    """spa_decoder_step validates its arguments before touching the device; the workspace
    size query answers 0 for a shape it does not take."""
    import ctypes

    from attention_b200 import _lib

    p = _lib.DecoderStepParams()
    p.dtype, p.batch, p.d_model, p.heads, p.ffn, p.vocab, p.layers = _lib.SPA_BF16, 1, 512, 8, 2048, 4096, 4
    p.local_window, p.top_m, p.n_pages, p.max_pages = 128, 8, 100, 130
    p.kv.page_size = 128
    assert _lib.lib.spa_decoder_step_workspace_size(ctypes.byref(p)) > 0
    assert _lib.lib.spa_decoder_step(ctypes.byref(p), None) == _lib.SPA_ERR_INVALID  # no pointers
    for field, value, code in (("batch", 5, _lib.SPA_ERR_UNSUPPORTED), ("batch", 0, _lib.SPA_ERR_INVALID),
                               ("heads", 2, _lib.SPA_ERR_UNSUPPORTED), ("d_model", 1024, _lib.SPA_ERR_UNSUPPORTED),
                               ("n_pages", 131, _lib.SPA_ERR_UNSUPPORTED), ("top_m", 33, _lib.SPA_ERR_UNSUPPORTED),
                               ("vocab", 4090, _lib.SPA_ERR_UNSUPPORTED), ("layers", 9, _lib.SPA_ERR_UNSUPPORTED)):
        old = getattr(p, field)
        setattr(p, field, value)
        assert _lib.lib.spa_decoder_step_workspace_size(ctypes.byref(p)) == 0, field
        assert _lib.lib.spa_decoder_step(ctypes.byref(p), None) == code, field
        setattr(p, field, old)
