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
