"""Causal sliding-window prefill on the GPU against the oracle.

Tolerances: fp32 within 1e-5 absolute; fp16/bf16 within 2e-2 absolute + 1e-2 relative."""

import numpy as np
import pytest
import torch

import attention_b200 as spa
import oracle
from attention_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"


def assert_close(out, ref, dtype):
    atol, rtol = (1e-5, 0.0) if dtype == torch.float32 else (2e-2, 1e-2)
    o, r = out.double().cpu(), ref.double().cpu()
    assert torch.isfinite(o).all()
    err = (o - r).abs()
    assert (err <= atol + rtol * r.abs()).all(), f"max err {err.max().item():.3e}"


@pytest.fixture(autouse=True)
def _no_device_errors():
    yield
    assert spa.device_error_flags() == 0


def test_prefill_golden(golden_dir):
    fx = dict(np.load(golden_dir / "prefill_small.npz"))
    b, h, s, d, w = fx["shape"].tolist()
    torch.manual_seed(int(fx["seed"]))
    q = torch.randn(b, h, s, d)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    out = spa.local_causal_prefill(q.to(DEV), k.to(DEV), v.to(DEV), w)
    assert_close(out, torch.from_numpy(fx["out"]), torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("dim", [64, 128, 32])
@pytest.mark.parametrize("seq,window", [(1, 16), (100, 32), (300, 128), (1000, 256), (2500, 2048), (777, 1)])
def test_prefill_shapes(dtype, dim, seq, window):
    gen = torch.Generator().manual_seed(seq + dim)
    shape = (2, 3, seq, dim)
    q, k, v = ((torch.randn(shape, generator=gen) * 0.5).to(dtype) for _ in range(3))
    out = spa.local_causal_prefill(q.to(DEV), k.to(DEV), v.to(DEV), window)
    ref = oracle.local_reference_chunked(q, k, v, window, chunk=512)
    assert_close(out, ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("halo", [2048, 128, 57])
def test_prefill_with_halo(dtype, halo):
    """A sequence chunk with the previous chunk's last keys equals the full prefill rows."""
    gen = torch.Generator().manual_seed(halo)
    window, start, seq = 2048, 2304, 1536
    shape = (1, 4, start + seq, 128)
    q, k, v = ((torch.randn(shape, generator=gen) * 0.5).to(dtype) for _ in range(3))
    sl = slice(start, start + seq)
    hsl = slice(start - halo, start)
    out = spa.local_causal_prefill(q[:, :, sl].contiguous().to(DEV), k[:, :, sl].contiguous().to(DEV),
                                   v[:, :, sl].contiguous().to(DEV), window,
                                   k_halo=k[:, :, hsl].contiguous().to(DEV), v_halo=v[:, :, hsl].contiguous().to(DEV))
    ref = oracle.local_reference_chunked(q[:, :, sl], k[:, :, sl], v[:, :, sl], window, chunk=512,
                                         k_halo=k[:, :, hsl], v_halo=v[:, :, hsl])
    assert_close(out, ref, dtype)
    if halo >= window - 1:
        full = oracle.local_reference_chunked(q, k, v, window, chunk=512)[:, :, sl]
        assert_close(out, full, dtype)


@pytest.mark.parametrize("seq", [4096, 16384, 32768, 131072, 262144])
def test_prefill_benchmark_shapes_sampled_rows(seq):
    """The benchmark's prefill shapes: batch 1, 32 heads, head_dim 128, bf16, window 2048,
    S = 4k .. 256k.  Row blocks at the sequence start, around the window boundary, at a
    128-row tile boundary in the middle, and the last rows of the sequence (the last work
    items of the persistent scheduler: the last tile pairs of the last head) are compared
    on every head with the chunked local_reference (fp64), within the bf16 tolerance."""
    window, heads, dim = 2048, 32, 128
    wl = workloads.local_prefill_workload(seq, heads=heads, head_dim=dim, seed=seq % 1000)
    q, k, v = wl["q"], wl["k"], wl["v"]
    out = spa.local_causal_prefill(q, k, v, window)
    mid = (seq // 2) // 128 * 128
    blocks = [(0, 160), (window - 96, window + 96), (mid - 64, mid + 64), (seq - 192, seq)]
    for i0, i1 in blocks:
        h0 = max(0, i0 - window + 1)
        qc = q[:, :, i0:i1].cpu()
        kc, vc = k[:, :, i0:i1].cpu(), v[:, :, i0:i1].cpu()
        kh, vh = (k[:, :, h0:i0].cpu(), v[:, :, h0:i0].cpu()) if i0 > 0 else (None, None)
        ref = oracle.local_reference_chunked(qc, kc, vc, window, chunk=64, k_halo=kh, v_halo=vh)
        got = out[:, :, i0:i1].double().cpu()
        err = (got - ref).abs()
        assert (err <= 2e-2 + 1e-2 * ref.abs()).all(), (seq, i0, err.max().item())
    assert spa.device_error_flags() == 0
