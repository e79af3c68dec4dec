"""spa_rms_norm (the integrated decoder's norm in one launch) against a plain PyTorch fp32
reference of the same formula; its fused forms (residual add + norm, embedding lookup +
norm) bit-exact against the separate ops they replace; the few-row linear layer against
a plain PyTorch fp32 reference."""

import pytest
import torch

import attention_b200 as spa
from attention_b200.decoder import add_rms_norm, argmax_advance, embed_rms_norm, linear, norm_linear, rms_norm

pytestmark = pytest.mark.gpu


def _ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 512), (3, 7, 128), (5, 1000), (1, 4096)])
def test_rms_norm_matches_fp32_reference(dtype, shape):
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = (torch.randn(shape, device="cuda", generator=g) * 3).to(dtype)
    w = (torch.rand(shape[-1], device="cuda", generator=g) + 0.5).to(dtype)
    y = rms_norm(x, w, 1e-5)
    assert y.dtype == dtype and y.shape == x.shape
    r = _ref(x, w, 1e-5)
    # fp32: 1e-5 absolute + relative; 16-bit: one rounding of the output (2^-8 relative)
    atol, rtol = (1e-5, 1e-5) if dtype == torch.float32 else (1e-3, 8e-3)
    assert ((y.float() - r).abs() <= atol + rtol * r.abs()).all()
    assert spa.device_error_flags() == 0


def test_rms_norm_zero_rows_and_validation():
    x = torch.empty(0, 64, device="cuda")
    w = torch.ones(64, device="cuda")
    assert rms_norm(x, w, 1e-5).shape == (0, 64)
    with pytest.raises(ValueError):
        rms_norm(torch.ones(2, 64), torch.ones(64), 1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 512), (3, 1000), (4, 4096)])
@pytest.mark.parametrize("in_place", [False, True])
def test_add_rms_norm_equals_add_then_norm(dtype, shape, in_place):
    g = torch.Generator(device="cuda").manual_seed(7 * sum(shape))
    x = (torch.randn(shape, device="cuda", generator=g) * 3).to(dtype)
    d = (torch.randn(shape, device="cuda", generator=g) * 2).to(dtype)
    w = (torch.rand(shape[-1], device="cuda", generator=g) + 0.5).to(dtype)
    want_x = x + d
    want = rms_norm(want_x, w, 1e-5)
    x_out = x.clone() if in_place else torch.empty_like(x)
    src = x_out if in_place else x
    y = add_rms_norm(src, d, w, 1e-5, x_out=x_out)
    assert torch.equal(x_out, want_x)
    assert torch.equal(y, want)
    assert spa.device_error_flags() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_embed_rms_norm_equals_lookup_add_norm(dtype):
    g = torch.Generator(device="cuda").manual_seed(3)
    vocab, n_pos, dim, rows = 4096, 300, 512, 5
    table = (torch.randn(vocab, dim, device="cuda", generator=g) * 0.02).to(dtype)
    pos = (torch.randn(n_pos, dim, device="cuda", generator=g) * 0.02).to(dtype)
    w = (torch.rand(dim, device="cuda", generator=g) + 0.5).to(dtype)
    ids = torch.tensor([0, 4095, 17, 17, 2048], dtype=torch.int64, device="cuda")
    positions = torch.tensor([0, 299, 5, 6, 150], dtype=torch.int32, device="cuda")
    x_out = torch.empty(rows, dim, dtype=dtype, device="cuda")
    y = embed_rms_norm(table, ids, pos, positions, w, 1e-5, x_out=x_out)
    want_x = table.index_select(0, ids) + pos.index_select(0, positions.long())
    assert torch.equal(x_out, want_x)
    assert torch.equal(y, rms_norm(want_x, w, 1e-5))
    assert spa.device_error_flags() == 0


def test_embed_rms_norm_out_of_range_id_is_flagged():
    """The kernel's own bounds check: an id past its table gives a zero row and device
    error bit 4; the other rows are unaffected."""
    dim = 64
    table = torch.randn(10, dim, device="cuda")
    pos = torch.randn(4, dim, device="cuda")
    w = torch.ones(dim, device="cuda")
    ids = torch.tensor([3, 10], dtype=torch.int64, device="cuda")
    positions = torch.tensor([1, 2], dtype=torch.int32, device="cuda")
    x_out = torch.full((2, dim), 7.0, device="cuda")
    y = embed_rms_norm(table, ids, pos, positions, w, 1e-5, x_out=x_out)
    assert spa.device_error_flags() == 4
    assert torch.equal(x_out[1], torch.zeros(dim, device="cuda")) and torch.equal(y[1], torch.zeros(dim, device="cuda"))
    assert torch.equal(x_out[0], table[3] + pos[1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,k,n", [(1, 512, 1536), (2, 2048, 512), (4, 512, 4096), (3, 100, 37), (1, 4104, 24)])
@pytest.mark.parametrize("gelu", [False, True])
def test_linear_rows_matches_fp32_reference(dtype, rows, k, n, gelu):
    g = torch.Generator(device="cuda").manual_seed(rows * 131 + k + n)
    x = torch.randn(rows, k, device="cuda", generator=g).to(dtype)
    w = (torch.randn(n, k, device="cuda", generator=g) * k ** -0.5).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    y = linear(x, w, b, gelu=gelu)
    ref = x.float() @ w.float().T + b.float()
    # the kernel rounds the sum to dtype before the activation, as the GEMM's output is
    ref_r = ref.to(dtype).float()
    if gelu:
        ref_r = torch.nn.functional.gelu(ref_r)
    # fp32: summation order only; 16-bit: one or two roundings (2^-8 relative) plus the
    # flip of a rounding when the fp32 sums differ in their last bits
    atol, rtol = (1e-4, 1e-4) if dtype == torch.float32 else (2e-2, 1.6e-2)
    assert y.dtype == dtype and y.shape == (rows, n)
    assert ((y.float() - ref_r).abs() <= atol + rtol * ref_r.abs()).all()
    assert spa.device_error_flags() == 0


def test_linear_fp32_out_holds_rounded_values():
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(2, 512, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, 512, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    out = torch.empty(2, 4096, device="cuda")
    linear(x, w, out=out)
    assert torch.equal(out, linear(x, w).float())
    with pytest.raises(ValueError):
        linear(torch.ones(5, 512, device="cuda", dtype=torch.bfloat16), w)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows", [1, 2, 4])
@pytest.mark.parametrize("with_delta", [False, True])
def test_norm_linear_equals_norm_then_linear(dtype, rows, with_delta):
    """The fused prologue normalises bit-identically to the separate norm kernels, so the
    product equals spa_linear of their output; x_out receives the summed rows."""
    g = torch.Generator(device="cuda").manual_seed(rows + 10 * with_delta)
    k, n = 512, 1536
    x = torch.randn(rows, k, device="cuda", generator=g).to(dtype)
    d = torch.randn(rows, k, device="cuda", generator=g).to(dtype) if with_delta else None
    nw = (torch.rand(k, device="cuda", generator=g) + 0.5).to(dtype)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(dtype)
    b = torch.randn(n, device="cuda", generator=g).to(dtype)
    x_out = torch.empty_like(x)
    y = norm_linear(x, w, b, norm_weight=nw, eps=1e-5, delta=d, x_out=x_out, gelu=True)
    if with_delta:
        ref_x = torch.empty_like(x)
        h = add_rms_norm(x, d, nw, 1e-5, x_out=ref_x)
        assert torch.equal(x_out, ref_x)
    else:
        h = rms_norm(x, nw, 1e-5)
        assert torch.equal(x_out, x)
    assert torch.equal(y, linear(h, w, b, gelu=True))
    logits = torch.empty(rows, n, device="cuda")
    norm_linear(x, w, norm_weight=nw, eps=1e-5, delta=d, out=logits)
    assert torch.equal(logits, linear(h, w).float())
    with pytest.raises(ValueError):
        norm_linear(x, w, b, norm_weight=nw, eps=1e-5, delta=d, x_out=x)
    assert spa.device_error_flags() == 0


def test_norm_linear_embedding_mode():
    g = torch.Generator(device="cuda").manual_seed(5)
    vocab, n_pos, k, n = 4096, 200, 512, 1536
    table = (torch.randn(vocab, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    pos = (torch.randn(n_pos, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    nw = (torch.rand(k, device="cuda", generator=g) + 0.5).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(n, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.tensor([7, 4095], dtype=torch.int64, device="cuda")
    positions = torch.tensor([0, 199], dtype=torch.int32, device="cuda")
    x_out = torch.empty(2, k, dtype=torch.bfloat16, device="cuda")
    y = norm_linear(table, w, b, norm_weight=nw, eps=1e-5, delta=pos, ids=ids, positions=positions, x_out=x_out)
    ref_x = torch.empty_like(x_out)
    h = embed_rms_norm(table, ids, pos, positions, nw, 1e-5, x_out=ref_x)
    assert torch.equal(x_out, ref_x)
    assert torch.equal(y, linear(h, w, b))
    assert spa.device_error_flags() == 0
    bad = torch.tensor([7, 4096], dtype=torch.int64, device="cuda")
    y = norm_linear(table, w, b, norm_weight=nw, eps=1e-5, delta=pos, ids=bad, positions=positions, x_out=x_out)
    assert spa.device_error_flags() == 4
    assert torch.equal(x_out[1], torch.zeros(k, dtype=torch.bfloat16, device="cuda"))
    assert torch.equal(y[1], b)  # a zero row times the weight, plus the bias


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_norm_linear_appends_kv_like_kv_append(dtype):
    """The QKV product's K and V columns stored into the paged pools by the epilogue equal
    spa_kv_append of the same columns; a negative position stores nothing."""
    from attention_b200.cache import kv_append

    g = torch.Generator(device="cuda").manual_seed(21)
    rows, heads, dh, page, max_pages = 3, 4, 32, 16, 6
    d = heads * dh
    x = torch.randn(rows, d, device="cuda", generator=g).to(dtype)
    delta = torch.randn(rows, d, device="cuda", generator=g).to(dtype)
    nw = (torch.rand(d, device="cuda", generator=g) + 0.5).to(dtype)
    w = (torch.randn(3 * d, d, device="cuda", generator=g) * 0.05).to(dtype)
    b = torch.randn(3 * d, device="cuda", generator=g).to(dtype)
    table = torch.randperm(rows * max_pages, generator=torch.Generator().manual_seed(2)).to(torch.int32).view(
        rows, max_pages).cuda()
    pos = torch.tensor([5, 37, -1], dtype=torch.int32, device="cuda")
    k1 = torch.zeros(rows * max_pages, heads, page, dh, dtype=dtype, device="cuda")
    v1, k2, v2 = torch.zeros_like(k1), torch.zeros_like(k1), torch.zeros_like(k1)
    x_out = torch.empty_like(x)
    y = norm_linear(x, w, b, norm_weight=nw, eps=1e-5, delta=delta, x_out=x_out,
                    append=(k1, v1, table, pos, d, 2 * d))
    qkv = y.view(rows, 3, heads, dh)
    kv_append(k2, v2, table, qkv[:, 1].contiguous(), qkv[:, 2].contiguous(), pos)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    assert k1.abs().sum() > 0
    assert torch.equal(y, norm_linear(x, w, b, norm_weight=nw, eps=1e-5, delta=delta))
    assert spa.device_error_flags() == 0


def test_argmax_advance_matches_torch_argmax():
    g = torch.Generator(device="cuda").manual_seed(8)
    logits = torch.randn(4, 4096, device="cuda", generator=g)
    logits[1, 100] = logits[1, 3000] = 50.0  # a tie: the first index wins
    logits[2, 7] = float("nan")              # NaN counts as the largest value
    logits[2, 9] = float("nan")
    logits[3] = 0.0                          # all equal
    token = torch.full((4,), -5, dtype=torch.int64, device="cuda")
    counters = torch.tensor([3, 4, 5, 6, 7], dtype=torch.int32, device="cuda")
    argmax_advance(logits, token, counters)
    assert torch.equal(token, torch.argmax(logits, dim=-1))
    assert token.tolist() == [int(logits[0].argmax()), 100, 7, 0]
    assert counters.tolist() == [4, 5, 6, 7, 8]
    assert spa.device_error_flags() == 0


@pytest.mark.parametrize("cols", [4096, 5000, 37])
def test_argmax_advance_log_matches_torch_argmax(cols):
    """The logged form: one CTA serves every row, reads each row's position before the
    counters (which hold the positions) advance, and writes the token at that position."""
    g = torch.Generator(device="cuda").manual_seed(9)
    logits = torch.randn(4, cols, device="cuda", generator=g)
    logits[1, 3] = logits[1, cols - 1] = 50.0  # a tie: the first index wins
    logits[2, 5] = float("nan")
    logits[3] = 0.0
    token = torch.full((4,), -5, dtype=torch.int64, device="cuda")
    counters = torch.tensor([3, 4, 9, 6, 7, 8, 9, 10, 11], dtype=torch.int32, device="cuda")
    log = torch.full((9, 4), -1, dtype=torch.int64, device="cuda")
    argmax_advance(logits, token, counters, log=log, positions=counters[:4])
    exp = torch.argmax(logits, dim=-1)
    assert torch.equal(token, exp)
    assert token.tolist()[1:] == [3, 5, 0]
    assert counters.tolist() == [4, 5, 10, 7, 8, 9, 10, 11, 12]
    want = torch.full((9, 4), -1, dtype=torch.int64)
    for r, p in enumerate([3, 4, 9, 6]):
        if p < 9:  # position 9 lies outside the log: not stored
            want[p, r] = exp[r]
    assert torch.equal(log.cpu(), want)
    assert spa.device_error_flags() == 0
