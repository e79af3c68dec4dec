"""Integrated sparse decoder on the GPU (fp32 run of the same pipeline) against the CPU
oracle decoder: per-step logits within 2e-3 absolute, selected pages and promotion
tables identical, over a prompt and a run of greedy steps that cross page boundaries."""

import numpy as np
import pytest
import torch

import attention_b200 as spa  # noqa: F401  (loads the library)
from attention_b200.decoder import DecoderConfig, SparseDecoder, init_weights
from oracle.decoder import OracleDecoder

pytestmark = pytest.mark.gpu


def test_decoder_matches_oracle_step_by_step():
    cfg = DecoderConfig(vocab=512, d_model=128, heads=4, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=1024 + 160)
    w = init_weights(cfg, seed=3)
    batch = 2
    gen = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, cfg.vocab, (batch, 1024), generator=gen)
    gpu = SparseDecoder(cfg, w, batch, dtype=torch.float32)
    ref = OracleDecoder(cfg, w, batch)
    lg = gpu.prefill(prompt.cuda()).cpu()
    lr = ref.prefill(prompt)
    assert (lg - lr).abs().max().item() < 2e-3
    tok = lr.argmax(-1)
    for step in range(150):
        lg, sg = gpu.decode_step(tok.cuda())
        lr, sr = ref.decode_step(tok)
        assert torch.equal(sg.cpu(), sr), step
        assert (lg.cpu() - lr).abs().max().item() < 2e-3, step
        assert np.array_equal(gpu.promotion.pages.cpu().numpy(), ref.pages), step
        assert np.array_equal(gpu.promotion.last_hit.cpu().numpy(), ref.last), step
        tok = lr.argmax(-1)  # both sides are fed the oracle's greedy token
    assert spa.device_error_flags() == 0


def test_decoder_bf16_runs_full_size_prompt_pages():
    """bf16 at the benchmark's width (d_model 512, 8 heads, vocab 4096) on a shorter prompt:
    finite logits and valid page ids in range for every layer."""
    cfg = DecoderConfig(max_context=4096 + 64)
    w = init_weights(cfg, seed=0)
    dec = SparseDecoder(cfg, w, 1)
    prompt = torch.randint(0, cfg.vocab, (1, 4096), generator=torch.Generator().manual_seed(1)).cuda()
    logits = dec.prefill(prompt)
    tok = logits.argmax(-1)
    for _ in range(8):
        logits, sel = dec.decode_step(tok)
        assert torch.isfinite(logits).all()
        assert ((sel >= 0) & (sel < dec.n_routable)).all()
        tok = logits.argmax(-1)
    assert spa.device_error_flags() == 0


def test_graphed_generation_equals_eager():
    """generate() replays one captured graph per step; it must produce the eager tokens,
    pages and promotion table, across pages becoming routable."""
    cfg = DecoderConfig(vocab=512, d_model=128, heads=4, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=1024 + 300)
    w = init_weights(cfg, seed=5)
    prompt = torch.randint(0, cfg.vocab, (2, 1024), generator=torch.Generator().manual_seed(6)).cuda()
    a = SparseDecoder(cfg, w, 2)
    b = SparseDecoder(cfg, w, 2)
    tok_a = a.prefill(prompt).argmax(-1)
    tok_b = b.prefill(prompt).argmax(-1)
    eager = []
    for _ in range(140):
        logits, _ = a.decode_step(tok_a)
        tok_a = logits.argmax(-1)
        eager.append(tok_a)
    graphed = b.generate(tok_b, 140, graphed=True)
    assert torch.equal(torch.stack(eager), graphed)
    assert torch.equal(a.promotion.pages, b.promotion.pages)
    assert torch.equal(a.promotion.last_hit, b.promotion.last_hit)
    assert len(b._graphs) >= 2  # a page became routable during the run
