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


ENGINES = ("persistent", "kernels")


@pytest.mark.parametrize("engine", ENGINES)
def test_decoder_matches_oracle_step_by_step(engine):
    cfg = DecoderConfig(vocab=512, d_model=128, heads=4, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=1024 + 160)
    w = init_weights(cfg, seed=3)
    batch = 2
    gen = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, cfg.vocab, (batch, 1024), generator=gen)
    gpu = SparseDecoder(cfg, w, batch, dtype=torch.float32, engine=engine)
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


@pytest.mark.parametrize("engine", ENGINES)
def test_decoder_full_size_fp32_matches_oracle_256_steps(engine):
    """The benchmark configuration at full size -- 4 layers, d_model 512, 8 heads x 64,
    vocab 4096, a 16384-token prompt in 128-token pages, router top-8 over the routable
    pages + 128-token window, 64 promoted slots with TTL 32 -- run in fp32 through the
    same kernels and graphs, against the CPU oracle decoder for 256 greedy steps: the
    pages every layer selects and both promotion tables identical at every step, logits
    within 2e-3 absolute.  (In bf16 the step computes in bf16 and its pages are not
    comparable to an fp32 oracle bit for bit; the fp32 instance checks the pipeline.)"""
    steps = 256
    cfg = DecoderConfig(max_context=16384 + steps + 8)
    w = init_weights(cfg, seed=0)
    prompt = torch.randint(0, cfg.vocab, (1, 16384), generator=torch.Generator().manual_seed(0))
    gpu = SparseDecoder(cfg, w, 1, dtype=torch.float32, engine=engine)
    ref = OracleDecoder(cfg, w, 1)
    lg = gpu.prefill(prompt.cuda()).cpu()
    lr = ref.prefill(prompt)
    assert (lg - lr).abs().max().item() < 2e-3
    tok = lr.argmax(-1)
    for step in range(steps):
        lg, sg = gpu.decode_step(tok.cuda())
        lr, sr = ref.decode_step(tok)
        assert torch.equal(sg.cpu(), sr), step
        assert (lg.cpu() - lr).abs().max().item() < 2e-3, step
        assert np.array_equal(gpu.promotion.pages.cpu().numpy(), ref.pages), step
        assert np.array_equal(gpu.promotion.last_hit.cpu().numpy(), ref.last), step
        tok = lr.argmax(-1)
    assert spa.device_error_flags() == 0


@pytest.mark.parametrize("engine", ENGINES)
def test_decoder_bf16_runs_full_size_prompt_pages(engine):
    """bf16 at the benchmark's width (d_model 512, 8 heads, vocab 4096) on a shorter prompt:
    finite logits and valid page ids in range for every layer."""
    cfg = DecoderConfig(max_context=4096 + 64)
    w = init_weights(cfg, seed=0)
    dec = SparseDecoder(cfg, w, 1, engine=engine)
    prompt = torch.randint(0, cfg.vocab, (1, 4096), generator=torch.Generator().manual_seed(1)).cuda()
    logits = dec.prefill(prompt)
    tok = logits.argmax(-1)
    for _ in range(8):
        logits, sel = dec.decode_step(tok)
        assert torch.isfinite(logits).all()
        assert ((sel >= 0) & (sel < dec.n_routable)).all()
        tok = logits.argmax(-1)
    assert spa.device_error_flags() == 0


@pytest.mark.parametrize("engine", ENGINES)
def test_graphed_generation_equals_eager(engine):
    """generate() replays one captured graph per step; it must produce the eager tokens,
    pages and promotion table, across pages becoming routable."""
    cfg = DecoderConfig(vocab=512, d_model=128, heads=4, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=1024 + 300)
    w = init_weights(cfg, seed=5)
    prompt = torch.randint(0, cfg.vocab, (2, 1024), generator=torch.Generator().manual_seed(6)).cuda()
    a = SparseDecoder(cfg, w, 2, engine=engine)
    b = SparseDecoder(cfg, w, 2, engine=engine)
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


@pytest.mark.parametrize("engine", ENGINES)
def test_rewind_replays_cached_graphs_with_current_summaries(engine):
    """After rewind() to the prompt end, generate() replays the graphs captured on the first
    pass (no new captures) and reproduces its tokens: the summaries a replayed graph reads
    are the current ones, not those of the capture."""
    cfg = DecoderConfig(vocab=512, d_model=128, heads=4, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=1024 + 300)
    w = init_weights(cfg, seed=7)
    prompt = torch.randint(0, cfg.vocab, (2, 1024), generator=torch.Generator().manual_seed(8)).cuda()
    dec = SparseDecoder(cfg, w, 2, engine=engine)
    tok = dec.prefill(prompt).argmax(-1)
    first = dec.generate(tok, 280)
    n_graphs = len(dec._graphs)
    assert n_graphs >= 3
    dec.rewind(dec.prompt_len)
    second = dec.generate(tok, 280)
    assert len(dec._graphs) == n_graphs
    assert torch.equal(first, second)


def test_generation_past_max_context_is_rejected():
    cfg = DecoderConfig(vocab=256, d_model=64, heads=2, layers=1, page_size=128, local_window=128, top_m=2,
                        promo_slots=4, promo_ttl=3, max_context=256 + 8)
    dec = SparseDecoder(cfg, init_weights(cfg, seed=1), 1)
    tok = dec.prefill(torch.randint(0, cfg.vocab, (1, 256), generator=torch.Generator().manual_seed(2)).cuda())
    with pytest.raises(ValueError):
        dec.generate(tok.argmax(-1), 9)
    with pytest.raises(ValueError):
        dec.rewind(dec.prompt_len + 1)


@pytest.mark.parametrize("batch", [1, 4])
def test_persistent_step_bf16_as_accurate_as_kernel_chain(batch):
    """The one-launch step against the multi-launch step in bf16 at the benchmark's width
    (d_model 512, 8 heads x 64, vocab 4096), both and the fp32 oracle decoder fed the same
    tokens.  The embedding, norms, linear layers and router are the same arithmetic in both
    engines, so layer 0's pages are identical at every step.  The attention's split
    structure differs (another fp32 summation order before the bf16 rounding), so deeper
    layers may see queries one bf16 bit apart and rank a near-tie the other way, and the
    logits drift apart by bf16 noise.  Required: the one-launch step's largest logit error
    against the fp32 oracle at most 1.25x the chain's (+2e-3), and the deeper layers'
    selected page sets identical to the chain's in at least 90 % of (step, layer, row)
    cases (measured: about 91 % in rank order)."""
    cfg = DecoderConfig(max_context=2048 + 160)
    w = init_weights(cfg, seed=2)
    prompt = torch.randint(0, cfg.vocab, (batch, 2048), generator=torch.Generator().manual_seed(3))
    one = SparseDecoder(cfg, w, batch, engine="persistent")
    chain = SparseDecoder(cfg, w, batch, engine="kernels")
    ref = OracleDecoder(cfg, w, batch)
    one.prefill(prompt.cuda())
    chain.prefill(prompt.cuda())
    tok = ref.prefill(prompt).argmax(-1)
    err_one = err_chain = 0.0
    same = total = 0
    for step in range(140):  # page 16 becomes routable at step 128
        l1, s1 = one.decode_step(tok.cuda())
        l2, s2 = chain.decode_step(tok.cuda())
        lr, _ = ref.decode_step(tok)
        assert torch.equal(s1[0], s2[0]), step
        same += (s1[1:].sort(-1).values == s2[1:].sort(-1).values).all(-1).sum().item()
        total += s1[1:, :, 0].numel()
        err_one = max(err_one, (l1.cpu() - lr).abs().max().item())
        err_chain = max(err_chain, (l2.cpu() - lr).abs().max().item())
        tok = lr.argmax(-1)
    assert err_one <= 1.25 * err_chain + 2e-3, (err_one, err_chain)
    assert same >= 0.90 * total, (same, total)
    assert spa.device_error_flags() == 0


def test_persistent_step_without_routable_pages():
    """A prompt shorter than window + one page: no page is routable, the step attends to the
    window only and reports -1 selections; fp32 against the oracle decoder."""
    cfg = DecoderConfig(vocab=256, d_model=128, heads=2, layers=2, page_size=128, local_window=128, top_m=4,
                        promo_slots=8, promo_ttl=5, max_context=256 + 40)
    w = init_weights(cfg, seed=9)
    prompt = torch.randint(0, cfg.vocab, (2, 128), generator=torch.Generator().manual_seed(10))
    gpu = SparseDecoder(cfg, w, 2, dtype=torch.float32, engine="persistent")
    ref = OracleDecoder(cfg, w, 2)
    lg = gpu.prefill(prompt.cuda()).cpu()
    lr = ref.prefill(prompt)
    tok = lr.argmax(-1)
    for step in range(140):  # the first page becomes routable at position 256
        lg, sg = gpu.decode_step(tok.cuda())
        lr, sr = ref.decode_step(tok)
        assert torch.equal(sg.cpu(), sr), step
        assert (lg.cpu() - lr).abs().max().item() < 2e-3, step
        assert np.array_equal(gpu.promotion.pages.cpu().numpy(), ref.pages), step
        tok = lr.argmax(-1)
    assert spa.device_error_flags() == 0
