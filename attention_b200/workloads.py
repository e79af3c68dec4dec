"""Seeded synthetic inputs with the shapes of the benchmark configurations.

No dataset is involved anywhere: every tensor is drawn from a seeded generator.

* sparse_decode_128k -- tree-routed gathered sparse decode: batch 4, 32 q heads /
  8 kv heads, head_dim 128, bf16, pages of 256 tokens (512 pages = 131072 tokens),
  256-token local window (the last page), superblocks of 16 pages, top-4
  superblocks, then top-m pages.  K/V/q ~ N(0,1)*0.5; 8 needle pages per
  (sequence, kv head) get K += 2*0.5*q_hat, q_hat the normalised mean of that kv
  head's query heads.  ``groups`` independent batches share one page pool
  through scattered (seeded permutation) page tables.
* dense_decode_32k -- batch 8, 32/8 heads, head_dim 128, bf16, 256 pages of 128
  tokens per sequence scattered through a 4096-page pool.
* local_prefill -- batch 1, 32 heads, head_dim 128, bf16, window 2048.
* cpu_sparse_decode -- batch 1, 8 heads, head_dim 64, fp32, 4096 tokens, seed 0.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class SparseDecodeConfig:
    batch: int = 4
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    page_size: int = 256
    pages_per_seq: int = 512
    local_window: int = 256
    superblock: int = 16
    top_super: int = 4
    top_m: int = 4
    needles: int = 8
    dtype: torch.dtype = torch.bfloat16

    @property
    def context(self) -> int:
        return self.page_size * self.pages_per_seq

    @property
    def routable_pages(self) -> int:
        return (self.context - self.local_window) // self.page_size

    @property
    def n_super(self) -> int:
        return -(-self.routable_pages // self.superblock)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def sparse_decode_workload(cfg: SparseDecodeConfig, *, groups: int = 1, seed: int = 0, device="cuda") -> dict:
    """Page pool + per-group page tables, queries and needle-planted keys.

    Returns k_pool/v_pool [groups*B*pages, Hkv, P, D], page_table [groups, B, pages]
    (int32), query [groups, B, Hq, D], context_lens [B] (int32)."""
    b, hq, hkv, d, p, npg = cfg.batch, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.page_size, cfg.pages_per_seq
    n_pages = groups * b * npg
    g = _gen(device, seed)
    k_pool = torch.randn(n_pages, hkv, p, d, generator=g, device=device, dtype=torch.float32).mul_(0.5)
    k_pool = k_pool.to(cfg.dtype)
    v_pool = torch.randn(n_pages, hkv, p, d, generator=g, device=device, dtype=torch.float32).mul_(0.5)
    v_pool = v_pool.to(cfg.dtype)
    perm = torch.randperm(n_pages, generator=g, device=device).to(torch.int32)
    page_table = perm.view(groups, b, npg).contiguous()
    query = (torch.randn(groups, b, hq, d, generator=g, device=device) * 0.5).to(cfg.dtype)
    # needles: shift every token of 8 historical pages per (group, b, kv head) along q_hat
    qf = query.float().view(groups, b, hkv, hq // hkv, d).mean(3)
    q_hat = qf / qf.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    needle_pages = torch.stack([
        torch.randperm(cfg.routable_pages, generator=g, device=device)[: cfg.needles]
        for _ in range(groups * b * hkv)
    ]).view(groups, b, hkv, cfg.needles)
    phys = torch.gather(page_table.long().unsqueeze(2).expand(groups, b, hkv, npg), 3, needle_pages.long())
    kv_idx = torch.arange(hkv, device=device).view(1, 1, hkv, 1).expand_as(phys)
    shift = (2 * 0.5) * q_hat.unsqueeze(3).expand(groups, b, hkv, cfg.needles, d)
    flat_pages, flat_heads = phys.reshape(-1), kv_idx.reshape(-1)
    k_pool[flat_pages, flat_heads] = (k_pool[flat_pages, flat_heads].float()
                                      + shift.reshape(-1, 1, d)).to(cfg.dtype)
    ctx = torch.full((b,), cfg.context, dtype=torch.int32, device=device)
    return {"k_pool": k_pool, "v_pool": v_pool, "page_table": page_table, "query": query, "context_lens": ctx,
            "needle_pages": needle_pages}


@dataclass
class DenseDecodeConfig:
    batch: int = 8
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    page_size: int = 128
    pages_per_seq: int = 256
    pool_pages: int = 4096
    dtype: torch.dtype = torch.bfloat16

    @property
    def context(self) -> int:
        return self.page_size * self.pages_per_seq


def dense_decode_workload(cfg: DenseDecodeConfig, *, seed: int = 0, device="cuda") -> dict:
    g = _gen(device, seed)
    shape = (cfg.pool_pages, cfg.kv_heads, cfg.page_size, cfg.head_dim)
    k_pool = (torch.randn(shape, generator=g, device=device) * 0.5).to(cfg.dtype)
    v_pool = (torch.randn(shape, generator=g, device=device) * 0.5).to(cfg.dtype)
    perm = torch.randperm(cfg.pool_pages, generator=g, device=device).to(torch.int32)
    table = perm[: cfg.batch * cfg.pages_per_seq].view(cfg.batch, cfg.pages_per_seq).contiguous()
    query = (torch.randn(cfg.batch, cfg.q_heads, cfg.head_dim, generator=g, device=device) * 0.5).to(cfg.dtype)
    ctx = torch.full((cfg.batch,), cfg.context, dtype=torch.int32, device=device)
    return {"k_pool": k_pool, "v_pool": v_pool, "page_table": table, "query": query, "context_lens": ctx}


def local_prefill_workload(seq_len: int, *, batch: int = 1, heads: int = 32, head_dim: int = 128,
                           dtype=torch.bfloat16, seed: int = 0, device="cuda") -> dict:
    g = _gen(device, seed)
    shape = (batch, heads, seq_len, head_dim)
    q = (torch.randn(shape, generator=g, device=device) * 0.5).to(dtype)
    k = (torch.randn(shape, generator=g, device=device) * 0.5).to(dtype)
    v = (torch.randn(shape, generator=g, device=device) * 0.5).to(dtype)
    return {"q": q, "k": k, "v": v}


def cpu_sparse_decode_inputs() -> dict:
    """Configuration 1 inputs: seed 0, draw order K, V, q (CPU, fp32)."""
    torch.manual_seed(0)
    keys = torch.randn(1, 8, 4096, 64)
    values = torch.randn(1, 8, 4096, 64)
    query = torch.randn(1, 8, 64)
    return {"keys": keys, "values": values, "query": query, "page_size": 128, "local_window": 128, "top_m": 4}


def prefill_flops(seq_len: int, window: int, heads: int = 32, head_dim: int = 128, batch: int = 1) -> float:
    """Unmasked (query, key) pairs x 4*D: 4*B*H*D*sum_i min(i+1, W)."""
    w = min(window, seq_len)
    pairs = seq_len * w - w * (w - 1) // 2
    return 4.0 * batch * heads * head_dim * pairs


def sparse_decode_bytes(cfg: SparseDecodeConfig) -> int:
    """Algorithmic HBM bytes of one tree-routed sparse decode step.

    K+V of W + m*P candidate tokens per (b, kv head), the fp32 superblock
    summaries, the fp32 summaries of the top_super*superblock candidate pages,
    the query and the output."""
    es = torch.tensor([], dtype=cfg.dtype).element_size()
    kv = 2 * cfg.batch * cfg.kv_heads * (cfg.local_window + cfg.top_m * cfg.page_size) * cfg.head_dim * es
    sup = cfg.batch * cfg.kv_heads * cfg.n_super * cfg.head_dim * 4
    pages = cfg.batch * cfg.kv_heads * cfg.top_super * cfg.superblock * cfg.head_dim * 4
    qo = 2 * cfg.batch * cfg.q_heads * cfg.head_dim * es
    return kv + sup + pages + qo


def dense_decode_bytes(cfg: DenseDecodeConfig) -> int:
    es = torch.tensor([], dtype=cfg.dtype).element_size()
    kv = 2 * cfg.batch * cfg.kv_heads * cfg.context * cfg.head_dim * es
    return kv + 2 * cfg.batch * cfg.q_heads * cfg.head_dim * es + cfg.batch * cfg.pages_per_seq * 4
