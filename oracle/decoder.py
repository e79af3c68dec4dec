"""CPU oracle of the integrated sparse decoder -- TEST INFRASTRUCTURE ONLY.

Same math as attention_b200/decoder.py on contiguous fp32 caches: the tiny decoder
block of train_tiny_transformer.py:134-190 (RMSNorm for LayerNorm), prompt prefill
with full causal attention (local_reference), then per decode step and layer the
reference's routed page decode (select_blocks + make_candidates + reference_attention,
triton_paged_gather_decode_benchmark.py:16-28, with the local window) and the
promotion-table policy (promotion_update).  Parity-unpinned for the promotion table
(the reference keeps no table)."""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from .sparse_paged import gather_decode, local_reference_chunked, promotion_update, select_blocks, summaries_fp64


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


class OracleDecoder:
    def __init__(self, cfg, weights: dict, batch: int):
        self.cfg, self.batch = cfg, batch
        self.w = {k: v.float() for k, v in weights.items()}
        h, dh = cfg.heads, cfg.head_dim
        self.k = [torch.zeros(batch, h, cfg.max_context, dh) for _ in range(cfg.layers)]
        self.v = [torch.zeros(batch, h, cfg.max_context, dh) for _ in range(cfg.layers)]
        self.ctx = 0
        # per layer: fp32 summaries of the completed pages so far (a page's keys never change
        # once it is complete, so each page is summarised once, with summaries_fp64's arithmetic)
        self.summ = [torch.zeros(batch, h, 0, dh) for _ in range(cfg.layers)]
        self.pages = np.full((cfg.layers * batch, cfg.promo_slots), -1, np.int32)
        self.last = np.zeros((cfg.layers * batch, cfg.promo_slots), np.int32)
        self.step_index = 0

    def _lin(self, x, name):
        return F.linear(x, self.w[f"{name}.w"], self.w[f"{name}.b"])

    def _mlp(self, x, i):
        return self._lin(F.gelu(self._lin(_rms(x, self.w[f"l{i}.norm2"], self.cfg.eps), f"l{i}.fc1")), f"l{i}.fc2")

    def prefill(self, tokens: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        b, s = tokens.shape
        h, dh = cfg.heads, cfg.head_dim
        x = self.w["emb"][tokens] + self.w["pos"][torch.arange(s)]
        for i in range(cfg.layers):
            qkv = self._lin(_rms(x, self.w[f"l{i}.norm1"], cfg.eps), f"l{i}.qkv").view(b, s, 3, h, dh)
            q, k, v = qkv.permute(2, 0, 3, 1, 4)
            self.k[i][:, :, :s] = k
            self.v[i][:, :, :s] = v
            att = local_reference_chunked(q, k, v, s, chunk=512).float()
            x = x + self._lin(att.transpose(1, 2).reshape(b, s, cfg.d_model), f"l{i}.out")
            x = x + self._mlp(x, i)
        self.ctx = s
        return F.linear(_rms(x[:, -1], self.w["norm_f"], cfg.eps), self.w["head"])

    def decode_step(self, token: torch.Tensor):
        cfg = self.cfg
        b, h, dh, p, win = self.batch, cfg.heads, cfg.head_dim, cfg.page_size, cfg.local_window
        pos = self.ctx
        x = self.w["emb"][token] + self.w["pos"][pos]
        n = max(0, (pos + 1 - win) // p)
        sels = []
        for i in range(cfg.layers):
            qkv = self._lin(_rms(x, self.w[f"l{i}.norm1"], cfg.eps), f"l{i}.qkv").view(b, 3, h, dh)
            q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
            self.k[i][:, :, pos] = k
            self.v[i][:, :, pos] = v
            m = min(cfg.top_m, n)
            if m > 0:
                have = self.summ[i].size(2)
                if have < n:
                    new_pages, _ = summaries_fp64(self.k[i][:, :, have * p:n * p], p, n - have)
                    self.summ[i] = torch.cat((self.summ[i], new_pages), dim=2)
                sel = select_blocks(q, self.summ[i][:, :, :n], m, scale=1.0 / math.sqrt(dh))
            else:
                sel = torch.full((b, 1), -1, dtype=torch.int64)
            att = gather_decode(q, self.k[i][:, :, : pos + 1], self.v[i][:, :, : pos + 1], sel, local_window=win,
                                block_size=p, context_lens=[pos + 1] * b).float()
            x = x + self._lin(att.reshape(b, cfg.d_model), f"l{i}.out")
            x = x + self._mlp(x, i)
            sels.append(sel)
        sel_all = torch.stack(sels)
        promotion_update(self.pages, self.last, sel_all.reshape(cfg.layers * b, -1).numpy(), self.step_index,
                         cfg.promo_ttl)
        self.step_index += 1
        self.ctx = pos + 1
        return F.linear(_rms(x, self.w["norm_f"], cfg.eps), self.w["head"]), sel_all
