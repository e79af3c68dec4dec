"""Promotion refresh gates -- TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Restates the reference's refresh decisions for promotion reuse:
* evaluate_promotion_ttl.py:125-139 -- a step refreshes when nothing is promoted, or
  (ttl) when ``step % ttl == 0``, or (signature) when the last-three-token signature
  differs from the one at the last refresh (``torch.equal`` over the batch), or (drift)
  when the batch mean of ``1 - cosine_similarity(state, state at last refresh)``
  exceeds the threshold; a refresh promotes the fresh selection and caches the state
  and signature;
* train_refresh_head.py:24-31 (``RefreshHead``: Linear(4W, H) -> GELU -> Linear(H, 1)
  over [current, cached, |current - cached|, current * cached]) with the decision of its
  evaluate(): ``sigmoid(head(state, cached)).mean() >= threshold``.
Pinned by tests/golden/refresh_gate.npz (the reference's RefreshHead and drift distance).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def drift_distance(state: torch.Tensor, cached: torch.Tensor) -> torch.Tensor:
    """Per-row ``1 - cosine_similarity`` (evaluate_promotion_ttl.py:130), fp32."""
    return 1.0 - F.cosine_similarity(state.float(), cached.float(), dim=-1)


def refresh_probability(state: torch.Tensor, cached: torch.Tensor, w1, b1, w2, b2) -> torch.Tensor:
    """Per-row ``sigmoid(RefreshHead(state, cached))`` (train_refresh_head.py:24-31), fp32."""
    c, p = state.float(), cached.float()
    features = torch.cat((c, p, (c - p).abs(), c * p), dim=-1)
    hidden = F.gelu(features @ torch.as_tensor(w1).float().T + torch.as_tensor(b1).float())
    logit = hidden @ torch.as_tensor(w2).float().reshape(1, -1).T + torch.as_tensor(b2).float()
    return torch.sigmoid(logit.squeeze(-1))


class GateSim:
    """Step-by-step restatement of the promotion-reuse loop with one refresh policy.

    ``step(fresh, ...)`` takes the router's fresh selection of this step and returns
    ``(used selection, refreshed)``."""

    def __init__(self, mode: str, *, ttl: int = 0, threshold: float = 0.0, head=None):
        self.mode, self.ttl, self.threshold, self.head = mode, ttl, threshold, head
        self.promoted = None
        self.cached_state = None
        self.cached_signature = None
        self.refreshes = 0

    def decide(self, *, step=None, signature=None, state=None) -> bool:
        if self.promoted is None:
            return True
        if self.mode == "ttl":
            return step % self.ttl == 0
        if self.mode == "signature":
            return not torch.equal(signature, self.cached_signature)
        if self.mode == "drift":
            return bool(drift_distance(state, self.cached_state).mean() > self.threshold)
        if self.mode == "learned":
            prob = refresh_probability(state, self.cached_state, *self.head)
            return bool(prob.mean() >= self.threshold)
        raise ValueError(self.mode)

    def step(self, fresh: torch.Tensor, *, step=None, signature=None, state=None):
        refresh = self.decide(step=step, signature=signature, state=state)
        if refresh:
            self.promoted = fresh.clone()
            self.cached_signature = None if signature is None else signature.clone()
            self.cached_state = None if state is None else state.clone()
            self.refreshes += 1
        return self.promoted, refresh
