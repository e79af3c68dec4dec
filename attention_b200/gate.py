"""Promotion refresh gate: decide on the device whether a decode step re-routes.

The reference evaluates refresh policies for promotion reuse on the host
(experiments/evaluate_promotion_ttl.py:125-139: fixed TTL, query signature, embedding
drift; experiments/train_refresh_head.py:24-31 and its evaluate(): a learned head).
``RefreshGate`` runs the same decision as one small kernel per step and keeps its state
(the cached state or signature at the last refresh, the promoted selection) in device
memory, so the whole loop can be captured in a CUDA graph.  Pass the gate to
``select_blocks``, ``select_blocks_tree`` or ``sparse_decode_step``: a closed gate makes
the router copy the promoted pages instead of reading any summary.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._util import stream_ptr

_MODES = {"ttl": _lib.GATE_TTL, "signature": _lib.GATE_SIGNATURE, "drift": _lib.GATE_DRIFT,
          "learned": _lib.GATE_LEARNED}


class RefreshGate:
    """Device-side refresh decision for a batch of ``batch`` rows.

    ``mode``: ``"ttl"`` (refresh when ``step % ttl == 0``), ``"signature"`` (refresh when
    the token-id signature ``[batch, sig_len]`` changed), ``"drift"`` (refresh when the
    batch mean of ``1 - cosine_similarity(state, cached_state)`` exceeds ``threshold``) or
    ``"learned"`` (refresh when the batch mean of ``sigmoid(head(state, cached_state))``
    reaches ``threshold``).  ``head`` for the learned mode is the reference's refresh head,
    either a module with ``network = Sequential(Linear(4W, H), GELU(), Linear(H, 1))`` or a
    dict with ``w1 [H, 4W]``, ``b1 [H]``, ``w2 [1, H]``, ``b2 [1]``.  The first step always
    routes."""

    def __init__(self, mode: str, batch: int, *, width: int = 0, sig_len: int = 0, ttl: int = 0,
                 threshold: float = 0.0, head=None, device="cuda"):
        if mode not in _MODES:
            raise ValueError(f"mode must be one of {sorted(_MODES)}")
        if batch <= 0:
            raise ValueError("batch must be positive")
        dev = torch.device(device)
        self.mode, self.batch, self.device = mode, batch, dev
        self.ttl, self.threshold = int(ttl), float(threshold)
        self.flags = torch.zeros(2, dtype=torch.int32, device=dev)  # [decision, promoted]
        self.score = torch.zeros(1, dtype=torch.float32, device=dev)
        self._promoted: torch.Tensor | None = None
        self.width, self.sig_len, self.hidden = int(width), int(sig_len), 0
        self.cached_state = self.cached_signature = None
        self._w = None
        if mode == "ttl" and ttl <= 0:
            raise ValueError("ttl must be positive")
        if mode == "signature":
            if sig_len <= 0:
                raise ValueError("sig_len must be positive")
            self.cached_signature = torch.zeros(batch, sig_len, dtype=torch.int64, device=dev)
        if mode in ("drift", "learned"):
            if width <= 0:
                raise ValueError("width must be positive")
            self.cached_state = torch.zeros(batch, width, dtype=torch.float32, device=dev)
        if mode == "learned":
            if head is None:
                raise ValueError("the learned gate needs a refresh head")
            if isinstance(head, dict):
                w1, b1, w2, b2 = head["w1"], head["b1"], head["w2"], head["b2"]
            else:
                w1, b1 = head.network[0].weight, head.network[0].bias
                w2, b2 = head.network[2].weight, head.network[2].bias
            w1 = w1.detach().to(dev, torch.float32).contiguous()
            if w1.dim() != 2 or w1.size(1) != 4 * width:
                raise ValueError("w1 must be [hidden, 4 * width]")
            self.hidden = w1.size(0)
            self._w = (w1, b1.detach().to(dev, torch.float32).reshape(-1).contiguous(),
                       w2.detach().to(dev, torch.float32).reshape(-1).contiguous(),
                       b2.detach().to(dev, torch.float32).reshape(-1).contiguous())
            if self._w[1].numel() != self.hidden or self._w[2].numel() != self.hidden or self._w[3].numel() != 1:
                raise ValueError("refresh head shapes do not match")

    def promoted_for(self, batch: int, top_m: int) -> torch.Tensor:
        """The device buffer of promoted pages ``[batch, top_m]`` (int64) the gated
        routers read and write."""
        if batch != self.batch:
            raise ValueError("the gate was built for another batch size")
        if self._promoted is None or self._promoted.size(1) != top_m:
            self._promoted = torch.full((batch, top_m), -1, dtype=torch.int64, device=self.device)
            self.flags[1].zero_()
        return self._promoted

    def reset(self) -> None:
        """Forget the promoted selection: the next step routes."""
        self.flags.zero_()

    def decide(self, *, state: torch.Tensor | None = None, signature: torch.Tensor | None = None,
               step=None) -> None:
        """Evaluate the gate for this step (asynchronous, on the current stream).
        ``step`` is an int or a one-element device int32 tensor (graph replay)."""
        a = _lib.RefreshGateArgs()
        a.mode, a.batch = _MODES[self.mode], self.batch
        a.gate = self.flags.data_ptr()
        a.score_out = self.score.data_ptr()
        a.threshold = self.threshold
        keep = []
        if self.mode == "ttl":
            a.ttl = self.ttl
            if isinstance(step, torch.Tensor):
                if step.dtype != torch.int32 or not step.is_cuda or step.numel() != 1:
                    raise ValueError("a device step must be a one-element int32 CUDA tensor")
                a.step_dev = step.data_ptr()
                keep.append(step)
            elif step is None or int(step) < 0:
                raise ValueError("the ttl gate needs a non-negative step")
            else:
                a.step = int(step)
        elif self.mode == "signature":
            if signature is None or signature.shape != (self.batch, self.sig_len):
                raise ValueError("signature must be [batch, sig_len]")
            sig = signature.to(self.device, torch.int64).contiguous()
            keep.append(sig)
            a.signature, a.cached_signature, a.sig_len = sig.data_ptr(), self.cached_signature.data_ptr(), self.sig_len
        else:
            if state is None or state.shape != (self.batch, self.width):
                raise ValueError("state must be [batch, width]")
            st = state.to(self.device, torch.float32).contiguous()
            keep.append(st)
            a.state, a.cached_state, a.width = st.data_ptr(), self.cached_state.data_ptr(), self.width
            if self.mode == "learned":
                w1, b1, w2, b2 = self._w
                a.w1, a.b1, a.w2, a.b2, a.hidden = (w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(),
                                                    self.hidden)
        _lib.check(_lib.lib.spa_refresh_gate(ctypes.byref(a), stream_ptr(self.device)), "spa_refresh_gate")
        self._keep = keep  # inputs stay alive until the next decision

    @property
    def refreshed(self) -> bool:
        """The last decision (synchronises)."""
        return bool(self.flags[0].item())
