"""Multi-GPU plumbing for the path (one process per GPU, torch.distributed).

* Decode shards over (sequence, kv head) pairs (``DecodeShard``): the B x Hkv pairs,
  sequence-major, are cut into equal contiguous ranges, one per rank, each a block of
  whole sequences or a group of kv heads inside one sequence.  A rank holds the K/V
  pages of its pairs only.  The router's score of a page averages over all query
  heads of the sequence, so every rank keeps the query rows and the (small) page
  summaries of its sequences for all heads and computes the selection itself:
  ranks that share a sequence run the same deterministic kernel on the same inputs
  and pick the same pages, with no collective.  The decode then reads only the
  rank's kv heads and their query heads.  Gathering the outputs (``gather``) is
  optional; the step itself exchanges nothing.
* Long-context prefill splits the sequence into contiguous chunks.  Query i of a
  chunk needs the window-1 keys before it, so rank r receives the last
  ``window`` K/V tokens of rank r-1 (the halo, 2 x H x window x D elements per
  sequence) into a local buffer over NCCL (NVLink on B200): peer data lands in
  local HBM and every kernel reads only local memory.  Rows that need no halo
  are computed while the exchange is in flight.
"""

from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from . import _lib


def shard_rows(n: int, world: int, rank: int) -> slice:
    """Contiguous, balanced split of n rows over world ranks."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def decode_shard(batch: int, kv_heads: int, world: int, rank: int) -> tuple[slice, slice]:
    """The (sequence, kv head) pairs of ``rank``: (sequences, kv heads) slices.

    Pairs are numbered sequence-major and split into ``world`` equal contiguous
    ranges; each must be whole sequences or one sequence's kv-head group."""
    pairs = batch * kv_heads
    if world < 1 or pairs % world:
        raise ValueError(f"{batch} x {kv_heads} (sequence, kv head) pairs do not split evenly over {world} ranks")
    per = pairs // world
    p0 = rank * per
    if per >= kv_heads:
        if per % kv_heads:
            raise ValueError(f"{per} pairs per rank is not a whole number of sequences of {kv_heads} kv heads")
        return slice(p0 // kv_heads, (p0 + per) // kv_heads), slice(0, kv_heads)
    if kv_heads % per:
        raise ValueError(f"{per} pairs per rank does not divide {kv_heads} kv heads")
    h0 = p0 % kv_heads
    return slice(p0 // kv_heads, p0 // kv_heads + 1), slice(h0, h0 + per)


class DecodeShard:
    """One rank's (sequence, kv head) block of a decode batch (see the module notes).

    ``rows`` and ``kv`` select the sequences and kv heads; ``q_heads`` the query heads
    of those kv heads (GQA groups are contiguous: q head h reads kv head h // group)."""

    def __init__(self, batch: int, q_heads: int, kv_heads: int, world: int, rank: int, *, group=None):
        if q_heads % kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")
        self.batch, self.n_q_heads, self.n_kv_heads = batch, q_heads, kv_heads
        self.world, self.rank, self.group = world, rank, group
        self.rows, self.kv = decode_shard(batch, kv_heads, world, rank)
        self.q_heads = self._q_slice(self.kv)
        self.full_heads = self.kv.start == 0 and self.kv.stop == kv_heads

    def _q_slice(self, kv: slice) -> slice:
        g = self.n_q_heads // self.n_kv_heads
        return slice(kv.start * g, kv.stop * g)

    def local(self, t: torch.Tensor, heads: str = "q") -> torch.Tensor:
        """The shard's block of a [B, heads, ...] tensor: query heads (``"q"``) or kv heads."""
        return t[self.rows, self.q_heads if heads == "q" else self.kv].contiguous()

    def gather(self, out_local: torch.Tensor) -> torch.Tensor:
        """All ranks' output blocks assembled into [B, Hq, D] (one all_gather)."""
        parts = [torch.empty_like(out_local) for _ in range(self.world)]
        dist.all_gather(parts, out_local.contiguous(), group=self.group)
        full = out_local.new_empty(self.batch, self.n_q_heads, out_local.size(-1))
        for r, part in enumerate(parts):
            rows, kv = decode_shard(self.batch, self.n_kv_heads, self.world, r)
            full[rows, self._q_slice(kv)] = part
        return full


def _device_compute(q, k, v, out, window, rows, k_halo, v_halo):
    from .prefill import local_causal_prefill

    local_causal_prefill(q, k, v, window, k_halo=k_halo, v_halo=v_halo, out=out, rows=rows)


class PrefillShard:
    """Sequence-parallel causal sliding-window prefill of one contiguous chunk.

    ``compute(q, k, v, out, window, rows, k_halo, v_halo)`` fills ``out`` rows;
    the default runs the sm_100a kernel.  Every rank calls ``forward`` with its
    chunk; ranks exchange halos pairwise (r -> r+1) with one batched send/recv."""

    TILE = 128
    # SMs the prefill leaves to the halo exchange's copy kernels while it is in flight
    sm_reserve = 8

    def __init__(self, rank: int, world: int, window: int, *, group=None, compute: Callable | None = None):
        self.rank, self.world, self.window, self.group = rank, world, window, group
        self.halo = window
        self.compute = compute or _device_compute
        self._kh = self._vh = None
        self._side = None

    def halo_free_from(self, seq: int) -> int:
        """First row whose window lies inside the chunk (rounded up to the kernel's tile)."""
        need = self.window - 1
        return min(seq, -(-need // self.TILE) * self.TILE)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, out: torch.Tensor) -> torch.Tensor:
        seq = q.size(2)
        if self.world > 1 and seq < self.halo:
            raise ValueError("each chunk must hold at least `window` tokens")
        ops = []
        if self.rank + 1 < self.world:
            k_tail = k[:, :, seq - self.halo:].contiguous()
            v_tail = v[:, :, seq - self.halo:].contiguous()
            ops += [dist.P2POp(dist.isend, k_tail, self.rank + 1, self.group),
                    dist.P2POp(dist.isend, v_tail, self.rank + 1, self.group)]
        if self.rank > 0:
            shape = (q.size(0), q.size(1), self.halo, q.size(3))
            if self._kh is None or self._kh.shape != shape or self._kh.dtype != k.dtype:
                self._kh = torch.empty(shape, dtype=k.dtype, device=k.device)
                self._vh = torch.empty_like(self._kh)
            ops += [dist.P2POp(dist.irecv, self._kh, self.rank - 1, self.group),
                    dist.P2POp(dist.irecv, self._vh, self.rank - 1, self.group)]
        reqs = dist.batch_isend_irecv(ops) if ops else []
        # while the exchange is in flight the prefill leaves SMs to its copy kernels (they
        # would otherwise wait for the persistent prefill's last CTA)
        reserve = self.sm_reserve if ops and q.is_cuda else 0
        prev = _lib.lib.spa_set_prefill_sm_reserve(reserve) if reserve else None
        if self.rank == 0:
            self.compute(q, k, v, out, self.window, (0, seq), None, None)
            if prev is not None:
                _lib.lib.spa_set_prefill_sm_reserve(prev)
        elif q.is_cuda:
            # The rows that need the halo run on a side stream that waits for the inputs and
            # the halo receive only: their CTAs take the SMs that the interior rows' persistent
            # CTAs leave as those run out of work (one CTA per SM fits), instead of a second
            # launch behind the first one's last wave.  The two launches write disjoint rows.
            split = self.halo_free_from(seq)
            main = torch.cuda.current_stream(q.device)
            if self._side is None:
                self._side = torch.cuda.Stream(device=q.device)
            inputs_ready = torch.cuda.Event()
            inputs_ready.record(main)
            if split < seq:
                self.compute(q, k, v, out, self.window, (split, seq), None, None)
            if prev is not None:
                _lib.lib.spa_set_prefill_sm_reserve(prev)
            with torch.cuda.stream(self._side):
                self._side.wait_event(inputs_ready)
                for r in reqs:
                    r.wait()
                reqs = []
                self.compute(q, k, v, out, self.window, (0, split), self._kh, self._vh)
            main.wait_stream(self._side)
        else:
            split = self.halo_free_from(seq)
            if split < seq:
                self.compute(q, k, v, out, self.window, (split, seq), None, None)
            for r in reqs:
                r.wait()
            reqs = []
            self.compute(q, k, v, out, self.window, (0, split), self._kh, self._vh)
        for r in reqs:
            r.wait()
        return out
