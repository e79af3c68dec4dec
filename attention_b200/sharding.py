"""Multi-GPU plumbing for the path (one process per GPU, torch.distributed).

* Decode needs no exchange: ranks own disjoint batch rows (``shard_rows``) or run
  independent replicas; the router of a row sees all of that row's heads on one
  rank, so selections never need a collective.
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


def shard_rows(n: int, world: int, rank: int) -> slice:
    """Contiguous, balanced split of n rows over world ranks."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def _device_compute(q, k, v, out, window, rows, k_halo, v_halo):
    from .prefill import local_causal_prefill

    local_causal_prefill(q, k, v, window, k_halo=k_halo, v_halo=v_halo, out=out, rows=rows)


class PrefillShard:
    """Sequence-parallel causal sliding-window prefill of one contiguous chunk.

    ``compute(q, k, v, out, window, rows, k_halo, v_halo)`` fills ``out`` rows;
    the default runs the sm_100a kernel.  Every rank calls ``forward`` with its
    chunk; ranks exchange halos pairwise (r -> r+1) with one batched send/recv."""

    TILE = 128

    def __init__(self, rank: int, world: int, window: int, *, group=None, compute: Callable | None = None):
        self.rank, self.world, self.window, self.group = rank, world, window, group
        self.halo = window
        self.compute = compute or _device_compute
        self._kh = self._vh = None

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
        if self.rank == 0:
            self.compute(q, k, v, out, self.window, (0, seq), None, None)
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
