"""Benchmark: 128k tree-routed sparse paged decode (+ local prefill) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the tree-routed sparse decode configuration -- batch 4,
32 query / 8 kv heads, head_dim 128, bf16, 131072-token contexts in pages of 256,
256-token local window, superblocks of 16 pages, top-4 superblocks, top-m pages
(m=4 by default) -- one two-level router launch plus one fused page-gather
split-K decode over the selected pages, for one batch.  Consecutive steps cycle
through `--groups` independent batches (different sequences and queries) stored
in one page pool, so the pages a step reads were last touched ~groups steps ago
and the re-read footprint (groups x ~22.6 MB) exceeds the 126 MB L2.

`value` is aggregate algorithmic HBM GB/s (bytes of one step x steps x ranks /
max-over-ranks device time); `us_per_step` is the per-step latency.  Multi-GPU
runs are weak-scaled replicas (each rank decodes its own batches; decode needs
no collective).  A `prefill` object reports the 128k causal sliding-window
prefill (window 2048, 32 heads, head_dim 128, bf16) in TFLOP/s; with N > 1 the
sequence is split in contiguous chunks and each rank receives a 2048-token K/V
halo from the previous rank over NCCL.

`--impl reference` times the reference's PyTorch path restated for the CPU
(router einsum/mean/top-k, candidate assembly, dense attention) on the host
cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "128k sparse decode µs/step & HBM GB/s; local prefill TFLOP/s @1/2/4/8 GPU"


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(PEAKS_FALLBACK), "fallback"


def read_profile_traffic(name: str):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock, power draw and clocks-event reasons of one GPU through NVML (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clocks_setting",
    }

    def __init__(self, index: int, period_s: float = 0.02):
        self.samples: list[tuple[int, int, int | None]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._nv = None
        self._period = period_s
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nv
        mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
        try:
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
        except Exception:
            reasons = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
        try:
            mw = nv.nvmlDeviceGetPowerUsage(self._h)
        except Exception:
            mw = None
        self.samples.append((mhz, reasons, mw))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self._stop.wait(self._period)

    def __enter__(self):
        if self._ok:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._ok:
            self._thread.join(timeout=2)
            if not self.samples:
                try:
                    self._sample()
                except Exception:
                    pass

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [m for m, _, _ in self.samples]
        watts = [w / 1000.0 for _, _, w in self.samples if w is not None]
        mask = 0
        for _, r, _ in self.samples:
            mask |= r
        names = [n for bit, n in self.REASONS.items() if mask & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples),
                "power_w": round(statistics.median(watts), 1) if watts else None}


# ------------------------------------------------------------------ distributed
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ CPU path of the reference
def cpu_reference_step(q, k_c, v_c, supers, summaries, cfg):
    """The reference's decode step restated for the CPU in its own ops: router
    einsum -> mean over heads -> top-k at two levels (select_blocks,
    triton_paged_gather_decode_benchmark.py:16-17), candidate assembly
    (make_candidates, :20-28) and dense softmax attention
    (reference_attention, triton_paged_attention.py:227-231), GQA-expanded."""
    b, hq, d = q.shape
    hkv = k_c.size(1)
    group = hq // hkv
    qf = q.float()
    qg = qf.view(b, hkv, group, d).sum(2)
    s1 = torch.einsum("bkd,bksd->bs", qg, supers) / hq
    top_s = torch.sort(s1, dim=1, descending=True, stable=True).indices[:, : cfg.top_super]
    pages = (top_s.unsqueeze(-1) * cfg.superblock + torch.arange(cfg.superblock)).flatten(1)
    pages = pages.clamp_max(cfg.routable_pages - 1)
    cand = summaries[torch.arange(b)[:, None, None], torch.arange(hkv)[None, :, None], pages[:, None, :]]
    s2 = torch.einsum("bkd,bkpd->bp", qg, cand) / hq
    order = torch.sort(s2, dim=1, descending=True, stable=True).indices[:, : cfg.top_m]
    sel = torch.gather(pages, 1, order)
    hist = cfg.context - cfg.local_window
    pk = k_c[:, :, :hist].view(b, hkv, hist // cfg.page_size, cfg.page_size, d).permute(0, 2, 1, 3, 4)
    pv = v_c[:, :, :hist].view(b, hkv, hist // cfg.page_size, cfg.page_size, d).permute(0, 2, 1, 3, 4)
    bi = torch.arange(b).unsqueeze(1)
    ck = torch.cat((k_c[:, :, hist:], pk[bi, sel].permute(0, 2, 1, 3, 4).flatten(2, 3)), dim=2).float()
    cv = torch.cat((v_c[:, :, hist:], pv[bi, sel].permute(0, 2, 1, 3, 4).flatten(2, 3)), dim=2).float()
    ck = ck.repeat_interleave(group, dim=1)
    cv = cv.repeat_interleave(group, dim=1)
    scores = torch.einsum("bhd,bhld->bhl", qf, ck) * d ** -0.5
    out = torch.einsum("bhl,bhld->bhd", scores.softmax(-1), cv)
    return sel, out.to(q.dtype)


def cpu_inputs_from_pool(wl, group: int, cfg):
    """Contiguous CPU copies [B, Hkv, L, D] of one group's sequences (plus its fp32 summaries)."""
    table = wl["page_table"][group].long()
    b, npg = table.shape
    k = wl["k_pool"][table.reshape(-1)].view(b, npg, cfg.kv_heads, cfg.page_size, cfg.head_dim)
    v = wl["v_pool"][table.reshape(-1)].view(b, npg, cfg.kv_heads, cfg.page_size, cfg.head_dim)
    k = k.permute(0, 2, 1, 3, 4).reshape(b, cfg.kv_heads, npg * cfg.page_size, cfg.head_dim).cpu()
    v = v.permute(0, 2, 1, 3, 4).reshape(b, cfg.kv_heads, npg * cfg.page_size, cfg.head_dim).cpu()
    return wl["query"][group].cpu(), k, v


def cpu_summaries(k_c, cfg):
    b, hkv, _, d = k_c.shape
    n = cfg.routable_pages
    summ = k_c[:, :, : n * cfg.page_size].float().view(b, hkv, n, cfg.page_size, d).mean(3)
    nsup = cfg.n_super
    pad = nsup * cfg.superblock - n
    sums = summ * cfg.page_size
    sums = torch.cat((sums, torch.zeros(b, hkv, pad, d)), dim=2).view(b, hkv, nsup, cfg.superblock, d).sum(3)
    counts = torch.full((nsup,), float(cfg.superblock * cfg.page_size))
    counts[-1] = (n - (nsup - 1) * cfg.superblock) * cfg.page_size
    return sums / counts.view(1, 1, nsup, 1), summ


def time_cpu_steps(q, k_c, v_c, sup, summ, cfg, *, steps: int, budget_s: float):
    cpu_reference_step(q, k_c, v_c, sup, summ, cfg)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    for _ in range(steps):
        t0 = time.perf_counter()
        cpu_reference_step(q, k_c, v_c, sup, summ, cfg)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    return statistics.mean(times), len(times)


# ------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    import attention_b200 as spa
    from attention_b200 import workloads

    dev = torch.device("cuda", local)
    peaks, peaks_src = load_peaks()
    cfg = workloads.SparseDecodeConfig(top_m=args.top_m)
    groups = args.groups
    wl = workloads.sparse_decode_workload(cfg, groups=groups, seed=1000 + rank, device=dev)
    k_pool, v_pool, ctx = wl["k_pool"], wl["v_pool"], wl["context_lens"]
    sup, summ = [], []
    for g in range(groups):
        s, u = spa.page_summaries(k_pool, block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                  page_table=wl["page_table"][g], superblock=cfg.superblock)
        summ.append(s)
        sup.append(u)
    scale = cfg.head_dim ** -0.5
    out_buf = [torch.empty_like(wl["query"][g]) for g in range(groups)]
    sel_buf = [torch.empty(cfg.batch, cfg.top_m, dtype=torch.int64, device=dev) for _ in range(groups)]

    def step(g):
        spa.sparse_decode_step(wl["query"][g], k_pool, v_pool, summ[g], super_summaries=sup[g],
                               superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
                               local_window=cfg.local_window, block_size=cfg.page_size, router_scale=scale,
                               page_table=wl["page_table"][g], context_lens=ctx, out=out_buf[g],
                               selected=sel_buf[g])

    def attention_only(g, sel):
        spa.paged_gather_decode_attention(wl["query"][g], k_pool, v_pool, sel, local_window=cfg.local_window,
                                          block_size=cfg.page_size, page_table=wl["page_table"][g],
                                          context_lens=ctx)

    warm = max(args.warmup, 3)
    for i in range(max(warm, groups)):
        step(i % groups)
    torch.cuda.synchronize()
    fixed_sel = [s.clone() for s in sel_buf]
    # capture: one graph per group (one step each) and one graph of all groups
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for g in range(groups):
            step(g)
    torch.cuda.current_stream(dev).wait_stream(stream)
    torch.cuda.synchronize()
    g_all = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_all):
        for g in range(groups):
            step(g)
    g_one = []
    for g in range(groups):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(g)
        g_one.append(gr)
    g_att = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_att):
        for g in range(groups):
            attention_only(g, fixed_sel[g])
    for _ in range(2):
        g_all.replay()
        g_att.replay()
    torch.cuda.synchronize()

    steps = args.steps
    full, rem = divmod(steps, groups)
    bytes_step = workloads.sparse_decode_bytes(cfg)
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks, torch.cuda.nvtx.range("sparse_step"):
        ev0.record()
        for _ in range(full):
            g_all.replay()
        for g in range(rem):
            g_one[g].replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, world)
    us_step = ms_max * 1e3 / steps
    value = bytes_step * steps * world / (ms_max * 1e-3) / 1e9

    # dominant kernel: the fused gather decode (split kernel + split merge), timed alone
    att_reps = max(1, min(200, steps // groups + 1))
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.nvtx.range("decode_roofline"):
        ea.record()
        for _ in range(att_reps):
            g_att.replay()
        eb.record()
        torch.cuda.synchronize()
    att_us = ea.elapsed_time(eb) * 1e3 / (att_reps * groups)
    es = 2
    att_bytes = (2 * cfg.batch * cfg.kv_heads * (cfg.local_window + cfg.top_m * cfg.page_size) * cfg.head_dim * es
                 + 2 * cfg.batch * cfg.q_heads * cfg.head_dim * es)
    att_gbs = att_bytes / (att_us * 1e-6) / 1e9
    hbm_peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    traffic = read_profile_traffic("sparse_decode_128k_attention_ncu.md")

    gated = None
    if not args.skip_gated:
        gated = run_gated(cfg, wl, summ, sup, sel_buf, out_buf, scale, groups, dev, world, att_reps)

    # end to end through the public API: pinned host query in, output + pages out, every step
    e2e = None
    if not args.skip_e2e:
        host_q = [wl["query"][g].cpu().pin_memory() for g in range(groups)]
        host_out = [torch.empty_like(host_q[g]).pin_memory() for g in range(groups)]
        host_sel = [torch.empty(cfg.batch, cfg.top_m, dtype=torch.int64).pin_memory() for g in range(groups)]
        dq = [torch.empty_like(wl["query"][g]) for g in range(groups)]
        e2e_steps = max(1, min(steps, args.e2e_steps))

        def e2e_step(g):
            dq[g].copy_(host_q[g], non_blocking=True)
            out, sel = spa.sparse_decode_step(dq[g], k_pool, v_pool, summ[g], super_summaries=sup[g],
                                              superblock=cfg.superblock, top_super=cfg.top_super,
                                              top_blocks=cfg.top_m, local_window=cfg.local_window,
                                              block_size=cfg.page_size, router_scale=scale,
                                              page_table=wl["page_table"][g], context_lens=ctx)
            host_out[g].copy_(out, non_blocking=True)
            host_sel[g].copy_(sel, non_blocking=True)

        def timed(fn):
            for i in range(3):
                fn(i % groups)
            torch.cuda.synchronize()
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(e2e_steps):
                fn(i % groups)
            e1.record()
            torch.cuda.synchronize()
            barrier(world)
            return max_over_ranks(e0.elapsed_time(e1), world)

        # the per-call API: three copies and one library call per step from Python
        call_ms = timed(e2e_step)
        # the prepared session: the same copies and step captured once, one replay per step
        sessions = [spa.SparseDecodeSession(k_pool, v_pool, summ[g], q_heads=cfg.q_heads, super_summaries=sup[g],
                                            superblock=cfg.superblock, top_super=cfg.top_super,
                                            top_blocks=cfg.top_m, local_window=cfg.local_window,
                                            block_size=cfg.page_size, router_scale=scale,
                                            page_table=wl["page_table"][g], context_lens=ctx)
                    for g in range(groups)]
        for g in range(groups):  # each group's query staged once in its session's pinned buffers
            for hq in sessions[g].host_query:
                hq.copy_(host_q[g])
        e_ms = timed(lambda g: sessions[g].step())
        qbytes = host_q[0].numel() * host_q[0].element_size()
        e2e = {"value": round(bytes_step * e2e_steps * world / (e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
               "us_per_step": round(e_ms * 1e3 / e2e_steps, 3), "steps": e2e_steps,
               "h2d_bytes_per_step": qbytes,
               "d2h_bytes_per_step": qbytes + cfg.batch * cfg.top_m * 8,
               "path": "attention_b200.SparseDecodeSession.step: one call into the native session (C ABI "
                       "spa_session_step): the fused step, whose kernels read the query from pinned host memory "
                       "over PCIe, and a copy kernel (spa_copy) writing output + page ids into pinned host "
                       "memory; one synchronisation at the end",
               "per_call_api": {"us_per_step": round(call_ms * 1e3 / e2e_steps, 3),
                                "value": round(bytes_step * e2e_steps * world / (call_ms * 1e-3) / 1e9, 2),
                                "path": "attention_b200.sparse_decode_step from Python with the same copies"}}
        del sessions

    # CPU baseline: the reference's path on the host cores, rank 0 at N=1
    cpu = None
    if world == 1 and not args.skip_cpu:
        q_c, k_c, v_c = cpu_inputs_from_pool(wl, 0, cfg)
        sup_c, summ_c = cpu_summaries(k_c, cfg)
        t, n = time_cpu_steps(q_c, k_c, v_c, sup_c, summ_c, cfg, steps=1000, budget_s=args.cpu_budget)
        cpu = {"value": round(bytes_step / t / 1e9, 3), "unit": "GB/s", "us_per_step": round(t * 1e6, 1),
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} full steps of the same workload (batch group 0): router + candidate assembly + "
                         "attention in torch CPU ops, wall clock mean"}
        del k_c, v_c

    prefill = None
    if not args.skip_prefill:
        prefill = run_prefill(args, world, rank, dev, peaks)
    integrated = None
    if not args.skip_integrated:
        integrated = run_integrated(args, dev)

    dense = None
    if not args.skip_dense:
        dense = run_dense(args, world, rank, dev, peaks)

    # kernels per step: the router, then the decode (plus a merge kernel when its splits
    # do not merge on chip)
    nsplit, on_chip = spa._lib.decode_plan(cfg.batch, cfg.q_heads, cfg.kv_heads,
                                           cfg.local_window + cfg.top_m * cfg.page_size)
    decode_kernels = "decode_mma_kernel" if (nsplit == 1 or on_chip) else "decode_mma_kernel + decode_combine_kernel"
    launches_per_step = 2 + (0 if (nsplit == 1 or on_chip) else 1)
    result = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(us_step / 1e3, 6),
        "us_per_step": round(us_step, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.5) K/V/q with planted needle pages)",
        "config": {"workload": f"tree-routed sparse decode 128k: B{cfg.batch} Hq{cfg.q_heads}/Hkv{cfg.kv_heads} "
                               f"D{cfg.head_dim} bf16, P{cfg.page_size} x {cfg.pages_per_seq} pages, W{cfg.local_window}, "
                               f"superblock {cfg.superblock} top-{cfg.top_super}, top-m {cfg.top_m}",
                   "batch": cfg.batch, "context": cfg.context, "top_m": cfg.top_m, "groups": groups,
                   "bytes_per_step": bytes_step,
                   "l2": f"inputs larger than L2: {groups} rotating batches, {groups * bytes_step / 1e6:.0f} MB "
                         "re-read footprint vs 126 MB L2",
                   "parallelism": f"replicas x{world} (no collective)", "graph": "CUDA graph replay"},
        "roofline": {"bound": "hbm", "kernel": decode_kernels,
                     "split_plan": f"{nsplit} splits per (sequence, kv head)"
                                   + (", merged on chip in a cluster" if on_chip and nsplit > 1 else ""),
                     "achieved": round(att_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(att_gbs / hbm_peak, 4), "traffic": traffic,
                     "peak_source": f"{peaks_src} (MEASURED_PEAKS.json hbm_gbs)" if peaks_src == "measured"
                     else "fallback 6650 GB/s",
                     "algorithmic_bytes_per_launch": att_bytes, "us_per_launch": round(att_us, 3)},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "prefill": prefill,
        "gated_step": gated,
        "dense_decode": dense,
        "integrated_decode": integrated,
        "clocks": clocks.summary(),
        "gpu_launches": steps * launches_per_step,
    }
    if rank == 0:
        print(json.dumps(result))


def run_prefill(args, world, rank, dev, peaks):
    import attention_b200 as spa
    from attention_b200 import sharding, workloads

    seq, window, heads, dim = args.prefill_seq, 2048, 32, 128
    flops = workloads.prefill_flops(seq, window, heads, dim)
    chunk = seq // world
    wl = workloads.local_prefill_workload(seq, heads=heads, head_dim=dim, seed=7, device=dev)
    sl = slice(rank * chunk, (rank + 1) * chunk)
    q, k, v = (wl[n][:, :, sl].contiguous() for n in ("q", "k", "v"))
    del wl
    out = torch.empty_like(q)
    runner = sharding.PrefillShard(rank, world, window) if world > 1 else None

    def run():
        if runner is None:
            spa.local_causal_prefill(q, k, v, window, out=out)
        else:
            runner.forward(q, k, v, out=out)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    reps = args.prefill_reps
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0, period_s=0.005) as clocks, \
            torch.cuda.nvtx.range("prefill"):
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
    # periodic causal router over the same chunk (reference: prefill + router overhead benchmark)
    router_ms = None
    if world == 1:
        for _ in range(2):
            spa.periodic_router(q, k, block_size=256, router_stride=256, top_blocks=4)
        torch.cuda.synchronize()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for _ in range(5):
            spa.periodic_router(q, k, block_size=256, router_stride=256, top_blocks=4)
        r1.record()
        torch.cuda.synchronize()
        router_ms = r0.elapsed_time(r1) / 5
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    tf = flops / (ms * 1e-3) / 1e12
    return {"seq_len": seq, "window": window, "heads": heads, "head_dim": dim, "ms": round(ms, 4),
            "tflops": round(tf, 1), "peak_tflops": peak * world, "frac": round(tf / (peak * world), 4),
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst) x GPUs",
            "traffic_16k": read_profile_traffic("local_prefill_tc_16k_ncu.md"),
            "traffic_source": "profiles/local_prefill_tc_16k_ncu.md (dram read+write of one S=16384 launch)",
            "flops": flops, "clocks": clocks.summary(), "sharding": f"{world} contiguous chunks, 2048-token K/V halo over NCCL" if world > 1
            else "single GPU", "reps": reps,
            "periodic_router_ms": round(router_ms, 4) if router_ms is not None else None,
            "periodic_router": "block 256, stride 256, top-4, summaries included" if router_ms is not None else None}


def run_gated(cfg, wl, summ, sup, sel_buf, out_buf, scale, groups, dev, world, reps):
    """The decode step behind an embedding-drift refresh gate evaluated on the device
    (state = the step's query, B x Hq*D): with the gate closed the router copies the
    promoted pages and reads no summary; with it open every step routes."""
    import attention_b200 as spa

    states = [wl["query"][g].float().reshape(cfg.batch, -1).contiguous() for g in range(groups)]
    result = {}
    # cosine distance lies in [0, 2]: threshold 3 never refreshes after the first step,
    # threshold -1 refreshes every step
    for name, thr in (("reuse", 3.0), ("route", -1.0)):
        gate = spa.RefreshGate("drift", cfg.batch, width=cfg.q_heads * cfg.head_dim, threshold=thr, device=dev)

        def gstep(g):
            gate.decide(state=states[g])
            spa.sparse_decode_step(wl["query"][g], wl["k_pool"], wl["v_pool"], summ[g], super_summaries=sup[g],
                                   superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
                                   local_window=cfg.local_window, block_size=cfg.page_size, router_scale=scale,
                                   page_table=wl["page_table"][g], context_lens=wl["context_lens"],
                                   out=out_buf[g], selected=sel_buf[g], gate=gate)

        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for g in range(groups):
                gstep(g)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for g in range(groups):
                gstep(g)
        graph.replay()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.nvtx.range(f"gated_{name}"):
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
        barrier(world)
        result[f"{name}_us_per_step"] = round(max_over_ranks(e0.elapsed_time(e1), world) * 1e3 / (reps * groups), 3)
        del graph
    result["gate"] = "embedding drift (1 - cosine) of the step's query, one device decision per step"
    result["launches_per_step"] = 3
    return result


def run_dense(args, world, rank, dev, peaks):
    """Dense paged decode at 32k: B8, Hq32/Hkv8, D128, bf16, 256 pages of 128 tokens per
    sequence in a 4096-page pool behind a random page table.  A step appends one token per
    (sequence, kv head) in place (the last position, so the context stays 32k) and attends
    over the whole context; the 2.1 GB pool is far larger than L2."""
    import attention_b200 as spa
    from attention_b200 import workloads

    cfg = workloads.DenseDecodeConfig()
    wl = workloads.dense_decode_workload(cfg, seed=11 + rank, device=dev)
    q, kp, vp, table, lens = (wl[n] for n in ("query", "k_pool", "v_pool", "page_table", "context_lens"))
    g = torch.Generator(device=dev).manual_seed(12 + rank)
    k_new = (torch.randn(cfg.batch, cfg.kv_heads, cfg.head_dim, generator=g, device=dev) * 0.5).to(cfg.dtype)
    v_new = (torch.randn(cfg.batch, cfg.kv_heads, cfg.head_dim, generator=g, device=dev) * 0.5).to(cfg.dtype)
    pos = (lens - 1).contiguous()

    def step():
        spa.kv_append(kp, vp, table, k_new, v_new, pos)
        return spa.paged_decode_attention(q, kp, vp, page_table=table, context_lens=lens)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):  # warm-up on the capture stream: its workspace exists before capture
        for _ in range(3):
            step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    reps = args.dense_steps
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.nvtx.range("dense_decode"):
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
    kv_bytes = 2 * cfg.batch * cfg.kv_heads * cfg.context * cfg.head_dim * 2
    io_bytes = 2 * cfg.batch * cfg.q_heads * cfg.head_dim * 2 + cfg.batch * cfg.pages_per_seq * 4
    append_bytes = 2 * 2 * cfg.batch * cfg.kv_heads * cfg.head_dim * 2
    step_bytes = kv_bytes + io_bytes + append_bytes
    gbs = step_bytes / (ms * 1e-3) / 1e9
    peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    nsplit, on_chip = spa._lib.decode_plan(cfg.batch, cfg.q_heads, cfg.kv_heads, cfg.context)
    del wl, kp, vp, graph
    torch.cuda.empty_cache()
    return {"workload": f"dense paged decode 32k: B{cfg.batch} Hq{cfg.q_heads}/Hkv{cfg.kv_heads} D{cfg.head_dim} "
                        f"bf16, {cfg.pages_per_seq} pages x {cfg.page_size} in a {cfg.pool_pages}-page pool, "
                        "one appended token per step",
            "us_per_step": round(ms * 1e3, 2), "bytes_per_step": step_bytes,
            "value": round(gbs * world, 1), "unit": "GB/s (all GPUs)", "frac": round(gbs / peak, 4),
            "peak": peak, "peak_source": "MEASURED_PEAKS.json hbm_gbs",
            "traffic": read_profile_traffic("dense_decode_32k_ncu.md"),
            "traffic_source": "profiles/dense_decode_32k_ncu.md (dram read+write per decode launch)",
            "kernels": "kv_append_kernel + decode_mma_kernel" + ("" if (nsplit == 1 or on_chip) else " + decode_combine_kernel"),
            "split_plan": f"{nsplit} splits per (sequence, kv head)" + (", merged on chip" if on_chip and nsplit > 1 else ""),
            "steps": reps, "graph": "CUDA graph replay"}


def run_integrated(args, dev):
    """Integrated 4-layer decoder (d_model 512, 8 heads, vocab 4096, bf16): a 16k-token
    prompt prefilled into 128-token pages, then greedy decode steps with router top-8 +
    128-token local window per layer and the 64-slot TTL-32 promotion table."""
    from attention_b200.decoder import DecoderConfig, SparseDecoder, init_weights

    steps = args.integrated_steps
    cfg = DecoderConfig(max_context=16384 + 2 * steps + 8)
    weights = init_weights(cfg, seed=0)
    prompt = torch.randint(0, cfg.vocab, (1, 16384), generator=torch.Generator().manual_seed(0)).to(dev)
    warm = SparseDecoder(cfg, weights, 1, device=dev)  # first-call costs (cuBLAS handles, modules)
    warm.generate(warm.prefill(prompt).argmax(-1), 4)
    del warm
    dec = SparseDecoder(cfg, weights, 1, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    logits = dec.prefill(prompt)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    tok = logits.argmax(-1)
    # untimed pass: captures the step graphs of these positions (one per routable-page
    # count); then the same positions again, timed, as pure graph replays
    dec.generate(tok, steps)
    dec.rewind(dec.prompt_len)
    torch.cuda.synchronize()
    e0.record()
    dec.generate(tok, steps)
    e1.record()
    torch.cuda.synchronize()
    return {"config": "4 layers, d_model 512, 8 heads x 64, vocab 4096, bf16, prompt 16384 in 128-token pages, "
                      "router top-8 + 128-token window, promotion 64 slots TTL 32",
            "prefill_ms": round(prefill_ms, 3), "decode_steps": steps,
            "decode_us_per_step": round(e0.elapsed_time(e1) * 1e3 / steps, 2),
            "mode": "one CUDA-graph replay per step (cuBLAS GEMMs + library kernels), greedy tokens on the "
                    f"device; the first {steps} positions after the prompt, decoded once untimed (graph "
                    "captures) and again timed after a rewind"}


# ------------------------------------------------------------------ reference arm
def run_reference(args, world, rank, local):
    if rank != 0:
        return
    from attention_b200 import workloads

    cfg = workloads.SparseDecodeConfig(top_m=args.top_m)
    if torch.cuda.is_available():
        wl = workloads.sparse_decode_workload(cfg, groups=1, seed=1000, device=torch.device("cuda", local))
        q_c, k_c, v_c = cpu_inputs_from_pool(wl, 0, cfg)
        del wl
        torch.cuda.empty_cache()
    else:
        wl = workloads.sparse_decode_workload(cfg, groups=1, seed=1000, device="cpu")
        q_c, k_c, v_c = cpu_inputs_from_pool(wl, 0, cfg)
    sup_c, summ_c = cpu_summaries(k_c, cfg)
    for _ in range(max(args.warmup, 1)):
        cpu_reference_step(q_c, k_c, v_c, sup_c, summ_c, cfg)
    t, n = time_cpu_steps(q_c, k_c, v_c, sup_c, summ_c, cfg, steps=args.steps, budget_s=args.cpu_budget * 4)
    bytes_step = workloads.sparse_decode_bytes(cfg)
    value = bytes_step / t / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": max(args.warmup, 1), "ms_per_step": round(t * 1e3, 4),
        "us_per_step": round(t * 1e6, 1), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,0.5) K/V/q with planted needle pages)",
        "config": {"workload": f"tree-routed sparse decode 128k: B{cfg.batch} Hq{cfg.q_heads}/Hkv{cfg.kv_heads} "
                               f"D{cfg.head_dim} bf16, P{cfg.page_size}, W{cfg.local_window}, top-m {cfg.top_m}",
                   "batch": cfg.batch, "context": cfg.context, "top_m": cfg.top_m, "bytes_per_step": bytes_step},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{n} full steps (router + candidate assembly + attention), torch CPU ops"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--top-m", type=int, default=4)
    ap.add_argument("--groups", type=int, default=16)
    ap.add_argument("--e2e-steps", type=int, default=2000)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--prefill-seq", type=int, default=131072)
    ap.add_argument("--prefill-reps", type=int, default=20)
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-integrated", action="store_true")
    ap.add_argument("--skip-dense", action="store_true")
    ap.add_argument("--skip-gated", action="store_true")
    ap.add_argument("--dense-steps", type=int, default=200)
    ap.add_argument("--integrated-steps", type=int, default=256)
    args = ap.parse_args()
    world, rank, local = init_dist()
    if world != args.gpus and rank == 0:
        print(f"note: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    try:
        if args.impl == "reference":
            run_reference(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
