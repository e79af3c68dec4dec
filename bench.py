"""Benchmark: 128k tree-routed sparse paged decode (+ dense decode, local prefill,
integrated decoder) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the tree-routed sparse decode configuration -- batch 4,
32 query / 8 kv heads, head_dim 128, bf16, 131072-token contexts in pages of 256,
256-token local window, superblocks of 16 pages, top-4 superblocks, top-m pages
(m=4 by default) -- the two-level router plus the fused page-gather split-K decode
over the selected pages, for one batch.  Consecutive steps cycle through
`--groups` independent batches (different sequences and queries) stored in one
page pool, so the pages a step reads were last touched ~groups steps ago and the
re-read footprint (groups x ~22.6 MB) exceeds the 126 MB L2.

`value` is aggregate algorithmic HBM GB/s (bytes of one step x steps / max-over-
ranks device time); `us_per_step` is the step latency.  With N > 1 GPUs the same
batch is split over the ranks by (sequence, kv head) pairs (strong scaling: the
total work per step is fixed): each rank holds the K/V pages of its pairs, keeps
its sequences' query rows and page summaries for all heads, routes them itself
and decodes its own kv heads; no collective runs inside a step.  The dense 32k
decode is split the same way, and the 128k prefill in contiguous sequence
chunks with a 2048-token K/V halo from the previous rank over NCCL.

`--impl reference` times the reference's PyTorch path on the host cores (rank 0
only): the oracle's restatement of select_blocks at two levels, make_candidates
and reference_attention, in fp32, on the same configuration.  It never loads the
CUDA library.
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "128k sparse decode µs/step & HBM GB/s; local prefill TFLOP/s @1/2/4/8 GPU"
PREFILL_SEQS = (4096, 16384, 32768, 131072, 262144)


def load_workloads():
    """attention_b200/workloads.py loaded on its own (it needs only torch): importing it
    through the package would load the CUDA library, which the reference arm must not."""
    spec = importlib.util.spec_from_file_location("spa_workloads", ROOT / "attention_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["spa_workloads"] = mod
    spec.loader.exec_module(mod)
    return mod


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


def sparse_config(cfg, groups: int, world: int) -> dict:
    """The `config` object of both arms (identical by construction)."""
    wk = load_workloads()
    bytes_step = wk.sparse_decode_bytes(cfg)
    return {"workload": f"tree-routed sparse decode 128k: B{cfg.batch} Hq{cfg.q_heads}/Hkv{cfg.kv_heads} "
                        f"D{cfg.head_dim} bf16, P{cfg.page_size} x {cfg.pages_per_seq} pages, W{cfg.local_window}, "
                        f"superblock {cfg.superblock} top-{cfg.top_super}, top-m {cfg.top_m}",
            "batch": cfg.batch, "context": cfg.context, "top_m": cfg.top_m, "superblock": cfg.superblock,
            "top_super": cfg.top_super, "groups": groups, "bytes_per_step": bytes_step,
            "l2": f"inputs larger than L2: {groups} rotating batches, {groups * bytes_step / 1e6:.0f} MB "
                  "re-read footprint vs 126 MB L2",
            "parallelism": "single GPU" if world == 1 else
            f"(sequence, kv head) shards x{world}, strong scaling, no collective in the step"}


def time_graph(graph, reps: int, world: int) -> float:
    """ms per replay of ``graph`` (CUDA events, barrier + synchronise around, max over ranks)."""
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / reps, world)


def capture(fn):
    """Warm ``fn`` on a side stream, then capture it once into a CUDA graph."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


# ------------------------------------------------------------------ sparse decode: inputs of this rank
class SparseShardInputs:
    """The rank's share of the rotating 128k batches: its sequences' query rows and
    page summaries for all heads (router inputs), its kv heads' query heads, and a
    compact pool holding only its (sequence, kv head) pages."""

    def __init__(self, spa, wk, cfg, groups, world, rank, dev):
        from attention_b200.sharding import DecodeShard

        self.shard = DecodeShard(cfg.batch, cfg.q_heads, cfg.kv_heads, world, rank)
        rows = self.shard.rows
        wl = wk.sparse_decode_workload(cfg, groups=groups, seed=1000, device=dev)
        self.summ, self.sup = [], []
        for g in range(groups):
            s, u = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                      page_table=wl["page_table"][g], superblock=cfg.superblock)
            self.summ.append(s[rows].contiguous())
            self.sup.append(u[rows].contiguous())
        self.q_rows = [wl["query"][g][rows].contiguous() for g in range(groups)]
        self.q_local = [q[:, self.shard.q_heads].contiguous() for q in self.q_rows]
        if world == 1:
            self.k_pool, self.v_pool, self.table = wl["k_pool"], wl["v_pool"], wl["page_table"]
        else:
            tab = wl["page_table"][:, rows]
            phys = tab.reshape(-1).long()
            self.k_pool = wl["k_pool"][phys][:, self.shard.kv].contiguous()
            self.v_pool = wl["v_pool"][phys][:, self.shard.kv].contiguous()
            self.table = torch.arange(phys.numel(), dtype=torch.int32, device=dev).view(tab.shape).contiguous()
        self.ctx = wl["context_lens"][rows].contiguous()
        self.n_rows = rows.stop - rows.start
        del wl
        torch.cuda.empty_cache()


def make_step(spa, cfg, x: SparseShardInputs, g: int, m: int, out, sel):
    """One sparse step of batch group g for this rank (m selected pages)."""
    scale = cfg.head_dim ** -0.5
    # a kv-head group of one sequence: routed over all of the sequence's heads, decoded over
    # this rank's kv heads (kv_head_range)
    rng = None if x.shard.full_heads else (x.shard.kv.start, x.shard.kv.stop - x.shard.kv.start)

    def step():
        spa.sparse_decode_step(x.q_rows[g], x.k_pool, x.v_pool, x.summ[g], super_summaries=x.sup[g],
                               superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=m,
                               router_scale=scale, out=out, selected=sel, local_window=cfg.local_window,
                               block_size=cfg.page_size, page_table=x.table[g], context_lens=x.ctx,
                               kv_head_range=rng)
    return step


# ------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    import attention_b200 as spa

    wk = load_workloads()
    dev = torch.device("cuda", local)
    peaks, peaks_src = load_peaks()
    hbm_peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    cfg = wk.SparseDecodeConfig(top_m=args.top_m)
    groups = args.groups
    x = SparseShardInputs(spa, wk, cfg, groups, world, rank, dev)
    out_buf = [torch.empty_like(x.q_local[g]) for g in range(groups)]
    sel_buf = {m: [torch.empty(x.n_rows, m, dtype=torch.int64, device=dev) for _ in range(groups)]
               for m in (2, 4, 8)}

    def all_groups(m):
        fns = [make_step(spa, cfg, x, g, m, out_buf[g], sel_buf[m][g]) for g in range(groups)]
        return lambda: [f() for f in fns]

    def one_group(m, g):
        return make_step(spa, cfg, x, g, m, out_buf[g], sel_buf[m][g])

    warm = max(args.warmup, 3)
    m0 = cfg.top_m
    run_all = all_groups(m0)
    for _ in range(warm):
        run_all()
    torch.cuda.synchronize()
    g_all = capture(run_all)
    g_one = [capture(one_group(m0, g)) for g in range(groups)]
    for _ in range(2):
        g_all.replay()
    torch.cuda.synchronize()

    steps = args.steps
    full, rem = divmod(steps, groups)
    bytes_step = wk.sparse_decode_bytes(cfg)
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
    ms_max = max_over_ranks(ev0.elapsed_time(ev1), world)
    us_step = ms_max * 1e3 / steps
    value = bytes_step * steps / (ms_max * 1e-3) / 1e9
    del g_one

    # dominant kernel: the fused gather decode (split kernel + split merge), timed alone, and
    # the step at m = 2, 4, 8
    reps = max(3, min(200, steps // groups + 1))
    es = 2
    local_pairs = x.n_rows * (x.shard.kv.stop - x.shard.kv.start)
    local_q_heads = x.q_local[0].size(1)

    def att_bytes(m):
        return (2 * local_pairs * (cfg.local_window + m * cfg.page_size) * cfg.head_dim * es
                + 2 * x.n_rows * local_q_heads * cfg.head_dim * es)

    per_m = {}
    att_us = {}
    for m in (2, 4, 8):
        if m == m0:
            step_us = us_step
        else:
            gm = capture(all_groups(m))
            step_us = time_graph(gm, reps, world) * 1e3 / groups
            del gm
        fixed = [s.clone() for s in sel_buf[m]]  # this m's selections, for the decode alone
        ga = capture(lambda: [spa.paged_gather_decode_attention(
            x.q_local[g], x.k_pool, x.v_pool, fixed[g], local_window=cfg.local_window, block_size=cfg.page_size,
            page_table=x.table[g], context_lens=x.ctx) for g in range(groups)])
        with torch.cuda.nvtx.range(f"decode_roofline_m{m}"):
            a_us = time_graph(ga, reps, world) * 1e3 / groups
        del ga
        att_us[m] = a_us
        mcfg = wk.SparseDecodeConfig(top_m=m)
        sb = wk.sparse_decode_bytes(mcfg)
        per_m[str(m)] = {"us_per_step": round(step_us, 3), "bytes_per_step": sb,
                         "value": round(sb / (step_us * 1e-6) / 1e9, 1), "unit": "GB/s",
                         "frac": round(sb / (step_us * 1e-6) / 1e9 / hbm_peak, 4),
                         "decode_kernel_us": round(a_us, 3),
                         "decode_kernel_gbs": round(att_bytes(m) / (a_us * 1e-6) / 1e9, 1),
                         "decode_kernel_frac": round(att_bytes(m) / (a_us * 1e-6) / 1e9 / hbm_peak, 4)}
    att_gbs = att_bytes(m0) / (att_us[m0] * 1e-6) / 1e9
    traffic = read_profile_traffic("sparse_decode_128k_attention_ncu.md")

    gated = None
    if world == 1 and not args.skip_gated:
        gated = run_gated(spa, cfg, x, groups, dev, reps)

    e2e = None
    if not args.skip_e2e:
        e2e = run_e2e(spa, cfg, x, groups, world, bytes_step, steps, args)

    cpu = None
    if world == 1 and not args.skip_cpu:
        cpu = run_cpu_baseline(wk, cfg, args.cpu_budget, seed=1000, device=dev)

    prefill = None
    if not args.skip_prefill:
        prefill = run_prefill(args, world, rank, dev, peaks)
    integrated = None
    if world == 1 and not args.skip_integrated:
        integrated = run_integrated(args, dev, hbm_peak)
    dense = None
    if not args.skip_dense:
        dense = run_dense(args, world, rank, dev, peaks)

    # kernels per step as the library dispatches this shape: 1 (routing inside the decode
    # kernel), else the router, the decode and, when its splits do not merge on chip, a merge
    launches_per_step = spa._lib.sparse_step_launches(
        spa._lib.SPA_BF16, x.n_rows, cfg.q_heads, cfg.kv_heads, cfg.head_dim,
        kv_head_count=x.shard.kv.stop - x.shard.kv.start, local_window=cfg.local_window, page_size=cfg.page_size,
        top_m=m0)
    nsplit, on_chip = spa._lib.decode_plan(x.n_rows, local_q_heads, x.shard.kv.stop - x.shard.kv.start,
                                           cfg.local_window + m0 * cfg.page_size)
    merged = nsplit == 1 or on_chip
    decode_kernels = "decode_mma_kernel" if merged else "decode_mma_kernel + decode_combine_kernel"
    peak_src = (f"{peaks_src} (MEASURED_PEAKS.json hbm_gbs)" if peaks_src == "measured" else "fallback 6650 GB/s")
    decode_alone = {"kernel": decode_kernels, "achieved": round(att_gbs, 1), "frac": round(att_gbs / hbm_peak, 4),
                    "algorithmic_bytes_per_launch": att_bytes(m0), "us_per_launch": round(att_us[m0], 3),
                    "traffic": traffic if world == 1 else None,
                    "what": "the gather decode alone over the steps' selections (no routing)"}
    if launches_per_step == 1:
        # the step is one kernel: its algorithmic bytes are the step's (this rank's share at N > 1)
        rank_bytes = bytes_step * local_pairs // (cfg.batch * cfg.kv_heads) if world > 1 else bytes_step
        step_gbs = rank_bytes / (ms_max * 1e-3 / steps) / 1e9
        roofline = {"bound": "hbm", "kernel": "decode_mma_kernel (route instantiation: routing + gather decode)",
                    "split_plan": f"{nsplit if nsplit > 1 else 8} splits per (sequence, kv head), merged on chip in a "
                                  "cluster",
                    "achieved": round(step_gbs, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(step_gbs / hbm_peak, 4),
                    "traffic": read_profile_traffic("sparse_step_128k_fused_ncu.md") if world == 1 else None,
                    "peak_source": peak_src, "algorithmic_bytes_per_launch": rank_bytes,
                    "us_per_launch": round(ms_max * 1e3 / steps, 3),
                    "duration_source": "CUDA events over the timed region / launches (one launch per step)",
                    "per_rank": world > 1, "decode_alone": decode_alone}
    else:
        roofline = {"bound": "hbm", "kernel": decode_kernels,
                    "split_plan": f"{nsplit} splits per (sequence, kv head)"
                                  + (", merged on chip in a cluster" if on_chip and nsplit > 1 else ""),
                    "achieved": round(att_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(att_gbs / hbm_peak, 4), "traffic": traffic if world == 1 else None,
                    "peak_source": peak_src, "algorithmic_bytes_per_launch": att_bytes(m0),
                    "us_per_launch": round(att_us[m0], 3), "per_rank": world > 1}
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
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.5) K/V/q with planted needle pages)",
        "config": sparse_config(cfg, groups, world),
        "roofline": roofline,
        "per_m": per_m,
        "e2e": e2e,
        "cpu_baseline": cpu,
        "prefill": prefill,
        "gated_step": gated,
        "dense_decode": dense,
        "integrated_decode": integrated,
        "clocks": clocks.summary(),
        "gpu_launches": steps * launches_per_step,
        "step_kernels": "decode_mma_kernel (route instantiation: routing + gather decode in one launch)"
                        if launches_per_step == 1 else "router_cluster_kernel + " + decode_kernels,
    }
    if rank == 0:
        print(json.dumps(result))


def run_e2e(spa, cfg, x, groups, world, bytes_step, steps, args):
    """End to end through the public API: each step's query from pinned host memory in,
    output + page ids to pinned host memory out, inside the timed region."""
    e2e_steps = max(1, min(steps, args.e2e_steps))
    host_q = [x.q_rows[g].cpu().pin_memory() for g in range(groups)]
    scale = cfg.head_dim ** -0.5

    def timed(fn, sync_each=False):
        for i in range(max(3, groups)):  # every group once: a serving loop prepares its tensors once
            fn(i % groups)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(e2e_steps):
            fn(i % groups)
            if sync_each:
                torch.cuda.current_stream().synchronize()
        e1.record()
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(e0.elapsed_time(e1), world)

    qbytes = host_q[0].numel() * host_q[0].element_size()
    out_bytes = x.q_local[0].numel() * x.q_local[0].element_size()
    res = {"unit": "GB/s", "steps": e2e_steps, "h2d_bytes_per_step": qbytes,
           "d2h_bytes_per_step": out_bytes + x.n_rows * cfg.top_m * 8}
    if x.shard.full_heads:
        sessions = [spa.SparseDecodeSession(x.k_pool, x.v_pool, x.summ[g], q_heads=cfg.q_heads,
                                            super_summaries=x.sup[g], superblock=cfg.superblock,
                                            top_super=cfg.top_super, top_blocks=cfg.top_m,
                                            local_window=cfg.local_window, block_size=cfg.page_size,
                                            router_scale=scale, page_table=x.table[g], context_lens=x.ctx)
                    for g in range(groups)]
        for g in range(groups):  # each group's query staged once in its session's pinned buffers
            for hq in sessions[g].host_query:
                hq.copy_(host_q[g])
        e_ms = timed(lambda g: sessions[g].step())
        s_ms = timed(lambda g: sessions[g].step(), sync_each=True)
        # the per-call API: one sparse_decode_step call per step from Python with pinned host
        # query, output and page-id buffers (a serving loop's buffers, allocated once)
        host_out = [torch.empty_like(host_q[g]).pin_memory() for g in range(groups)]
        host_sel = [torch.empty(x.n_rows, cfg.top_m, dtype=torch.int64).pin_memory() for g in range(groups)]
        tables = [x.table[g] for g in range(groups)]

        def per_call(g):
            spa.sparse_decode_step(host_q[g], x.k_pool, x.v_pool, x.summ[g], super_summaries=x.sup[g],
                                   superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
                                   local_window=cfg.local_window, block_size=cfg.page_size, router_scale=scale,
                                   page_table=tables[g], context_lens=x.ctx, out=host_out[g], selected=host_sel[g])

        c_ms = timed(per_call)
        # headline: the drop-in call a user of the reference's API makes each step
        res.update(value=round(bytes_step * e2e_steps / (c_ms * 1e-3) / 1e9, 2),
                   us_per_step=round(c_ms * 1e3 / e2e_steps, 3),
                   path="attention_b200.sparse_decode_step called from Python every step with pinned host "
                        "query, output and page-id tensors (spa_sparse_decode_step_host: a copy kernel reads the "
                        "query from host memory, the one-launch step writes output and page ids into host memory; "
                        "prepared arguments cached per pool, table and summaries); the host may run ahead of the "
                        "device",
                   session={"us_per_step": round(e_ms * 1e3 / e2e_steps, 3),
                            "value": round(bytes_step * e2e_steps / (e_ms * 1e-3) / 1e9, 2),
                            "path": "attention_b200.SparseDecodeSession.step: one call into the native session "
                                    "(C ABI spa_session_step) that launches the CUDA graph of its host-buffer "
                                    "slot: a copy kernel brings the step's query from pinned mapped host memory "
                                    "into device memory, the router and the gather decode run, and a copy kernel "
                                    "(spa_copy) writes output + page ids into pinned host memory; the host may "
                                    "enqueue one step ahead (two buffer slots)"},
                   per_step_sync={"us_per_step": round(s_ms * 1e3 / e2e_steps, 3),
                                  "value": round(bytes_step * e2e_steps / (s_ms * 1e-3) / 1e9, 2),
                                  "path": "the session step, followed every step by a host synchronisation "
                                          "before the next step is enqueued (results read on the host each "
                                          "step)"})
        for s in sessions:
            s.close()
        del sessions
    else:
        dq = [torch.empty_like(x.q_rows[g]) for g in range(groups)]
        host_out = [torch.empty(x.q_local[g].shape, dtype=x.q_local[g].dtype).pin_memory() for g in range(groups)]
        host_sel = [torch.empty(x.n_rows, cfg.top_m, dtype=torch.int64).pin_memory() for g in range(groups)]

        def call(g):
            dq[g].copy_(host_q[g], non_blocking=True)
            out, sel = spa.sparse_decode_step(dq[g], x.k_pool, x.v_pool, x.summ[g], super_summaries=x.sup[g],
                                              superblock=cfg.superblock, top_super=cfg.top_super,
                                              top_blocks=cfg.top_m, local_window=cfg.local_window,
                                              block_size=cfg.page_size, router_scale=scale,
                                              page_table=x.table[g], context_lens=x.ctx,
                                              kv_head_range=(x.shard.kv.start, x.shard.kv.stop - x.shard.kv.start))
            host_out[g].copy_(out, non_blocking=True)
            host_sel[g].copy_(sel, non_blocking=True)

        e_ms = timed(call)
        res.update(value=round(bytes_step * e2e_steps / (e_ms * 1e-3) / 1e9, 2),
                   us_per_step=round(e_ms * 1e3 / e2e_steps, 3),
                   path="per call from Python: host->device copy of the sequences' query rows, "
                        "sparse_decode_step over this rank's kv heads (routed over all heads), device->host "
                        "copies of output and page ids")
    return res


def run_cpu_baseline(wk, cfg, budget_s, *, seed, device):
    """The reference's path on the host cores (bounded sample of the same workload)."""
    import oracle

    q_c, k_c, v_c, sup_c, summ_c = reference_inputs(wk, cfg, seed, device)
    t, n = time_reference_steps(oracle, q_c, k_c, v_c, sup_c, summ_c, cfg, steps=1000, budget_s=budget_s)
    bytes_step = wk.sparse_decode_bytes(cfg)
    return {"value": round(bytes_step / t / 1e9, 3), "unit": "GB/s", "us_per_step": round(t * 1e6, 1),
            "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} full steps of batch group 0 of the same workload: oracle.reference_decode_step "
                      "(select_blocks at two levels, make_candidates, reference_attention; fp32 torch CPU "
                      "ops), wall clock mean"}


def reference_inputs(wk, cfg, seed, device):
    """Contiguous CPU copies [B, Hkv, L, D] of batch group 0 and its oracle summaries."""
    import oracle

    wl = wk.sparse_decode_workload(cfg, groups=1, seed=seed, device=device)
    table = wl["page_table"][0].long()
    b, npg = table.shape
    k = wl["k_pool"][table.reshape(-1)].view(b, npg, cfg.kv_heads, cfg.page_size, cfg.head_dim)
    v = wl["v_pool"][table.reshape(-1)].view(b, npg, cfg.kv_heads, cfg.page_size, cfg.head_dim)
    k = k.permute(0, 2, 1, 3, 4).reshape(b, cfg.kv_heads, npg * cfg.page_size, cfg.head_dim).cpu()
    v = v.permute(0, 2, 1, 3, 4).reshape(b, cfg.kv_heads, npg * cfg.page_size, cfg.head_dim).cpu()
    q = wl["query"][0].cpu()
    del wl
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    summ, sums = oracle.summaries_fp64(k, cfg.page_size, cfg.routable_pages)
    sup = oracle.super_summaries(sums, cfg.superblock, cfg.page_size)
    return q, k, v, sup, summ


def time_reference_steps(oracle, q, k_c, v_c, sup, summ, cfg, *, steps: int, budget_s: float):
    def one():
        oracle.reference_decode_step(q, k_c, v_c, sup, summ, superblock=cfg.superblock, top_super=cfg.top_super,
                                     top_blocks=cfg.top_m, local_window=cfg.local_window,
                                     block_size=cfg.page_size)

    one()  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    for _ in range(steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    return statistics.mean(times), len(times)


def run_prefill(args, world, rank, dev, peaks):
    import attention_b200 as spa
    from attention_b200 import sharding

    wk = load_workloads()
    window, heads, dim = 2048, 32, 128
    peak = float(peaks.get("bf16_tflops", PEAKS_FALLBACK["bf16_tflops"]))
    peak_s = float(peaks.get("bf16_tflops_sustained", PEAKS_FALLBACK["bf16_tflops_sustained"]))
    seqs = [args.prefill_seq] if (world > 1 or args.prefill_seq != 131072) else list(PREFILL_SEQS)
    runs = {}
    head = None
    for seq in seqs:
        flops = wk.prefill_flops(seq, window, heads, dim)
        chunk = seq // world
        wl = wk.local_prefill_workload(seq, heads=heads, head_dim=dim, seed=7, device=dev)
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
        reps = max(3, min(args.prefill_reps, int(20 * 131072 / seq)))
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index if dev.index is not None else 0, period_s=0.005) as clocks, \
                torch.cuda.nvtx.range(f"prefill_{seq}"):
            e0.record()
            for _ in range(reps):
                run()
            e1.record()
            torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / reps, world)
        tf = flops / (ms * 1e-3) / 1e12
        runs[str(seq)] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / (peak * world), 4),
                          "frac_sustained": round(tf / (peak_s * world), 4), "flops": flops, "reps": reps,
                          "clocks": clocks.summary()}
        if seq == args.prefill_seq:
            head = (seq, ms, tf, flops, clocks.summary(), reps, q, k)
        del q, k, v, out
        torch.cuda.empty_cache()
    seq, ms, tf, flops, clk, reps, q, k = head
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
    return {"seq_len": seq, "window": window, "heads": heads, "head_dim": dim, "ms": round(ms, 4),
            "tflops": round(tf, 1), "peak_tflops": peak * world, "frac": round(tf / (peak * world), 4),
            "frac_sustained": round(tf / (peak_s * world), 4),
            "peak_source": "MEASURED_PEAKS.json bf16_tflops (burst) and bf16_tflops_sustained, x GPUs",
            "traffic_16k": read_profile_traffic("local_prefill_tc_16k_ncu.md"),
            "traffic_source": "profiles/local_prefill_tc_16k_ncu.md (dram read+write of one S=16384 launch)",
            "flops": flops, "clocks": clk, "reps": reps,
            "sharding": f"{world} contiguous chunks, 2048-token K/V halo over NCCL" if world > 1 else "single GPU",
            "by_seq_len": runs,
            "periodic_router_ms": round(router_ms, 4) if router_ms is not None else None,
            "periodic_router": "block 256, stride 256, top-4, summaries included" if router_ms is not None else None}


def run_gated(spa, cfg, x, groups, dev, reps):
    """The decode step behind an embedding-drift refresh gate evaluated on the device
    (state = the step's query, B x Hq*D): with the gate closed the router copies the
    promoted pages and reads no summary; with it open every step routes."""
    states = [x.q_rows[g].float().reshape(cfg.batch, -1).contiguous() for g in range(groups)]
    out = [torch.empty_like(x.q_rows[g]) for g in range(groups)]
    sel = [torch.empty(cfg.batch, cfg.top_m, dtype=torch.int64, device=dev) for _ in range(groups)]
    result = {}
    # cosine distance lies in [0, 2]: threshold 3 never refreshes after the first step,
    # threshold -1 refreshes every step
    for name, thr in (("reuse", 3.0), ("route", -1.0)):
        gate = spa.RefreshGate("drift", cfg.batch, width=cfg.q_heads * cfg.head_dim, threshold=thr, device=dev)

        def gstep(g):
            gate.decide(state=states[g])
            spa.sparse_decode_step(x.q_rows[g], x.k_pool, x.v_pool, x.summ[g], super_summaries=x.sup[g],
                                   superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
                                   local_window=cfg.local_window, block_size=cfg.page_size,
                                   router_scale=cfg.head_dim ** -0.5, page_table=x.table[g], context_lens=x.ctx,
                                   out=out[g], selected=sel[g], gate=gate)

        graph = capture(lambda: [gstep(g) for g in range(groups)])
        graph.replay()
        with torch.cuda.nvtx.range(f"gated_{name}"):
            result[f"{name}_us_per_step"] = round(time_graph(graph, reps, 1) * 1e3 / groups, 3)
        del graph
    result["gate"] = "embedding drift (1 - cosine) of the step's query, one device decision per step"
    result["launches_per_step"] = 3
    return result


def run_dense(args, world, rank, dev, peaks):
    """Dense paged decode at 32k: B8, Hq32/Hkv8, D128, bf16, 256 pages of 128 tokens per
    sequence in a 4096-page pool behind a random page table.  A step appends one token per
    (sequence, kv head) in place (the last position, so the context stays 32k) and attends
    over the whole context; the 2.1 GB pool is far larger than L2.  With N > 1 GPUs each
    rank holds the pages of its (sequence, kv head) pairs and decodes them (strong
    scaling: the batch is fixed)."""
    import attention_b200 as spa
    from attention_b200.sharding import DecodeShard

    wk = load_workloads()
    cfg = wk.DenseDecodeConfig()
    shard = DecodeShard(cfg.batch, cfg.q_heads, cfg.kv_heads, world, rank)
    wl = wk.dense_decode_workload(cfg, seed=11, device=dev)
    g = torch.Generator(device=dev).manual_seed(12)
    k_new = (torch.randn(cfg.batch, cfg.kv_heads, cfg.head_dim, generator=g, device=dev) * 0.5).to(cfg.dtype)
    v_new = (torch.randn(cfg.batch, cfg.kv_heads, cfg.head_dim, generator=g, device=dev) * 0.5).to(cfg.dtype)
    q, kp, vp, table, lens = (wl[n] for n in ("query", "k_pool", "v_pool", "page_table", "context_lens"))
    if world > 1:
        tab = table[shard.rows]
        phys = tab.reshape(-1).long()
        kp = kp[phys][:, shard.kv].contiguous()
        vp = vp[phys][:, shard.kv].contiguous()
        table = torch.arange(phys.numel(), dtype=torch.int32, device=dev).view(tab.shape).contiguous()
        q, lens = shard.local(q), lens[shard.rows].contiguous()
        k_new, v_new = shard.local(k_new, "kv"), shard.local(v_new, "kv")
    del wl
    torch.cuda.empty_cache()
    pos = (lens - 1).contiguous()

    def step():
        spa.kv_append(kp, vp, table, k_new, v_new, pos)
        return spa.paged_decode_attention(q, kp, vp, page_table=table, context_lens=lens)

    for _ in range(3):
        step()
    graph = capture(step)
    for _ in range(3):
        graph.replay()
    with torch.cuda.nvtx.range("dense_decode"):
        ms = time_graph(graph, args.dense_steps, world)
    kv_bytes = 2 * cfg.batch * cfg.kv_heads * cfg.context * cfg.head_dim * 2
    io_bytes = 2 * cfg.batch * cfg.q_heads * cfg.head_dim * 2 + cfg.batch * cfg.pages_per_seq * 4
    append_bytes = 2 * 2 * cfg.batch * cfg.kv_heads * cfg.head_dim * 2
    step_bytes = kv_bytes + io_bytes + append_bytes
    gbs = step_bytes / (ms * 1e-3) / 1e9
    peak = float(peaks.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    n_rows, n_kv = shard.rows.stop - shard.rows.start, shard.kv.stop - shard.kv.start
    nsplit, on_chip = spa._lib.decode_plan(n_rows, q.size(1), n_kv, cfg.context)
    del kp, vp, graph
    torch.cuda.empty_cache()
    return {"workload": f"dense paged decode 32k: B{cfg.batch} Hq{cfg.q_heads}/Hkv{cfg.kv_heads} D{cfg.head_dim} "
                        f"bf16, {cfg.pages_per_seq} pages x {cfg.page_size} in a {cfg.pool_pages}-page pool, "
                        "one appended token per step",
            "us_per_step": round(ms * 1e3, 2), "bytes_per_step": step_bytes,
            "value": round(gbs, 1), "unit": "GB/s (all GPUs)", "frac": round(gbs / (peak * world), 4),
            "peak": peak * world, "peak_source": "MEASURED_PEAKS.json hbm_gbs x GPUs",
            "traffic": read_profile_traffic("dense_decode_32k_ncu.md") if world == 1 else None,
            "traffic_source": "profiles/dense_decode_32k_ncu.md (dram read+write per decode launch)",
            "kernels": "kv_append_kernel + decode_mma_kernel" + ("" if (nsplit == 1 or on_chip) else " + decode_combine_kernel"),
            "split_plan": f"{nsplit} splits per (sequence, kv head)" + (", merged on chip" if on_chip and nsplit > 1 else ""),
            "sharding": "single GPU" if world == 1 else f"(sequence, kv head) shards x{world}: {n_rows} sequences x "
                                                         f"{n_kv} kv heads per rank, strong scaling",
            "steps": args.dense_steps, "graph": "CUDA graph replay"}


def decoder_step_bytes(cfg, routable_pages: int) -> int:
    """Algorithmic HBM bytes of one decode step of the integrated model (bf16): every
    weight matrix, bias and norm read once (embedding and position tables: one row),
    per layer the K/V of the window + top-m pages and the fp32 summaries the router
    scores, the appended K/V, the fp32 logits."""
    d, f, v, hd = cfg.d_model, cfg.mlp_mult * cfg.d_model, cfg.vocab, cfg.head_dim
    per_layer_w = (3 * d * d + 3 * d) + (d * d + d) + (f * d + f) + (d * f + d) + 2 * d
    weights = (cfg.layers * per_layer_w + v * d + d + 2 * d) * 2
    kv = cfg.layers * 2 * cfg.heads * (cfg.local_window + cfg.top_m * cfg.page_size) * hd * 2
    summaries = cfg.layers * cfg.heads * routable_pages * hd * 4
    append = cfg.layers * 2 * cfg.heads * hd * 2
    return weights + kv + summaries + append + v * 4


def run_integrated(args, dev, hbm_peak):
    """Integrated 4-layer decoder (d_model 512, 8 heads, vocab 4096, bf16): a 16k-token
    prompt prefilled into 128-token pages, then greedy decode steps with router top-8 +
    128-token local window per layer and the 64-slot TTL-32 promotion table.  The headline
    is the default engine (the chained kernels); the one-launch step (spa_decoder_step) is
    timed beside it."""
    from attention_b200.decoder import DecoderConfig, SparseDecoder, init_weights

    steps = args.integrated_steps
    cfg = DecoderConfig(max_context=16384 + 2 * steps + 8)
    weights = init_weights(cfg, seed=0)
    prompt = torch.randint(0, cfg.vocab, (1, 16384), generator=torch.Generator().manual_seed(0)).to(dev)
    warm = SparseDecoder(cfg, weights, 1, device=dev)  # first-call costs (library handles, modules)
    warm.generate(warm.prefill(prompt).argmax(-1), 4)
    del warm
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    timed = {}
    for engine in ("persistent", "kernels"):
        dec = SparseDecoder(cfg, weights, 1, device=dev, engine=engine)
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
        timed[engine] = (e0.elapsed_time(e1) * 1e3 / steps, prefill_ms)
        del dec
    us, prefill_ms = timed["kernels"]
    # routable pages: the historical pages before the local window, 16384 / 128 - 1 at the
    # first step (one more page becomes routable every 128 steps)
    nbytes = decoder_step_bytes(cfg, (16384 + steps // 2) // cfg.page_size - 1)
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"config": "4 layers, d_model 512, 8 heads x 64, vocab 4096, bf16, prompt 16384 in 128-token pages, "
                      "router top-8 + 128-token window, promotion 64 slots TTL 32",
            "prefill_ms": round(prefill_ms, 3), "decode_steps": steps,
            "decode_us_per_step": round(us, 2), "bytes_per_step": nbytes, "gbs": round(gbs, 1),
            "frac": round(gbs / hbm_peak, 4),
            "mode": "one CUDA-graph replay per step (the default engine): the library's few-row linear kernels "
                    "(spa_norm_linear / spa_linear, norms and residual adds fused in front, QKV epilogue append), "
                    "one routed gather decode per layer, promotion update, vocabulary head and argmax, chained as "
                    f"programmatic dependents; the first {steps} positions after the prompt, decoded once untimed "
                    "(graph captures) and again timed after a rewind",
            "persistent_step": {"decode_us_per_step": round(timed["persistent"][0], 2), "launches_per_step": 1,
                                "mode": "the same step as one cooperative kernel (spa_decoder_step), phases "
                                        "exchanging data through global memory"}}


# ------------------------------------------------------------------ reference arm
def run_reference(args, world, rank, local):
    """The reference's PyTorch CPU path on the host cores, rank 0 only, on the same
    configuration and `config` as our arm; nothing here loads the CUDA library."""
    if rank != 0:
        return
    import oracle

    # every host core for the one rank that runs (torchrun sets one thread per process)
    try:
        import psutil

        torch.set_num_threads(psutil.cpu_count(logical=False) or os.cpu_count() or 1)
    except Exception:
        torch.set_num_threads(os.cpu_count() or 1)

    wk = load_workloads()
    cfg = wk.SparseDecodeConfig(top_m=args.top_m)
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    q, k_c, v_c, sup, summ = reference_inputs(wk, cfg, 1000, device)
    for _ in range(max(args.warmup, 1)):
        oracle.reference_decode_step(q, k_c, v_c, sup, summ, superblock=cfg.superblock, top_super=cfg.top_super,
                                     top_blocks=cfg.top_m, local_window=cfg.local_window, block_size=cfg.page_size)
    t, n = time_reference_steps(oracle, q, k_c, v_c, sup, summ, cfg, steps=args.steps, budget_s=args.cpu_budget * 4)
    bytes_step = wk.sparse_decode_bytes(cfg)
    value = bytes_step / t / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": max(args.warmup, 1), "ms_per_step": round(t * 1e3, 4),
        "us_per_step": round(t * 1e6, 1), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (seeded N(0,0.5) K/V/q with planted needle pages)",
        "config": sparse_config(cfg, args.groups, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{n} full steps of batch group 0: oracle.reference_decode_step (select_blocks "
                                   "at two levels, make_candidates, reference_attention; fp32 torch CPU ops)"},
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
