"""Sequence-parallel prefill and (sequence, kv head)-sharded sparse decode over NCCL on 2+ GPUs
(skipped on a single-GPU host).

Each rank holds a contiguous chunk, receives the previous rank's last `window` K/V
tokens through the NCCL halo exchange, and runs the tensor-core kernel; rank 0
gathers the chunks and compares them with one single-GPU prefill of the whole
sequence.  Tolerance: bf16, 2e-2 absolute + 1e-2 relative."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, seq, window, result_dir):
    import datetime

    import torch.distributed as dist

    import attention_b200 as spa
    from attention_b200.sharding import PrefillShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        gen = torch.Generator(device=dev).manual_seed(0)
        shape = (1, 4, seq, 128)
        q, k, v = ((torch.randn(shape, generator=gen, device=dev) * 0.5).to(torch.bfloat16) for _ in range(3))
        chunk = seq // world
        sl = slice(rank * chunk, (rank + 1) * chunk)
        qc, kc, vc = (t[:, :, sl].contiguous() for t in (q, k, v))
        out = torch.empty_like(qc)
        PrefillShard(rank, world, window).forward(qc, kc, vc, out=out)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        if rank == 0:
            full = spa.local_causal_prefill(q, k, v, window)
            got = torch.cat(gathered, dim=2)
            err = (got.double() - full.double()).abs()
            ok = bool((err <= 2e-2 + 1e-2 * full.double().abs()).all())
            with open(os.path.join(result_dir, "result.txt"), "w") as f:
                f.write(f"{ok} {err.max().item():.3e} {spa.device_error_flags()}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("seq,window", [(8192, 2048), (6144, 1000)])
def test_sequence_parallel_prefill_matches_single_gpu(tmp_path, seq, window):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), seq, window, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ok, err, flags = (tmp_path / "result.txt").read_text().split()
    assert ok == "True", err
    assert flags == "0"


def _decode_worker(rank, world, port, result_dir):
    """One (sequence, kv head) shard of the 128k-shape sparse step per GPU (its own kv
    heads' pages only, the sequences' summaries and query rows for all heads), outputs
    gathered over NCCL and compared on rank 0 with the single-GPU step."""
    import datetime

    import torch.distributed as dist

    import attention_b200 as spa
    from attention_b200 import workloads
    from attention_b200.sharding import DecodeShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        cfg = workloads.SparseDecodeConfig(top_m=4, pages_per_seq=128)
        wl = workloads.sparse_decode_workload(cfg, groups=1, seed=5, device=dev)  # same seed: same batch everywhere
        table, q, ctx = wl["page_table"][0], wl["query"][0], wl["context_lens"]
        summ, sup = spa.page_summaries(wl["k_pool"], block_size=cfg.page_size, n_pages=cfg.routable_pages,
                                       page_table=table, superblock=cfg.superblock)
        kw = dict(superblock=cfg.superblock, top_super=cfg.top_super, top_blocks=cfg.top_m,
                  local_window=cfg.local_window, block_size=cfg.page_size, router_scale=cfg.head_dim ** -0.5)
        shard = DecodeShard(cfg.batch, cfg.q_heads, cfg.kv_heads, world, rank)
        tab = table[shard.rows]
        phys = tab.reshape(-1).long()
        kp = wl["k_pool"][phys][:, shard.kv].contiguous()
        vp = wl["v_pool"][phys][:, shard.kv].contiguous()
        local_tab = torch.arange(phys.numel(), dtype=torch.int32, device=dev).view(tab.shape)
        out, sel = spa.sparse_decode_step(q[shard.rows].contiguous(), kp, vp, summ[shard.rows].contiguous(),
                                          super_summaries=sup[shard.rows].contiguous(), page_table=local_tab,
                                          context_lens=ctx[shard.rows].contiguous(),
                                          kv_head_range=(shard.kv.start, shard.kv.stop - shard.kv.start), **kw)
        full = shard.gather(out)
        sels = [torch.empty_like(sel) for _ in range(world)]
        dist.all_gather(sels, sel)
        if rank == 0:
            ref_out, ref_sel = spa.sparse_decode_step(q, wl["k_pool"], wl["v_pool"], summ, super_summaries=sup,
                                                      page_table=table, context_lens=ctx, **kw)
            sel_ok = all(torch.equal(sels[r], ref_sel[DecodeShard(cfg.batch, cfg.q_heads, cfg.kv_heads, world,
                                                                  r).rows]) for r in range(world))
            err = (full.double() - ref_out.double()).abs()
            ok = sel_ok and bool((err <= 2e-2 + 1e-2 * ref_out.double().abs()).all())
            with open(os.path.join(result_dir, "result.txt"), "w") as f:
                f.write(f"{ok} {err.max().item():.3e} {spa.device_error_flags()}")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_sparse_decode_matches_single_gpu(tmp_path):
    world = 2
    mp.start_processes(_decode_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    ok, err, flags = (tmp_path / "result.txt").read_text().split()
    assert ok == "True", err
    assert flags == "0"
