"""Sequence-parallel prefill over NCCL on 2+ GPUs (skipped on a single-GPU host).

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
