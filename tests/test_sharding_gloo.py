"""Host-side multi-rank logic on CPU ranks (gloo): the prefill halo exchange and
batch sharding.  The chunk compute is the oracle, so no GPU is involved."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from attention_b200.sharding import PrefillShard, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_compute(q, k, v, out, window, rows, k_halo, v_halo):
    full = oracle.local_reference_chunked(q, k, v, window, chunk=64, k_halo=k_halo, v_halo=v_halo)
    out[:, :, rows[0]:rows[1]] = full[:, :, rows[0]:rows[1]].to(out.dtype)


def _worker(rank, world, port, seq, window, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gen = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(1, 2, seq, 16, generator=gen, dtype=torch.float64) for _ in range(3))
        chunk = seq // world
        sl = slice(rank * chunk, (rank + 1) * chunk)
        out = torch.zeros(1, 2, chunk, 16, dtype=torch.float64)
        PrefillShard(rank, world, window, compute=_cpu_compute).forward(
            q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous(), out=out)
        torch.save(out, os.path.join(result_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,seq,window", [(2, 512, 128), (4, 1024, 200), (3, 768, 256)])
def test_prefill_halo_exchange_matches_full_sequence(tmp_path, world, seq, window):
    mp.start_processes(_worker, args=(world, _free_port(), seq, window, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    got = torch.cat([torch.load(tmp_path / f"rank{r}.pt") for r in range(world)], dim=2)
    gen = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(1, 2, seq, 16, generator=gen, dtype=torch.float64) for _ in range(3))
    ref = oracle.local_reference_chunked(q, k, v, window, chunk=128)
    assert (got - ref).abs().max().item() < 1e-12


def test_halo_free_rows_round_up_to_tile():
    assert PrefillShard(1, 2, 2048).halo_free_from(16384) == 2048
    assert PrefillShard(1, 2, 200).halo_free_from(16384) == 256
    assert PrefillShard(1, 2, 129).halo_free_from(100) == 100


def test_shard_rows_cover_exactly_once():
    for n in (1, 4, 7, 64):
        for world in (1, 2, 3, 8):
            cover = []
            for r in range(world):
                s = shard_rows(n, world, r)
                cover.extend(range(n)[s])
            assert cover == list(range(n))


def _late_worker(rank, world, port, result_dir):
    """Rank 1 never joins the exchange: rank 0's receive must fail on the process-group
    timeout instead of waiting forever."""
    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    try:
        if rank == 1:
            q = torch.zeros(1, 1, 64, 8)
            out = torch.zeros_like(q)
            try:
                PrefillShard(1, 2, 32, compute=_cpu_compute).forward(q, q, q, out=out)
                status = "completed"
            except Exception as exc:  # noqa: BLE001 - any transport error is the expected outcome
                status = f"error: {type(exc).__name__}"
            with open(os.path.join(result_dir, "status.txt"), "w") as f:
                f.write(status)
        # rank 0 leaves without sending its halo
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_missing_peer_surfaces_as_error_not_hang(tmp_path):
    mp.start_processes(_late_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn",
                       join=True)
    assert (tmp_path / "status.txt").read_text().startswith("error")


# ---------------------------------------------------------------- (sequence, kv head) decode shards
def test_decode_shard_layout():
    from attention_b200.sharding import decode_shard

    # 4 sequences x 8 kv heads: whole sequences up to 4 ranks, kv-head halves at 8
    assert decode_shard(4, 8, 1, 0) == (slice(0, 4), slice(0, 8))
    assert decode_shard(4, 8, 2, 1) == (slice(2, 4), slice(0, 8))
    assert decode_shard(4, 8, 4, 3) == (slice(3, 4), slice(0, 8))
    assert decode_shard(4, 8, 8, 5) == (slice(2, 3), slice(4, 8))
    assert decode_shard(8, 8, 8, 7) == (slice(7, 8), slice(0, 8))
    covered = set()
    for r in range(8):
        rows, kv = decode_shard(4, 8, 8, r)
        covered |= {(b, h) for b in range(rows.start, rows.stop) for h in range(kv.start, kv.stop)}
    assert covered == {(b, h) for b in range(4) for h in range(8)}
    with pytest.raises(ValueError):
        decode_shard(4, 8, 3, 0)
    with pytest.raises(ValueError):
        decode_shard(2, 6, 3, 0)  # 4 pairs per rank: not a divisor of 6 kv heads


def _sparse_inputs(seed=0):
    gen = torch.Generator().manual_seed(seed)
    b, hq, hkv, d, page, n_pages, win, sb = 4, 16, 8, 32, 16, 37, 16, 8
    ctx = n_pages * page + win
    keys = torch.randn(b, hkv, ctx, d, generator=gen, dtype=torch.float64)
    values = torch.randn(b, hkv, ctx, d, generator=gen, dtype=torch.float64)
    q = torch.randn(b, hq, d, generator=gen, dtype=torch.float64)
    return dict(q=q, keys=keys, values=values, page=page, n_pages=n_pages, win=win, sb=sb)


def _decode_worker(rank, world, port, result_dir):
    """Each rank: the router over its sequences' full query rows and summaries (the
    oracle's canonical router), then the gather decode over its own kv heads only."""
    from attention_b200.sharding import DecodeShard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = _sparse_inputs()
        q, keys, values = x["q"], x["keys"], x["values"]
        shard = DecodeShard(q.size(0), q.size(1), keys.size(1), world, rank)
        # replicated router inputs of the shard's sequences (all heads)
        summ, sums = oracle.summaries_fp64(keys[shard.rows], x["page"], x["n_pages"])
        sup = oracle.super_summaries(sums, x["sb"], x["page"])
        sel = oracle.select_blocks_tree(q[shard.rows], sup, summ, superblock=x["sb"], top_super=2, top_blocks=3)
        # the rank holds only its kv heads' pages
        k_local, v_local = shard.local(keys, "kv"), shard.local(values, "kv")
        out_local = oracle.gather_decode(shard.local(q), k_local, v_local, sel, local_window=x["win"],
                                         block_size=x["page"])
        full = shard.gather(out_local)
        sels = [torch.empty_like(sel) for _ in range(world)]
        dist.all_gather(sels, sel)
        if rank == 0:
            torch.save({"out": full, "sel": sels}, os.path.join(result_dir, "decode.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_shards_match_single_process(tmp_path, world):
    mp.start_processes(_decode_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    got = torch.load(tmp_path / "decode.pt")
    x = _sparse_inputs()
    summ, sums = oracle.summaries_fp64(x["keys"], x["page"], x["n_pages"])
    sup = oracle.super_summaries(sums, x["sb"], x["page"])
    sel = oracle.select_blocks_tree(x["q"], sup, summ, superblock=x["sb"], top_super=2, top_blocks=3)
    ref = oracle.gather_decode(x["q"], x["keys"], x["values"], sel, local_window=x["win"], block_size=x["page"])
    assert (got["out"] - ref).abs().max().item() < 1e-12
    # ranks that share a sequence selected the same pages, equal to the single-process ones
    from attention_b200.sharding import decode_shard

    for r in range(world):
        rows, _ = decode_shard(4, 8, world, r)
        assert torch.equal(got["sel"][r], sel[rows])
