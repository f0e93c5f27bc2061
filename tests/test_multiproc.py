"""Multi-process (batch, head) sharding on CPU with the gloo backend.

World size 2 (and 3) stand in for GPUs: each rank takes its shard of the
units, generates its units' inputs from per-unit seeds, computes sample rows
with the CPU oracle, and rank 0 gathers them.  The result must equal a
single-process computation of the same rows (the partition covers every unit
once and the data does not depend on the world size), the MAX-over-ranks
timing rule must hold, and a rank that dies makes the others' next
collective fail instead of hanging.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


B, H, S, D = 2, 3, 64, 64  # 6 units


def _rows_of_units(u0, u1, q, k, v, oracle):
    """Oracle output of rows {0, S-1} of every unit in [u0, u1) (local tensors)."""
    rows = []
    for i in range(u1 - u0):
        rows += [i * S, i * S + S - 1]
    u16 = lambda t: t.view(__import__("torch").int16).numpy().view(np.uint16)
    return oracle.attention_rows(u16(q), u16(k), u16(v), np.array(rows), bn_tile=32, nthreads=1)


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    from attnprofile_b200 import shard
    from oracle import oracle
    _init(rank, world, port)
    u0, u1 = shard.shard_range(B * H, world, rank)
    q, k, v, _ = shard.generate_units(u0, u1, S, D, torch.float16, "cpu", 77)
    local = _rows_of_units(u0, u1, q, k, v, oracle) if u1 > u0 else np.zeros((0, D), np.uint16)
    parts = [None] * world
    dist.all_gather_object(parts, (u0, u1, local))
    t = shard.max_over_ranks(float(rank + 1))
    n = shard.sum_over_ranks(u1 - u0)
    if rank == 0:
        np.save(Path(out_dir) / "gathered.npy",
                np.concatenate([p[2] for p in sorted(parts, key=lambda p: p[0])]))
        np.save(Path(out_dir) / "meta.npy", np.array([t, n]))
    dist.destroy_process_group()


def _dying_worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    _init(rank, world, port, timeout_s=10)
    dist.barrier()
    if rank == 1:
        os._exit(3)  # a rank that leaves between steps, with nothing in flight
    try:
        dist.all_reduce(torch.ones(1))
        msg = "no error"
    except Exception as e:  # noqa: BLE001
        msg = "error: " + type(e).__name__
    (Path(out_dir) / f"rank{rank}.txt").write_text(msg)


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_shards_equal_single_process(tmp_path, world, oracle_mod):
    import torch
    import torch.multiprocessing as mp
    from attnprofile_b200 import shard
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    got = np.load(tmp_path / "gathered.npy")
    q, k, v, _ = shard.generate_units(0, B * H, S, D, torch.float16, "cpu", 77)
    ref = _rows_of_units(0, B * H, q, k, v, oracle_mod)
    assert np.array_equal(got, ref)
    t, n = np.load(tmp_path / "meta.npy")
    assert t == world and n == B * H


def test_rank_failure_is_seen_by_the_others(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_dying_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in ctx.processes)
    assert (tmp_path / "rank0.txt").read_text().startswith("error")


def _gather_worker(rank, world, port, out_dir):
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist
    from attnprofile_b200 import shard
    _init(rank, world, port)
    units = 7  # uneven shards (and an empty one at world 8 would be allowed)
    u0, u1 = shard.shard_range(units, world, rank)
    # stand-in output: each unit's block filled with its unit index
    O = torch.arange(u0, u1, dtype=torch.float32).view(1, -1, 1, 1).expand(1, u1 - u0, 5, 4)
    O = O.contiguous().to(torch.float16)
    full = shard.gather_output(O, units, dst=world - 1)
    if rank == world - 1:
        torch.save(full, Path(out_dir) / "full.pt")
    else:
        assert full is None
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_output_collects_every_shard(tmp_path, world):
    import torch
    import torch.multiprocessing as mp
    mp.start_processes(_gather_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    full = torch.load(tmp_path / "full.pt")
    assert tuple(full.shape) == (1, 7, 5, 4)
    for u in range(7):
        assert torch.all(full[0, u] == u)
