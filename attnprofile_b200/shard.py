"""(batch, head) sharding across GPUs -- host side, no collective on the data path.

Attention is independent per (batch, head) unit u = b * H + h, so a job of
U = B * H units is split into contiguous ranges, GPU g owning
[floor(g * U / n), floor((g + 1) * U / n)) -- the rule of attn_shard_range in
the C ABI (mirrored here in Python so CPU-only processes can use it).  Each
GPU generates its own units' inputs from a per-unit seed, so a unit's data is
the same whatever the number of GPUs, and runs the kernel on local memory.
The only collectives are control-plane ones outside the timed region (a
barrier around timing and a MAX of the per-rank times).

The reference has no multi-GPU code; this is the partition the benchmark
configurations C4 (8x32x8192x128) and C5 (1x64x32768x128) run on 1/2/4/8 GPUs.
"""
from __future__ import annotations


def shard_range(units: int, world: int, rank: int) -> tuple[int, int]:
    """Units [begin, end) of `rank` (same rule as attn_shard_range)."""
    if units < 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad partition: units={units} world={world} rank={rank}")
    return units * rank // world, units * (rank + 1) // world


def unit_seed(base_seed: int, set_index: int, unit: int) -> int:
    """Seed of one (batch, head) unit's inputs: independent of the world size."""
    return base_seed * 1000003 + set_index * 7919 + unit


def generate_units(u0: int, u1: int, S: int, D: int, dtype, device, base_seed: int,
                   set_index: int = 0, sigma: float = 1.0):
    """Seeded N(0, sigma^2) Q, K, V for units [u0, u1), shaped [1, u1 - u0, S, D],
    plus an empty O.  Unit u's values depend only on (base_seed, set_index, u)."""
    import torch
    n = u1 - u0
    Q = torch.empty(1, n, S, D, dtype=dtype, device=device)
    K, V = torch.empty_like(Q), torch.empty_like(Q)
    for i, u in enumerate(range(u0, u1)):
        g = torch.Generator(device=device).manual_seed(unit_seed(base_seed, set_index, u))
        for t in (Q, K, V):
            t[0, i].copy_((torch.randn(S, D, generator=g, device=device) * sigma).to(dtype))
    return Q, K, V, torch.empty_like(Q)


def max_over_ranks(value: float, device=None) -> float:
    """MAX of a per-rank float over the default process group (identity when
    torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(value: float, device=None) -> list[float]:
    """Every rank's value of a per-rank float, in rank order, on every rank
    ([value] when torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(value)]
    t = torch.zeros(dist.get_world_size(), dtype=torch.float64, device=device)
    t[dist.get_rank()] = float(value)
    dist.all_reduce(t)
    return [float(x) for x in t.tolist()]


def sum_over_ranks(value: int, device=None) -> int:
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return int(value)
    t = torch.tensor([int(value)], dtype=torch.int64, device=device)
    dist.all_reduce(t)
    return int(t.item())


def gather_output(O_local, units_total: int, dst: int = 0):
    """Collect the sharded output on one rank: every rank holds O for its
    units [u0, u1) as [1, u1 - u0, S, D]; rank `dst` returns the whole
    [1, units_total, S, D] (other ranks return None).  Point-to-point sends of
    each shard straight into its slice of the destination tensor (NCCL over
    NVLink on GPUs, gloo on CPU) -- the optional consumer-side step after the
    collective-free compute.  Identity with one rank."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return O_local
    world, rank = dist.get_world_size(), dist.get_rank()
    u0, u1 = shard_range(units_total, world, rank)
    if O_local.shape[1] != u1 - u0:
        raise ValueError(f"rank {rank} holds {O_local.shape[1]} units, its range is [{u0}, {u1})")
    if rank != dst:
        if u1 > u0:
            dist.send(O_local.contiguous(), dst)
        return None
    S, D = O_local.shape[2], O_local.shape[3]
    out = torch.empty(1, units_total, S, D, dtype=O_local.dtype, device=O_local.device)
    out[:, u0:u1].copy_(O_local)
    ops = []
    for r in range(world):
        r0, r1 = shard_range(units_total, world, r)
        if r != dst and r1 > r0:
            ops.append(dist.P2POp(dist.irecv, out[:, r0:r1], r))
    for req in (dist.batch_isend_irecv(ops) if ops else []):
        req.wait()
    return out
