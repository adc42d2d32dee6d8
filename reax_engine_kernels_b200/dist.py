"""Multi-GPU host logic: one process per GPU, work sharded with no data-path collective.

The kernels themselves never communicate.  This module only decides which shard of a layer each rank owns and
reduces per-rank timings (a barrier and a MAX all-reduce), with NCCL tensors on GPUs or gloo tensors on CPU (the
CPU test suite runs it as world-size-2 gloo).

Sharding (the partitions the hot path has naturally):
  * gate-up GEMM: column-parallel along N2 in whole groups of 4 gate/up rows (w_g4 rows [8j, 8j+8) stay together);
  * sliced / plain GEMM: column-parallel along N;
  * attention: by (batch x kv-head) units;
  * linear-attention kernels: by rows / channel units / chunks.
"""
from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def split_even(total: int, world: int, rank: int, granule: int = 1) -> Shard:
    """Contiguous shard of [0, total) for `rank`, boundaries on multiples of `granule`; sizes differ by at most one
    granule (the first ranks get the extra granules)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if total % granule:
        raise ValueError(f"total {total} is not a multiple of granule {granule}")
    units = total // granule
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    n = base + (1 if rank < extra else 0)
    return Shard(start * granule, (start + n) * granule)


def gate_up_columns(N2: int, world: int, rank: int) -> Shard:
    """Output columns of the gate-up layer owned by `rank` (groups of 4 features never split)."""
    return split_even(N2, world, rank, granule=4)


def gate_up_weight_rows(N2: int, world: int, rank: int) -> Shard:
    """Rows of the interleaved w_g4 [2*N2, K] owned by `rank`: the 8 rows of each 4-feature group together."""
    c = gate_up_columns(N2, world, rank)
    return Shard(2 * c.start, 2 * c.stop)


def attention_units(B: int, Hkv: int, world: int, rank: int) -> list[tuple[int, int]]:
    """(batch, kv head) pairs owned by `rank`."""
    s = split_even(B * Hkv, world, rank)
    return [(u // Hkv, u % Hkv) for u in range(s.start, s.stop)]


def env_world() -> tuple[int, int, int]:
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0"))


def max_over_ranks(value: float, world: int, device=None) -> float:
    """MAX of a per-rank scalar over all ranks (identity at world 1).  device=None: CPU tensor (gloo)."""
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device=None):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    if device is not None and torch.cuda.is_available():
        torch.cuda.synchronize()
