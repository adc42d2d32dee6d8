"""Multi-process host logic on CPU (gloo, world size 2): sharding covers every unit exactly once, the max-over-ranks
timing reduction returns the slowest rank, and the gate-up weight shard keeps the groups of 4 together."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from reax_engine_kernels_b200 import dist as rd
from reax_engine_kernels_b200 import synth


def test_split_even_covers_everything():
    for total, world, g in [(14336, 8, 4), (14336, 3, 4), (100, 7, 1), (32, 8, 1)]:
        shards = [rd.split_even(total, world, r, g) for r in range(world)]
        assert shards[0].start == 0 and shards[-1].stop == total
        for a, b in zip(shards, shards[1:]):
            assert a.stop == b.start
        assert all(s.start % g == 0 and s.stop % g == 0 for s in shards)
        assert max(s.size for s in shards) - min(s.size for s in shards) <= g


def test_gate_up_shard_is_a_valid_layer():
    # a column shard of the packed weights, fed to the oracle alone, reproduces exactly those output columns
    from oracle import oracle as orc

    M, N2, K, world = 4, 48, 32, 3
    x = synth.bf16_normal(1, (M, K))
    w = synth.bf16_normal(2, (2 * N2, K), 0.1)
    full, _, _ = orc.gv(x, w, intervals=False)
    for r in range(world):
        c, rows = rd.gate_up_columns(N2, world, r), rd.gate_up_weight_rows(N2, world, r)
        part, _, _ = orc.gv(x, np.ascontiguousarray(w[rows.start:rows.stop]), intervals=False)
        assert np.array_equal(part, full[:, c.start:c.stop])


def test_attention_units_partition():
    got = sorted(u for r in range(8) for u in rd.attention_units(4, 8, 8, r))
    assert got == [(b, h) for b in range(4) for h in range(8)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        rd.barrier(world)
        m = rd.max_over_ranks(10.0 + rank, world)
        shard = rd.gate_up_columns(14336, world, rank)
        out[rank] = (m, shard.start, shard.stop)
        rd.barrier(world)
    finally:
        dist.destroy_process_group()


def test_gloo_world2_max_and_shards():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert out[0][0] == out[1][0] == 11.0  # the slowest rank's time
    assert (out[0][1], out[0][2], out[1][1], out[1][2]) == (0, 7168, 7168, 14336)
