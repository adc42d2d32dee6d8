"""Sequence-parallel attention host logic on CPU: zigzag sharding covers the sequence once with equal causal work per
rank, the all-gather + reassembly puts every key back at its position, and a world-2 gloo run with a reference
attention gives the single-process result for every query row."""
import socket

import pytest
import torch
import torch.multiprocessing as mp

from reax_engine_kernels_b200 import seqpar


def ref_attend(q, k, v, scale, qpos, G, out):
    """fp32 causal attention with the kernel's visibility rule (key j visible to row i iff j <= qpos[b, i // G])."""
    B, H, M, D = q.shape
    N = k.shape[2]
    s = torch.einsum("bhmd,bhnd->bhmn", q.double(), k.double()) * scale
    rowpos = qpos.long()[:, torch.arange(M) // G]  # [B, M]
    vis = torch.arange(N)[None, None, None, :] <= rowpos[:, None, :, None]
    p = torch.softmax(s.masked_fill(~vis, float("-inf")), dim=-1)
    out.copy_(torch.einsum("bhmn,bhnd->bhmd", p, v.double()).to(out.dtype))
    return out


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_zigzag_partition_and_balance(world):
    S = 2 * world * 16
    seen = torch.cat([seqpar.local_positions(S, world, r) for r in range(world)])
    assert torch.equal(seen.sort().values, torch.arange(S, dtype=torch.int32))
    work = [int((seqpar.local_positions(S, world, r).long() + 1).sum()) for r in range(world)]
    assert max(work) == min(work)  # causal (row, key) pairs per rank
    with pytest.raises(ValueError):
        seqpar.zigzag_chunks(S + 1, world, 0)


def test_assemble_restores_positions():
    world, B, H, S, D = 4, 2, 3, 64, 5
    full = torch.arange(B * H * S * D, dtype=torch.float32).reshape(B, H, S, D)
    shards = []
    for r in range(world):
        pos = seqpar.local_positions(S, world, r).long()
        shards.append(full[:, :, pos])
    assert torch.equal(seqpar.assemble(torch.stack(shards), world), full)


def test_single_rank_equals_full_attention():
    B, H, G, S, D = 1, 2, 2, 32, 8
    g = torch.Generator().manual_seed(3)
    q = torch.randn(B, H, S * G, D, generator=g)
    k = torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    full = ref_attend(q, k, v, 0.3, torch.arange(S, dtype=torch.int32)[None], G, torch.empty_like(q))
    pos = seqpar.local_positions(S, 1, 0).long()
    rows = (pos[:, None] * G + torch.arange(G)).reshape(-1)
    o = seqpar.attention(q[:, :, rows], k[:, :, pos], v[:, :, pos], 0.3, S, 1, 0, G=G, k_full=k, v_full=v,
                         attend=ref_attend)
    assert torch.allclose(o, full[:, :, rows], atol=1e-6)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, H, G, S, D = 2, 2, 2, 48, 8
        g = torch.Generator().manual_seed(11)  # every rank draws the same full problem and keeps its shard
        q = torch.randn(B, H, S * G, D, generator=g)
        k = torch.randn(B, H, S, D, generator=g)
        v = torch.randn(B, H, S, D, generator=g)
        pos = seqpar.local_positions(S, world, rank).long()
        rows = (pos[:, None] * G + torch.arange(G)).reshape(-1)
        o = seqpar.attention(q[:, :, rows].contiguous(), k[:, :, pos].contiguous(), v[:, :, pos].contiguous(), 0.25,
                             S, world, rank, G=G, attend=ref_attend)
        outs = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(outs, o)
        if rank == 0:
            full = ref_attend(q, k, v, 0.25, torch.arange(S, dtype=torch.int32).repeat(B, 1), G, torch.empty_like(q))
            got = torch.empty_like(full)
            for r in range(world):
                pr = seqpar.local_positions(S, world, r).long()
                got[:, :, (pr[:, None] * G + torch.arange(G)).reshape(-1)] = outs[r]
            out["maxdiff"] = float((got - full).abs().max())
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_gloo_world2_sequence_parallel_matches_full():
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
    assert out["maxdiff"] < 1e-6
