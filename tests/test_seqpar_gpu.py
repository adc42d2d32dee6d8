"""Sequence-parallel attention on the GPU through the attention kernel.

* one GPU, 4 ranks emulated: each rank's zigzag shard runs through seqpar.attention with the whole position-ordered K
  and V handed in (what the all-gather produces); the reassembled output is compared with the kernel run on the whole
  sequence (same keys in the same 128-key blocks for every row, so the same arithmetic) and with the oracle on
  sampled rows;
* two GPUs (skipped with fewer): two processes over NCCL, each holding only its shard of K and V, all-gathering them
  inside seqpar.attention; the outputs gathered to rank 0 must equal the single-GPU whole-sequence kernel output.
"""
import math
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as orc
from reax_engine_kernels_b200 import kernels as rk
from reax_engine_kernels_b200 import seqpar, synth
from tests.tolerance import assert_close, assert_close_interval

pytestmark = pytest.mark.gpu
bf = synth.bf16_bits_to_f32
B, H, G, S, D = 1, 2, 4, 4096, 128


def problem(device="cuda"):
    q = synth.device_normal_bf16((B, H, S * G, D), 1.0, 1600, device=device)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, 1601, device=device)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, 1602, device=device)
    return q, k, v


def shard(t, world, rank, per_token):
    pos = seqpar.local_positions(S, world, rank).long().to(t.device)
    idx = (pos[:, None] * per_token + torch.arange(per_token, device=t.device)).reshape(-1)
    return t[:, :, idx].contiguous(), idx


def test_emulated_four_ranks_match_whole_sequence():
    world = 4
    q, k, v = problem()
    scale = 1 / math.sqrt(D)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
    full = rk.fmha(q, k, v, scale, qpos=qpos, G=G)
    got = torch.empty_like(full)
    for r in range(world):
        ql, rows = shard(q, world, r, G)
        kl, _ = shard(k, world, r, 1)
        vl, _ = shard(v, world, r, 1)
        o = seqpar.attention(ql, kl, vl, scale, S, world, r, G=G, k_full=k, v_full=v)
        got[:, :, rows] = o
        # the all-gather's reassembly, emulated: every rank's shard stacked rank-major
    ks = torch.stack([shard(k, world, r, 1)[0] for r in range(world)])
    assert torch.equal(seqpar.assemble(ks, world), k)
    torch.cuda.synchronize()
    g, f = synth.from_torch_bf16(got), synth.from_torch_bf16(full)
    assert_close(bf(g), bf(f))
    qh, kh, vh = (synth.from_torch_bf16(t) for t in (q, k, v))
    for r0 in (0, 5000, S * G - 3):
        ref, lo, hi = orc.fmha(qh, kh, vh, scale, qpos=qpos.cpu().numpy(), G=G, qpBs=S, rows=(r0, r0 + 3),
                               intervals=True)
        sl = (slice(None), slice(None), slice(r0, r0 + 3))
        assert_close_interval(bf(g[sl]), bf(ref[sl]), bf(lo[sl]), bf(hi[sl]))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import datetime
    import os

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        q, k, v = problem()
        scale = 1 / math.sqrt(D)
        ql, rows = shard(q, world, rank, G)
        kl, _ = shard(k, world, rank, 1)
        vl, _ = shard(v, world, rank, 1)
        del k, v
        o = seqpar.attention(ql, kl, vl, scale, S, world, rank, G=G)
        outs = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(outs, o)
        if rank == 0:
            q, k, v = problem()
            qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
            full = rk.fmha(q, k, v, scale, qpos=qpos, G=G)
            got = torch.empty_like(full)
            for r in range(world):
                got[:, :, shard(q, world, r, G)[1]] = outs[r]
            torch.cuda.synchronize()
            g, f = synth.from_torch_bf16(got), synth.from_torch_bf16(full)
            out["exact"] = float(np.mean(g == f))
            out["g"], out["f"] = bf(g), bf(f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_nccl_all_gather():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    assert_close(out["g"], out["f"])
