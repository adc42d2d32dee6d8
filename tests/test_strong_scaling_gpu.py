"""BASELINE's multi-GPU splits, reassembled over NCCL and compared bit for bit with one GPU's output.

Config 2 (gate-up GEMM) is split column-parallel along N2 (each rank owns whole groups of 4 gate/up features) and
config 3's attention by (batch x kv-head) units; no collective runs on the data path.  The shards are all-gathered over
NCCL only to check them: the reassembled layer must equal rank 0's single-GPU output exactly.  Two ranks, one process
per GPU (spawned), NVLS off; skipped with fewer than two GPUs.  The single-GPU emulation of every split width
(tests/test_gemm_gpu.py::test_gv_column_shards_reproduce_full_layer_bitwise) covers 2, 4 and 8 ranks on one GPU.
"""
import math
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

M, K, N2 = 2048, 4096, 14336
B, HKV, G, S, D = 4, 8, 4, 2048, 128  # config 3's heads and batches, 2048 positions (the split is per unit)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gate_up(rank_rows=None):
    from reax_engine_kernels_b200 import synth

    x = synth.device_normal_bf16((M, K), 1.0, 41)
    w = synth.device_normal_bf16((2 * N2, K), 0.02, 42)
    return x, (w if rank_rows is None else w[rank_rows.start:rank_rows.stop].contiguous())


def _attention_inputs():
    from reax_engine_kernels_b200 import synth

    q = synth.device_normal_bf16((B, HKV, S * G, D), 1.0, 43)
    k = synth.device_normal_bf16((B, HKV, S, D), 1.0, 44)
    v = synth.device_normal_bf16((B, HKV, S, D), 1.0, 45)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
    return q, k, v, qpos


def _worker(rank, world, port, out):
    import datetime
    import os

    import torch.distributed as dist

    from reax_engine_kernels_b200 import dist as rd
    from reax_engine_kernels_b200 import kernels as rk

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        # ---- config 2: this rank's gate-up columns
        rows = rd.gate_up_weight_rows(N2, world, rank)
        x, w = _gate_up(rows)
        part = rk.gv(x, w, cfg=0)
        parts = [torch.empty_like(part) for _ in range(world)]  # N2 / world columns each (14336 divides evenly)
        dist.all_gather(parts, part)
        # ---- config 3 heads: this rank's (batch, kv head) units, a contiguous run of whole batches here
        q, k, v, qpos = _attention_inputs()
        units = rd.attention_units(B, HKV, world, rank)
        b0, b1 = units[0][0], units[-1][0] + 1
        assert [u for u in units] == [(b, h) for b in range(b0, b1) for h in range(HKV)]
        o = rk.fmha(q[b0:b1], k[b0:b1], v[b0:b1], 1 / math.sqrt(D), qpos=qpos[b0:b1], G=G)
        os_ = [torch.empty_like(o) for _ in range(world)]
        dist.all_gather(os_, o)
        if rank == 0:
            x, wf = _gate_up()
            full = rk.gv(x, wf, cfg=0)
            got = torch.cat(parts, 1)
            out["gv_bitwise"] = bool(torch.equal(got.view(torch.int16), full.view(torch.int16)))
            fo = rk.fmha(q, k, v, 1 / math.sqrt(D), qpos=qpos, G=G)
            go = torch.cat(os_, 0)
            out["attn_bitwise"] = bool(torch.equal(go.view(torch.int16), fo.view(torch.int16)))
            out["status"] = rk.status("libreax_gv") | rk.status("libreax_fmha_post")
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_shards_reassemble_bitwise():
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
    assert out["gv_bitwise"], "gate-up shards differ from the single-GPU layer"
    assert out["attn_bitwise"], "attention units differ from the single-GPU output"
    assert out["status"] == 0
