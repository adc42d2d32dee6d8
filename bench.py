#!/usr/bin/env python
"""Benchmark of the REAX kernel set on B200 (driver contract: one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--scaling strong|weak]

Headline workload (the configuration the metric is quoted on): the gate-up GEMM with the fused
SiLU*mul epilogue, X [2048, 4096] ~ N(0,1), gate/up weights [14336, 4096] each ~ N(0, 0.02) packed into reax_gv's
interleaved layout, bf16 output [2048, 14336], fp32 accumulation.  One step = one reax_gv call per rank.

Multi-GPU (torchrun, one process per GPU; NCCL carries the barrier, the MAX of the timings and -- outside every timed
region -- an all-gather that reassembles the sharded outputs for a bitwise check against one GPU's full output):
  strong (default): BASELINE's own splits -- config 2 column-parallel along N2 (14336/N columns per rank, whole groups
                    of 4 gate/up features), config 3 by (batch x kv-head) units (32/N per rank), config 1 by head,
                    config 4 along N;
  weak:             every rank runs a config-2-sized shard of an N-times wider layer (and full attention shapes).
The config-5 linear-attention kernels run the full BASELINE shapes on every rank (replicas).

Timing: W untimed warm-up steps, then K steps each bracketed by CUDA events on the launching stream, the L2 cache
flushed (a 256 MiB write) between steps outside the events, a barrier + synchronize before and after; the per-rank
sums are reduced with MAX over ranks.  `value` = total FLOPs of the job / that time.

Parity: rank 0 at N=1 runs the CPU-baseline leg, which times the fp64 oracle on a bounded row sample and then, as the
checker, compares every leg's device output with it on sampled rows (outside all timed regions): the `parity` object.

--impl reference: the reference kernels are GPU-only (sm_120 sources, no CPU path), so the reference arm is the fp64
C++ restatement of their math (oracle/, multithreaded over all host cores), each step a bounded row sample of the
same workload; rank 0 alone runs it.  When the reference's own kernels built for sm_100a (oracle/_ref) and a GPU are
present, the same line also carries their device times at the BASELINE shapes (`reference_kernels`); this arm's
`reference_point_shapes` counterpart is in the main line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K, N2 = 2048, 4096, 14336
SEED = 0x5EED0000 + 2
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "gate-up GEMM (fused SiLU*mul) TFLOP/s, whole job"
# the kernel reax_gv runs at config 2 on a 148-SM B200: 256 x 256 tiles on CTA pairs (cta_group::2 MMAs), 896 tiles
# on 74 pairs = 12.1 waves, the k-blocks of the last two waves and the partial one shared out evenly
GV_KERNEL = "gemm_kernel<256,6,EPI_GV,split,pair> (CTA pairs, cta_group::2)"
ATTN = dict(B=4, Hkv=8, G=4, S=8192, D=128)   # GQA causal prefill, Hq = 32
ATTN1 = dict(B=1, Hkv=8, G=1, S=1024, D=128)  # causal MHA
SLICED = dict(K=4096, N=4096, S=4, Ms=(16, 256, 4096))  # BASELINE config 4 (S = 4 slices of 1024)
LINEAR = dict(B=2, S=16384, H=16, HV=32, D=128, hidden=2048)  # BASELINE config 5 (linear-attention block)
FLUSH_BYTES = 256 << 20


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return FALLBACK_PEAKS, "fallback"


def traffic_per_launch(name):
    """DRAM bytes (read + write) of one launch of a bench workload, from the committed ncu summaries."""
    p = os.path.join(ROOT, "profiles", "dram_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(name, {}).get("dram_bytes_per_launch")
    return None


class ClockSampler:
    """SM clock and clock-event (throttle) reasons read through NVML every 2 ms by a background thread while the
    timed region runs (read-only queries; no GPU setting is touched)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap",
               "hw_power_brake": "nvmlClocksEventReasonHwPowerBrakeSlowdown"}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.max_mhz = None
        self.stop = None
        self.err = None

    def __enter__(self):
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            bits = {k: getattr(nv, v) for k, v in self.REASONS.items()}

            def poll():
                while not self.stop.is_set():
                    try:
                        mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                        r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, [k for k, b in bits.items() if r & b]))
                    except Exception as e:  # pragma: no cover
                        self.err = str(e)
                    self.stop.wait(0.002)

            self.stop = threading.Event()
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
        except Exception as e:  # pragma: no cover
            self.err = str(e)
        return self

    def __exit__(self, *a):
        if self.stop is not None:
            self.stop.set()
            self.t.join(1.0)

    def summary(self):
        sm = [m for m, _ in self.samples]
        reasons = sorted({r for _, rs in self.samples for r in rs})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
               "samples": len(sm), "source": "NVML, 2 ms polling during the timed region"}
        if self.err:
            out["error"] = self.err
        return out


# ------------------------------------------------------------------------------------------------ process group
def dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    from reax_engine_kernels_b200 import dist as rd

    rd.barrier(world, device="cuda")


def max_over_ranks(x, world):
    from reax_engine_kernels_b200 import dist as rd

    return rd.max_over_ranks(x, world, device="cuda")


class Ctx:
    """Per-process state shared by the legs."""

    def __init__(self, args, world, rank, local):
        import torch

        self.args, self.world, self.rank, self.local = args, world, rank, local
        self.stream = torch.cuda.current_stream()
        self.flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
        self.pk, self.pk_kind = peaks()
        self.keep = {}  # device outputs kept for the parity checks of the CPU-baseline leg (rank 0, N = 1)

    @property
    def strong(self):
        return self.args.scaling == "strong"

    def timed(self, fn, steps, flush=True, sleep_ns=50_000_000):
        """Per-launch device times (ms) of `fn` on the current stream: warm-up, barrier, then `steps` launches each
        between two CUDA events, the L2 flushed before each (outside the events) when `flush`; the GPU is kept
        busy while the host enqueues so no host gap falls inside an event pair."""
        import torch

        for _ in range(self.args.warmup):
            fn()
        barrier(self.world)
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        torch.cuda._sleep(sleep_ns)
        for a, b in evs:
            if flush:
                self.flush.zero_()
            a.record(self.stream)
            fn()
            b.record(self.stream)
        barrier(self.world)
        return [a.elapsed_time(b) for a, b in evs]

    def gather_check(self, local_flat, full_fn, reorder=None):
        """Reassembly check: all-gather every rank's output shard (a flat tensor; shards padded to the largest) over
        NCCL and compare, on rank 0, the reassembled output with `full_fn()` -- the whole problem run on rank 0's
        GPU alone -- bit for bit.  `reorder(list of per-rank shards)` builds the full output from the shards.  Runs
        outside every timed region; every rank takes the same collective steps."""
        import torch
        import torch.distributed as dist

        if self.world == 1:
            return None
        n = torch.tensor([local_flat.numel()], dtype=torch.int64, device="cuda")
        sizes = [torch.zeros_like(n) for _ in range(self.world)]
        dist.all_gather(sizes, n)
        sizes = [int(s.item()) for s in sizes]
        mx = max(sizes)
        buf = torch.zeros(mx, dtype=local_flat.dtype, device="cuda")
        buf[:local_flat.numel()] = local_flat
        out = torch.empty(self.world * mx, dtype=local_flat.dtype, device="cuda")
        dist.all_gather_into_tensor(out, buf)
        ok = None
        if self.rank == 0:
            shards = [out[r * mx:r * mx + sizes[r]] for r in range(self.world)]
            whole = reorder(shards) if reorder else torch.cat(shards)
            full = full_fn().reshape(-1)
            ok = bool(whole.numel() == full.numel() and torch.equal(whole.view(torch.int16), full.view(torch.int16)))
        del out, buf
        torch.cuda.synchronize()
        barrier(self.world)
        return ok

    def roof_tensor(self, flops, ms, kernel):
        ach = flops / (ms * 1e-3) / 1e12
        return {"bound": "tensor", "achieved": round(ach, 2), "peak": self.pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": round(ach / self.pk["bf16_tflops"], 4),
                "peak_source": f"{self.pk_kind} bf16 burst (kernel timed alone)", "kernel": kernel,
                "algorithmic_flops_per_launch": flops}

    def roof_hbm(self, nbytes, ms, kernel):
        gbs = nbytes / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(gbs, 1), "peak": self.pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(gbs / self.pk["hbm_gbs"], 4), "peak_source": f"{self.pk_kind} HBM copy bandwidth",
                "kernel": kernel, "algorithmic_bytes_per_launch": int(nbytes)}


# ------------------------------------------------------------------------------------------------ config 2 (headline)
def gate_up_weights():
    """The packed gate/up weights of the full config-2 layer (every rank generates the same layer)."""
    import torch

    from reax_engine_kernels_b200 import synth

    wg = synth.device_normal_bf16((N2, K), 0.02, SEED + 1000)
    wu = synth.device_normal_bf16((N2, K), 0.02, SEED + 1001)
    w = torch.stack([wg.view(N2 // 4, 4, K), wu.view(N2 // 4, 4, K)], 1).reshape(2 * N2, K)
    del wg, wu
    return w


def leg_gate_up(c):
    """Config 2 through the C ABI (reax_gv): device-resident timing, the end-to-end loop with host buffers, the
    reassembly check.  Returns the headline fields of the JSON line."""
    import torch
    import torch.distributed as dist

    from reax_engine_kernels_b200 import abi, synth
    from reax_engine_kernels_b200 import dist as rd

    args, world, rank = c.args, c.world, c.rank
    lib = abi.load("libreax_gv")
    s = c.stream.cuda_stream
    x = synth.device_normal_bf16((M, K), 1.0, SEED)
    w_full = None
    if c.strong:
        cols, rows = rd.gate_up_columns(N2, world, rank), rd.gate_up_weight_rows(N2, world, rank)
        w_full = gate_up_weights()
        w = w_full[rows.start:rows.stop].contiguous()
        if rank != 0 or world == 1:
            w_full = None
        n2 = cols.size
    else:
        n2 = N2
        wg = synth.device_normal_bf16((n2, K), 0.02, SEED + 1000 + 2 * rank)
        wu = synth.device_normal_bf16((n2, K), 0.02, SEED + 1001 + 2 * rank)
        w = torch.stack([wg.view(n2 // 4, 4, K), wu.view(n2 // 4, 4, K)], 1).reshape(2 * n2, K).contiguous()
        del wg, wu
    torch.cuda.empty_cache()
    out = torch.empty(M, n2, dtype=torch.bfloat16, device="cuda")
    flops_rank = 2.0 * M * (2 * n2) * K
    flops_job = 2.0 * M * 2 * N2 * K * (1 if c.strong else world)

    def step(xb=x, ob=out):
        rc = lib.reax_gv(args.cfg, xb.data_ptr(), w.data_ptr(), ob.data_ptr(), M, n2, K, s)
        if rc:
            raise RuntimeError(f"reax_gv returned {rc}")

    with ClockSampler(c.local) as clk:
        times = c.timed(step, args.steps, flush=True, sleep_ns=100_000_000)
    clocks = clk.summary()
    total_ms = max_over_ranks(sum(times), world)
    mean_launch_ms = sum(times) / len(times)
    status = lib.reax_b200_status(s)
    if status:
        raise RuntimeError(f"device status word {status:#x}")

    # ---- end to end: the C-ABI call with host buffers (pinned), copies inside the timed region.  The packed weights
    # are the layer's parameters and stay resident, as the engine holds them; every step's input (activations X)
    # crosses host->device and its result (this rank's [M, n2] activation output) device->host.  Steps are pipelined
    # as a serving loop runs them: host->device copies on one stream, the kernel on the compute stream, the
    # device->host copies on a third, with two device buffers each for X and the output.
    # With the layer split over N ranks (strong scaling), every rank needs all of X: each rank brings its M / N rows in
    # from the host and an NCCL all-gather over NVLink assembles X on every GPU -- the exchange a column-parallel layer
    # makes -- instead of N ranks each pulling the whole of X through their host links.
    gather_x = c.strong and world > 1 and M % world == 0
    xr = rd.split_even(M, world, rank) if gather_x else None
    x_h = torch.empty_like(x[xr.start:xr.stop] if gather_x else x, device="cpu").pin_memory()
    x_h.copy_(x[xr.start:xr.stop] if gather_x else x)
    out_h = torch.empty(M, n2, dtype=torch.bfloat16).pin_memory()
    x_ds = [torch.empty_like(x) for _ in range(2)]
    x_sl = [torch.empty(x_h.shape, dtype=x.dtype, device="cuda") for _ in range(2)] if gather_x else None
    out_ds = [torch.empty_like(out) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_run(nsteps, start_ev=None, end_ev=None):
        comp_done, out_done = [None, None], [None, None]
        if start_ev is not None:
            s_in.wait_event(start_ev)
        for i in range(nsteps):
            b = i & 1
            with torch.cuda.stream(s_in):
                if comp_done[b] is not None:
                    s_in.wait_event(comp_done[b])  # the kernel of step i-2 has finished reading x_ds[b]
                if gather_x:
                    x_sl[b].copy_(x_h, non_blocking=True)
                    dist.all_gather_into_tensor(x_ds[b], x_sl[b])  # ordered after the copy, before e_in, on s_in
                else:
                    x_ds[b].copy_(x_h, non_blocking=True)
                e_in = torch.cuda.Event()
                e_in.record(s_in)
            c.stream.wait_event(e_in)
            if out_done[b] is not None:
                c.stream.wait_event(out_done[b])  # step i-2's result has left out_ds[b]
            step(x_ds[b], out_ds[b])
            e_c = torch.cuda.Event()
            e_c.record(c.stream)
            comp_done[b] = e_c
            with torch.cuda.stream(s_out):
                s_out.wait_event(e_c)
                out_h.copy_(out_ds[b], non_blocking=True)
                e_o = torch.cuda.Event()
                e_o.record(s_out)
                out_done[b] = e_o
        if end_ev is not None:
            end_ev.record(s_out)  # after the last result copy, which follows every kernel and input copy
        torch.cuda.synchronize()

    e2e_run(args.warmup)
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(100_000_000)
    e0.record(c.stream)
    e2e_run(args.steps, e0, e1)
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_bitwise = bool(torch.equal(out_h.view(torch.int16), out.cpu().view(torch.int16)))
    h2d_bytes = x_h.numel() * x_h.element_size()
    del x_h, out_h, x_ds, out_ds, x_sl

    # ---- reassembly check (strong scaling): shards all-gathered over NCCL, compared with rank 0's full layer
    reassembled = None
    if c.strong and world > 1:
        def reorder(shards):
            return torch.cat([sh.view(M, -1) for sh in shards], 1).reshape(-1)

        def full():
            f = torch.empty(M, N2, dtype=torch.bfloat16, device="cuda")
            assert lib.reax_gv(args.cfg, x.data_ptr(), w_full.data_ptr(), f.data_ptr(), M, N2, K, s) == 0
            return f

        reassembled = c.gather_check(out.reshape(-1), full, reorder)
    if world == 1:
        c.keep["gv"] = (x, w, out)
        c.keep["gv_ms"] = mean_launch_ms
    w_full = None

    achieved = flops_rank / (mean_launch_ms * 1e-3) / 1e12
    roof = c.roof_tensor(flops_rank, mean_launch_ms, GV_KERNEL)
    roof["traffic"] = traffic_per_launch("gv_config2") if n2 == N2 else None
    res = {
        "metric": METRIC,
        "value": round(flops_job * args.steps / (total_ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 5),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights, generated on device)",
        "config": {"workload": "gate-up GEMM + SiLU*mul, BASELINE config 2", "M": M, "K": K,
                   "N2_total": N2 if c.strong else N2 * world, "N2_per_gpu": n2, "cfg": args.cfg,
                   "parallelism": f"column-parallel along N2 x{world} ({args.scaling})",
                   "l2": "flushed between timed steps (256 MiB write outside the events)"},
        "per_gpu_tflops": round(achieved, 2),
        "pct_bf16_peak": round(100.0 * achieved / c.pk["bf16_tflops"], 1),
        "roofline": roof,
        "e2e": {"value": round(flops_job * args.steps / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": out.numel() * 2,
                "result_bitwise_equal_to_device_run": e2e_bitwise,
                "x_all_gathered_over_nccl": gather_x,
                "path": "ctypes reax_gv (C ABI), pinned host X in (with N > 1 ranks: this rank's M/N rows, then an "
                        "NCCL all-gather of X over NVLink) / this rank's output out every step, weights resident; "
                        "steps pipelined over three streams (input copy, kernel, result copy; two device buffers "
                        "each), as a serving loop runs them"},
        "gpu_launches": args.steps * 2,
        "clocks": clocks,
    }
    if reassembled is not None:
        res["reassembled_bitwise"] = reassembled
    return res


# ------------------------------------------------------------------------------------------------ attention
def attn_flops(B, Hkv, G, S, D):
    """4 * D * (visible (row, key) pairs): causal, row r of a kv head sees keys 0..r/G."""
    return 4.0 * D * B * Hkv * G * S * (S + 1) / 2


def _attention_problem(cfg, seed, D):
    import torch

    from reax_engine_kernels_b200 import synth

    B, H, G, S = cfg["B"], cfg["Hkv"], cfg["G"], cfg["S"]
    Mr = S * G
    q = synth.device_normal_bf16((B, H, Mr, D), 1.0, seed)
    k = synth.device_normal_bf16((B, H, S, D), 1.0, seed + 1)
    v = synth.device_normal_bf16((B, H, S, D), 1.0, seed + 2)
    qpos = torch.arange(S, dtype=torch.int32, device="cuda").repeat(B, 1).contiguous()
    return q, k, v, qpos


def _attention_step(c, q, k, v, qpos, o, G, units, D):
    """One rank's (batch, kv head) units: one reax_fmha_q_hd call per batch segment of consecutive heads."""
    from reax_engine_kernels_b200 import abi

    lib = abi.load("libreax_fmha_post")
    st = c.stream.cuda_stream
    H = q.shape[1]
    Mr = q.shape[2]
    S = k.shape[2]
    scale = 1.0 / math.sqrt(D)
    segs = {}
    for b, h in units:
        segs.setdefault(b, []).append(h)
    calls = []  # (b0, b1, h0, h1): one launch over batches [b0, b1) x heads [h0, h1)
    for b, hs in segs.items():
        h0, h1 = min(hs), max(hs) + 1
        assert hs == list(range(h0, h1))
        if calls and (h0, h1) == (0, H) and calls[-1][2:] == (0, H) and calls[-1][1] == b:
            calls[-1] = (calls[-1][0], b + 1, 0, H)  # whole batches merge into one launch
        else:
            calls.append((b, b + 1, h0, h1))
    strides = lambda t: (t.stride(0), t.stride(1), t.stride(2))

    def step():
        for b0, b1, h0, h1 in calls:
            qq, kk, vv, oo = q[b0:b1, h0:h1], k[b0:b1, h0:h1], v[b0:b1, h0:h1], o[b0:b1, h0:h1]
            rc = lib.reax_fmha_q_hd(qq.data_ptr(), kk.data_ptr(), vv.data_ptr(), qpos[b0:b1].data_ptr(), G, S,
                                    oo.data_ptr(), scale, b1 - b0, h1 - h0, Mr, S, *strides(qq), *strides(kk),
                                    *strides(vv), *strides(oo), D, st)
            if rc:
                raise RuntimeError(f"reax_fmha_q_hd returned {rc}")

    return step, len(calls)


def leg_attention(c, cfg, seed, label, D=None, flush=True, steps=None, keep=None, shard=True, floor=False):
    """Attention (qpos mode, causal) through reax_fmha_q_hd.  strong: the rank's (batch x kv-head) units of the
    BASELINE shape; weak: the full shape on every rank.  Reassembly over NCCL checked against rank 0's full run.
    floor: also time an empty kernel (torch's spin kernel for 0 cycles) the same way -- after the same L2 flush,
    between the same two events -- which is the least any launch can measure here, and the TFLOP/s it would allow."""
    import torch

    from reax_engine_kernels_b200 import dist as rd

    world, rank = c.world, c.rank
    B, H, G, S = cfg["B"], cfg["Hkv"], cfg["G"], cfg["S"]
    D = D or cfg["D"]
    q, k, v, qpos = _attention_problem(cfg, seed, D)
    o = torch.zeros_like(q)
    split = c.strong and shard
    units = rd.attention_units(B, H, world, rank) if split else [(b, h) for b in range(B) for h in range(H)]
    step, ncalls = _attention_step(c, q, k, v, qpos, o, G, units, D)
    steps = steps or max(3, c.args.steps // 10)
    times = c.timed(step, steps, flush=flush)
    total_ms = max_over_ranks(sum(times), world)
    fl_rank = attn_flops(1, len(units), G, S, D)
    fl_job = attn_flops(B, H, G, S, D) * (1 if split else world)
    ms = sum(times) / steps
    two_tile = D == 128 and (S * G // 256) * len(units) >= 2 * 148
    res = {"workload": label, "value": round(fl_job * steps / (total_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "steps": steps, "ms_per_step": round(total_ms / steps, 5), "units_per_rank": len(units),
           "per_gpu_tflops": round(fl_rank / (ms * 1e-3) / 1e12, 2),
           "roofline": c.roof_tensor(fl_rank, ms, "fmha2_kernel<1,true>" if two_tile else f"fmha_kernel<{D},1,true>"),
           "l2": "flushed between launches (256 MiB write)" if flush else "inputs larger than L2 per step",
           "gpu_launches": steps * ncalls}
    if floor:
        ft = c.timed(lambda: torch.cuda._sleep(0), steps, flush=flush)
        fms = sum(ft) / len(ft)
        res["launch_floor"] = {"ms": round(fms, 5), "tflops_if_kernel_took_no_time": round(fl_rank / (fms * 1e-3) / 1e12, 1),
                               "what": "an empty kernel timed like the leg: the per-launch cost no kernel can go below"}
    if split and world > 1:
        ulo = rd.split_even(B * H, world, rank)
        flat = o.view(B * H, -1)[ulo.start:ulo.stop].reshape(-1)

        def full():
            f = torch.zeros_like(q)
            st, _ = _attention_step(c, q, k, v, qpos, f, G, [(b, h) for b in range(B) for h in range(H)], D)
            st()
            return f

        res["reassembled_bitwise"] = c.gather_check(flat, full)
    if keep and world == 1:
        c.keep[keep] = (q, k, v, qpos, o, G)
    return res


# ------------------------------------------------------------------------------------------------ config 4
def leg_gate_up_shards(c):
    """The config-2 shard that one rank of an N-GPU strong-scaling job runs (N = 2, 4, 8: N2 / N output columns),
    timed on this GPU, with the single-GPU time of the whole layer from the headline leg.  reax_gv runs 256 x 256
    tiles on CTA pairs (74 pairs on 148 SMs): a shard leaves 6.05, 3.03 or 1.51 waves of them, and the k-blocks of the
    last waves are shared out evenly (partial accumulators handed between clusters through scratch memory).  Each
    shard's output is checked bit for bit against its columns of the whole layer (the layer of the headline leg), and
    each shard is also timed on the one-SM kernel (REAX_GEMM_PAIR=0) and with the split turned off, as comparisons."""
    import torch

    from reax_engine_kernels_b200 import abi
    from reax_engine_kernels_b200 import dist as rd

    x, w, full_out = c.keep["gv"]
    lib = abi.load("libreax_gv")
    s = c.stream.cuda_stream
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    out = {"note": "per-rank shard of BASELINE config 2 on one GPU; projected_efficiency = whole-layer time / "
                   "(N x shard time), i.e. the strong-scaling efficiency an N-GPU job of these shards would reach "
                   "with no other cost"}
    launches = 0
    for world in (2, 4, 8):
        cols, rows = rd.gate_up_columns(N2, world, 0), rd.gate_up_weight_rows(N2, world, 0)
        n2 = cols.size
        ws = w[rows.start:rows.stop]
        o = torch.empty(M, n2, dtype=torch.bfloat16, device="cuda")

        def step(ws=ws, o=o, n2=n2):
            rc = lib.reax_gv(c.args.cfg, x.data_ptr(), ws.data_ptr(), o.data_ptr(), M, n2, K, s)
            if rc:
                raise RuntimeError(f"reax_gv returned {rc}")

        tiles = (M // 256) * (2 * n2 // 256)  # pair tiles
        t_default = c.timed(step, c.args.steps)
        launches += c.args.steps
        bitwise = bool(torch.equal(o.view(torch.int16), full_out[:, cols.start:cols.stop].view(torch.int16)))
        other = {}
        for name, env in (("unsplit_ms", {"REAX_GEMM_SPLIT": "0"}), ("one_sm_ms", {"REAX_GEMM_PAIR": "0"})):
            old = {k: os.environ.get(k) for k in env}
            os.environ.update(env)
            try:
                t = c.timed(step, c.args.steps)
                launches += c.args.steps
            finally:
                for k, v in old.items():
                    if v is None:
                        del os.environ[k]
                    else:
                        os.environ[k] = v
            other[name] = round(sum(t) / len(t), 5)
            bitwise = bitwise and bool(torch.equal(o.view(torch.int16),
                                                   full_out[:, cols.start:cols.stop].view(torch.int16)))
        ms = sum(t_default) / len(t_default)
        flops = 2.0 * M * 2 * n2 * K
        out[f"N={world}"] = {
            "N2_per_gpu": n2, "pair_tiles": tiles, "waves": round(tiles / (sms // 2), 3),
            "split_last_waves": bool(tiles > sms // 2 and tiles % (sms // 2)),
            "ms": round(ms, 5), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            **other,
            "projected_efficiency": round(c.keep["gv_ms"] / (world * ms), 3),
            "bitwise_equal_to_full_layer_columns": bitwise,
        }
    status = lib.reax_b200_status(s)
    if status:
        raise RuntimeError(f"device status word {status:#x}")
    out["gpu_launches"] = launches
    return out


def leg_sliced(c):
    """reax_slices over all 16 SLICE_CFGS indices x M in {16, 256, 4096}, K = N = 4096, S = 4 slices
    of 1024, bf16 partials.  strong: N split column-parallel over the ranks.  Per M: the time of every cfg (L2 flushed
    between launches), the roofline of the best (HBM for M = 16: W is read once; tensor otherwise); every cfg's output
    is checked bitwise against cfg 0's outside the timed region."""
    import torch

    from reax_engine_kernels_b200 import abi, synth
    from reax_engine_kernels_b200 import dist as rd

    Kc, Nc, S = SLICED["K"], SLICED["N"], SLICED["S"]
    kps = Kc // S
    lib = abi.load("libreax_slices")
    st = c.stream.cuda_stream
    ncol = rd.split_even(Nc, c.world, c.rank, granule=16) if c.strong else rd.Shard(0, Nc)
    n = ncol.size
    w_full = synth.device_normal_bf16((Nc, Kc), 0.02, 0x5EED0000 + 4 + 1)
    w = w_full[ncol.start:ncol.stop].contiguous()
    steps = max(3, c.args.steps // 4)
    out = {}
    launches = 0
    all_identical = True
    for Mi in SLICED["Ms"]:
        x = synth.device_normal_bf16((Mi, Kc), 1.0, 0x5EED0000 + 4 + Mi)
        p = torch.empty(S, Mi, n, dtype=torch.bfloat16, device="cuda")
        ref = None
        per_cfg = []
        for cfg in range(16):
            def step(cfg=cfg):
                rc = lib.reax_slices(cfg, 0, x.data_ptr(), w.data_ptr(), p.data_ptr(), Mi, n, kps, S, Kc, st)
                if rc:
                    raise RuntimeError(f"reax_slices returned {rc}")

            times = c.timed(step, steps, flush=True, sleep_ns=5_000_000)
            launches += steps
            per_cfg.append(max_over_ranks(sum(times) / steps, c.world))
            if ref is None:
                ref = p.clone()
            elif not torch.equal(p.view(torch.int16), ref.view(torch.int16)):
                all_identical = False
        best = min(range(16), key=lambda i: per_cfg[i])
        ms = per_cfg[best]
        fl_rank = 2.0 * Mi * n * Kc
        fl_job = 2.0 * Mi * Nc * Kc * (1 if c.strong else c.world)
        nbytes = 2 * Mi * Kc + 2 * n * Kc + S * Mi * n * 2
        kern = ("gemm_kernel<32,10,EPI_BF16_T> (swapped, M <= 64)" if Mi <= 64 else
                "gemm_kernel<BN,ST,EPI_BF16> (one SM per tile, M <= 256)" if Mi <= 256 else
                "gemm_kernel<BN,ST,EPI_BF16> (CTA pairs)")
        roof = c.roof_hbm(nbytes, ms, kern) if Mi <= 64 else c.roof_tensor(fl_rank, ms, kern)
        e = {"ms_best": round(ms, 5), "best_cfg": best, "ms_mean_over_cfgs": round(sum(per_cfg) / 16, 5),
             "ms_worst": round(max(per_cfg), 5), "value": round(fl_job / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
             "roofline": roof}
        if c.strong and c.world > 1:
            def full(x=x, Mi=Mi):
                f = torch.empty(S, Mi, Nc, dtype=torch.bfloat16, device="cuda")
                assert lib.reax_slices(0, 0, x.data_ptr(), w_full.data_ptr(), f.data_ptr(), Mi, Nc, kps, S, Kc, st) == 0
                return f

            def reorder(shards, Mi=Mi):
                return torch.cat([sh.view(S, Mi, -1) for sh in shards], 2).reshape(-1)

            e["reassembled_bitwise"] = c.gather_check(ref.reshape(-1), full, reorder)
        if c.world == 1:
            c.keep[f"sliced_{Mi}"] = (x, w, ref)
        out[f"M={Mi}"] = e
    return {"workload": "sliced GEMM sweep, BASELINE config 4 (K = N = 4096, S = 4 x 1024, bf16 partials, cfg 0-15)",
            "per_M": out, "all_cfgs_bitwise_identical": all_identical, "steps_per_cfg": steps,
            "l2": "flushed between launches (256 MiB write)", "gpu_launches": launches}


# ------------------------------------------------------------------------------------------------ config 5
def leg_linear(c):
    """Memory-bound leg (B=2 x 16384 tokens, 16 key heads / 32 value heads of 128): the RMSNorm
    (reax_rarn), depthwise conv + SiLU + L2 (reax_conv_l2), KKT inverse (reax_kkt), chunked delta rule (reax_howu)
    and the delta rule with the gated RMSNorm (reax_howu_norm), each timed alone with the L2 flushed between launches;
    achieved = algorithmic DRAM bytes / mean launch time, against the measured HBM copy bandwidth.  Every rank runs
    the full shapes (replicas, no collective)."""
    import numpy as np
    import torch

    from reax_engine_kernels_b200 import kernels as rk, synth

    L = LINEAR
    T, hid = L["B"] * L["S"], L["hidden"]
    KD = VD = L["H"] * L["D"]
    SX = 2 * KD + VD
    seed = 0x5EED0000 + 5 + 131 * c.rank
    steps = max(3, c.args.steps // 10)
    out = {}

    def run(name, kernel, fn, nbytes, what):
        ms = max_over_ranks(sum(c.timed(fn, steps)) / steps, c.world)
        out[name] = {"kernel": kernel, "ms": round(ms, 4), "algorithmic_bytes": int(nbytes), "bytes": what,
                     "roofline": c.roof_hbm(nbytes, ms, kernel)}

    part = synth.device_normal_bf16((2, T, hid), 0.5, seed)
    res = synth.device_normal_bf16((T, hid), 1.0, seed + 1)
    wn = synth.device_normal_bf16((hid,), 0.1, seed + 2, mean=1.0)
    h = torch.empty(T, hid, dtype=torch.bfloat16, device="cuda")
    o = torch.empty_like(h)
    run("rmsnorm", "rarn_kernel", lambda: rk.rarn(part, res, wn, 1e-6, 1.0 / hid, h_out=h, out=o), 5 * T * hid * 2,
        "2 partials + residual read, h + normed written (bf16)")
    if c.world == 1:
        c.keep["rarn"] = (part, res, wn, h, o)
    qkv = synth.device_normal_bf16((T, SX), 1.0, seed + 3)
    cw = synth.device_normal_bf16((SX, 4), 0.5, seed + 4)
    meta = torch.from_numpy(np.array([(p_, 0, s_ * L["S"], 0) for s_ in range(L["B"]) for p_ in range(L["S"])],
                                     np.int32)).cuda()
    q = torch.empty(T, KD, dtype=torch.bfloat16, device="cuda")
    k = torch.empty_like(q)
    v = torch.empty(T, VD, dtype=torch.bfloat16, device="cuda")
    run("conv", "conv_kernel<1,false>", lambda: rk.conv_l2(qkv, meta, cw, KD, VD, q=q, k=k, v=v), T * SX * 2 * 2,
        "qkv read once, q/k/v written once (bf16)")
    if c.world == 1:
        c.keep["conv"] = (qkv, meta, cw, q, k, v, KD, VD)
    d = synth.delta_rule_inputs([L["S"]] * L["B"], L["H"], L["HV"], seed + 5)
    kt = synth.to_torch_bf16(d["k"])
    g = torch.from_numpy(d["g"]).cuda()
    beta = synth.to_torch_bf16(d["beta"])
    cu = torch.from_numpy(d["cu"]).cuda()
    cidx = torch.from_numpy(d["cidx"]).cuda()
    A = torch.zeros(T, L["HV"], 64, dtype=torch.bfloat16, device="cuda")
    run("kkt", "kkt_kernel", lambda: rk.kkt(kt, g, beta, cu, cidx, L["HV"], A=A),
        T * L["H"] * 128 * 2 + T * L["HV"] * 6 + T * L["HV"] * 40 * 2,
        "k read, g/beta read, the 10 written 16x16 blocks of A (40 of 64 columns per row on average)")
    qq = synth.to_torch_bf16(d["q"])
    vv = synth.device_normal_bf16((T, L["HV"], 128), 1.0, seed + 6)
    oo = torch.empty_like(vv)
    sc = 1 / math.sqrt(128)
    hb = T * (2 * L["H"] * 128 * 2 + 2 * L["HV"] * 128 * 2 + L["HV"] * 64 * 2)
    run("delta_rule", "howu_tc_kernel", lambda: rk.howu(qq, kt, vv, beta, A, g, cu, sc, o=oo), hb,
        "q, k, v, A read, o written (bf16)")
    # the gated-RMSNorm entry: every token's row is written (f2s = identity), z [T, HV*128] read, out written
    f2s = torch.arange(T, dtype=torch.int32, device="cuda")
    z = synth.device_normal_bf16((T, L["HV"] * 128), 1.0, seed + 7)
    nw = synth.device_normal_bf16((128,), 0.1, seed + 8, mean=1.0)
    on = torch.empty(T, L["HV"], 128, dtype=torch.bfloat16, device="cuda")
    run("delta_rule_norm", "howu_tc_kernel (reax_howu_norm)",
        lambda: rk.howu_norm(qq, kt, vv, beta, A, g, cu, sc, f2s, z, nw, 1e-6, 1.0 / 128, on),
        hb + T * L["HV"] * 128 * 2 + T * 4, "q, k, v, A, z, f2s read, normed o written (bf16)")
    if c.world == 1:
        c.keep["delta"] = (d, A, vv, oo, z, nw, on, sc)
        c.keep["delta_dev"] = (qq, kt, beta, g, cu, f2s)
    return {"workload": "linear-attention block, BASELINE config 5 (B=2, S=16384, 16 heads x 128)", "steps": steps,
            "parallelism": "replicas (every rank runs the full shapes)",
            "l2": "flushed between launches (256 MiB write)", "kernels": out, "gpu_launches": 5 * steps}


def leg_reference_point_shapes(c):
    """This package's kernels at the shapes the reference arm's `reference_kernels` times the reference's own sm_100a
    build on (where BASELINE's shape is one the reference cannot run, its nearest runnable shape): attention at head
    dim 256 on the config-3 shape, RMSNorm at D = 2560, the config-5 qkv projection as a plain GEMM."""
    import torch

    from reax_engine_kernels_b200 import kernels as rk, synth

    steps = max(3, c.args.steps // 10)
    out = {}
    a = leg_attention(c, ATTN, 0x5EED0000 + 33, "config 3 at head dim 256", D=256, steps=steps, shard=False)
    out["fmha_q_d256"] = {"ms": a["ms_per_step"], "tflops": a["per_gpu_tflops"]}
    n, D = 32768, 2560
    part = synth.device_normal_bf16((2, n, D), 0.5, 7)
    res = synth.device_normal_bf16((n, D), 1.0, 8)
    wn = synth.device_normal_bf16((D,), 0.1, 9, mean=1.0)
    h, o = torch.empty(n, D, dtype=torch.bfloat16, device="cuda"), torch.empty(n, D, dtype=torch.bfloat16, device="cuda")
    ms = sum(c.timed(lambda: rk.rarn(part, res, wn, 1e-6, 1.0 / D, h_out=h, out=o), steps)) / steps
    out["rarn_d2560"] = {"ms": round(ms, 4), "gbs": round(5 * n * D * 2 / ms / 1e6, 1)}
    del part, res, h, o
    Mp, Kp, Np = 32768, 2048, 6144
    x = synth.device_normal_bf16((Mp, Kp), 1.0, 3)
    w = synth.device_normal_bf16((Np, Kp), 0.02, 4)
    dd = torch.empty(Mp, Np, dtype=torch.bfloat16, device="cuda")
    ms = sum(c.timed(lambda: rk.gemm(x, w, cfg=0, out=dd), steps)) / steps
    out["gemm_qkv_projection"] = {"ms": round(ms, 4), "tflops": round(2.0 * Mp * Np * Kp / ms / 1e9, 1),
                                  "roofline": c.roof_tensor(2.0 * Mp * Np * Kp, ms, "gemm_kernel<256,6,EPI_BF16,pair> (CTA pairs)")}
    return {"what": "ours at the reference arm's reference_kernels shapes (per GPU)", "steps": steps, "kernels": out,
            "gpu_launches": steps * 3}


# ------------------------------------------------------------------------------------------------ CPU leg
def calibrate_rows(fn, seconds, limit=M):
    """Rows of X whose oracle evaluation takes about `seconds` on this host (at least 1, at most `limit`)."""
    t0 = time.perf_counter()
    fn(2)
    t1 = time.perf_counter()
    fn(10)
    t2 = time.perf_counter()
    per_row = max(((t2 - t1) - (t1 - t0)) / 8, (t2 - t1) / 10 * 0.5, 1e-4)
    return int(min(limit, max(1, round(seconds / per_row))))


def cpu_baseline(c, seconds):
    """The fp64 C++ oracle on the host cores: (1) timed on a bounded row sample of the headline workload (the CPU
    baseline); (2) as the checker, every leg's device output compared with it on sampled rows -- the parity objects.
    Runs after every timed region (rank 0, N = 1)."""
    import numpy as np
    import torch

    from oracle import oracle as orc
    from oracle.tolerance import parity_stats
    from reax_engine_kernels_b200 import synth

    bf = synth.bf16_bits_to_f32
    h = synth.from_torch_bf16
    cores = len(os.sched_getaffinity(0))
    orc.set_threads(cores)
    parity = {}
    x, w, out = c.keep["gv"]
    wh, xh = h(w), h(x)
    n2 = wh.shape[0] // 2
    rows = calibrate_rows(lambda r: orc.gv(xh[:r], wh, intervals=False), seconds)
    t0 = time.perf_counter()
    orc.gv(xh[:rows], wh, intervals=False)
    dt = time.perf_counter() - t0
    base = {"value": round(2.0 * rows * 2 * n2 * K / dt / 1e12, 6), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of {M} rows x all {n2} outputs x K={K} (fp64 oracle, {dt:.1f} s)"}
    # ---- gate-up: rows at M-tile edges and the last tile, with the rounding interval
    sel = np.r_[0:4, 126:130, 1022:1026, 2044:2048]
    ref, lo, hi = orc.gv(np.ascontiguousarray(xh[sel]), wh)
    parity["gate_up"] = parity_stats(bf(h(out)[sel]), bf(ref), bf(lo), bf(hi))
    # ---- attention, configs 3 and 1: sampled query rows of every (batch, kv head), with the interval
    for key, rsel in (("attention", ((0, 4), (252, 260), (32764, 32768))), ("attention_config1", ((0, 1024),))):
        if key not in c.keep:
            continue
        q, k, v, qpos, o, G = c.keep[key]
        qh, kh, vh, oh = h(q), h(k), h(v), h(o)
        S = kh.shape[2]
        ys, rs, los, his = [], [], [], []
        for r0, r1 in rsel:
            ref, lo, hi = orc.fmha(qh, kh, vh, 1.0 / math.sqrt(qh.shape[3]), qpos=qpos.cpu().numpy(), G=G, qpBs=S,
                                   rows=(r0, r1), intervals=True)
            sl = (slice(None), slice(None), slice(r0, r1))
            ys.append(bf(oh[sl]).ravel())
            rs.append(bf(ref[sl]).ravel())
            los.append(bf(lo[sl]).ravel())
            his.append(bf(hi[sl]).ravel())
        parity[key] = parity_stats(np.concatenate(ys), np.concatenate(rs), np.concatenate(los), np.concatenate(his))
    # ---- sliced GEMM (cfg 0; every cfg was checked bitwise equal to it): rows of each M
    for Mi in SLICED["Ms"]:
        if f"sliced_{Mi}" not in c.keep:
            continue
        x4, w4, p4 = c.keep[f"sliced_{Mi}"]
        r = np.r_[0:min(Mi, 16)] if Mi <= 256 else np.r_[0:4, 2046:2050, 4092:4096]
        ref = orc.slices(np.ascontiguousarray(h(x4)[r]), h(w4), SLICED["S"], SLICED["K"] // SLICED["S"],
                         part_fp32=False)
        parity[f"sliced_M{Mi}"] = parity_stats(bf(h(p4)[:, r]), bf(ref))
    if "rarn" in c.keep:
        # ---- config 5: RMSNorm rows, conv tokens, KKT chunks, the delta rule on a prefix of one sequence / key head
        part, res, wn, hh, o = c.keep["rarn"]
        n_, D_ = 256, part.shape[2]
        ph = np.ascontiguousarray(h(part[:, :n_]))
        _, ref = orc.rarn(ph, 2, 0, n_ * D_, h(res[:n_]), h(wn), n_, D_, 1e-6, 1.0 / D_)
        parity["rmsnorm"] = parity_stats(bf(h(o[:n_])), bf(ref))
        qkv, meta, cw, q, k, v, KD, VD = c.keep["conv"]
        Tf = 2048
        rq, rk_, rv = orc.conv(h(qkv[:Tf]), qkv.shape[1], None, 0, meta[:Tf].cpu().numpy(), h(cw), Tf, 1e-6, KD, VD,
                               1, 0)
        parity["conv"] = parity_stats(bf(np.concatenate([h(q[:Tf]), h(k[:Tf]), h(v[:Tf])], 1)),
                                      bf(np.concatenate([rq, rk_, rv], 1)))
        d, A, vv, oo, z, nw, on, sc = c.keep["delta"]
        Tp = 2048  # prefix of sequence 0: its first 32 chunks depend on nothing after them
        Ar = orc.kkt(d["k"][:Tp], d["g"][:Tp], d["beta"][:Tp], np.array([0, Tp], np.int64),
                     np.array([(0, j) for j in range(Tp // 64)], np.int64), LINEAR["H"], LINEAR["HV"])
        parity["kkt"] = parity_stats(bf(h(A[:Tp])), bf(Ar))
        H1, HV1 = 1, 2  # key head 0 and its value heads 0, 1
        sub = lambda a, nh: np.ascontiguousarray(a[:Tp, :nh])
        Ah, vh = h(A[:Tp]), h(vv[:Tp])
        args = (sub(d["q"], H1), sub(d["k"], H1), sub(vh, HV1), sub(d["beta"], HV1), sub(Ah, HV1), sub(d["g"], HV1),
                np.array([0, Tp], np.int64), sc, H1, HV1)
        oref = orc.howu(*args)
        zs = np.ascontiguousarray(h(z[:Tp]).reshape(Tp, -1, 128)[:, :HV1].reshape(Tp, -1))
        nref = orc.howu(*args, norm=dict(f2s=np.arange(Tp, dtype=np.int32), z=zs, ZS=zs.shape[1], nw=h(nw), eps=1e-6,
                                         factor=1.0 / 128, rows=Tp))
        theirs = reference_delta_rule(c, oo, on)
        if theirs is None:
            parity["delta_rule"] = parity_stats(bf(h(oo[:Tp, :HV1])), bf(oref))
            parity["delta_rule_norm"] = parity_stats(bf(h(on[:Tp, :HV1])), bf(nref))
        else:
            # the chain criterion, pinned to the reference's own kernel run on the same inputs (oracle/tolerance.py)
            from oracle.tolerance import reference_matched_stats

            t_o, t_n = theirs
            for key, ours_t, ref_t, orc_o in (("delta_rule", oo, t_o, oref), ("delta_rule_norm", on, t_n, nref)):
                st = reference_matched_stats(bf(h(ours_t[:Tp, :HV1])), bf(orc_o), bf(h(ref_t[:Tp, :HV1])))
                st["bitwise_equal_to_reference_kernel_frac_all_outputs"] = float(
                    (ours_t.view(torch.int16) == ref_t.view(torch.int16)).float().mean())
                parity[key] = st
    return base, parity


def reference_delta_rule(c, oo, on):
    """The reference's own reax_howu / reax_howu_norm (oracle/_ref, built for sm_100a) on the bench's config-5 inputs,
    as the checker of the delta-rule parity; None when that build is absent."""
    import ctypes as C

    import torch

    from oracle.build import ref_path

    if not os.path.exists(ref_path("libreax_howu")) or "delta_dev" not in c.keep:
        return None
    d, A, vv, _, z, nw, _, sc = c.keep["delta"]
    qq, kt, beta, g, cu, f2s = c.keep["delta_dev"]
    ref = C.CDLL(ref_path("libreax_howu"))
    P = lambda t: C.c_void_p(t.data_ptr())
    s = C.c_void_p(c.stream.cuda_stream)
    H, HV = LINEAR["H"], LINEAR["HV"]
    t_o, t_n = torch.empty_like(oo), torch.empty_like(on)
    rc = ref.reax_howu(P(qq), P(kt), P(vv), P(beta), P(A), P(g), P(t_o), P(cu), C.c_float(sc), C.c_int(LINEAR["B"]),
                       C.c_int(H), C.c_int(HV), s)
    rc |= ref.reax_howu_norm(P(qq), P(kt), P(vv), P(beta), P(A), P(g), P(t_n), P(cu), C.c_float(sc),
                             C.c_int(LINEAR["B"]), C.c_int(H), C.c_int(HV), s, P(f2s), P(z), C.c_longlong(z.stride(0)),
                             P(nw), C.c_float(1e-6), C.c_float(1.0 / 128))
    torch.cuda.synchronize()
    return None if rc else (t_o, t_n)


# ------------------------------------------------------------------------------------------------ reference arm
def run_reference(args, world, rank):
    """Reference arm: the fp64 C++ restatement of reax_gv on all host cores, a bounded row sample per step (the
    reference has no CPU path).  Also, when a GPU and oracle/_ref are present, the reference's own kernels built for
    sm_100a timed on this GPU at the BASELINE shapes (a second reference point; never feeds `value`)."""
    if rank != 0:
        return None
    import numpy as np

    from oracle import oracle as orc
    from reax_engine_kernels_b200 import synth

    n2 = N2 if args.scaling == "weak" else -(-N2 // world)
    rng = np.random.default_rng(SEED)
    bfn = lambda shape, std: synth.f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
    wh = synth.gv_pack_g4(bfn((n2, K), 0.02), bfn((n2, K), 0.02))
    cores = len(os.sched_getaffinity(0))
    orc.set_threads(cores)
    rows = calibrate_rows(lambda r: orc.gv(bfn((r, K), 1.0), wh, intervals=False), args.cpu_seconds_per_step)
    xs = bfn((rows, K), 1.0)
    for _ in range(args.warmup):
        orc.gv(xs, wh, intervals=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.gv(xs, wh, intervals=False)
    dt = time.perf_counter() - t0
    flops = 2.0 * rows * 2 * n2 * K
    v = round(flops * args.steps / dt / 1e12, 6)
    res = {
        "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * dt / args.steps, 3), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "bf16 in / fp64 math", "data": "synthetic (seeded, host generator)",
        "config": {"workload": "gate-up GEMM + SiLU*mul, BASELINE config 2", "M": M, "K": K, "N2_per_gpu": n2,
                   "sample_rows_per_step": rows},
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": f"{rows} of {M} rows x all {n2} outputs x K={K} per step"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference ships GPU-only sm_120 kernels without a CPU path; this arm is the fp64 C++ oracle",
    }
    if not args.no_reference_kernels:
        try:
            from oracle import ref_kernels

            res["reference_kernels"] = ref_kernels.time_all(args.ref_kernel_steps)
        except Exception as e:  # the second reference point is optional (no GPU, no oracle/_ref)
            res["reference_kernels"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong")
    ap.add_argument("--cfg", type=int, default=0)
    ap.add_argument("--no-shards", action="store_true", help="skip the config-2 per-rank shard leg (N = 1 only)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample size (seconds of oracle work)")
    ap.add_argument("--cpu-seconds-per-step", type=float, default=3.0, help="reference arm: oracle seconds per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-attention", action="store_true", help="skip the attention legs (configs 3 and 1)")
    ap.add_argument("--no-sliced", action="store_true", help="skip the sliced-GEMM leg (config 4)")
    ap.add_argument("--no-linear", action="store_true", help="skip the linear-attention leg (config 5)")
    ap.add_argument("--no-reference-shapes", action="store_true", help="skip ours at the reference arm's shapes")
    ap.add_argument("--no-reference-kernels", action="store_true", help="reference arm: skip the oracle/_ref GPU timing")
    ap.add_argument("--ref-kernel-steps", type=int, default=5)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        res = run_reference(args, world, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup()
    try:
        c = Ctx(args, world, rank, local)
        res = leg_gate_up(c)
        if world == 1 and c.strong and not args.no_shards:
            res["gate_up_shards"] = leg_gate_up_shards(c)
            res["gpu_launches"] += res["gate_up_shards"].pop("gpu_launches")
        if not args.no_attention:
            res["attention"] = leg_attention(c, ATTN, 0x5EED0000 + 3,
                                             "GQA causal prefill attention, BASELINE config 3 (B=4, S=8192, Hq=32, "
                                             "Hkv=8, D=128)", keep="attention")
            res["attention_config1"] = leg_attention(c, ATTN1, 0x5EED0000 + 1,
                                                     "causal MHA attention, BASELINE config 1 (B=1, S=1024, H=8, "
                                                     "D=128)", steps=max(5, args.steps // 2), keep="attention_config1",
                                                     floor=True)
            res["gpu_launches"] += res["attention"]["gpu_launches"] + res["attention_config1"]["gpu_launches"]
        if not args.no_sliced:
            res["sliced"] = leg_sliced(c)
            res["gpu_launches"] += res["sliced"]["gpu_launches"]
        if not args.no_linear:
            res["linear_attention"] = leg_linear(c)
            res["gpu_launches"] += res["linear_attention"]["gpu_launches"]
        if not args.no_reference_shapes:
            res["reference_point_shapes"] = leg_reference_point_shapes(c)
            res["gpu_launches"] += res["reference_point_shapes"]["gpu_launches"]
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            base, parity = cpu_baseline(c, args.cpu_seconds)
            res["cpu_baseline"] = base
            res["parity"] = parity
            res["parity_all_within_tolerance"] = all(p["within_tolerance"] for p in parity.values())
        c.keep.clear()
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        del torch


if __name__ == "__main__":
    main()
