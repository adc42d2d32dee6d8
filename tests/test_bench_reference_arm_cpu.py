"""The benchmark's reference arm (`bench.py --impl reference`) on CPU: the driver runs it beside the GPU arm, so its
one JSON line must carry the GPU arm's metric, unit and config with the reference-arm keys (impl, cpu_baseline, e2e
with zero copy bytes), and under torchrun every rank but 0 must exit without work or output."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--cpu-seconds-per-step", "0.3"], capture_output=True, text=True, env=env,
                       timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.strip()]


def test_reference_arm_line():
    lines = _run({})
    assert len(lines) == 1
    d = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench

    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "TFLOP/s"
    assert d["higher_is_better"] is True and d["n_gpus"] == 1 and d["value"] > 0
    assert d["config"]["workload"].startswith("gate-up GEMM") and d["config"]["N2_per_gpu"] == bench.N2
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the second reference point (the reference's sm_100a kernels on the GPU) is reported, or says why not
    assert "kernels" in d["reference_kernels"] or "unavailable" in d["reference_kernels"]


def test_reference_arm_other_ranks_are_silent():
    assert _run({"WORLD_SIZE": "2", "RANK": "1"}) == []
