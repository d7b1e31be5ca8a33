"""bench.py's reference arms on the host cores: one JSON line with the keys
the benchmark contract names (run small here; the driver runs it at 8192),
nothing from ranks other than 0, and for the one-GPU workloads the
reference's own CPU matmul rather than the GPU library."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                          capture_output=True, text=True, timeout=300, env=env, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    out = _run({}, "--size", "256", "--steps", "2", "--warmup", "1")
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1
    assert "256x256x256" in d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_stay_silent():
    out = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--size", "256", "--steps", "1")
    assert out.returncode == 0 and out.stdout.strip() == ""



@pytest.mark.parametrize("workload", ["batched", "linear", "attention"])
def test_small_workload_reference_arms(workload):
    """The one-GPU workloads' reference arm times the reference's own CPU
    matmul and backward on a sample of the step, never the GPU library."""
    out = _run({}, "--workload", workload, "--steps", "1", "--warmup", "1")
    assert out.returncode == 0, out.stderr
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["metric"] == f"{workload} fwd+bwd GEMM TFLOP/s" and d["value"] > 0
    assert d["cpu_baseline"]["cores"] == 1 and d["cpu_baseline"]["kind"] in ("reference", "port")
    assert d["e2e"]["h2d_bytes_per_step"] == 0


def test_decoder_reference_arm():
    """The decoder workload's reference arm: the reference's own CPU training
    step (drop-in build on "cpu") on one sequence, as tokens/s."""
    from macrograd_b200 import training

    if not os.path.exists(training.SEAM):
        pytest.skip("drop-in build not available (needs the reference sources at build time)")
    out = _run({}, "--workload", "decoder", "--steps", "1", "--warmup", "1")
    assert out.returncode == 0, out.stderr
    d = json.loads(out.stdout.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["value"] > 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] == 1
