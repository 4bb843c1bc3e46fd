"""bench.py's output contract, checked on the CPU: the reference arm (the CPU
restatement of the reference block timed on the host cores) prints exactly one
JSON line on stdout with the keys a benchmark driver reads, for one process
and for rank 0 of a weak-scaling multi-GPU run; other ranks print nothing.
The launch-count helper matches the kernels each batch size takes."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _run(env_extra, *args):
    env = dict(os.environ, OMP_NUM_THREADS=os.environ.get("OMP_NUM_THREADS", "4"), **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, cwd=ROOT, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [ln for ln in r.stdout.splitlines() if ln.strip()]


def test_reference_arm_prints_one_contract_line():
    lines = _run({}, "--steps", "1", "--warmup", "3", "--batch", "8")
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert REQUIRED <= d.keys(), REQUIRED - d.keys()
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["global_batch"] == 8 and d["n_gpus"] == 1


def test_reference_arm_weak_scaling_rank0_only():
    env = {"WORLD_SIZE": "2", "RANK": "0", "LOCAL_RANK": "0"}
    d = json.loads(_run(env, "--gpus", "2", "--steps", "1", "--warmup", "3", "--batch", "4")[0])
    assert d["scaling"] == "weak" and d["config"]["global_batch"] == 8  # 4 tokens per GPU x 2
    assert _run(dict(env, RANK="1", LOCAL_RANK="1"), "--gpus", "2", "--steps", "1", "--warmup", "3") == []


@pytest.mark.parametrize("T,world,expect", [
    (1, 1, 2 + 0 + 1 + 3),       # logits, fused top-k + dispatch, gather, gate/up, down, combine
    (8, 1, 2 + 0 + 1 + 3),
    (64, 1, 2 + 1 + 1 + 3),      # logits, top-k, one dispatch kernel, gather, 3 expert / combine kernels
    (128, 2, 1 + 1 + 2 + 1 + 3),  # + the expert-parallel fence and row gather
    (4096, 1, 1 + 3 + 1 + 3),    # tensor-core router, three-kernel dispatch
])
def test_launch_count(T, world, expect):
    sys.path.insert(0, ROOT)
    import bench
    assert bench.launches_per_forward(T, True, world) == expect
