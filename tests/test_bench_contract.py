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


class _FakeNvml:
    """Stands in for pynvml: a device whose SM clock and clock-event reasons
    follow a script, so the bench's sampler is tested without a GPU (read-only
    queries only; nothing here changes a setting)."""
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonSwPowerCap = 0x4
    nvmlClocksEventReasonHwSlowdown = 0x8
    nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nvmlClocksEventReasonHwThermalSlowdown = 0x40

    def __init__(self, script):
        self.script, self.i, self.calls = script, 0, []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        self.calls.append(("pci", bus))
        return "h"

    def nvmlDeviceGetHandleByIndex(self, i):
        self.calls.append(("index", i))
        return "h"

    def nvmlDeviceGetMaxClockInfo(self, h, which):
        return 1965

    def nvmlDeviceGetClockInfo(self, h, which):
        return self.script[min(self.i, len(self.script) - 1)][0]

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        r = self.script[min(self.i, len(self.script) - 1)][1]
        self.i += 1
        return r


def test_clock_sampler_reads_nvml(monkeypatch):
    import time
    sys.path.insert(0, ROOT)
    import bench
    fake = _FakeNvml([(1965, 0), (1965, 0x4), (1890, 0x4)])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(0, "00000000:1b:00.0", period_s=0.002) as cs:
        time.sleep(0.05)
    s = cs.summary()
    assert s["source"] == "nvml" and s["samples"] >= 3 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]  # power cap seen; no slowdown reason
    assert fake.calls[0] == "init" and ("pci", "00000000:1b:00.0") in fake.calls and fake.calls[-1] == "shutdown"

    fake = _FakeNvml([(1000, 0x8 | 0x40)])
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    with bench.ClockSampler(2) as cs:
        time.sleep(0.02)
    s = cs.summary()
    assert s["sm_mhz"] == 1000.0 and s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]
    assert ("index", 2) in fake.calls
