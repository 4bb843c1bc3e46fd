#!/usr/bin/env python
"""bench.py -- MoE-layer throughput on B200.

Headline (the JSON line's `value`): config 1, decode.  48 stacked MoE blocks of
the Qwen3-30B-A3B-like shape (hidden 2048, 128 experts, top-8 renormalised
softmax, expert intermediate 768, SwiGLU, 4-bit affine group 64, bf16
scales/biases), single-token decode steps at batch 64, batches 1/8/32 in
`sweep`.  A step is one pass of the 48-layer chain h_{l+1} = h_l + MoE_l(h_l)
over one batch, replayed as one CUDA graph with inputs resident in HBM.

Also measured, each against its roofline:
* `prefill` (config 2): the same stack at 4096 and 16,384 tokens (batch 1
  and 4 of 4096-token sequences), against the measured bf16 tensor peak;
* `configs.config3`: E=512, K=10, I=512 with a sigmoid-gated shared expert
  (I=512), decode 64 and prefill 2048;
* `configs.config4`: config 1's shape with 8-bit weights and a Zipf(1.2)
  skewed router, decode 256 and prefill 8192, with the per-GPU pair load;
* `strong` (N > 1): config 1 decode at 64 tokens in all.

Weights and tokens come from senmoe.synth (seeded hash values in MLX layout,
identical on the CPU and the GPU): 16.3 GB (config 1), 43.5 GB (config 3)
and 30.8 GB (config 4) of packed weights, far larger than L2, so every step
streams them from HBM (no L2 flush needed).

On N GPUs (torchrun, one rank per GPU) every stack runs expert parallel:
rank r holds experts [r*E/N, (r+1)*E/N) of every layer, every rank takes the
whole batch and routes it, runs its experts' pairs, combines the batch's r-th
block of tokens reading the other ranks' expert rows over NVLink, and sends
the combined rows to every peer (senmoe.ep).  The headline batch is 64 tokens
per GPU, 64*N in all (weak scaling); `--scaling strong` keeps 64 in all.
Configs 2-4 run at their stated sizes in all.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl senmoe|reference]

`--impl reference` times the CPU restatement of the reference block (oracle/,
the reference itself is Rust + MLX/Metal and cannot run here) on all host
cores: every step is the real 48-layer residual chain over a sample of the
headline batch (its first 64 tokens), with config 1's layer 0 weights.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "sen-mlx_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

from senmoe import synth  # noqa: E402  (numpy only at import)

SPEC = synth.CONFIG1
H, E, K, I, BITS, G, LAYERS = SPEC.hidden, SPEC.experts, SPEC.top_k, SPEC.intermediate, SPEC.bits, 64, 48
METRIC = "MoE-layer decode tokens/s (48-layer stack, batch 64)"
UNIT = "tokens/s"
WORKLOAD = "config1-decode: 48 x MoE(H=2048,E=128,K=8,I=768,4-bit g64), batch 64"
REF_SAMPLE = 64  # tokens per reference-arm step

# Algorithmic bytes per touched expert (packed words + bf16 scales + biases).
BYTES_GATE_UP = 2 * (I * H * BITS // 8 + 2 * I * (H // G) * 2)
BYTES_DOWN = H * I * BITS // 8 + 2 * H * (I // G) * 2
BYTES_EXPERT = BYTES_GATE_UP + BYTES_DOWN  # 2,654,208


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense 16-bit tensor peak (TFLOP/s): the burst figure, as the expert GEMMs
    are timed as individual launches."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def measured_traffic():
    """DRAM bytes (read + write) of one gate/up launch at batch 64 from the
    committed ncu summary, or None."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", "qmma_decode_b64.md")) as f:
            m = re.search(r"traffic_bytes_per_launch_gate_up:\s*(\d+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


def headline_config(world: int, batch: int, scaling: str, layers: int) -> dict:
    """The `config` object of both arms' JSON lines."""
    return {"workload": WORKLOAD if world == 1 else
            f"{WORKLOAD} per GPU ({batch} tokens in all)" if scaling == "weak" else WORKLOAD,
            "global_batch": batch, "batch_per_gpu": batch / world, "layers": layers,
            "parallelism": f"ep{world}" if world > 1 else "single", "experts_per_gpu": E // world,
            "l2": "weights 16.3 GB per step >> 126 MB L2 (no flush needed)", "cuda_graph": True,
            "weights": "senmoe.synth seed 0 (hash-generated MLX layout)"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons during the timed region, read-only:
    NVML polled from a background thread every 5 ms (a sample from the first
    millisecond on), or `nvidia-smi -lms 20` where NVML is unavailable (its
    start-up takes ~100 ms, so short regions get few samples)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    NVML_BITS = ("nvmlClocksEventReasonHwSlowdown", "nvmlClocksEventReasonHwThermalSlowdown",
                 "nvmlClocksEventReasonSwThermalSlowdown", "nvmlClocksEventReasonSwPowerCap")

    def __init__(self, gpu_index: int, pci_bus_id: str | None = None, period_s: float = 0.005):
        self.gpu, self.pci, self.period = gpu_index, pci_bus_id, period_s
        self.proc = None
        self.nv = None
        self.samples = []   # NVML: (sm_mhz, reason bits)
        self.lines = []     # nvidia-smi: csv lines

    def __enter__(self):
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByPciBusId(self.pci) if self.pci else nv.nvmlDeviceGetHandleByIndex(self.gpu)
            self.smax = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.nv, self.stop = nv, threading.Event()

            def poll():
                while True:
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM), reasons(h)))
                    except Exception:
                        pass
                    if self.stop.wait(self.period):
                        return

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nv = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "20"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.nv is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        if self.nv is not None:
            bits = [getattr(self.nv, b, 0) for b in self.NVML_BITS]
            for mhz, r in self.samples:
                sm.append(float(mhz))
                for n, b in zip(self.NAMES, bits):
                    if b and (r & b):
                        reasons.add(n)
            smax, source = float(self.smax), "nvml"
        else:
            source = "nvidia-smi"
            for ln in self.lines:
                f = [x.strip() for x in ln.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    smax = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(self.NAMES, f[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "source": source}


def pci_bus_id(torch, device: int) -> str | None:
    """The device's PCI bus id in NVML's form, or None."""
    try:
        p = torch.cuda.get_device_properties(device)
        return f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:
        return None


# --------------------------------------------------------------- weights
def make_stack(torch, senmoe, device, spec, layers, max_tokens, rank=0, world=1, weights=None, expert_slots=0):
    """The rank's share of a synthetic `layers`-deep stack of `spec` on the
    device: this rank's experts of every layer (all of them on one GPU), the
    router and shared expert whole.  `weights` reuses already built tensors;
    `expert_slots` caps each layer's per-pair scratch (expert parallelism)."""
    from senmoe import ep
    bnd = ep.expert_bounds(spec.experts, world)
    eb, ee = bnd[rank], bnd[rank + 1]
    if weights is None:
        weights = [synth.moe_weights(spec, l, device, experts=(eb, ee)) for l in range(layers)]
    args = synth.moe_args(spec, expert_slots=expert_slots)
    blocks = [senmoe.DeepseekMoe(args, w, max_tokens=max_tokens, device=device, expert_range=(eb, ee))
              for w in weights]
    if world > 1:
        ep.connect(blocks)
    return blocks, weights


def launches_per_forward(T, tensor_cores, world, shared=False, shared_gate=False):
    """Kernels one forward launches: the router (one kernel from 128 tokens,
    where top-k runs in the logits kernel's last CTAs or the tensor-core
    router; logits + top-k below), dispatch (one kernel up to 2048 pairs,
    else three; up to 8 tokens top-k and dispatch share one launch), the
    expert-parallel fence and row gather, the gathered-activation copy
    (tensor-core paths), gate/up, down, the shared expert (two GEMV launches,
    plus the gate's dot product and sigmoid), combine."""
    router = 1 if T >= 128 else 2
    disp = 1 if (T * K + 1023) // 1024 <= 2 else 3
    if T <= 8 and T * K <= 2048:
        router, disp = 2, 0  # logits, then top-k and dispatch in one launch
    sh = (2 + (2 if shared_gate else 0)) if shared else 0
    return router + disp + (2 if world > 1 else 0) + (1 if tensor_cores else 0) + 3 + sh


# --------------------------------------------------------- CPU baseline
def _oracle_layer(spec):
    """Layer 0 of a spec as oracle (numpy) weights, built with torch on the
    host (multithreaded) and converted; same bits as the GPU arm's layer 0."""
    import numpy as np
    import torch
    from oracle import oracle as O
    t = synth.layer_tensors(spec, 0, None, "cpu")
    np_t = {k: (v.numpy().view(np.uint32) if v.dtype == torch.int32 else v.view(torch.int16).numpy().view(np.uint16))
            for k, v in t.items()}
    cfg = O.MoeConfig(hidden=spec.hidden, intermediate=spec.intermediate, num_experts=spec.experts,
                      top_k=spec.top_k, bits=spec.bits, group_size=64, shared_intermediate=spec.shared,
                      shared_gate=spec.shared_gate)
    return cfg, O.weights_from_synth(np_t)


def _host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _chain_step(O, cfg, mw, x, layers):
    h = x
    for _ in range(layers):
        h, _ = O.moe_residual(cfg, mw, h, mode=0)
    return h


def cpu_baseline(T=REF_SAMPLE, steps=3, layers=LAYERS):
    """The CPU restatement (oracle/, OpenMP over all host cores) timed on the
    headline workload: `steps` real 48-layer residual chains over the first T
    tokens of the headline batch (config 1 layer 0 weights chained), after one
    warm-up step; plus config 0 (one layer, 16 tokens) at all cores and at
    one core."""
    import numpy as np
    from oracle import oracle as O
    O.build()
    cores = _host_cores()
    O.set_threads(cores)
    cfg, mw = _oracle_layer(SPEC)
    x = synth.spec_tokens(SPEC, T)
    _chain_step(O, cfg, mw, x, layers)
    t0 = time.perf_counter()
    for _ in range(steps):
        _chain_step(O, cfg, mw, x, layers)
    per_step = (time.perf_counter() - t0) / steps
    x16 = synth.spec_tokens(SPEC, 16)
    c0 = {}
    for n in (cores, 1):
        O.set_threads(n)
        O.moe_forward(cfg, mw, x16, mode=0)
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < 2.0:
            O.moe_forward(cfg, mw, x16, mode=0)
            reps += 1
        c0["all_cores_ms" if n == cores else "one_core_ms"] = (time.perf_counter() - t0) / reps * 1e3
    O.set_threads(cores)
    c0["cores"] = cores
    return {"value": T / per_step, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{steps} steps (+1 warm-up) of the 48-layer residual chain over {T} tokens of the headline "
                      f"batch, config 1 layer-0 weights chained x{layers}, {per_step:.2f} s per step; MLX-rounding "
                      f"CPU restatement (oracle/), OpenMP on {cores} cores",
            "config0_one_layer_16_tokens": c0}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    cores = _host_cores()
    O.set_threads(cores)  # torchrun sets OMP_NUM_THREADS=1; the CPU arm takes every host core
    world = int(os.environ.get("WORLD_SIZE", "1"))
    batch = args.batch * (world if args.scaling == "weak" else 1)  # the GPU arm's whole batch
    sample = min(batch, REF_SAMPLE)
    cfg, mw = _oracle_layer(SPEC)
    x = synth.spec_tokens(SPEC, sample)
    for _ in range(args.warmup):
        _chain_step(O, cfg, mw, x, args.layers)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _chain_step(O, cfg, mw, x, args.layers)
    dt = (time.perf_counter() - t0) / args.steps
    value = sample / dt
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "u4 weights / bf16 activations (fp32 accumulate)",
            "data": "synthetic (senmoe.synth, the GPU arm's layer-0 weights and first tokens)", "impl": "reference",
            "config": headline_config(world, batch, args.scaling, args.layers),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"each step: the {args.layers}-layer residual chain h <- h + MoE(h) over the "
                                       f"first {sample} of the batch's {batch} tokens (config 1 layer 0 chained); "
                                       "CPU restatement of the reference block with MLX's rounding points "
                                       "(the reference is Rust + MLX/Metal, not runnable on this box)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


# ------------------------------------------------------------ GPU arm
_JSON_OUT = None


def emit(line: dict) -> None:
    """Writes the result line to the process's original stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


class Gpu:
    """Per-process GPU context: device, rank, world and the collective
    helpers every measurement uses (same steps on every rank)."""

    def __init__(self, torch, dist, local, rank, world):
        self.torch, self.dist, self.rank, self.world, self.local = torch, dist, rank, world, local
        self.dev = torch.device("cuda", local)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def log(self, *a):
        if self.rank == 0:
            print("[bench]", *a, file=sys.stderr, flush=True)


def timed_steps(g, stk, x, steps, warmup):
    """Device time (s) of `steps` replays of the stack's graph for x, inputs
    resident; max over ranks."""
    T = x.shape[0]
    for _ in range(warmup):
        stk.forward(x)
    g.barrier()
    s = stk.stream
    torch = g.torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(steps):
            stk.bufs[0][:T].copy_(x, non_blocking=True)
            stk._graph(T).replay()
        e1.record(s)
    e1.synchronize()
    g.barrier()
    return g.max_over_ranks(e0.elapsed_time(e1) / 1e3)


def routing_per_layer(g, lays, x, bounds):
    """Touched experts per layer and each rank's pair count per layer for
    the chain's actual routing (plain forwards on every rank)."""
    torch = g.torch
    E_ = lays[0].args.n_routed_experts
    h = x.clone()
    offs = torch.empty(E_ + 1, dtype=torch.int32, device=g.dev)
    touched, pairs = [], []
    for L in lays:
        L.forward(h, debug={"offsets": offs})
        o = offs.cpu().tolist()
        touched.append(sum(1 for e in range(E_) if o[e + 1] > o[e]))
        pairs.append([o[bounds[r + 1]] - o[bounds[r]] for r in range(len(bounds) - 1)])
        h = L.forward_residual(h)
    return touched, pairs


def stage_profile(g, lays, x, nrep):
    """Per-stage milliseconds summed over nrep steps x layers, from CUDA
    events between the stages of plain (non-graph) forwards; the host
    enqueues a whole step long before the GPU finishes it, so the deltas
    are kernel time.  The shared-expert stage is left out for layers
    without one."""
    import senmoe
    for L in lays:
        L.set_profiling(True)
    stages = [s for s in senmoe.DeepseekMoe.STAGES if s != "shared" or lays[0].args.n_shared_experts]
    acc = {k: 0.0 for k in stages}
    for _ in range(nrep):
        h = x
        for L in lays:
            h = L.forward_residual(h)
        g.torch.cuda.synchronize()
        for L in lays:
            for k, v in L.stage_times().items():
                if k in acc:
                    acc[k] += v
    for L in lays:
        L.set_profiling(False)
    return acc


def decode_point(g, spec, stk, lays, x, steps, warmup, hbm_peak, bounds, profile=True):
    """One decode batch of a stack: tokens/s, algorithmic HBM bytes of the
    touched experts (+ shared expert, router, activations) per step against
    the measured copy bandwidth of all ranks, and the per-rank pair load."""
    T = x.shape[0]
    touched, pairs = routing_per_layer(g, lays, x, bounds)
    secs = timed_steps(g, stk, x, steps, warmup)
    step = secs / steps
    per_layer = [n * spec.expert_bytes() + spec.shared_bytes() + spec.experts * spec.hidden * 2
                 + (spec.hidden * 2 if spec.shared_gate else 0) + 2 * T * spec.hidden * 2 for n in touched]
    alg = sum(per_layer)
    load = [sum(p[r] for p in pairs) / len(pairs) for r in range(g.world)]
    out = {"tokens": T, "tokens_per_s": T / step, "ms_per_step": step * 1e3,
           "touched_experts_per_layer": sum(touched) / len(touched), "alg_bytes_per_step": alg,
           "hbm_gbs": alg / step / 1e9, "hbm_frac": alg / step / 1e9 / (g.world * hbm_peak),
           "expert_kernels": __import__("senmoe").PATH_NAMES[lays[0].expert_path(T)]}
    if g.world > 1:
        out["pairs_per_gpu"] = {"mean": sum(load) / len(load), "max": max(load), "max_over_mean":
                                max(load) / max(sum(load) / len(load), 1e-9)}
    if profile:
        sp = stage_profile(g, lays, x, 3)
        out["stage_us_per_layer"] = {k: round(v / (3 * len(lays)) * 1e3, 2) for k, v in sp.items()}
    return out


def prefill_point(g, spec, stk, lays, x, steps, warmup, total_tokens=None):
    """One prefill pass of a stack: tokens/s and algorithmic TFLOP/s per GPU
    (routed experts' 6 H I flops per pair, the shared expert's per token, the
    router's 2 H E per token) against the measured bf16 burst peak.
    total_tokens: token-local stack (x holds this rank's tokens, the call
    all ranks' total_tokens); stage timings are then left out."""
    T = x.shape[0] if total_tokens is None else total_tokens
    psteps = max(2, min(steps, 5))
    secs = timed_steps(g, stk, x, psteps, warmup)
    step = secs / psteps
    Hh, Ii = spec.hidden, spec.intermediate
    flops_layer = T * spec.top_k * 6 * Hh * Ii + T * 6 * Hh * spec.shared + 2 * T * Hh * spec.experts
    peak_t, src = tensor_peak()
    per_gpu = flops_layer * len(lays) / step / 1e12 / g.world
    out = {"tokens": T, "tokens_per_s": T / step, "ms_per_step": step * 1e3, "tflops_per_gpu": per_gpu,
           "frac": per_gpu / peak_t, "peak_tflops": peak_t, "peak_source": src,
           "expert_kernels": __import__("senmoe").PATH_NAMES[lays[0].expert_path(T)],
           "scaling": None if g.world == 1 else "strong: the same tokens on every rank" if total_tokens is None
           else f"weak, token-local: {x.shape[0]} own tokens per rank"}
    if total_tokens is None:
        pst = stage_profile(g, lays, x, 2)
        gu_s = pst["gate_up"] / 1e3 / (2 * len(lays))
        dn_s = pst["down"] / 1e3 / (2 * len(lays))
        # this rank's share of the expert pairs, over its gate/up and down stage times
        out["gate_up_tflops_per_gpu"] = T * spec.top_k * 4 * Hh * Ii / g.world / gu_s / 1e12
        out["down_tflops_per_gpu"] = T * spec.top_k * 2 * Hh * Ii / g.world / dn_s / 1e12
        out["stage_share"] = {k: v / max(sum(pst.values()), 1e-12) for k, v in pst.items()}
    return out


def arena_bytes(spec, max_tokens, expert_slots=0):
    """About the scratch one layer allocates for max_tokens tokens (per
    expert slot: gathered activations, h twice, d, group sums; per pair:
    routing and permutation; per token: logits, rows)."""
    H_, I_, K_, E_ = spec.hidden, spec.intermediate, spec.top_k, spec.experts
    slots = expert_slots or max_tokens * K_
    return int(slots * (4 * H_ + 4 * I_ + H_ // 16) + max_tokens * K_ * 24 + max_tokens * (4 * E_ + 4 * H_)
               + (1 << 20))


def free_stack(g, stk, lays):
    if stk is not None:
        stk.release()
    for L in lays:
        L.close()
    g.torch.cuda.synchronize()
    g.torch.cuda.empty_cache()


def extra_config(g, senmoe, spec, layers, dec_T, pre_T, args, hbm_peak, bounds_fn):
    """Decode at dec_T and prefill at pre_T tokens (in all) of a 48-layer
    stack of `spec`, built, measured and freed."""
    lays, wts = make_stack(g.torch, senmoe, g.local, spec, layers, max(dec_T, pre_T), g.rank, g.world)
    stk = senmoe.MoeStack(lays, max(dec_T, pre_T), use_graph=True)
    bounds = bounds_fn(spec.experts)
    x = synth.spec_tokens(spec, max(dec_T, pre_T), device=g.dev)
    out = {"spec": {k: getattr(spec, k) for k in ("hidden", "experts", "top_k", "intermediate", "bits", "shared",
                                                  "shared_gate", "zipf")},
           "decode": decode_point(g, spec, stk, lays, x[:dec_T], args.steps, args.warmup, hbm_peak, bounds),
           "prefill": prefill_point(g, spec, stk, lays, x[:pre_T], args.steps, args.warmup)}
    if spec.zipf:
        _, pairs = routing_per_layer(g, lays, x[:pre_T], list(range(spec.experts + 1)))
        top = max(1, spec.experts // 10)
        shares = [sum(sorted(p, reverse=True)[:top]) / max(sum(p), 1) for p in pairs]
        out["skew"] = {"top10pct_expert_pair_share": sum(shares) / len(shares), "tokens": pre_T}
        if g.world > 1:
            _, rp = routing_per_layer(g, lays, x[:pre_T], bounds)
            load = [sum(p[r] for p in rp) / len(rp) for r in range(g.world)]
            out["prefill"]["pairs_per_gpu"] = {"mean": sum(load) / len(load), "max": max(load),
                                               "max_over_mean": max(load) / max(sum(load) / len(load), 1e-9)}
    g.log(f"{spec.name}: {out}")
    free_stack(g, stk, lays)
    del wts
    g.torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="senmoe", choices=["senmoe", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="decode batch per GPU (weak) or in all (strong)")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="N > 1: batch per GPU fixed (weak) or total batch fixed (strong)")
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-tokens", default="4096,16384",
                    help="config-2 prefill token counts (48 layers x each); empty to skip")
    ap.add_argument("--configs", default="3,4", help="extra BASELINE configs to measure (3, 4); empty to skip")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: plain (non-graph) forwards of the workload, W warm-up + K steps, no "
                         "timing or JSON")
    args = ap.parse_args()
    # stdout carries only the JSON line: anything else written to fd 1 (NCCL's
    # version banner, library prints) goes to stderr
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    import senmoe
    from senmoe import ep

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    g = Gpu(torch, dist, local, rank, world)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=g.dev)
    bounds_fn = lambda e: ep.expert_bounds(e, world)

    if args.ncu:
        layers, _keep = make_stack(torch, senmoe, local, SPEC, args.layers, args.batch, rank, world)
        x = synth.spec_tokens(SPEC, args.batch, device=g.dev)
        for _ in range(args.warmup + args.steps):
            h = x
            for L in layers:
                h = L.forward_residual(h)
        torch.cuda.synchronize()
        return

    scale = world if args.scaling == "weak" else 1
    per_gpu = args.batch
    args.batch = per_gpu * scale  # the whole batch of a step
    batches = [args.batch] if args.no_sweep else sorted({b * scale for b in (1, 8, 32, per_gpu)})
    tmax = max(batches + [64])
    layers, wts = make_stack(torch, senmoe, local, SPEC, args.layers, tmax, rank, world)
    stack = senmoe.MoeStack(layers, tmax, use_graph=True)
    x_all = synth.spec_tokens(SPEC, tmax, device=g.dev)  # the same tokens on every rank
    hbm_peak, hbm_kind = peaks()
    bounds = bounds_fn(E)

    results = {}
    clocks = None
    for T in batches:
        if T == args.batch:
            with ClockSampler(local, pci_bus_id(torch, local)) as cs:
                results[T] = decode_point(g, SPEC, stack, layers, x_all[:T], args.steps, args.warmup, hbm_peak,
                                          bounds)
            clocks = cs.summary()
        else:
            results[T] = decode_point(g, SPEC, stack, layers, x_all[:T], args.steps, args.warmup, hbm_peak, bounds)
        g.log(f"batch {T}: {results[T]}")

    # ---- dominant decode kernel (gate/up) from in-graph stage events
    T = args.batch
    nrep = max(3, min(args.steps, 10))
    stage_ms = stage_profile(g, layers, x_all[:T], nrep)
    touched, _ = routing_per_layer(g, layers, x_all[:T], bounds)
    launches = nrep * len(layers)
    gate_up_s = stage_ms["gate_up"] / 1e3 / launches
    # this rank's share of the touched experts and pairs (all of them on one GPU)
    gate_up_bytes = sum(n * BYTES_GATE_UP + T * K * (H + I) * 2 for n in touched) / len(touched) / world
    achieved = gate_up_bytes / gate_up_s / 1e9
    stage_share = {k: v / max(sum(stage_ms.values()), 1e-12) for k, v in stage_ms.items()}
    g.log(f"decode stage ms (sum over {nrep} steps x {len(layers)} layers): {stage_ms}")

    strong = token_local = None
    if world > 1:  # latency view: 64 tokens in all, each rank 1/N of the experts
        strong = decode_point(g, SPEC, stack, layers, x_all[:64], args.steps, args.warmup, hbm_peak, bounds)
        g.log(f"strong 64: {strong}")
        # token-local form: each rank routes and combines only its own tokens
        # (rank r: tokens [r * per_gpu, (r + 1) * per_gpu) of the same batch)
        lstack = senmoe.MoeStack(layers, per_gpu, use_graph=True, tokens_per_rank=[per_gpu] * world)
        secs = timed_steps(g, lstack, x_all[rank * per_gpu:(rank + 1) * per_gpu], args.steps, args.warmup)
        step = secs / args.steps
        alg = results[args.batch]["alg_bytes_per_step"]
        token_local = {"tokens": args.batch, "tokens_per_s": args.batch / step, "ms_per_step": step * 1e3,
                       "hbm_frac": alg / step / 1e9 / (world * hbm_peak),
                       "form": f"token-local: {per_gpu} own tokens per rank (senmoe_layer_forward_tokens)"}
        g.log(f"token-local decode: {token_local}")
        lstack.release()

    # ---- e2e through the public API with host buffers
    x_host = x_all[:T].cpu().pin_memory()
    for _ in range(args.warmup):
        stack.forward(x_host)
    g.barrier()
    t0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stack.stream)
    for _ in range(args.steps):
        y_host = stack.forward(x_host)  # H2D copy, graph replay, D2H copy, sync
    e1.record(stack.stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    g.barrier()
    e2e_s = g.max_over_ranks(max(e0.elapsed_time(e1) / 1e3, wall) / args.steps)
    if not torch.isfinite(y_host.float()).all():
        raise RuntimeError("non-finite output from the 48-layer chain")
    stack.release()

    # ---- config 2: prefill of the same stack (layers sharing its weights)
    prefill = {}
    for TP in [int(v) for v in args.prefill_tokens.split(",") if v.strip()]:
        pl, _ = make_stack(torch, senmoe, local, SPEC, args.layers, TP, rank, world, weights=wts)
        pstack = senmoe.MoeStack(pl, TP, use_graph=True)
        xp = synth.spec_tokens(SPEC, TP, device=g.dev)
        prefill[str(TP)] = prefill_point(g, SPEC, pstack, pl, xp, args.steps, args.warmup)
        g.log(f"prefill {TP}: {prefill[str(TP)]}")
        free_stack(g, pstack, pl)
        del xp
    # token-local prefill (N > 1): each rank its own sequence of TL tokens,
    # TL = the first prefill size unless the 48 layers' scratch for all
    # ranks' tokens would not fit the free device memory (then halved)
    if world > 1 and args.prefill_tokens.strip():
        TL = int(args.prefill_tokens.split(",")[0])
        free_b = torch.cuda.mem_get_info(g.dev)[0]
        # expert slots: twice a rank's even share of the pairs (TL * K)
        while TL > 256 and args.layers * arena_bytes(SPEC, TL * world, 2 * TL * K) > 0.7 * free_b:
            TL //= 2
        TL = int(-g.max_over_ranks(-TL))  # every rank takes the smallest
        pl, _ = make_stack(torch, senmoe, local, SPEC, args.layers, TL * world, rank, world, weights=wts,
                           expert_slots=2 * TL * K)
        pstack = senmoe.MoeStack(pl, TL, use_graph=True, tokens_per_rank=[TL] * world)
        xp = synth.spec_tokens(SPEC, TL, device=g.dev, first=rank * TL)
        prefill[f"token_local_{TL}_per_gpu"] = prefill_point(g, SPEC, pstack, pl, xp, args.steps, args.warmup,
                                                               total_tokens=TL * world)
        g.log(f"token-local prefill {TL}/GPU: {prefill[f'token_local_{TL}_per_gpu']}")
        free_stack(g, pstack, pl)
        del xp

    head = results[args.batch]
    line = {
        "metric": METRIC, "value": head["tokens_per_s"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "u4 weights / bf16 activations (fp32 accumulate)",
        "data": "synthetic (senmoe.synth: hash-generated 4-bit MLX-layout weights, x ~ N(0,1))",
        "config": headline_config(world, args.batch, args.scaling, args.layers),
        "sweep": {str(t): r for t, r in results.items()},
        "roofline": {"bound": "hbm", "kernel": f"expert gate/up (+SwiGLU), {head['expert_kernels']} path",
                     "achieved": achieved, "peak": hbm_peak,
                     "unit": "GB/s", "frac": achieved / hbm_peak,
                     "traffic": (measured_traffic() if args.batch == 64 and world == 1
                                 and head["expert_kernels"] == "mma" else None),
                     "traffic_source": "profiles/qmma_decode_b64.md (ncu dram__bytes_read+write, one launch)",
                     "peak_source": hbm_kind,
                     "algorithmic_bytes_per_launch": gate_up_bytes, "avg_launch_ms": gate_up_s * 1e3,
                     "step_hbm_gbs": head["hbm_gbs"], "step_frac": head["hbm_gbs"] / hbm_peak},
        "stage_share": stage_share,
        "strong": strong,
        "token_local": token_local,
        "prefill": prefill,
        "gpu_launches": launches_per_forward(args.batch, head["expert_kernels"] != "gemv", world) * args.layers
        * args.steps,
        "clocks": clocks,
        "e2e": {"value": args.batch / e2e_s, "unit": UNIT, "h2d_bytes_per_step": args.batch * H * 2,
                "d2h_bytes_per_step": args.batch * H * 2, "api": "senmoe.MoeStack.forward(host tensor)"},
    }

    # ---- configs 3 and 4 (config 1's weights freed first)
    for L in layers:
        L.close()
    del layers, wts, stack
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    extra = {}
    want = [c.strip() for c in args.configs.split(",") if c.strip()]
    if "3" in want:
        extra["config3"] = extra_config(g, senmoe, synth.CONFIG3, args.layers, 64, 2048, args, hbm_peak, bounds_fn)
    if "4" in want:
        extra["config4"] = extra_config(g, senmoe, synth.CONFIG4, args.layers, 256, 8192, args, hbm_peak, bounds_fn)
    line["configs"] = extra

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(T=min(args.batch, REF_SAMPLE), layers=args.layers)
    if rank == 0:
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
