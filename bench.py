#!/usr/bin/env python
"""bench.py -- MoE-layer decode throughput on B200.

Workload: 48 stacked MoE blocks of the Qwen3-30B-A3B-like shape
(hidden 2048, 128 experts, top-8 renormalised softmax, expert intermediate
768, SwiGLU, 4-bit affine group 64, bf16 scales/biases), single-token decode
steps at batch 64 (the headline), with batches 1/8/32 reported in `sweep`.
A step is one pass of the 48-layer chain h_{l+1} = h_l + MoE_l(h_l) over one
batch.  Weights are synthetic (random 4-bit codes, per-group scales/biases
spanning the range of N(0, 0.02) weights), router N(0, 1/sqrt(H)) so logits
are ~N(0, 1), tokens x ~ N(0, 1): 16.3 GB of packed weights, far larger than
L2, so every step streams them from HBM (no L2 flush needed).

On N GPUs (torchrun, one rank per GPU) the same 48-layer stack runs expert
parallel: rank r holds experts [r*128/N, (r+1)*128/N) of every layer, every
rank takes the whole batch and routes it, runs its experts' pairs, combines
the batch's r-th block of tokens reading the other ranks' expert rows over
NVLink, and sends the combined rows to every peer (senmoe.ep).  By default
the batch is 64 tokens per GPU, 64*N in all (weak scaling: each GPU's share
of the expert pairs and of the combine stays fixed as N grows); `value` is
the whole batch's tokens/s.  `--scaling strong` keeps the batch at 64 in all.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl senmoe|reference]

`--impl reference` times the CPU restatement of the reference block
(oracle/, the reference itself is Rust + MLX/Metal and cannot run here) on
the host cores, one layer per step, scaled to the 48-layer step.
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

H, E, K, I, BITS, G, LAYERS = 2048, 128, 8, 768, 4, 64, 48
METRIC = "MoE-layer decode tokens/s (48-layer stack, batch 64)"
UNIT = "tokens/s"
WORKLOAD = "config1-decode: 48 x MoE(H=2048,E=128,K=8,I=768,4-bit g64), batch 64"

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


def tensor_peak():
    """Dense 16-bit tensor peak (TFLOP/s): the burst figure, as the expert GEMMs
    are timed as individual launches."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


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
EXPERT_CHUNK = 16  # experts generated per seed: the model is the same for N = 1, 2, 4, 8


def make_stack(torch, senmoe, device, layers, max_tokens, seed=0, rank=0, world=1):
    """Synthetic 48-layer stack in MLX layout on the device: this rank's
    experts of every layer (all of them on one GPU), the router whole."""
    from senmoe import ep
    gen = torch.Generator(device=device)
    blocks, keep = [], []
    args = senmoe.MoeArgs(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, num_experts_per_tok=K,
                          bits=BITS, group_size=G)
    bnd = ep.expert_bounds(E, world)
    eb, ee = bnd[rank], bnd[rank + 1]
    chunk = EXPERT_CHUNK if eb % EXPERT_CHUNK == 0 and ee % EXPERT_CHUNK == 0 else 1

    def proj(l, which, rows, cols, gain=1.0):
        ws, ss, bs = [], [], []
        for c0 in range(eb, ee, chunk):
            gen.manual_seed(((seed * 1000 + l) * 4 + which) * 4096 + c0 // chunk)
            ws.append(torch.randint(-2**31, 2**31 - 1, (chunk, rows, cols * BITS // 32), generator=gen,
                                    device=device, dtype=torch.int32))
            # groups of N(0, 0.02) values span about +-0.05: scale ~ 0.1/15, bias ~ -7.5 scale
            s = (torch.rand((chunk, rows, cols // G), generator=gen, device=device) * 0.002 + 0.006) * gain
            b = -(s * 7.5) + torch.randn((chunk, rows, cols // G), generator=gen, device=device) * (1e-3 * gain)
            ss.append(s.to(torch.bfloat16))
            bs.append(b.to(torch.bfloat16))
        return senmoe.SwitchLinear(torch.cat(ws), torch.cat(ss), torch.cat(bs))

    for l in range(layers):
        gen.manual_seed(seed * 1000 + l)
        rw = (torch.randn((E, H), generator=gen, device=device) / math.sqrt(H)).to(torch.bfloat16)
        # The stack has no RMSNorm between blocks (that is the caller's), so the
        # down projection is scaled to keep each block's output small next to
        # the residual stream; routing inputs then stay ~N(0, 1) at every layer.
        wt = senmoe.MoeWeights(router_weight=rw, gate_proj=proj(l, 0, I, H), up_proj=proj(l, 1, I, H),
                               down_proj=proj(l, 2, H, I, gain=0.01))
        keep.append(wt)
        blocks.append(senmoe.DeepseekMoe(args, wt, max_tokens=max_tokens, device=device, expert_range=(eb, ee)))
    if world > 1:
        ep.connect(blocks)
    return blocks, keep


def launches_per_forward(T, tensor_cores, world):
    """Kernels one forward launches: the router (one kernel from 128 tokens,
    where top-k runs in the logits kernel's last CTAs or the tensor-core
    router; logits + top-k below), dispatch (one kernel up to 2048 pairs,
    else three; up to 8 tokens top-k and dispatch share one launch), the
    expert-parallel fence and row gather, the gathered-activation copy
    (tensor-core paths), gate/up, down, combine."""
    router = 1 if T >= 128 else 2
    disp = 1 if (T * K + 1023) // 1024 <= 2 else 3
    if T <= 8 and T * K <= 2048:
        router, disp = 2, 0  # logits, then top-k and dispatch in one launch
    return router + disp + (2 if world > 1 else 0) + (1 if tensor_cores else 0) + 3


# --------------------------------------------------------- CPU baseline
def cpu_baseline(T=64, min_seconds=10.0, reps=None):
    """Times the CPU restatement (oracle/, OpenMP over all host threads) on one
    layer of the workload shape; tokens/s scaled to the 48-layer step."""
    from oracle import oracle as O
    O.build()
    cfg = O.MoeConfig(hidden=H, intermediate=I, num_experts=E, top_k=K, bits=BITS, group_size=G)
    mw = O.make_layer(cfg, seed=0, router_std=1.0 / math.sqrt(H))
    x = O.make_tokens(T, H, seed=1)
    O.moe_forward(cfg, mw, x, mode=1)  # warm
    times = []
    t_all = time.perf_counter()
    while (reps is None and time.perf_counter() - t_all < min_seconds) or (reps is not None and len(times) < reps):
        t0 = time.perf_counter()
        O.moe_forward(cfg, mw, x, mode=1)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    return {"value": T / (per_layer * LAYERS), "unit": UNIT, "cores": O.num_threads(), "kind": "port",
            "sample": f"{len(times)} forwards of one layer (H=2048,E=128,K=8,I=768,4-bit) at batch {T}, "
                      f"median {per_layer * 1e3:.1f} ms/layer, scaled x{LAYERS} layers; fp32 oracle, OpenMP"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    args.batch *= world if args.scaling == "weak" else 1  # the GPU arm's whole batch
    cfg = O.MoeConfig(hidden=H, intermediate=I, num_experts=E, top_k=K, bits=BITS, group_size=G)
    mw = O.make_layer(cfg, seed=0, router_std=1.0 / math.sqrt(H))
    x = O.make_tokens(args.batch, H, seed=1)
    for _ in range(args.warmup):
        O.moe_forward(cfg, mw, x, mode=1)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.moe_forward(cfg, mw, x, mode=1)
    dt = (time.perf_counter() - t0) / args.steps  # one layer per step
    value = args.batch / (dt * LAYERS)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * LAYERS * 1e3, "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None, "dtype": "u4/bf16 (fp32 accumulate)", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": args.batch, "layers": LAYERS},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": O.num_threads(), "kind": "port",
                             "sample": f"one layer per step ({args.steps} steps) at batch {args.batch}, scaled x48; "
                                       "CPU restatement of the reference block (the reference is Rust+MLX/Metal, "
                                       "not runnable on this box)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


# ------------------------------------------------------------ GPU arm
_JSON_OUT = None


def emit(line: dict) -> None:
    """Writes the result line to the process's original stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


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
    ap.add_argument("--prefill-tokens", type=int, default=4096,
                    help="config-2 prefill measurement (48 layers x this many tokens); 0 to skip")
    ap.add_argument("--ncu", action="store_true",
                    help="profiling mode: plain (non-graph) forwards of the workload, W warm-up + K steps, no "
                         "timing or JSON; every step launches 6 kernels per layer in order")
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

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.ncu:
        layers, _keep = make_stack(torch, senmoe, local, args.layers, args.batch, rank=rank, world=world)
        x = torch.randn((args.batch, H), device=dev).to(torch.bfloat16)
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
    tmax = max(batches)
    layers, _keep = make_stack(torch, senmoe, local, args.layers, tmax, rank=rank, world=world)
    stack = senmoe.MoeStack(layers, tmax, use_graph=True)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)  # the same tokens on every rank
    x_all = torch.randn((max(tmax, args.prefill_tokens), H), generator=gen, device=dev).to(torch.bfloat16)

    def timed_steps(stk, T, steps, warmup):
        """Device time of `steps` replays of the 48-layer chain, inputs resident."""
        x = x_all[:T]
        for _ in range(warmup):
            stk.forward(x)
        barrier()
        s = stk.stream
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(steps):
                stk.bufs[0][:T].copy_(x, non_blocking=True)
                stk._graph(T).replay()
            e1.record(s)
        e1.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1) / 1e3)

    def touched_per_layer(lays, T):
        """Touched experts per layer for the chain's actual routing."""
        h = x_all[:T].clone()
        offs = torch.empty(E + 1, dtype=torch.int32, device=dev)
        counts = []
        for L in lays:
            L.forward(h, debug={"offsets": offs})
            counts.append(int((offs[1:] - offs[:-1] > 0).sum().item()))
            h = L.forward_residual(h)
        return counts

    def stage_profile(lays, T, nrep):
        """Per-stage milliseconds summed over nrep steps x layers, from CUDA
        events between the stages of plain (non-graph) forwards; the host
        enqueues a whole step long before the GPU finishes it, so the deltas
        are kernel time."""
        for L in lays:
            L.set_profiling(True)
        x = x_all[:T]
        acc = {k: 0.0 for k in senmoe.DeepseekMoe.STAGES}
        for _ in range(nrep):
            h = x
            for L in lays:
                h = L.forward_residual(h)
            torch.cuda.synchronize()
            for L in lays:
                for k, v in L.stage_times().items():
                    acc[k] += v
        for L in lays:
            L.set_profiling(False)
        return acc

    hbm_peak, hbm_kind = peaks()
    results = {}
    clocks = None
    for T in batches:
        touched = touched_per_layer(layers, T)
        if T == args.batch:
            with ClockSampler(local, pci_bus_id(torch, local)) as cs:
                secs = timed_steps(stack, T, args.steps, args.warmup)
            clocks = cs.summary()
        else:
            secs = timed_steps(stack, T, args.steps, args.warmup)
        step = secs / args.steps
        alg_bytes = sum(n * BYTES_EXPERT + E * H * 2 + 2 * T * H * 2 for n in touched)
        sp = stage_profile(layers, T, 3)
        per_layer_us = {k: round(v / (3 * len(layers)) * 1e3, 2) for k, v in sp.items()}
        results[T] = {"tokens_per_s": T / step, "ms_per_step": step * 1e3,
                      "expert_kernels": senmoe.PATH_NAMES[layers[0].expert_path(T)],
                      "stage_us_per_layer": per_layer_us,
                      "touched_experts_per_layer": sum(touched) / len(touched),
                      "hbm_gbs": alg_bytes / step / 1e9, "hbm_frac": alg_bytes / step / 1e9 / (world * hbm_peak)}
        if rank == 0:
            print(f"[bench] batch {T}: {results[T]}", file=sys.stderr, flush=True)

    # ---- dominant decode kernel (gate/up) from in-graph stage events
    T = args.batch
    nrep = max(3, min(args.steps, 10))
    stage_ms = stage_profile(layers, T, nrep)
    touched = touched_per_layer(layers, T)
    launches = nrep * len(layers)
    gate_up_s = stage_ms["gate_up"] / 1e3 / launches
    # this rank's share of the touched experts and pairs (all of them on one GPU)
    gate_up_bytes = sum(n * BYTES_GATE_UP + T * K * (H + I) * 2 for n in touched) / len(touched) / world
    achieved = gate_up_bytes / gate_up_s / 1e9
    stage_share = {k: v / max(sum(stage_ms.values()), 1e-12) for k, v in stage_ms.items()}
    if rank == 0:
        print(f"[bench] decode stage ms (sum over {nrep} steps x {len(layers)} layers): {stage_ms}",
              file=sys.stderr, flush=True)

    # ---- prefill (config 2): 48 layers x prefill_tokens, tensor-core roofline
    prefill = None
    if args.prefill_tokens > 0:
        TP = args.prefill_tokens
        pl = [senmoe.DeepseekMoe(L.args, L.weights, max_tokens=TP, device=local, expert_range=L.expert_range)
              for L in layers]
        if world > 1:
            from senmoe import ep
            ep.connect(pl)
        pstack = senmoe.MoeStack(pl, TP, use_graph=True)
        psteps = max(2, min(args.steps, 5))
        secs = timed_steps(pstack, TP, psteps, args.warmup)
        step = secs / psteps
        flops_layer = TP * K * 6 * H * I + 2 * TP * H * E
        pst = stage_profile(pl, TP, 2)
        gu_s = pst["gate_up"] / 1e3 / (2 * len(pl))
        dn_s = pst["down"] / 1e3 / (2 * len(pl))
        peak_t = tensor_peak()
        prefill = {"tokens": TP, "tokens_per_s": TP / step, "ms_per_step": step * 1e3,
                   "tflops": flops_layer * len(pl) / step / 1e12,
                   "frac": flops_layer * len(pl) / step / 1e12 / (world * peak_t[0]),
                   "gate_up_tflops": TP * K * 4 * H * I / gu_s / 1e12,
                   "down_tflops": TP * K * 2 * H * I / dn_s / 1e12,
                   "peak_tflops": peak_t[0], "peak_source": peak_t[1],
                   "stage_share": {k: v / max(sum(pst.values()), 1e-12) for k, v in pst.items()}}
        if rank == 0:
            print(f"[bench] prefill: {prefill}", file=sys.stderr, flush=True)
        pstack.release()
        for L in pl:
            L.close()
        del pl

    # ---- e2e through the public API with host buffers
    x_host = x_all[:T].cpu().pin_memory()
    for _ in range(args.warmup):
        stack.forward(x_host)
    barrier()
    t0 = time.perf_counter()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stack.stream)
    for _ in range(args.steps):
        y_host = stack.forward(x_host)  # H2D copy, graph replay, D2H copy, sync
    e1.record(stack.stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    e2e_s = max_over_ranks(max(e0.elapsed_time(e1) / 1e3, wall) / args.steps)
    if not torch.isfinite(y_host.float()).all():
        raise RuntimeError("non-finite output from the 48-layer chain")

    head = results[args.batch]
    line = {
        "metric": METRIC, "value": head["tokens_per_s"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "u4 weights / bf16 activations (fp32 accumulate)",
        "data": "synthetic (random-init 4-bit MLX-layout weights, x ~ N(0,1))",
        "config": {"workload": WORKLOAD if world == 1 else
                   f"{WORKLOAD} per GPU ({args.batch} tokens in all)" if args.scaling == "weak" else WORKLOAD,
                   "global_batch": args.batch, "batch_per_gpu": args.batch / world, "layers": args.layers,
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "experts_per_gpu": E // world,
                   "l2": "weights 16.3 GB per step >> 126 MB L2 (no flush needed)", "cuda_graph": True},
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
        "prefill": prefill,
        "gpu_launches": launches_per_forward(args.batch, head["expert_kernels"] != "gemv", world) * args.layers
        * args.steps,
        "clocks": clocks,
        "e2e": {"value": args.batch / e2e_s, "unit": UNIT, "h2d_bytes_per_step": args.batch * H * 2,
                "d2h_bytes_per_step": args.batch * H * 2, "api": "senmoe.MoeStack.forward(host tensor)"},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(T=args.batch)
    stack.release()
    if rank == 0:
        emit(line)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
