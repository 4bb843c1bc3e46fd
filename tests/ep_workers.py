"""Rank bodies for the expert-parallel tests, run as spawned processes
(one per rank) joined in a torch.distributed group on 127.0.0.1.

CPU ranks use gloo; GPU ranks bind one GPU each and still use gloo for the
host-side table exchange (the data path is the library's peer-memory combine).
"""
from __future__ import annotations

import bisect
import hashlib
import os
import socket
import traceback
from datetime import timedelta

import numpy as np

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _entry(rank, world, port, fn_name, args, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        try:
            q.put((rank, "ok", globals()[fn_name](rank, world, *args)))
        finally:
            dist.destroy_process_group()
    except BaseException:
        q.put((rank, "err", traceback.format_exc()))


def spawn_ranks(fn_name: str, world: int, *args, timeout: float = 240.0) -> list:
    """Runs ``fn_name(rank, world, *args)`` on ``world`` spawned ranks and
    returns their results in rank order; raises with a rank's traceback."""
    import multiprocessing as mp
    import queue

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, world, port, fn_name, args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results, errors = {}, []
    try:
        for _ in range(world):
            rank, status, val = q.get(timeout=timeout)
            if status == "ok":
                results[rank] = val
            else:
                errors.append(f"rank {rank}:\n{val}")
    except queue.Empty:
        errors.append(f"ranks timed out after {timeout} s (got {sorted(results)})")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()  # this test's own child, by handle
                p.join()
    if errors:
        raise AssertionError("\n".join(errors))
    return [results[r] for r in range(world)]


# ------------------------------------------------------------------ CPU ranks
class FakeLayer:
    """Stands in for DeepseekMoe in the table exchange: a blob per (rank, layer)."""

    def __init__(self, rank: int, index: int):
        self.rank, self.index, self.connected = rank, index, None

    def peer_info(self) -> bytes:
        return f"r{self.rank}l{self.index}".encode()

    def connect_peers(self, rank: int, infos: list) -> None:
        self.connected = (rank, [b.decode() for b in infos])


def exchange(rank, world, n_layers, extra_on_rank=-1):
    from senmoe import ep

    layers = [FakeLayer(rank, i) for i in range(n_layers + (1 if rank == extra_on_rank else 0))]
    ep.connect(layers)
    return [L.connected for L in layers]


def decomposition(rank, world, bits):
    """The expert-parallel data flow on the CPU: every rank routes all tokens,
    computes the rows of its own experts at their global slots, the rows are
    all-gathered, each rank combines its own block of tokens (every pair's
    row from its owner, in slot order) and the combined rows are
    all-gathered into y.  Returns this rank's y (fp32)."""
    import torch
    import torch.distributed as dist

    from helpers import fixture_layer
    from oracle import numpy_ref as N
    from senmoe import ep

    d = np.load(os.path.join(GOLD, f"moe_block_small_{bits}bit.npz"))
    cfg, w = fixture_layer(d)
    H, E, K, g = cfg.hidden, cfg.num_experts, cfg.top_k, cfg.group_size
    x = N.bf16_val(d["x"]).reshape(-1, H)
    T, P = x.shape[0], x.shape[0] * K
    ids, wts = N.route(cfg, w, x)
    b = ep.expert_bounds(E, world)
    eb, ee = b[rank], b[rank + 1]
    # global slots: stable counting sort of the pairs by expert
    order = np.argsort(ids.reshape(-1), kind="stable")
    slot = np.empty(P, dtype=np.int64)
    slot[order] = np.arange(P)
    gd = N.dequantize(w.gate_w[eb:ee], w.gate_s[eb:ee], w.gate_b[eb:ee], g, cfg.bits).astype(np.float64)
    ud = N.dequantize(w.up_w[eb:ee], w.up_s[eb:ee], w.up_b[eb:ee], g, cfg.bits).astype(np.float64)
    dd = N.dequantize(w.down_w[eb:ee], w.down_s[eb:ee], w.down_b[eb:ee], g, cfg.bits).astype(np.float64)
    rows = np.zeros((P, H), dtype=np.float32)
    for p in range(P):
        e = int(ids.reshape(-1)[p])
        if eb <= e < ee:
            rows[slot[p]] = N.expert_mlp(x[p // K].astype(np.float64), gd[e - eb], ud[e - eb], dd[e - eb])
    gathered = [torch.zeros(P, H) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(rows))
    tb = [T * r // world for r in range(world + 1)]  # token blocks, as ep_token_begin
    mine = np.zeros((T, H), dtype=np.float32)
    sh = N.shared_out(cfg, w, x) if cfg.shared_intermediate else None
    for t in range(tb[rank], tb[rank + 1]):
        acc = np.zeros(H, dtype=np.float32)
        for j in range(K):
            p = t * K + j
            owner = bisect.bisect_right(b, int(ids[t, j])) - 1
            acc = (acc + gathered[owner][slot[p]].numpy() * wts[t, j]).astype(np.float32)
        mine[t] = acc if sh is None else (acc + sh[t]).astype(np.float32)
    blocks = [torch.zeros(T, H) for _ in range(world)]
    dist.all_gather(blocks, torch.from_numpy(mine))
    y = np.zeros((T, H), dtype=np.float32)
    for r in range(world):
        y[tb[r]:tb[r + 1]] = blocks[r].numpy()[tb[r]:tb[r + 1]]
    return y


# ------------------------------------------------------------------ GPU ranks
def two_cta_form(args, T, world, sms):
    """Whether a forward of T tokens takes the warp-MMA kernel's two-CTA
    (64-row) group-scaled form, by the layer's own choice (layer.cu: tokens
    per touched local expert, slots per tile, and whether the 128-row gate/up
    tiles fill the SMs).  An expert-parallel rank holds E / world experts, so
    it can take that form where one GPU does not; the two forms add a row's
    k-partitions in a different order (equal within the block tolerance, not
    bit for bit)."""
    K, E, I = args.num_experts_per_tok, args.n_routed_experts, args.moe_intermediate_size
    P = T * K
    e_local = E // world if world > 1 else E
    pairs = P * e_local // E if world > 1 else P
    pairs = max(pairs, 1)
    pe = pairs / min(pairs, e_local)
    tc_min = 16.0 if args.bits == 4 else 24.0  # layer.cu tc_min_tokens_per_expert
    if args.expert_path not in (0, 3) or (args.expert_path == 0 and pe >= tc_min):
        return False  # not the warp-MMA path
    return (args.bits == 4 and pe <= 8.0 and args.mma_form == 0 and min(P, e_local) * (I // 128) < sms)


def _gpu_setup(rank, world, H, I, E, K, bits, T, shared, seed, skew=False):
    import torch

    from helpers import device_weights, moe_args
    from oracle import oracle as O

    torch.cuda.set_device(rank)
    cfg = O.MoeConfig(hidden=H, intermediate=I, num_experts=E, top_k=K, bits=bits,
                      shared_intermediate=shared, shared_gate=bool(shared))
    mw = O.make_layer(cfg, seed=seed, router_std=1.0 / np.sqrt(H))
    x = O.make_tokens(T, H, seed=seed + 1)
    if skew:
        # Zipf(1.2) pull toward the low expert ids: x's column 0 is the
        # constant 1 and Wg's column 0 holds the per-expert offset, so a few
        # experts get many more slots than the mean (the hybrid split)
        x = x.copy()
        x[:, 0] = O.f32_to_bf16(np.ones(T, dtype=np.float32))
        rw = O.bf16_to_f32(mw.router_w)
        rw[:, 0] = 3.0 / np.arange(1, E + 1, dtype=np.float32) ** 1.2
        mw.router_w = O.f32_to_bf16(rw.astype(np.float32))
    return cfg, mw, x, moe_args(cfg), device_weights(mw, device=f"cuda:{rank}")


def ep_forward(rank, world, H, I, E, K, bits, Ts, shared, seed, expert_path, skew=False):
    """EP layer vs the one-GPU layer on every rank, for several batch sizes
    (also through a CUDA-graph stack).  Returns per T: bit-identity with the
    one-GPU layer, repeatability, a digest of the output (compared across
    ranks), max abs / rel L2 vs the one-GPU layer and max abs vs the oracle."""
    import torch

    import senmoe
    from helpers import moe_args, rel_l2, t_bf16, to_numpy_bf16, bf16_np_to_f32
    from oracle import oracle as O
    from senmoe import ep

    Tmax = max(Ts)
    cfg, mw, x_np, args, wd = _gpu_setup(rank, world, H, I, E, K, bits, Tmax, shared, seed, skew)
    args = moe_args(cfg, expert_path)
    full = senmoe.DeepseekMoe(args, wd, max_tokens=Tmax)
    epl = ep.make_layer(args, wd, Tmax, rank, world)
    ep.connect([epl])
    x = t_bf16(x_np, device=f"cuda:{rank}")
    out = {}
    for T in Ts:
        ref = full.forward(x[:T])
        y = epl.forward(x[:T])
        y2 = epl.forward(x[:T])  # a second call: the epoch/flag hand-over
        epl.check()
        full.check()
        orc = O.moe_forward(cfg, mw, x_np[:T])
        a, b2 = to_numpy_bf16(y), to_numpy_bf16(ref)
        sms = torch.cuda.get_device_properties(rank).multi_processor_count
        out[T] = dict(exact=bool(torch.equal(y, ref)), repeat=bool(torch.equal(y, y2)),
                      same_kernels=(two_cta_form(args, T, world, sms) == two_cta_form(args, T, 1, sms)
                                    and full.expert_path(T) == epl.expert_path(T)),
                      digest=hashlib.sha256(a.tobytes()).hexdigest(),
                      max_abs=float(np.abs(bf16_np_to_f32(a) - bf16_np_to_f32(b2)).max()),
                      rel_l2=float(rel_l2(bf16_np_to_f32(a), bf16_np_to_f32(b2))),
                      max_abs_oracle=float(np.abs(bf16_np_to_f32(a) - orc["y_f32"]).max()),
                      path=epl.expert_path(T))
    # a graph-captured two-layer stack with the residual add (the decode step)
    epl2 = ep.make_layer(args, wd, Tmax, rank, world)
    ep.connect([epl2])
    full2 = senmoe.DeepseekMoe(args, wd, max_tokens=Tmax)
    stack = senmoe.MoeStack([epl, epl2], max_tokens=Tmax)
    ref_stack = senmoe.MoeStack([full, full2], max_tokens=Tmax, use_graph=False)
    T = Ts[0]
    ys = [stack.forward(x[:T]).clone() for _ in range(3)]
    yr = ref_stack.forward(x[:T])
    epl.check()
    epl2.check()
    out["stack_repeat"] = all(bool(torch.equal(v, ys[0])) for v in ys)
    out["stack_digest"] = hashlib.sha256(to_numpy_bf16(ys[0]).tobytes()).hexdigest()
    out["stack_max_abs"] = float((ys[0].float() - yr.float()).abs().max())
    sms = torch.cuda.get_device_properties(rank).multi_processor_count
    out["stack_same_kernels"] = (two_cta_form(args, T, world, sms) == two_cta_form(args, T, 1, sms)
                                 and full.expert_path(T) == epl.expert_path(T))
    stack.release()
    torch.cuda.synchronize()
    import torch.distributed as dist
    dist.barrier()  # no rank frees its rows while a peer may still read them
    for L in (epl, epl2, full, full2):
        L.close()
    dist.barrier()
    return out


def ep_missing_rank(rank, world, H, I, E, K, bits, T, seed):
    """Rank world-1 skips one forward: the other ranks' bounded waits run out
    and their check() reports ERR_TIMEOUT; the skipping rank stays clean."""
    import torch
    import torch.distributed as dist

    import senmoe
    from helpers import moe_args, t_bf16
    from senmoe import ep

    cfg, mw, x_np, args, wd = _gpu_setup(rank, world, H, I, E, K, bits, T, 0, seed)
    epl = ep.make_layer(moe_args(cfg), wd, T, rank, world)
    ep.connect([epl])
    x = t_bf16(x_np, device=f"cuda:{rank}")
    epl.forward(x)
    epl.check()  # one good call on every rank
    dist.barrier()
    status = "ok"
    if rank != world - 1:
        epl.forward(x)
        try:
            epl.check()
        except senmoe.SenMoeError as e:
            status = f"status {e.status}"
    torch.cuda.synchronize()
    dist.barrier()
    epl.close()
    dist.barrier()
    return status


def ep_tokens_forward(rank, world, H, I, E, K, bits, count_lists, shared, seed, expert_path):
    """Token-local expert parallelism: rank r passes its own tokens (its
    slice of the call's tokens, rank order) and must get back exactly what
    one GPU returns for them when it runs every rank's tokens at once.
    count_lists: per case, every rank's token count.  Returns per case the
    bit-identity, repeatability and max abs vs the oracle, plus the same for
    a graph-captured two-layer residual stack of the first case."""
    import torch

    import senmoe
    from helpers import bf16_np_to_f32, moe_args, t_bf16, to_numpy_bf16
    from oracle import oracle as O
    from senmoe import ep

    from dataclasses import replace

    Tmax = max(sum(c) for c in count_lists)
    cfg, mw, x_np, args, wd = _gpu_setup(rank, world, H, I, E, K, bits, Tmax, shared, seed)
    args = moe_args(cfg, expert_path)
    full = senmoe.DeepseekMoe(args, wd, max_tokens=Tmax)
    # expert-slot capacity: twice a rank's even share of the pairs (the scratch
    # of an expert-parallel rank shrinks with the world size)
    args_ep = replace(args, expert_slots=max(64, 2 * Tmax * K // world))
    epl = ep.make_layer(args_ep, wd, Tmax, rank, world)
    ep.connect([epl])
    x = t_bf16(x_np, device=f"cuda:{rank}")
    out = {}
    for ci, counts in enumerate(count_lists):
        T = sum(counts)
        b = sum(counts[:rank])
        n = counts[rank]
        ref = full.forward(x[:T])[b:b + n]
        y = epl.forward_tokens(x[b:b + n], counts)
        y2 = epl.forward_tokens(x[b:b + n], counts)
        epl.check()
        full.check()
        orc = O.moe_forward(cfg, mw, x_np[b:b + n]) if n else {"y_f32": np.zeros((0, H), np.float32)}
        a = bf16_np_to_f32(to_numpy_bf16(y))
        sms = torch.cuda.get_device_properties(rank).multi_processor_count
        out[ci] = dict(exact=bool(torch.equal(y, ref)), repeat=bool(torch.equal(y, y2)),
                       same_kernels=(two_cta_form(args, T, world, sms) == two_cta_form(args, T, 1, sms)
                                    and full.expert_path(T) == epl.expert_path(T)),
                       max_abs_full=float((y.float() - ref.float()).abs().max()) if n else 0.0,
                       max_abs_oracle=float(np.abs(a - orc["y_f32"]).max()) if n else 0.0)
    # a graph-captured two-layer residual stack over the first case's tokens
    counts = count_lists[0]
    T, b, n = sum(counts), sum(counts[:rank]), counts[rank]
    epl2 = ep.make_layer(args_ep, wd, Tmax, rank, world)
    ep.connect([epl2])
    full2 = senmoe.DeepseekMoe(args, wd, max_tokens=Tmax)
    stack = senmoe.MoeStack([epl, epl2], max_tokens=Tmax, tokens_per_rank=counts)
    ref_stack = senmoe.MoeStack([full, full2], max_tokens=Tmax, use_graph=False)
    ys = [stack.forward(x[b:b + n]).clone() for _ in range(3)]
    yr = ref_stack.forward(x[:T])[b:b + n]
    epl.check()
    epl2.check()
    out["stack_repeat"] = all(bool(torch.equal(v, ys[0])) for v in ys)
    out["stack_exact"] = bool(torch.equal(ys[0], yr))
    out["stack_max_abs"] = float((ys[0].float() - yr.float()).abs().max()) if n else 0.0
    sms = torch.cuda.get_device_properties(rank).multi_processor_count
    out["stack_same_kernels"] = (two_cta_form(args, T, world, sms) == two_cta_form(args, T, 1, sms)
                                 and full.expert_path(T) == epl.expert_path(T))
    stack.release()
    torch.cuda.synchronize()
    import torch.distributed as dist
    dist.barrier()  # no rank frees its rows while a peer may still read them
    for L in (epl, epl2, full, full2):
        L.close()
    dist.barrier()
    return out
