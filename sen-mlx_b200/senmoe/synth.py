"""senmoe.synth -- seeded synthetic MoE weights and tokens in MLX layout.

Every value is a pure function of (seed, tensor, flat index) through a 32-bit
integer hash, evaluated with the same integer and IEEE float operations in
numpy (host) and in torch (any device), so a CPU process and a GPU process
build bit-identical tensors without shipping them.  bench.py builds its
workloads with it (the GPU arm on the device, the CPU baseline on the host)
and the tests use it to check the exact tensors the bench runs.

Shapes follow the MLX affine-quantized layout the block consumes
(src/engine/mlx_native.rs:3381-3389): codes u32 ``[E, out, in*bits/32]``,
bf16 scales and biases ``[E, out, in/64]``, router bf16 ``[E, H]``.

Values:
* codes: uniformly random words (every 4- or 8-bit code equally likely);
* scales/biases: what an MLX affine quantizer produces for groups of 64
  N(0, 0.02) weights: scale = 0.1/(2^bits-1) * (0.9 + 0.3 u), bias =
  -(2^bits-1)/2 * scale + 1e-3 z, both times ``gain``;
* router weight N(0, 1/sqrt(H)) so logits of N(0, 1) tokens are ~N(0, 1);
* tokens N(0, 1).
"Normal" values are Irwin-Hall sums of four hash uniforms, scaled to unit
variance (bounded tails at +-3.46, which routing does not notice).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

M32 = 0xFFFFFFFF
_C1, _C2 = 0x7FEB352D, 0x846CA68B
_TOKENS_LAYER = 0xFFFF  # key namespace of the token streams
PROJECTIONS = {"gate": 0, "up": 1, "down": 2, "shared_gate": 3, "shared_up": 4, "shared_down": 5}


def _mul32(x, c: int):
    """(x * c) mod 2^32 for 0 <= x < 2^32 held in int64, with every partial
    product below 2^63 (no signed overflow in numpy or torch)."""
    lo, hi = x & 0xFFFF, x >> 16
    return (lo * c + (((hi * c) & 0xFFFF) << 16)) & M32


def _mix(x):
    x = x ^ (x >> 16)
    x = _mul32(x, _C1)
    x = x ^ (x >> 15)
    x = _mul32(x, _C2)
    return x ^ (x >> 16)


def _mix_int(v: int) -> int:
    v &= M32
    v ^= v >> 16
    v = (v * _C1) & M32
    v ^= v >> 15
    v = (v * _C2) & M32
    return v ^ (v >> 16)


def _key(seed: int, layer: int, stream: int) -> int:
    return _mix_int(_mix_int(seed * 0x9E3779B1 + layer) ^ (stream * 0x85EBCA77))


class _Numpy:
    def arange(self, lo, hi):
        return np.arange(lo, hi, dtype=np.int64)

    def f64(self, h):
        return h.astype(np.float64)

    def bf16(self, v64):
        """float64 -> float32 -> bf16 bits (round to nearest even each time)."""
        u = v64.astype(np.float32).view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)

    def u32(self, h):
        return h.astype(np.uint32)

    def cat(self, parts):
        return np.concatenate(parts)


class _Torch:
    def __init__(self, device):
        import torch
        self.t, self.device = torch, device

    def arange(self, lo, hi):
        return self.t.arange(lo, hi, dtype=self.t.int64, device=self.device)

    def f64(self, h):
        return h.to(self.t.float64)

    def bf16(self, v64):
        return v64.to(self.t.float32).to(self.t.bfloat16)

    def u32(self, h):
        # same bits as uint32, stored as int32 (torch's packed-weight dtype here)
        return (h - ((h >> 31) << 32)).to(self.t.int32)

    def cat(self, parts):
        return self.t.cat(parts)


def backend(device=None):
    """numpy for device None or "numpy", else torch on that device."""
    return _Numpy() if device is None or device == "numpy" else _Torch(device)


def _hash(bk, key: int, lo: int, hi: int):
    x = bk.arange(lo, hi)
    return _mix(_mix((x + key) & M32) ^ _mix_int(key ^ 0x27D4EB2F))


def _uniform(bk, key, lo, hi):
    """(h + 0.5) / 2^32 in (0, 1), float64 (exact)."""
    return (bk.f64(_hash(bk, key, lo, hi)) + 0.5) * (1.0 / 4294967296.0)


def _normal(bk, key, lo, hi):
    """Irwin-Hall(4) of four independent uniform streams, unit variance."""
    s = _uniform(bk, key, lo, hi)
    for j in (1, 2, 3):
        s = s + _uniform(bk, _mix_int(key + j * 0x165667B1), lo, hi)
    return (s - 2.0) * math.sqrt(3.0)


def projection(seed: int, layer: int, which: str, rows: int, cols: int, bits: int, experts=None, gain: float = 1.0,
               device=None, chunk_elems: int = 1 << 25):
    """Quantized projection of experts [eb, ee) (``experts``; None: a dense
    projection with no expert dim): (codes, scales, biases).  Expert e's
    values depend only on its global index, so an expert-parallel rank builds
    exactly its slice of the one-GPU tensors."""
    bk = backend(device)
    words, groups = cols * bits // 32, cols // 64
    eb, ee = (0, 1) if experts is None else experts
    levels = (1 << bits) - 1
    p = PROJECTIONS[which]
    kc, ks, kb = (_key(seed, layer, 3 * p + i) for i in range(3))
    per_c, per_g = rows * words, rows * groups
    step = max(1, chunk_elems // max(per_c, 1))
    codes, scales, biases = [], [], []
    for e0 in range(eb, ee, step):
        e1 = min(ee, e0 + step)
        codes.append(bk.u32(_hash(bk, kc, e0 * per_c, e1 * per_c)))
        s = (_uniform(bk, ks, e0 * per_g, e1 * per_g) * 0.3 + 0.9) * (0.1 / levels) * gain
        b = s * (-levels / 2.0) + _normal(bk, kb, e0 * per_g, e1 * per_g) * (1e-3 * gain)
        scales.append(bk.bf16(s))
        biases.append(bk.bf16(b))
    shape_c, shape_g = (rows, words), (rows, groups)
    if experts is not None:
        shape_c, shape_g = (ee - eb, rows, words), (ee - eb, rows, groups)
    return (bk.cat(codes).reshape(shape_c), bk.cat(scales).reshape(shape_g), bk.cat(biases).reshape(shape_g))


def router_weight(seed: int, layer: int, num_experts: int, hidden: int, device=None, expert_offsets=None):
    """bf16 [E, H] ~ N(0, 1/sqrt(H)).  ``expert_offsets`` (E floats) adds
    offset_e / ZIPF_X0 to column 0, so tokens whose column 0 is ZIPF_X0
    (``tokens(..., zipf_column=True)``) get logit offset_e on expert e."""
    bk = backend(device)
    w = _normal(bk, _key(seed, layer, 20), 0, num_experts * hidden) * (1.0 / math.sqrt(hidden))
    w = w.reshape(num_experts, hidden)
    if expert_offsets is not None:
        off = np.asarray(expert_offsets, dtype=np.float64) / ZIPF_X0
        if isinstance(bk, _Numpy):
            w[:, 0] += off
        else:
            w[:, 0] += bk.t.from_numpy(off).to(w.device)
    return bk.bf16(w)


def shared_gate_vector(seed: int, layer: int, hidden: int, device=None):
    """bf16 [H] ~ N(0, 1/sqrt(H)): the sigmoid gate of a gated shared expert."""
    bk = backend(device)
    return bk.bf16(_normal(bk, _key(seed, layer, 21), 0, hidden) * (1.0 / math.sqrt(hidden)))


ZIPF_X0 = 4.0  # column-0 value of skewed-routing tokens


def tokens(seed: int, num_tokens: int, hidden: int, device=None, first: int = 0, zipf_column: bool = False):
    """bf16 [T, H] ~ N(0, 1): rows first .. first+T-1 of the seed's token
    stream (any row range of one stream agrees with the whole).  With
    ``zipf_column`` column 0 is ZIPF_X0, the input of the router offsets."""
    bk = backend(device)
    v = _normal(bk, _key(seed, _TOKENS_LAYER, 0), first * hidden, (first + num_tokens) * hidden)
    v = v.reshape(num_tokens, hidden)
    if zipf_column:
        v[:, 0] = ZIPF_X0
    return bk.bf16(v)


def zipf_offsets(seed: int, num_experts: int, s: float = 1.2, c: float = 1.0, layer: int = 0) -> np.ndarray:
    """Per-expert router logit offsets c * log(1 / rank_e^s) (rank 1 = 0,
    falling with rank), ranks a seeded permutation of 1..E per layer: a
    Zipf(s) preference so a few experts take most tokens (with c = 1 and
    N(0, 1) logits the top 10 % of 128 experts take ~80 % of the pairs)."""
    order = np.argsort(np.asarray([_mix_int(_key(seed, layer, 30) + e) for e in range(num_experts)]), kind="stable")
    rank = np.empty(num_experts, dtype=np.int64)
    rank[order] = np.arange(1, num_experts + 1)
    return -c * s * np.log(rank.astype(np.float64))


def bytes_per_expert(hidden: int, intermediate: int, bits: int, group: int = 64) -> int:
    """Packed codes + bf16 scales and biases of one expert's gate, up and down."""
    gate_up = 2 * (intermediate * hidden * bits // 8 + 2 * intermediate * (hidden // group) * 2)
    down = hidden * intermediate * bits // 8 + 2 * hidden * (intermediate // group) * 2
    return gate_up + down


@dataclass(frozen=True)
class LayerSpec:
    """Shape and routing of one synthetic MoE layer."""
    name: str
    hidden: int
    experts: int
    top_k: int
    intermediate: int
    bits: int
    shared: int = 0             # shared-expert intermediate (0: none)
    shared_gate: bool = False   # sigmoid-gated shared expert
    zipf: bool = False          # Zipf(1.2)-skewed router (tokens need zipf_column=True)
    down_gain: float = 0.01     # keeps each block's output small next to the residual stream
    seed: int = 0

    def expert_bytes(self) -> int:
        return bytes_per_expert(self.hidden, self.intermediate, self.bits)

    def shared_bytes(self) -> int:
        return bytes_per_expert(self.hidden, self.shared, self.bits) if self.shared else 0


# The BASELINE configurations (config 0 is config 1's layer on the CPU at 16 tokens).
CONFIG1 = LayerSpec("config1", 2048, 128, 8, 768, 4, seed=0)
CONFIG3 = LayerSpec("config3", 2048, 512, 10, 512, 4, shared=512, shared_gate=True, seed=3)
CONFIG4 = LayerSpec("config4", 2048, 128, 8, 768, 8, zipf=True, seed=4)


def layer_tensors(spec: LayerSpec, layer: int, experts=None, device=None) -> dict:
    """One layer's tensors: router_w, {gate,up,down}_{w,s,b} of experts
    [eb, ee) (``experts``; None: all), sh_{gate,up,down}_{w,s,b} and
    sh_gate_vec when the spec has them.  numpy (codes uint32, bf16 as uint16
    bits) for device None, else torch on ``device`` (codes int32, bfloat16)."""
    H, I, E, b = spec.hidden, spec.intermediate, spec.experts, spec.bits
    rng = (0, E) if experts is None else tuple(experts)
    off = zipf_offsets(spec.seed, E, layer=layer) if spec.zipf else None
    t = {"router_w": router_weight(spec.seed, layer, E, H, device, expert_offsets=off)}
    for name, rows, cols, gain in (("gate", I, H, 1.0), ("up", I, H, 1.0), ("down", H, I, spec.down_gain)):
        t[f"{name}_w"], t[f"{name}_s"], t[f"{name}_b"] = projection(spec.seed, layer, name, rows, cols, b, rng, gain,
                                                                    device)
    if spec.shared:
        Is = spec.shared
        for name, rows, cols, gain in (("gate", Is, H, 1.0), ("up", Is, H, 1.0), ("down", H, Is, spec.down_gain)):
            t[f"sh_{name}_w"], t[f"sh_{name}_s"], t[f"sh_{name}_b"] = projection(
                spec.seed, layer, f"shared_{name}", rows, cols, b, None, gain, device)
        if spec.shared_gate:
            t["sh_gate_vec"] = shared_gate_vector(spec.seed, layer, H, device)
    return t


def token_seed(spec: LayerSpec) -> int:
    return 1234 + spec.seed


def spec_tokens(spec: LayerSpec, num_tokens: int, device=None, first: int = 0):
    """The workload's tokens for a spec (column 0 set for a skewed router)."""
    return tokens(token_seed(spec), num_tokens, spec.hidden, device, first=first, zipf_column=spec.zipf)


def moe_args(spec: LayerSpec, **overrides):
    """senmoe.MoeArgs of a spec (one shared expert of width spec.shared)."""
    from . import MoeArgs
    kw = dict(hidden_size=spec.hidden, moe_intermediate_size=spec.intermediate, n_routed_experts=spec.experts,
              num_experts_per_tok=spec.top_k, bits=spec.bits, group_size=64,
              n_shared_experts=1 if spec.shared else 0, shared_gate=spec.shared_gate)
    if spec.shared and spec.shared != spec.intermediate:
        raise ValueError("the shared expert's width must equal moe_intermediate_size (n_shared_experts = 1)")
    kw.update(overrides)
    return MoeArgs(**kw)


def moe_weights(spec: LayerSpec, layer: int, device, experts=None):
    """senmoe.MoeWeights of one synthetic layer on a CUDA device (experts
    [eb, ee) only for an expert-parallel rank)."""
    from . import MoeWeights, SwitchLinear
    t = layer_tensors(spec, layer, experts, device)
    sl = lambda p: SwitchLinear(t[f"{p}_w"], t[f"{p}_s"], t[f"{p}_b"])
    w = MoeWeights(router_weight=t["router_w"], gate_proj=sl("gate"), up_proj=sl("up"), down_proj=sl("down"))
    if spec.shared:
        w.shared_gate_proj, w.shared_up_proj, w.shared_down_proj = sl("sh_gate"), sl("sh_up"), sl("sh_down")
        w.shared_gate_vector = t.get("sh_gate_vec")
    return w
