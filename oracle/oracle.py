"""TEST INFRASTRUCTURE ONLY -- ctypes wrapper around the C oracle.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module.  It restates sen-mlx's MoE block on the CPU
(src/engine/mlx_lm/models/deepseek_v2.rs:466-553, utils/moe.rs:20-77); see
moe_oracle.c for the rounding model.  Parity against MLX itself is unpinned
(MLX is not available here); the restatement is pinned to the reference's own
known-answer test (utils/moe.rs:89-146) via tests/golden/.

bf16 tensors cross this boundary as numpy uint16 arrays holding raw bf16 bits.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lib = None

ORC_OK, ORC_BAD_ARG, ORC_BAD_INDEX, ORC_NO_MEM = 0, 1, 2, 3


def build(force: bool = False) -> str:
    """Compile moe_oracle.c with the committed Makefile (gcc + OpenMP)."""
    src = os.path.join(_HERE, "moe_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class OrcConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32), ("intermediate", C.c_int32), ("num_experts", C.c_int32),
        ("top_k", C.c_int32), ("bits", C.c_int32), ("group_size", C.c_int32),
        ("norm_topk_prob", C.c_int32), ("routed_scaling_factor", C.c_float),
        ("shared_intermediate", C.c_int32), ("shared_gate", C.c_int32),
        ("mode", C.c_int32), ("activation", C.c_int32),
    ]


_P = C.c_void_p


class OrcGemmaRouterConfig(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
                ("group_size", C.c_int32), ("bits", C.c_int32), ("eps", C.c_float)]


class OrcGemmaRouterWeights(C.Structure):
    _fields_ = [("proj_w", C.c_void_p), ("proj_s", C.c_void_p), ("proj_b", C.c_void_p),
                ("scale", C.c_void_p), ("per_expert_scale", C.c_void_p)]


class OrcWeights(C.Structure):
    _fields_ = [
        ("router_w", _P), ("gate_w", _P), ("up_w", _P), ("down_w", _P),
        ("gate_s", _P), ("gate_b", _P), ("up_s", _P), ("up_b", _P), ("down_s", _P), ("down_b", _P),
        ("sh_gate_w", _P), ("sh_up_w", _P), ("sh_down_w", _P),
        ("sh_gate_s", _P), ("sh_gate_b", _P), ("sh_up_s", _P), ("sh_up_b", _P),
        ("sh_down_s", _P), ("sh_down_b", _P), ("sh_gate_vec", _P),
    ]


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(_LIB_PATH)
        i64, i32 = C.c_int64, C.c_int32
        L.orc_quantize_affine.argtypes = [_P, i64, i64, i32, i32, _P, _P, _P]
        L.orc_dequantize_affine.argtypes = [_P, _P, _P, i64, i64, i32, i32, _P]
        L.orc_gather_qmm.argtypes = [_P, i64, _P, _P, _P, _P, i64, i64, i64, i32, i32, i32, _P]
        L.orc_router.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcWeights), _P, i64, _P, _P, _P]
        L.orc_dispatch.argtypes = [_P, i64, i32, i32, _P, _P, _P]
        L.orc_moe_forward.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcWeights), _P, i64,
                                      _P, _P, _P, _P, _P, _P]
        L.orc_experts_forward.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcWeights), _P, i64, _P, _P, _P, _P]
        L.orc_gemma_router.argtypes = [C.POINTER(OrcGemmaRouterConfig), C.POINTER(OrcGemmaRouterWeights), _P, i64,
                                       _P, _P, _P]
        L.orc_f32_to_bf16.argtypes = [_P, _P, i64]
        L.orc_bf16_to_f32.argtypes = [_P, _P, i64]
        L.orc_fill_normal.argtypes = [C.c_uint64, _P, i64, C.c_float]
        L.orc_set_num_threads.argtypes = [C.c_int]
        L.orc_num_threads.restype = C.c_int
        _lib = L
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _check(rc, what):
    if rc != ORC_OK:
        raise RuntimeError(f"oracle {what} failed with status {rc}")


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# --------------------------------------------------------------- bf16 bits
def f32_to_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16(_ptr(a), _ptr(out), a.size)
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.float32)
    lib().orc_bf16_to_f32(_ptr(a), _ptr(out), a.size)
    return out


def normal(seed: int, shape, std: float = 1.0) -> np.ndarray:
    """Counter-based seeded N(0, std^2) float32 (reproducible under any thread count)."""
    out = np.empty(shape, dtype=np.float32)
    lib().orc_fill_normal(C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), _ptr(out), out.size, float(std))
    return out


# ------------------------------------------------------------- primitives
def quantize(w: np.ndarray, group: int = 64, bits: int = 4):
    """MLX-layout affine quantization of a float [..., rows, cols] array.

    Returns (wq uint32 [..., rows, cols*bits/32], scales bf16 bits, biases bf16 bits).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    *lead, cols = w.shape
    rows = int(np.prod(lead)) if lead else 1
    wq = np.empty((*lead, cols * bits // 32), dtype=np.uint32)
    s = np.empty((*lead, cols // group), dtype=np.uint16)
    b = np.empty_like(s)
    _check(lib().orc_quantize_affine(_ptr(w), rows, cols, group, bits, _ptr(wq), _ptr(s), _ptr(b)), "quantize")
    return wq, s, b


def dequantize(wq, s, b, group: int = 64, bits: int = 4) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    *lead, words = wq.shape
    cols = words * 32 // bits
    rows = int(np.prod(lead)) if lead else 1
    out = np.empty((*lead, cols), dtype=np.float32)
    _check(lib().orc_dequantize_affine(_ptr(wq), _ptr(np.ascontiguousarray(s)), _ptr(np.ascontiguousarray(b)),
                                       rows, cols, group, bits, _ptr(out)), "dequantize")
    return out


def gather_qmm(x_bf16, wq, s, b, idx, group: int = 64, bits: int = 4) -> np.ndarray:
    """utils/moe.rs:33-43 with transpose=true.  x [x_rows, in] bf16 bits;
    idx [n] int (n a multiple of x_rows); returns [n, out] bf16 bits."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    idx = np.ascontiguousarray(np.asarray(idx).reshape(-1), dtype=np.int32)
    E, out_f, _ = wq.shape
    in_f = x.shape[-1]
    y = np.empty((idx.size, out_f), dtype=np.uint16)
    _check(lib().orc_gather_qmm(_ptr(x), x.shape[0], _ptr(np.ascontiguousarray(wq)), _ptr(np.ascontiguousarray(s)),
                                _ptr(np.ascontiguousarray(b)), _ptr(idx), idx.size, in_f, out_f, E, group, bits,
                                _ptr(y)), "gather_qmm")
    return y


def dispatch(ids: np.ndarray, num_experts: int):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, K = ids.shape
    perm = np.empty(T * K, dtype=np.int32)
    inv = np.empty(T * K, dtype=np.int32)
    offs = np.empty(num_experts + 1, dtype=np.int32)
    _check(lib().orc_dispatch(_ptr(ids), T, K, num_experts, _ptr(perm), _ptr(offs), _ptr(inv)), "dispatch")
    return perm, offs, inv


# ------------------------------------------------------------------ block
@dataclass
class MoeWeights:
    """One layer's weights in MLX layout (numpy; bf16 as uint16 bits)."""
    router_w: np.ndarray            # [E, H] bf16
    gate_w: np.ndarray; gate_s: np.ndarray; gate_b: np.ndarray   # [E, I, H*bits/32], [E, I, H/g]
    up_w: np.ndarray; up_s: np.ndarray; up_b: np.ndarray
    down_w: np.ndarray; down_s: np.ndarray; down_b: np.ndarray   # [E, H, I*bits/32], [E, H, I/g]
    sh_gate_w: np.ndarray | None = None; sh_gate_s: np.ndarray | None = None; sh_gate_b: np.ndarray | None = None
    sh_up_w: np.ndarray | None = None; sh_up_s: np.ndarray | None = None; sh_up_b: np.ndarray | None = None
    sh_down_w: np.ndarray | None = None; sh_down_s: np.ndarray | None = None; sh_down_b: np.ndarray | None = None
    sh_gate_vec: np.ndarray | None = None

    def to_c(self) -> OrcWeights:
        self._keep = {k: (None if v is None else np.ascontiguousarray(v)) for k, v in self.__dict__.items()
                      if k != "_keep"}
        return OrcWeights(**{k: _ptr(v) for k, v in self._keep.items()})


@dataclass
class MoeConfig:
    hidden: int = 2048
    intermediate: int = 768
    num_experts: int = 128
    top_k: int = 8
    bits: int = 4
    group_size: int = 64
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    shared_intermediate: int = 0
    shared_gate: bool = False
    activation: int = 0  # 0 SwiGLU (DeepSeek), 1 GeGLU (Gemma)

    def to_c(self, mode: int = 0) -> OrcConfig:
        return OrcConfig(self.hidden, self.intermediate, self.num_experts, self.top_k, self.bits,
                         self.group_size, int(self.norm_topk_prob), float(self.routed_scaling_factor),
                         self.shared_intermediate, int(self.shared_gate), int(mode), int(self.activation))


def router(cfg: MoeConfig, w: MoeWeights, x_bf16: np.ndarray, mode: int = 0):
    """Returns (ids [T,K] int32, weights [T,K] f32, scores [T,E] f32)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, cfg.hidden)
    T = x.shape[0]
    ids = np.empty((T, cfg.top_k), dtype=np.int32)
    wts = np.empty((T, cfg.top_k), dtype=np.float32)
    scores = np.empty((T, cfg.num_experts), dtype=np.float32)
    c, cw = cfg.to_c(mode), w.to_c()
    _check(lib().orc_router(C.byref(c), C.byref(cw), _ptr(x), T, _ptr(ids), _ptr(wts), _ptr(scores)), "router")
    return ids, wts, scores


def moe_forward(cfg: MoeConfig, w: MoeWeights, x_bf16: np.ndarray, mode: int = 0):
    """DeepseekMoe::forward restated.  Returns a dict with y_f32 [T,H],
    y_bf16 [T,H] (bits), ids/weights [T,K], perm [T*K], offsets [E+1]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, cfg.hidden)
    T, H, K, E = x.shape[0], cfg.hidden, cfg.top_k, cfg.num_experts
    out = dict(
        y_f32=np.zeros((T, H), dtype=np.float32), y_bf16=np.zeros((T, H), dtype=np.uint16),
        ids=np.zeros((T, K), dtype=np.int32), weights=np.zeros((T, K), dtype=np.float32),
        perm=np.zeros(T * K, dtype=np.int32), offsets=np.zeros(E + 1, dtype=np.int32),
    )
    c, cw = cfg.to_c(mode), w.to_c()
    _check(lib().orc_moe_forward(C.byref(c), C.byref(cw), _ptr(x), T, _ptr(out["y_f32"]), _ptr(out["y_bf16"]),
                                 _ptr(out["ids"]), _ptr(out["weights"]), _ptr(out["perm"]), _ptr(out["offsets"])),
           "moe_forward")
    return out


def make_layer(cfg: MoeConfig, seed: int = 0, router_std: float = 0.02, expert_std: float = 0.02) -> MoeWeights:
    """Seeded synthetic layer: router N(0, router_std) bf16, expert weights
    N(0, expert_std) quantized with the MLX-style quantizer.  Each tensor gets
    its own sub-seed (seed * 64 + k) of the counter-based generator."""
    E, H, I, g, b = cfg.num_experts, cfg.hidden, cfg.intermediate, cfg.group_size, cfg.bits
    sub = lambda k: seed * 64 + k
    router_w = f32_to_bf16(normal(sub(0), (E, H), router_std))
    gw, gs, gb = quantize(normal(sub(1), (E, I, H), expert_std), g, b)
    uw, us, ub = quantize(normal(sub(2), (E, I, H), expert_std), g, b)
    dw, ds, db = quantize(normal(sub(3), (E, H, I), expert_std), g, b)
    mw = MoeWeights(router_w, gw, gs, gb, uw, us, ub, dw, ds, db)
    if cfg.shared_intermediate:
        Is = cfg.shared_intermediate
        mw.sh_gate_w, mw.sh_gate_s, mw.sh_gate_b = quantize(normal(sub(4), (Is, H), expert_std), g, b)
        mw.sh_up_w, mw.sh_up_s, mw.sh_up_b = quantize(normal(sub(5), (Is, H), expert_std), g, b)
        mw.sh_down_w, mw.sh_down_s, mw.sh_down_b = quantize(normal(sub(6), (H, Is), expert_std), g, b)
        if cfg.shared_gate:
            mw.sh_gate_vec = f32_to_bf16(normal(sub(7), (H,), router_std))
    return mw


def make_tokens(T: int, hidden: int, seed: int = 1) -> np.ndarray:
    """x ~ N(0, 1) as bf16 bits, [T, hidden]."""
    return f32_to_bf16(normal(seed * 64 + 63, (T, hidden), 1.0))


def experts_forward(cfg: MoeConfig, w: MoeWeights, x_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray,
                    mode: int = 0):
    """Experts::forward (gemma4.rs:842-848): the experts of the given routing
    ids / weights [T, K] and their f32 weighted sum (+ shared experts).
    Returns (y_f32 [T, H], y_bf16 bits [T, H])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, cfg.hidden)
    T, H = x.shape[0], cfg.hidden
    ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(T, cfg.top_k)
    weights = np.ascontiguousarray(weights, dtype=np.float32).reshape(T, cfg.top_k)
    y = np.zeros((T, H), dtype=np.float32)
    yb = np.zeros((T, H), dtype=np.uint16)
    c, cw = cfg.to_c(mode), w.to_c()
    _check(lib().orc_experts_forward(C.byref(c), C.byref(cw), _ptr(x), T, _ptr(ids), _ptr(weights), _ptr(y),
                                     _ptr(yb)), "experts_forward")
    return y, yb


@dataclass
class GemmaRouterConfig:
    hidden: int
    num_experts: int
    top_k: int
    group_size: int = 64
    bits: int = 8
    eps: float = 1e-6

    def to_c(self) -> OrcGemmaRouterConfig:
        return OrcGemmaRouterConfig(self.hidden, self.num_experts, self.top_k, self.group_size, self.bits,
                                    float(self.eps))


@dataclass
class GemmaRouterWeights:
    """Gemma Router parameters (gemma4.rs:683-700), numpy; bf16 as uint16 bits."""
    proj_w: np.ndarray   # [E, H*bits/32] u32
    proj_s: np.ndarray   # [E, H/group] bf16
    proj_b: np.ndarray
    scale: np.ndarray    # [H] bf16
    per_expert_scale: np.ndarray  # [E] bf16

    def to_c(self) -> OrcGemmaRouterWeights:
        self._keep = [np.ascontiguousarray(v) for v in (self.proj_w, self.proj_s, self.proj_b, self.scale,
                                                         self.per_expert_scale)]
        return OrcGemmaRouterWeights(*[_ptr(v) for v in self._keep])


def make_gemma_router(rc: GemmaRouterConfig, seed: int = 0) -> GemmaRouterWeights:
    """Seeded synthetic router: projection N(0, 1) quantized at rc.bits (the norm
    weight folds in H^-1/2, so logits come out ~N(0, 1)),
    norm scale around 1, per-expert scales in (0.5, 1.5)."""
    E, H = rc.num_experts, rc.hidden
    sub = lambda k: seed * 64 + 40 + k
    pw, ps, pb = quantize(normal(sub(0), (E, H), 1.0), rc.group_size, rc.bits)  # logits ~ N(0, 1)
    scale = f32_to_bf16(1.0 + normal(sub(1), (H,), 0.2))
    pes = f32_to_bf16(1.0 + 0.5 * np.tanh(normal(sub(2), (E,), 1.0)))
    return GemmaRouterWeights(pw, ps, pb, scale, pes)


def gemma_router(rc: GemmaRouterConfig, rw: GemmaRouterWeights, x_bf16: np.ndarray):
    """Router::forward (gemma4.rs:716-736).  Returns (ids [T,K] int32,
    weights [T,K] f32, scores [T,E] f32)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, rc.hidden)
    T = x.shape[0]
    ids = np.empty((T, rc.top_k), dtype=np.int32)
    wts = np.empty((T, rc.top_k), dtype=np.float32)
    scores = np.empty((T, rc.num_experts), dtype=np.float32)
    c, cw = rc.to_c(), rw.to_c()
    _check(lib().orc_gemma_router(C.byref(c), C.byref(cw), _ptr(x), T, _ptr(ids), _ptr(wts), _ptr(scores)),
           "gemma_router")
    return ids, wts, scores


def moe_residual(cfg: MoeConfig, w: MoeWeights, x_bf16: np.ndarray, mode: int = 0):
    """One decoder step of the MoE stack, h = x + DeepseekMoe::forward(x)
    (DecoderLayer::forward's residual add, deepseek_v2.rs:613-620), with the
    block's f32 sum and x added in f32 and rounded to bf16 once, as the GPU
    block's fused residual does.  Returns (h bf16 bits [T, H], the forward's
    dict)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16).reshape(-1, cfg.hidden)
    out = moe_forward(cfg, w, x, mode=mode)
    return f32_to_bf16(bf16_to_f32(x) + out["y_f32"]), out


def weights_from_synth(mw: dict) -> MoeWeights:
    """oracle MoeWeights from numpy tensors named as senmoe.synth.layer_numpy returns them."""
    u16 = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.uint16)
    u32 = lambda a: None if a is None else np.ascontiguousarray(a).view(np.uint32)
    w = MoeWeights(u16(mw["router_w"]), u32(mw["gate_w"]), u16(mw["gate_s"]), u16(mw["gate_b"]), u32(mw["up_w"]),
                   u16(mw["up_s"]), u16(mw["up_b"]), u32(mw["down_w"]), u16(mw["down_s"]), u16(mw["down_b"]))
    for k in ("sh_gate_w", "sh_up_w", "sh_down_w"):
        setattr(w, k, u32(mw.get(k)))
    for k in ("sh_gate_s", "sh_gate_b", "sh_up_s", "sh_up_b", "sh_down_s", "sh_down_b", "sh_gate_vec"):
        setattr(w, k, u16(mw.get(k)))
    return w
