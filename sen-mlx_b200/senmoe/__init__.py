"""senmoe -- Python host side of the B200 MoE block, over the C ABI in
include/senmoe.h (libsenmoe.so, loaded with ctypes).

Mirrors the reference's MoE interfaces (paths inside the sen-mlx project):

* ``gather_qmm(x, w, scales, biases, rhs_indices, transpose, group_size, bits,
  sorted_indices)`` -- src/engine/mlx_lm/utils/moe.rs:33-77, same argument
  names, meaning and broadcasting for the forms the reference uses
  (``x [..., 1, in]`` against ``rhs_indices [..., K]`` -> ``[..., K, 1, out]``,
  and ``x [..., K, 1, in]`` against ``[..., K]``).
* ``SwitchLinear`` / ``DeepseekMoe`` -- src/engine/mlx_lm/models/deepseek_v2.rs:400-553;
  ``DeepseekMoe.forward(x [B, L, H]) -> [B, L, H]``.
* Failures raise ``SenMoeError`` carrying the C status and message, as the
  reference's shim turns a non-zero status into ``Exception::custom``
  (utils/moe.rs:66-74).

torch is used only for device memory and streams.  There is no CPU path:
importing this module on a machine without the built library raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.abspath(os.path.join(_HERE, "..", "lib", "libsenmoe.so"))

OK, ERR_BAD_ARG, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_NO_MEMORY, ERR_DEVICE = range(8)
ROUTER_SOFTMAX_TOPK = 0
ACT_SWIGLU, ACT_GEGLU = 0, 1
# expert-product kernels (SenMoeConfig.reserved[0]): CUDA-core GEMV, tcgen05 GEMM, warp-MMA GEMM
PATH_AUTO, PATH_GEMV, PATH_TENSOR_CORE, PATH_MMA = 0, 1, 2, 3
PATH_SINGLE_TOKEN = 4  # reported only: one token on one GPU, the whole block in one launch
PATH_NAMES = {PATH_GEMV: "gemv", PATH_TENSOR_CORE: "tcgen05", PATH_MMA: "mma", PATH_SINGLE_TOKEN: "single-token"}


class SenMoeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"senmoe status {status}: {message}")
        self.status = status


class SenMoeConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32), ("moe_intermediate_size", C.c_int32), ("n_routed_experts", C.c_int32),
        ("num_experts_per_tok", C.c_int32), ("bits", C.c_int32), ("group_size", C.c_int32),
        ("router_kind", C.c_int32), ("activation", C.c_int32), ("norm_topk_prob", C.c_int32),
        ("routed_scaling_factor", C.c_float), ("shared_intermediate", C.c_int32), ("shared_gate", C.c_int32),
        ("max_tokens", C.c_int32), ("expert_begin", C.c_int32), ("expert_end", C.c_int32),
        ("reserved", C.c_int32 * 3),
    ]


_P = C.c_void_p
WEIGHT_FIELDS = [
    "router_weight", "gate_weight", "gate_scales", "gate_biases", "up_weight", "up_scales", "up_biases",
    "down_weight", "down_scales", "down_biases", "shared_gate_weight", "shared_gate_scales",
    "shared_gate_biases", "shared_up_weight", "shared_up_scales", "shared_up_biases", "shared_down_weight",
    "shared_down_scales", "shared_down_biases", "shared_gate_vector",
]


class SenMoeWeights(C.Structure):
    _fields_ = [(n, _P) for n in WEIGHT_FIELDS]


class SenMoeGemmaRouter(C.Structure):
    _fields_ = [("hidden_size", C.c_int32), ("num_experts", C.c_int32), ("top_k", C.c_int32),
                ("bits", C.c_int32), ("group_size", C.c_int32), ("rms_norm_eps", C.c_float),
                ("proj_weight", C.c_void_p), ("proj_scales", C.c_void_p), ("proj_biases", C.c_void_p),
                ("scale", C.c_void_p), ("per_expert_scale", C.c_void_p)]


class SenMoeDebug(C.Structure):
    _fields_ = [("topk_ids", _P), ("topk_weights", _P), ("perm", _P), ("offsets", _P)]


MAX_RANKS = 8  # SENMOE_MAX_RANKS


class SenMoePeerInfo(C.Structure):
    _fields_ = [("ipc_handle", C.c_uint8 * 64), ("rows_offset", C.c_int64), ("flags_offset", C.c_int64),
                ("arena_bytes", C.c_int64), ("expert_begin", C.c_int32), ("expert_end", C.c_int32),
                ("device", C.c_int32), ("reserved", C.c_int32)]


# Every symbol include/senmoe.h declares, with its ctypes signature.
_i64, _i32, _f32 = C.c_int64, C.c_int32, C.c_float
SIGNATURES = {
    "senmoe_last_error": (C.c_char_p, []),
    "senmoe_version": (C.c_char_p, []),
    "senmoe_selftest_sigmoid": (C.c_int, [C.POINTER(_i64), C.POINTER(_i64)]),
    "senmoe_layer_create": (C.c_int, [C.POINTER(SenMoeConfig), C.POINTER(SenMoeWeights), C.c_int, C.POINTER(_P)]),
    "senmoe_layer_destroy": (C.c_int, [_P]),
    "senmoe_layer_forward": (C.c_int, [_P, _P, _i64, _P, C.POINTER(SenMoeDebug), _P]),
    "senmoe_layer_check": (C.c_int, [_P, _P]),
    "senmoe_layer_peer_info": (C.c_int, [_P, C.POINTER(SenMoePeerInfo)]),
    "senmoe_layer_connect_peers": (C.c_int, [_P, _i32, _i32, C.POINTER(SenMoePeerInfo)]),
    "senmoe_layer_forward_residual": (C.c_int, [_P, _P, _i64, _P, _P]),
    "senmoe_layer_forward_tokens": (C.c_int, [_P, _P, _i64, _P, C.POINTER(_i64), _i32, _P]),
    "senmoe_layer_set_profiling": (C.c_int, [_P, C.c_int]),
    "senmoe_layer_expert_path": (C.c_int, [_P, _i64]),
    "senmoe_layer_stage_times": (C.c_int, [_P, C.POINTER(C.c_float), C.c_int]),
    "senmoe_router": (C.c_int, [_P, _i64, _P, _i32, _i32, _i32, _i32, _f32, _P, _P, _P, _P]),
    "senmoe_dispatch": (C.c_int, [_P, _i64, _i32, _i32, _P, _P, _P, _P, _P]),
    "senmoe_gather_qmm": (C.c_int, [_P, _i64, _P, _P, _P, _P, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _P,
                                    _P]),
    "senmoe_moe_forward_noalloc": (C.c_int, [C.POINTER(SenMoeConfig), C.POINTER(SenMoeWeights), _P, _i64, _P, _P]),
    "senmoe_gemma_router": (C.c_int, [C.c_void_p, _P, _i64, _P, _P, _P]),
    "senmoe_quantized_linear": (C.c_int, [_P, _i64, _P, _P, _P, _i64, _i64, C.c_int32, C.c_int32, _P, _P]),
    "senmoe_layer_experts_forward": (C.c_int, [_P, _P, _i64, _P, _P, _P, _P]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libsenmoe.so; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python sen-mlx_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != OK:
        raise SenMoeError(status, lib().senmoe_last_error().decode())


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _u32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype not in (torch.uint32, torch.int32):
        raise TypeError(f"packed weights must be uint32/int32, got {t.dtype}")
    return t


# ------------------------------------------------------------ gather_qmm
def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               rhs_indices: torch.Tensor, transpose: bool = True, group_size: int = 64, bits: int = 4,
               sorted_indices: bool = False, stream=None) -> torch.Tensor:
    """``out[b] = x[b] @ dequant(w[rhs_indices[b]]).T`` (utils/moe.rs:20-43).

    ``x`` is bf16 ``[*batch_x, 1, in]`` whose batch dims broadcast against
    ``rhs_indices [*batch_i]``; returns bf16 ``[*batch_i, 1, out]``.  Supported
    broadcasts are the ones the reference makes: ``batch_x`` equal to
    ``batch_i``, or equal to it with trailing dims of size 1.
    """
    if x.dtype != torch.bfloat16 or scales.dtype != torch.bfloat16 or biases.dtype != torch.bfloat16:
        raise TypeError("x, scales and biases must be bfloat16")
    if x.shape[-2] != 1:
        raise SenMoeError(ERR_UNSUPPORTED, f"gather_qmm: x rows per matmul must be 1 (got M={x.shape[-2]})")
    E, out_f, _ = w.shape
    in_f = x.shape[-1]
    bx, bi = tuple(x.shape[:-2]), tuple(rhs_indices.shape)
    n = rhs_indices.numel()
    if bx == bi:  # one x row per index (SwitchGlu's down call)
        x_rows = n
    elif len(bx) == len(bi) and len(bi) > 0 and bx[:-1] == bi[:-1] and bx[-1] == 1:
        x_rows = n // bi[-1] if bi[-1] else 0  # x broadcast over the last index dim (gate/up)
    else:
        raise SenMoeError(ERR_UNSUPPORTED, f"gather_qmm: x batch {bx} against indices {bi} is not a form the "
                                           "reference uses")
    if n == 0:
        return torch.empty((*bi, 1, out_f), dtype=torch.bfloat16, device=x.device)
    xc = x.contiguous().reshape(x_rows, in_f)
    idx = rhs_indices.to(torch.int32).contiguous()
    out = torch.empty((*bi, 1, out_f), dtype=torch.bfloat16, device=x.device)
    _check(lib().senmoe_gather_qmm(_ptr(xc), x_rows, _ptr(_u32(w).contiguous()), _ptr(scales.contiguous()),
                                   _ptr(biases.contiguous()), _ptr(idx), n, in_f, out_f, E, int(transpose),
                                   group_size, bits, int(sorted_indices), _ptr(out), _stream(stream)))
    return out


# ------------------------------------------------------------- the block
@dataclass
class MoeArgs:
    """The MoE fields of the reference's ModelArgs (deepseek_v2.rs:103-118)."""
    hidden_size: int = 2048
    moe_intermediate_size: int = 768
    n_routed_experts: int = 128
    num_experts_per_tok: int = 8
    n_shared_experts: int = 0
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    bits: int = 4
    group_size: int = 64
    activation: int = ACT_SWIGLU
    shared_gate: bool = False  # sigmoid-gated shared expert (no reference counterpart)
    expert_path: int = PATH_AUTO  # AUTO: GEMV (~1 token per expert), warp MMA (decode), tcgen05 (prefill)
    # warp-MMA form: 0 group-scaled 4-bit where supported (two CTAs per SM at 8-slot tiles),
    # 1 dequantise every weight to fp16, 2 group-scaled with one CTA per SM at every tile width,
    # 3 as 2 with 128-row down tiles instead of 256-row ones (same results)
    mma_form: int = 0
    # expert parallelism: the most (token, expert) pairs this rank's experts take per call
    # (per-pair scratch rows); 0 = max_tokens * num_experts_per_tok
    expert_slots: int = 0


@dataclass
class SwitchLinear:
    """Stacked quantized projection: weight u32 [E, out, in*bits/32], scales/biases bf16 [E, out, in/64]."""
    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor


@dataclass
class MoeWeights:
    router_weight: torch.Tensor | None  # bf16 [E, H]; None: experts_forward only
    gate_proj: SwitchLinear
    up_proj: SwitchLinear
    down_proj: SwitchLinear
    shared_gate_proj: SwitchLinear | None = None  # [Is, ...] (no expert dim)
    shared_up_proj: SwitchLinear | None = None
    shared_down_proj: SwitchLinear | None = None
    shared_gate_vector: torch.Tensor | None = None
    _keep: list = field(default_factory=list, repr=False)


class DeepseekMoe:
    """DeepseekMoe::forward on the B200 kernels (deepseek_v2.rs:520-553).

    Borrows the weight tensors (they must stay alive and in place) and owns
    the layer's device scratch, sized for ``max_tokens`` tokens per call.
    ``expert_range`` selects the locally held experts for expert parallelism;
    the expert tensors then hold only those experts.
    """

    def __init__(self, args: MoeArgs, weights: MoeWeights, max_tokens: int, device: int | None = None,
                 expert_range: tuple[int, int] | None = None):
        self.args, self.weights = args, weights
        self.device = torch.cuda.current_device() if device is None else device
        eb, ee = expert_range if expert_range is not None else (0, args.n_routed_experts)
        self.expert_range = (eb, ee)
        cfg = SenMoeConfig()
        cfg.hidden_size = args.hidden_size
        cfg.moe_intermediate_size = args.moe_intermediate_size
        cfg.n_routed_experts = args.n_routed_experts
        cfg.num_experts_per_tok = args.num_experts_per_tok
        cfg.bits = args.bits
        cfg.group_size = args.group_size
        cfg.router_kind = ROUTER_SOFTMAX_TOPK
        cfg.activation = args.activation
        cfg.norm_topk_prob = int(args.norm_topk_prob)
        cfg.routed_scaling_factor = float(args.routed_scaling_factor)
        cfg.shared_intermediate = args.moe_intermediate_size * args.n_shared_experts
        cfg.shared_gate = int(args.shared_gate)
        cfg.max_tokens = int(max_tokens)
        cfg.expert_begin, cfg.expert_end = eb, ee
        cfg.reserved[0] = int(args.expert_path)
        cfg.reserved[1] = int(args.mma_form)
        cfg.reserved[2] = int(args.expert_slots)
        self._cfg = cfg
        wt = SenMoeWeights()
        wt.router_weight = _ptr(weights.router_weight)
        for name in ("gate", "up", "down"):
            p = getattr(weights, f"{name}_proj")
            setattr(wt, f"{name}_weight", _ptr(_u32(p.weight)))
            setattr(wt, f"{name}_scales", _ptr(p.scales))
            setattr(wt, f"{name}_biases", _ptr(p.biases))
            sp = getattr(weights, f"shared_{name}_proj")
            if sp is not None:
                setattr(wt, f"shared_{name}_weight", _ptr(_u32(sp.weight)))
                setattr(wt, f"shared_{name}_scales", _ptr(sp.scales))
                setattr(wt, f"shared_{name}_biases", _ptr(sp.biases))
        wt.shared_gate_vector = _ptr(weights.shared_gate_vector)
        self._wt = wt
        handle = _P()
        _check(lib().senmoe_layer_create(C.byref(cfg), C.byref(wt), self.device, C.byref(handle)))
        self._handle = handle

    def forward(self, x: torch.Tensor, debug: dict | None = None, stream=None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, L, H] (or [T, H]) bf16 -> same shape bf16.  ``debug`` may map
        'topk_ids' / 'topk_weights' / 'perm' / 'offsets' to device tensors."""
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise TypeError("x must be a CUDA bfloat16 tensor")
        H = self.args.hidden_size
        if x.shape[-1] != H:
            raise SenMoeError(ERR_BAD_ARG, f"x last dim {x.shape[-1]} != hidden_size {H}")
        xc = x.contiguous()
        T = xc.numel() // H
        y = torch.empty_like(xc) if out is None else out
        dbg = None
        if debug:
            dbg = SenMoeDebug(*(_ptr(debug.get(k)) for k in ("topk_ids", "topk_weights", "perm", "offsets")))
        _check(lib().senmoe_layer_forward(self._handle, _ptr(xc), T, _ptr(y), C.byref(dbg) if dbg else None,
                                          _stream(stream)))
        return y

    __call__ = forward

    def experts_forward(self, x: torch.Tensor, indices: torch.Tensor, weights: torch.Tensor, stream=None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
        """Experts::forward(x, indices, weights) (gemma4.rs:842-848): the layer's
        experts over routing from the caller (e.g. GemmaRouter.forward), their
        weighted sum in fp32, bf16 out.  x [..., H] bf16, indices int32 /
        weights fp32 [..., K] on the device."""
        H, K = self.args.hidden_size, self.args.num_experts_per_tok
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != H:
            raise TypeError("x must be a CUDA bfloat16 tensor [..., hidden_size]")
        xc = x.contiguous()
        T = xc.numel() // H
        ids = indices.to(torch.int32).contiguous()
        w = weights.to(torch.float32).contiguous()
        if ids.numel() != T * K or w.numel() != T * K:
            raise SenMoeError(ERR_BAD_ARG, f"indices / weights must hold {T} x {K} entries")
        y = torch.empty_like(xc) if out is None else out
        _check(lib().senmoe_layer_experts_forward(self._handle, _ptr(xc), T, _ptr(ids), _ptr(w), _ptr(y),
                                                  _stream(stream)))
        return y

    def forward_residual(self, x: torch.Tensor, stream=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """h = x + forward(x): DecoderLayer::forward's residual add (deepseek_v2.rs:619) fused in."""
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != self.args.hidden_size:
            raise TypeError("x must be a CUDA bfloat16 tensor [..., hidden_size]")
        xc = x.contiguous()
        h = torch.empty_like(xc) if out is None else out
        _check(lib().senmoe_layer_forward_residual(self._handle, _ptr(xc), xc.numel() // self.args.hidden_size,
                                                   _ptr(h), _stream(stream)))
        return h

    def forward_tokens(self, x: torch.Tensor, tokens_per_rank, residual: bool = False, stream=None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Token-local expert parallelism: ``x`` [T_r, H] holds this rank's
        own tokens, ``tokens_per_rank[q]`` every rank's count (the same list
        on every rank); returns forward(x) (+ x with ``residual``) for them."""
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != self.args.hidden_size:
            raise TypeError("x must be a CUDA bfloat16 tensor [..., hidden_size]")
        xc = x.contiguous()
        T = xc.numel() // self.args.hidden_size
        counts = (C.c_int64 * max(len(tokens_per_rank), 1))(*[int(v) for v in tokens_per_rank])
        y = torch.empty_like(xc) if out is None else out
        _check(lib().senmoe_layer_forward_tokens(self._handle, _ptr(xc) if T else None, T, _ptr(y) if T else None,
                                                 counts, int(residual), _stream(stream)))
        return y

    def expert_path(self, num_tokens: int) -> int:
        """PATH_GEMV, PATH_MMA or PATH_TENSOR_CORE: the expert kernels a forward of num_tokens runs."""
        r = lib().senmoe_layer_expert_path(self._handle, int(num_tokens))
        if r < 0:
            _check(-r)
        return r

    STAGES = ("router", "dispatch", "gate_up", "down", "shared", "combine")

    def set_profiling(self, enable: bool) -> None:
        _check(lib().senmoe_layer_set_profiling(self._handle, int(enable)))

    def stage_times(self) -> dict:
        """Milliseconds per stage of the last profiled forward (waits for it)."""
        buf = (C.c_float * len(self.STAGES))()
        n = lib().senmoe_layer_stage_times(self._handle, buf, len(self.STAGES))
        if n < 0:
            _check(-n)
        return {k: float(buf[i]) for i, k in enumerate(self.STAGES)}

    def check(self, stream=None) -> None:
        """Synchronises and raises if a kernel recorded a device-side error."""
        _check(lib().senmoe_layer_check(self._handle, _stream(stream)))

    def peer_info(self) -> bytes:
        """This rank's expert-parallel table entry (an opaque, picklable blob)."""
        info = SenMoePeerInfo()
        _check(lib().senmoe_layer_peer_info(self._handle, C.byref(info)))
        return bytes(info)

    def connect_peers(self, rank: int, infos: list) -> None:
        """Expert-parallel form: ``infos[r]`` is rank r's ``peer_info()``.
        Afterwards every rank's forward takes the same tokens and returns the
        same output, each rank computing only its own experts."""
        n = len(infos)
        arr = (SenMoePeerInfo * max(n, 1))()
        for i, blob in enumerate(infos):
            if len(blob) != C.sizeof(SenMoePeerInfo):
                raise SenMoeError(ERR_BAD_ARG, f"peer info {i} has {len(blob)} bytes")
            C.memmove(C.byref(arr, i * C.sizeof(SenMoePeerInfo)), blob, len(blob))
        _check(lib().senmoe_layer_connect_peers(self._handle, int(rank), n, arr))

    def close(self) -> None:
        if getattr(self, "_handle", None):
            lib().senmoe_layer_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------- stage entry points
def router(x: torch.Tensor, router_weight: torch.Tensor, top_k: int, norm_topk_prob: bool = True,
           routed_scaling_factor: float = 1.0, stream=None):
    """Router half of DeepseekMoe::forward: returns (ids int32 [T, K], weights fp32 [T, K])."""
    H = x.shape[-1]
    E = router_weight.shape[0]
    xc = x.contiguous().reshape(-1, H)
    T = xc.shape[0]
    logits = torch.empty((T, E), dtype=torch.float32, device=x.device)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=x.device)
    wts = torch.empty((T, top_k), dtype=torch.float32, device=x.device)
    _check(lib().senmoe_router(_ptr(xc), T, _ptr(router_weight.contiguous()), H, E, top_k, int(norm_topk_prob),
                               float(routed_scaling_factor), _ptr(logits), _ptr(ids), _ptr(wts), _stream(stream)))
    return ids, wts


def quantized_linear(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     group_size: int = 64, bits: int = 4, stream=None) -> torch.Tensor:
    """nn::QuantizedLinear::forward without bias: x [..., in] bf16 @
    dequant(w [out, in*bits/32])^T -> [..., out] bf16."""
    if x.dtype != torch.bfloat16 or not x.is_cuda:
        raise TypeError("x must be a CUDA bfloat16 tensor")
    out_f, in_f = w.shape[0], x.shape[-1]
    xc = x.contiguous()
    T = xc.numel() // in_f
    y = torch.empty((*x.shape[:-1], out_f), dtype=torch.bfloat16, device=x.device)
    _check(lib().senmoe_quantized_linear(_ptr(xc), T, _ptr(_u32(w)), _ptr(scales.contiguous()),
                                         _ptr(biases.contiguous()), in_f, out_f, group_size, bits, _ptr(y),
                                         _stream(stream)))
    return y


@dataclass
class GemmaRouterWeights:
    """gemma4::Router parameters (gemma4.rs:683-700): the quantized ``proj``
    ([E, H*bits/32] u32, bf16 scales / biases [E, H/group]), the norm
    ``scale`` [H] and ``per_expert_scale`` [E], both bf16."""
    proj: SwitchLinear
    scale: torch.Tensor
    per_expert_scale: torch.Tensor


class GemmaRouter:
    """gemma4::Router::forward (gemma4.rs:716-736) on the GPU: rms_norm with
    weight scale * H^-1/2, quantized projection, top-k, softmax over the k,
    * per_expert_scale.  Borrows the weight tensors."""

    def __init__(self, hidden_size: int, num_experts: int, top_k: int, weights: GemmaRouterWeights,
                 rms_norm_eps: float = 1e-6, bits: int = 8, group_size: int = 64):
        self.top_k, self.weights = top_k, weights
        r = SenMoeGemmaRouter()
        r.hidden_size, r.num_experts, r.top_k, r.bits, r.group_size = hidden_size, num_experts, top_k, bits, group_size
        r.rms_norm_eps = float(rms_norm_eps)
        self._w32 = _u32(weights.proj.weight)
        r.proj_weight, r.proj_scales, r.proj_biases = _ptr(self._w32), _ptr(weights.proj.scales), _ptr(weights.proj.biases)
        r.scale, r.per_expert_scale = _ptr(weights.scale), _ptr(weights.per_expert_scale)
        self._r = r

    def forward(self, x: torch.Tensor, stream=None):
        """x [..., H] bf16 -> (indices int32 [..., K], weights fp32 [..., K])."""
        H = self._r.hidden_size
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.shape[-1] != H:
            raise TypeError("x must be a CUDA bfloat16 tensor [..., hidden_size]")
        xc = x.contiguous()
        T = xc.numel() // H
        ids = torch.empty((*x.shape[:-1], self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((*x.shape[:-1], self.top_k), dtype=torch.float32, device=x.device)
        _check(lib().senmoe_gemma_router(C.byref(self._r), _ptr(xc), T, _ptr(ids), _ptr(w), _stream(stream)))
        return ids, w

    __call__ = forward


def dispatch(topk_ids: torch.Tensor, num_experts: int, stream=None):
    """Expert-contiguous permutation: returns (perm, inverse, offsets, active_list)."""
    ids = topk_ids.to(torch.int32).contiguous()
    T, K = ids.shape
    dev = ids.device
    perm = torch.empty(T * K, dtype=torch.int32, device=dev)
    inv = torch.empty(T * K, dtype=torch.int32, device=dev)
    offs = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    scratch = torch.zeros(num_experts + 2, dtype=torch.int32, device=dev)
    _check(lib().senmoe_dispatch(_ptr(ids), T, K, num_experts, _ptr(perm), _ptr(inv), _ptr(offs), _ptr(scratch),
                                 _stream(stream)))
    n = int(scratch[num_experts].item())
    if int(scratch[num_experts + 1].item()):
        raise SenMoeError(ERR_DEVICE, f"dispatch saw an expert id outside [0, {num_experts})")
    return perm, inv, offs, scratch[:n].clone()


# ------------------------------------------------------------ layer stack
class MoeStack:
    """A stack of MoE blocks chained as in the decoder
    (``h_{l+1} = h_l + DeepseekMoe_l(h_l)``, deepseek_v2.rs:613-620 and the
    layer loop :665-687), with the residual add fused into each block's combine.

    ``forward`` accepts a host or device bf16 tensor ``[T, H]`` and returns the
    result on the same side.  With ``use_graph`` the whole chain for a given T
    is captured once into a CUDA graph and replayed, so a decode step costs one
    graph launch instead of ~6 kernel launches per layer.
    """

    def __init__(self, layers: list, max_tokens: int, use_graph: bool = True, tokens_per_rank=None):
        """``tokens_per_rank``: token-local expert parallelism (every rank
        chains its own tokens; forward(x) takes this rank's count of them)."""
        self.layers = layers
        self.tokens_per_rank = None if tokens_per_rank is None else [int(v) for v in tokens_per_rank]
        self.hidden = layers[0].args.hidden_size
        self.max_tokens = max_tokens
        self.use_graph = use_graph
        dev = torch.device("cuda", layers[0].device)
        self.bufs = [torch.zeros(max_tokens, self.hidden, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.stream = torch.cuda.Stream(device=dev)
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.outs: dict[int, torch.Tensor] = {}  # device view holding the chain's output per T
        self.host_out: dict[int, torch.Tensor] = {}

    def _run(self, T: int) -> torch.Tensor:
        a, b = self.bufs
        for L in self.layers:
            if self.tokens_per_rank is not None:
                L.forward_tokens(a[:T], self.tokens_per_rank, residual=True, stream=self.stream, out=b[:T])
            else:
                L.forward_residual(a[:T], stream=self.stream, out=b[:T])
            a, b = b, a
        return a[:T]

    def _graph(self, T: int) -> torch.cuda.CUDAGraph:
        g = self.graphs.get(T)
        if g is None:
            saved = self.bufs[0][:T].clone()
            with torch.cuda.stream(self.stream):
                self._run(T)  # warm-up outside capture (kernel attributes, lazy loading)
                self.bufs[0][:T].copy_(saved)
            self.stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                self.outs[T] = self._run(T)
            self.graphs[T] = g
        return g

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        if T > self.max_tokens:
            raise SenMoeError(ERR_BAD_ARG, f"T={T} exceeds max_tokens={self.max_tokens}")
        on_host = not x.is_cuda
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.bufs[0][:T].copy_(x, non_blocking=True)
            if self.use_graph:
                self._graph(T).replay()
                y = self.outs[T]
            else:
                y = self._run(T)
            if on_host:
                out = self.host_out.get(T)
                if out is None:
                    out = torch.empty((T, self.hidden), dtype=torch.bfloat16, pin_memory=True)
                    self.host_out[T] = out
                out.copy_(y, non_blocking=True)
                self.stream.synchronize()
                return out
        torch.cuda.current_stream().wait_stream(self.stream)
        return y

    def release(self) -> None:
        """Drops the captured graphs (before destroying layers or process groups)."""
        self.graphs.clear()
