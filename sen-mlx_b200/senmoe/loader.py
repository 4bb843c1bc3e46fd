"""MoE-block weights from MLX safetensors checkpoints: the load side of the
block, with the reference loaders' naming and config rules.

DeepSeek-V2 (``load_deepseek_v2_any``, src/engine/mlx_native.rs:3365-3530):
  * shards listed by ``model.safetensors.index.json`` (its ``weight_map``), or
    a single ``model.safetensors``;
  * ``config.json::quantization.{group_size, bits}``, default (64, 4)
    (:3381-3389);
  * MoE layers: ``n_routed_experts > 0``, ``i >= first_k_dense_replace`` and
    (``moe_layer_freq <= 0`` or ``i % moe_layer_freq == 0``)
    (models/deepseek_v2.rs:152-156), holding
    ``model.layers.{i}.mlp.gate.weight`` (the bf16 router),
    ``...mlp.switch_mlp.{gate,up,down}_proj.{weight,scales,biases}`` (stacked,
    already quantized) and, with ``n_shared_experts > 0``,
    ``...mlp.shared_experts.{gate,up,down}_proj.{weight,scales,biases}``.  The
    reference renames ``mlp.`` to ``moe.`` for these layers (:3422-3435);
    both spellings are accepted.

Gemma-4 (``load_gemma4_any``, mlx_native.rs:3090-3357):
  * ``config.json::text_config`` (or the top level) with ``enable_moe_block``,
    ``num_experts``, ``top_k_experts``, ``moe_intermediate_size``,
    ``rms_norm_eps`` (models/gemma4.rs:132-142, 264-273, 1430-1475);
  * keys may carry a ``language_model.`` prefix (:3180-3184);
  * per layer ``router.{proj.weight, proj.scales, proj.biases, scale,
    per_expert_scale}`` and ``experts.switch_glu.{gate,up,down}_proj.*``; the
    experts take the top-level quantization (gemma4.rs:1462-1474), the router
    projection its own width (8-bit in the shipped checkpoint), read here
    from the tensor's shape.

The checkpoint's tensors are used as stored (packed u32 codes, bf16 scales
and biases); fp16 / fp32 scales, biases or router weights are converted to
bf16, the only float layout the kernels take.
"""
from __future__ import annotations

import json
import os
import struct
import warnings
from dataclasses import dataclass

import numpy as np
import torch

from . import GemmaRouterWeights, MoeArgs, MoeWeights, SwitchLinear, ACT_GEGLU

_DTYPES = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "U32": np.uint32, "I32": np.int32,
           "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "F64": np.float64, "I64": np.int64}


class SafetensorsCheckpoint:
    """Read-only view of a checkpoint directory's safetensors shards; tensors
    are memory-mapped, returned as numpy arrays (bf16 as uint16 bits)."""

    def __init__(self, model_dir: str):
        self.dir = model_dir
        index = os.path.join(model_dir, "model.safetensors.index.json")
        self._where: dict[str, str] = {}
        if os.path.exists(index):
            with open(index) as f:
                for name, shard in json.load(f)["weight_map"].items():
                    self._where[name] = os.path.join(model_dir, shard)
        else:
            single = os.path.join(model_dir, "model.safetensors")
            if not os.path.exists(single):
                raise FileNotFoundError(f"no model.safetensors.index.json or model.safetensors in {model_dir}")
            for name in self._header(single)[0]:
                self._where[name] = single
        self._headers: dict[str, tuple[dict, int]] = {}

    @staticmethod
    def _header(path: str):
        with open(path, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            head = json.loads(f.read(n))
        head.pop("__metadata__", None)
        return head, 8 + n

    def keys(self):
        return self._where.keys()

    def __contains__(self, name: str) -> bool:
        return name in self._where

    def dtype(self, name: str) -> str:
        path = self._where[name]
        if path not in self._headers:
            self._headers[path] = self._header(path)
        return self._headers[path][0][name]["dtype"]

    def get(self, name: str) -> np.ndarray:
        path = self._where[name]
        if path not in self._headers:
            self._headers[path] = self._header(path)
        head, base = self._headers[path]
        meta = head[name]
        dt = _DTYPES.get(meta["dtype"])
        if dt is None:
            raise ValueError(f"{name}: unsupported dtype {meta['dtype']}")
        start, end = meta["data_offsets"]
        shape = tuple(meta["shape"])
        count = int(np.prod(shape)) if shape else 1
        if (end - start) != count * np.dtype(dt).itemsize:
            raise ValueError(f"{name}: data size {end - start} does not match shape {shape} x {meta['dtype']}")
        # a scalar tensor (shape []) is mapped as one element and reshaped
        m = np.memmap(path, dtype=dt, mode="r", offset=base + start, shape=shape if shape else (1,))
        return m if shape else m.reshape(())


def _bf16_bits(ckpt: SafetensorsCheckpoint, name: str) -> np.ndarray:
    a = ckpt.get(name)
    kind = ckpt.dtype(name)
    if kind == "BF16":
        return np.asarray(a)
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    out = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # round to nearest even
    # NaN stays a NaN of the same sign (rounding its payload could carry into
    # the exponent and give Inf or flip the sign); quiet NaN 0x7FC0 / 0xFFC0
    nan = np.isnan(f)
    if nan.any():
        out[nan] = np.where(np.signbit(f[nan]), 0xFFC0, 0x7FC0).astype(np.uint16)
    return out.reshape(np.shape(a))  # ascontiguousarray makes a 0-d input 1-d


def _to_device(a: np.ndarray, device, bf16: bool = False) -> torch.Tensor:
    # memory-mapped shards are read-only: a host tensor gets its own copy; a
    # device tensor is copied out of the mapping (the read-only host view
    # only feeds that copy, so torch's non-writable-array warning is moot)
    host = torch.device(device).type == "cpu"
    a = np.array(a, copy=True) if host else np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    elif bf16:
        a = a.view(np.int16)
    with warnings.catch_warnings():
        warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
        t = torch.from_numpy(a)
    if bf16:
        t = t.view(torch.bfloat16)
    return t.to(device)


def _switch_linear(ckpt, prefix: str, device) -> SwitchLinear:
    return SwitchLinear(_to_device(ckpt.get(f"{prefix}.weight"), device),
                        _to_device(_bf16_bits(ckpt, f"{prefix}.scales"), device, bf16=True),
                        _to_device(_bf16_bits(ckpt, f"{prefix}.biases"), device, bf16=True))


def _config(model_dir: str) -> dict:
    with open(os.path.join(model_dir, "config.json")) as f:
        return json.load(f)


def _quant(cfg: dict) -> tuple[int, int]:
    q = cfg.get("quantization") or cfg.get("quantization_config") or {}
    return int(q.get("group_size", 64)), int(q.get("bits", 4))


def _bits_from_shape(packed_cols: int, in_features: int) -> int:
    bits = packed_cols * 32 // in_features
    if bits not in (4, 8) or packed_cols * 32 != bits * in_features:
        raise ValueError(f"packed width {packed_cols} words does not fit {in_features} columns at 4 or 8 bits")
    return bits


@dataclass
class LoadedMoe:
    """One MoE layer of a checkpoint: its index, the block arguments and the
    weights (device tensors in MLX layout)."""
    layer: int
    args: MoeArgs
    weights: MoeWeights


@dataclass
class LoadedGemmaMoe:
    layer: int
    args: MoeArgs               # the experts (GeGLU); the router is separate
    weights: MoeWeights         # router_weight None: Experts::forward only
    router: GemmaRouterWeights
    router_bits: int
    rms_norm_eps: float


def load_deepseek_moe(model_dir: str, device="cuda", layers: list[int] | None = None) -> list[LoadedMoe]:
    """The MoE layers of a DeepSeek-V2 MLX checkpoint (all, or ``layers``)."""
    cfg = _config(model_dir)
    group, bits = _quant(cfg)
    E, n_layers = int(cfg["n_routed_experts"]), int(cfg["num_hidden_layers"])
    first_dense = int(cfg.get("first_k_dense_replace", 0))
    freq = int(cfg.get("moe_layer_freq", 1))
    n_shared = int(cfg.get("n_shared_experts") or 0)
    ckpt = SafetensorsCheckpoint(model_dir)
    out = []
    for i in range(n_layers):
        if not (E > 0 and i >= first_dense and (freq <= 0 or i % freq == 0)):
            continue
        if layers is not None and i not in layers:
            continue
        pre = next((p for p in (f"model.layers.{i}.mlp", f"model.layers.{i}.moe")
                    if f"{p}.switch_mlp.gate_proj.weight" in ckpt), None)
        if pre is None:
            raise KeyError(f"layer {i}: no switch_mlp tensors under model.layers.{i}.mlp / .moe")
        args = MoeArgs(hidden_size=int(cfg["hidden_size"]), moe_intermediate_size=int(cfg["moe_intermediate_size"]),
                       n_routed_experts=E, num_experts_per_tok=int(cfg["num_experts_per_tok"]),
                       n_shared_experts=n_shared, norm_topk_prob=bool(cfg.get("norm_topk_prob", False)),
                       routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)), bits=bits,
                       group_size=group)
        w = MoeWeights(router_weight=_to_device(_bf16_bits(ckpt, f"{pre}.gate.weight"), device, bf16=True),
                       gate_proj=_switch_linear(ckpt, f"{pre}.switch_mlp.gate_proj", device),
                       up_proj=_switch_linear(ckpt, f"{pre}.switch_mlp.up_proj", device),
                       down_proj=_switch_linear(ckpt, f"{pre}.switch_mlp.down_proj", device))
        if n_shared > 0:
            w.shared_gate_proj = _switch_linear(ckpt, f"{pre}.shared_experts.gate_proj", device)
            w.shared_up_proj = _switch_linear(ckpt, f"{pre}.shared_experts.up_proj", device)
            w.shared_down_proj = _switch_linear(ckpt, f"{pre}.shared_experts.down_proj", device)
        out.append(LoadedMoe(i, args, w))
    return out


def load_gemma4_moe(model_dir: str, device="cuda", layers: list[int] | None = None) -> list[LoadedGemmaMoe]:
    """The MoE blocks (router + routed experts) of a Gemma-4 MLX checkpoint."""
    root = _config(model_dir)
    cfg = root.get("text_config", root)
    group, bits = _quant(root)
    if not cfg.get("enable_moe_block"):
        return []
    E, K, I = cfg.get("num_experts"), cfg.get("top_k_experts"), cfg.get("moe_intermediate_size")
    if not (E and K and I and E > 0 and K > 0 and I > 0):
        return []  # a half-declared MoE counts as absent (gemma4.rs:260-273)
    H, eps = int(cfg["hidden_size"]), float(cfg.get("rms_norm_eps", 1e-6))
    ckpt = SafetensorsCheckpoint(model_dir)
    name = lambda k: k if k in ckpt else f"language_model.{k}"
    out = []
    for i in range(int(cfg["num_hidden_layers"])):
        if layers is not None and i not in layers:
            continue
        rp, ep = f"model.layers.{i}.router", f"model.layers.{i}.experts.switch_glu"
        if name(f"{rp}.proj.weight") not in ckpt:
            continue  # a dense layer
        args = MoeArgs(hidden_size=H, moe_intermediate_size=int(I), n_routed_experts=int(E),
                       num_experts_per_tok=int(K), norm_topk_prob=False, bits=bits, group_size=group,
                       activation=ACT_GEGLU)
        sl = lambda p: SwitchLinear(_to_device(ckpt.get(name(f"{p}.weight")), device),
                                    _to_device(_bf16_bits(ckpt, name(f"{p}.scales")), device, bf16=True),
                                    _to_device(_bf16_bits(ckpt, name(f"{p}.biases")), device, bf16=True))
        w = MoeWeights(router_weight=None, gate_proj=sl(f"{ep}.gate_proj"), up_proj=sl(f"{ep}.up_proj"),
                       down_proj=sl(f"{ep}.down_proj"))
        proj = sl(f"{rp}.proj")
        rw = GemmaRouterWeights(proj, _to_device(_bf16_bits(ckpt, name(f"{rp}.scale")), device, bf16=True),
                                _to_device(_bf16_bits(ckpt, name(f"{rp}.per_expert_scale")), device, bf16=True))
        out.append(LoadedGemmaMoe(i, args, w, rw, _bits_from_shape(proj.weight.shape[-1], H), eps))
    return out
