"""Generates the committed golden fixtures in this directory.

Run from the repository root:  python tests/golden/make_golden.py

Fixtures are produced by the pure-numpy restatement (oracle/numpy_ref.py),
independently of the C oracle, so the tests can check one against the other
and both against the CUDA kernels.

gather_qmm_kat.npz
    The reference's own known-answer test for the primitive,
    src/engine/mlx_lm/utils/moe.rs:89-146 (gather_qmm_matches_per_expert_reference),
    with its exact input formulas: E=4, out=32, in=64, group 64, 4 bits,
    w[i] = ((i % 7) - 3) * 0.05 over [E, out, in], x[i] = ((i % 5) - 2) * 0.1
    over [M=3, in], indices [0, 1, 2, 3, 1, 0] as [M, K=2].  The reference
    runs it in float32; this build's layout is bf16 (x, scales, biases), so x
    and the quantization parameters are bf16-rounded.  Expected output: the
    per-pair dequantize + matmul in float64 (the reference's check, moe.rs:118-144),
    compared with tolerance 1e-2 max abs as the reference does.

moe_block_small_{4,8}bit.npz
    A small DeepseekMoe block (H=128, I=64, E=8, K=2, T=5; 8-bit also has a
    sigmoid-gated shared expert with I_shared=64) with seeded inputs; outputs
    from the numpy restatement in MLX rounding mode.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from oracle import numpy_ref as N  # noqa: E402


def kat():
    e, out, k_in, group, bits = 4, 32, 64, 64, 4
    wf = ((np.arange(e * out * k_in) % 7).astype(np.float32) - 3.0) * np.float32(0.05)
    wf = wf.reshape(e, out, k_in)
    wq, s, b = N.quantize(wf, group, bits)
    m, k = 3, 2
    xf = ((np.arange(m * k_in) % 5).astype(np.float32) - 2.0) * np.float32(0.1)
    x = N.bf16_bits(xf.reshape(m, k_in))
    inds = np.array([0, 1, 2, 3, 1, 0], dtype=np.int32).reshape(m, k)
    wd = N.dequantize(wq, s, b, group, bits).astype(np.float64)
    xd = N.bf16_val(x).astype(np.float64)
    expected = np.stack([[wd[inds[mi, ki]] @ xd[mi] for ki in range(k)] for mi in range(m)])  # [M, K, out]
    y = N.gather_qmm(x, wq, s, b, inds, group, bits).reshape(m, k, out)
    np.savez(os.path.join(HERE, "gather_qmm_kat.npz"), w_float=wf, wq=wq, scales=s, biases=b, x=x, inds=inds,
             expected_f64=expected, y_bf16=y, group=group, bits=bits)


def small_block(bits: int):
    from types import SimpleNamespace
    H, I, E, K, T = 128, 64, 8, 2, 5
    shared = 64 if bits == 8 else 0
    cfg = SimpleNamespace(hidden=H, intermediate=I, num_experts=E, top_k=K, bits=bits, group_size=64,
                          norm_topk_prob=True, routed_scaling_factor=1.0 if bits == 4 else 2.5,
                          shared_intermediate=shared, shared_gate=bool(shared))
    rng = np.random.default_rng(1234 + bits)
    w = SimpleNamespace()
    w.router_w = N.bf16_bits(rng.standard_normal((E, H)).astype(np.float32) * np.float32(0.09))
    for name, shp in (("gate", (E, I, H)), ("up", (E, I, H)), ("down", (E, H, I))):
        q, s, b = N.quantize(rng.standard_normal(shp).astype(np.float32) * np.float32(0.05), 64, bits)
        setattr(w, f"{name}_w", q), setattr(w, f"{name}_s", s), setattr(w, f"{name}_b", b)
    for name in ("gate", "up", "down"):
        for sfx in ("w", "s", "b"):
            setattr(w, f"sh_{name}_{sfx}", None)
    w.sh_gate_vec = None
    if shared:
        for name, shp in (("gate", (shared, H)), ("up", (shared, H)), ("down", (H, shared))):
            q, s, b = N.quantize(rng.standard_normal(shp).astype(np.float32) * np.float32(0.05), 64, bits)
            setattr(w, f"sh_{name}_w", q), setattr(w, f"sh_{name}_s", s), setattr(w, f"sh_{name}_b", b)
        w.sh_gate_vec = N.bf16_bits(rng.standard_normal(H).astype(np.float32) * np.float32(0.05))
    x = N.bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    r = N.moe_forward(cfg, w, x, mode=0)
    arrays = {k: v for k, v in vars(w).items() if v is not None}
    np.savez(os.path.join(HERE, f"moe_block_small_{bits}bit.npz"), x=x, y_f32=r["y_f32"], y_bf16=r["y_bf16"],
             ids=r["ids"], weights=r["weights"],
             cfg=np.array([H, I, E, K, bits, 64, 1, shared, int(bool(shared))], dtype=np.int64),
             routed_scaling_factor=np.float32(cfg.routed_scaling_factor), **arrays)


if __name__ == "__main__":
    kat()
    small_block(4)
    small_block(8)
    print("fixtures written to", HERE)
