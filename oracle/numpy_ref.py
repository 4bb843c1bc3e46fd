"""TEST INFRASTRUCTURE ONLY -- an independent numpy restatement of the same
MoE block as moe_oracle.c, written separately so the two can check each other
(small sizes only; it is vectorised but not fast).

Follows src/engine/mlx_lm/models/deepseek_v2.rs:466-553,
src/engine/mlx_lm/models/gemma4.rs:716-736 (router) and :809-848 (GeGLU
experts) and src/engine/mlx_lm/utils/moe.rs:20-77 with the MLX rounding points
listed in moe_oracle.c.  bf16 values are carried as uint16 bit patterns.
"""
from __future__ import annotations

import numpy as np


def bf16_bits(a) -> np.ndarray:
    """float -> bf16 bits, round to nearest even (NaN kept quiet)."""
    f = np.ascontiguousarray(a, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_val(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rbf(a) -> np.ndarray:
    return bf16_val(bf16_bits(a))


def quantize(w: np.ndarray, group: int = 64, bits: int = 4):
    """MLX-style affine quantizer (same algorithm as orc_quantize_affine)."""
    w = np.asarray(w, dtype=np.float32)
    *lead, cols = w.shape
    g = w.reshape(*lead, cols // group, group)
    n_bins = np.float32((1 << bits) - 1)
    mx, mn = g.max(-1, keepdims=True), g.min(-1, keepdims=True)
    use_min = np.abs(mn) > np.abs(mx)
    scale = np.maximum((mx - mn) / n_bins, np.float32(1e-7)).astype(np.float32)
    scale = np.where(use_min, scale, -scale).astype(np.float32)
    edge = np.where(use_min, mn, mx)
    q0 = np.rint(edge / scale)
    nz = q0 != 0
    scale = np.where(nz, edge / np.where(nz, q0, 1), scale).astype(np.float32)
    bias = np.where(nz, edge, 0).astype(np.float32)
    q = np.clip(np.rint((g - bias) / scale), 0, n_bins).astype(np.uint32).reshape(*lead, cols)
    per = 32 // bits
    q = q.reshape(*lead, cols // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    wq = np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)
    return wq, bf16_bits(scale[..., 0]), bf16_bits(bias[..., 0])


def dequantize(wq, s, b, group: int = 64, bits: int = 4) -> np.ndarray:
    """w = q * scale + bias (fp32), MLX packing (lower columns in lower bits)."""
    wq = np.asarray(wq, dtype=np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = ((wq[..., None] >> shifts) & np.uint32((1 << bits) - 1)).reshape(*wq.shape[:-1], -1).astype(np.float32)
    cols = q.shape[-1]
    qg = q.reshape(*q.shape[:-1], cols // group, group)
    w = qg * bf16_val(s)[..., None] + bf16_val(b)[..., None]
    return w.reshape(*q.shape).astype(np.float32)


def gather_qmm(x_bits, wq, s, b, idx, group: int = 64, bits: int = 4) -> np.ndarray:
    """y[i] = bf16(x[i // rep] @ dequant(w[idx[i]]).T), float64 accumulation."""
    x = bf16_val(x_bits).astype(np.float64)
    idx = np.asarray(idx).reshape(-1)
    rep = idx.size // x.shape[0]
    wd = dequantize(wq, s, b, group, bits).astype(np.float64)
    out = np.stack([wd[idx[i]] @ x[i // rep] for i in range(idx.size)])
    return bf16_bits(out.astype(np.float32))


def rounding(mode: int):
    """The rounding applied at the MLX graph's bf16 points (mode 0) or none (mode 1)."""
    return rbf if mode == 0 else (lambda a: np.asarray(a, dtype=np.float32))


def route(cfg, w, x, mode: int = 0):
    """Router of deepseek_v2.rs:526-543 for x [T, H] fp32 (bf16 values):
    returns (ids [T, K] int32, weights [T, K] fp32)."""
    R = rounding(mode)
    E, K = cfg.num_experts, cfg.top_k
    logits = R((x.astype(np.float64) @ bf16_val(w.router_w).astype(np.float64).T).astype(np.float32))
    m = logits.max(-1, keepdims=True)
    ex = np.exp(logits - m).astype(np.float32)
    scores = R((ex / ex.sum(-1, keepdims=True, dtype=np.float64)).astype(np.float32))
    order = np.lexsort((np.broadcast_to(np.arange(E), scores.shape), -scores), axis=-1)  # score desc, id asc
    ids = order[:, :K].astype(np.int32)
    wts = np.take_along_axis(scores, ids, -1).astype(np.float32)
    if cfg.norm_topk_prob:
        den = R(wts.sum(-1, keepdims=True, dtype=np.float32)) + np.float32(1e-20)
        wts = (wts / den).astype(np.float32)
    if abs(cfg.routed_scaling_factor - 1.0) > 1.1920929e-7:
        wts = (wts * np.float32(cfg.routed_scaling_factor)).astype(np.float32)
    return ids, wts


def expert_mlp(xr, gd, ud, dd, mode: int = 0, activation: int = 0) -> np.ndarray:
    """One SwitchGlu expert on one token (deepseek_v2.rs:443-462; GeGLU:
    gemma4.rs:811-823): x row fp64, dequantised gate/up/down fp64; returns the
    down output (bf16 values, fp32)."""
    R = rounding(mode)
    g = R((gd @ xr).astype(np.float32))
    u = R((ud @ xr).astype(np.float32))
    if activation == 1:  # gelu_approximate, tanh form, rounded once
        g32 = g.astype(np.float32)
        a = R((np.float32(0.5) * g32 * (np.float32(1.0) + np.tanh(
            np.float32(0.7978845608028654) * (g32 + np.float32(0.044715) * g32 * g32 * g32)))).astype(np.float32))
    else:
        sg = R((1.0 / (1.0 + np.exp(-g.astype(np.float32)))).astype(np.float32))
        a = R(g * sg)
    h = R(a * u)
    return R((dd @ h.astype(np.float64)).astype(np.float32))


def shared_out(cfg, w, x, mode: int = 0) -> np.ndarray:
    """gate_t * shared_mlp(x_t) per token (deepseek_v2.rs:550-552), fp32 [T, H]."""
    sg_d = dequantize(w.sh_gate_w, w.sh_gate_s, w.sh_gate_b, cfg.group_size, cfg.bits).astype(np.float64)
    su_d = dequantize(w.sh_up_w, w.sh_up_s, w.sh_up_b, cfg.group_size, cfg.bits).astype(np.float64)
    sd_d = dequantize(w.sh_down_w, w.sh_down_s, w.sh_down_b, cfg.group_size, cfg.bits).astype(np.float64)
    out = np.zeros((x.shape[0], cfg.hidden), dtype=np.float32)
    for t in range(x.shape[0]):
        gate = np.float32(1.0)
        if cfg.shared_gate:
            a = float(x[t].astype(np.float64) @ bf16_val(w.sh_gate_vec).astype(np.float64))
            gate = np.float32(1.0 / (1.0 + np.exp(-np.float32(a))))
        out[t] = gate * expert_mlp(x[t].astype(np.float64), sg_d, su_d, sd_d, mode)
    return out


def moe_forward(cfg, w, x_bits, mode: int = 0, ids=None, wts=None):
    """cfg/w: oracle.MoeConfig / oracle.MoeWeights.  Same outputs as the C
    oracle; ids / wts [T, K] given: Experts::forward (gemma4.rs:842-848)."""
    H, K = cfg.hidden, cfg.top_k
    x = bf16_val(x_bits).reshape(-1, H)
    T = x.shape[0]
    if ids is None:
        ids, wts = route(cfg, w, x, mode)
    act = getattr(cfg, "activation", 0)
    g_d = dequantize(w.gate_w, w.gate_s, w.gate_b, cfg.group_size, cfg.bits).astype(np.float64)
    u_d = dequantize(w.up_w, w.up_s, w.up_b, cfg.group_size, cfg.bits).astype(np.float64)
    d_d = dequantize(w.down_w, w.down_s, w.down_b, cfg.group_size, cfg.bits).astype(np.float64)
    y = np.zeros((T, H), dtype=np.float32)
    for t in range(T):
        acc = np.zeros(H, dtype=np.float32)
        for j in range(K):
            e = ids[t, j]
            acc = (acc + expert_mlp(x[t].astype(np.float64), g_d[e], u_d[e], d_d[e], mode, act) *
                   wts[t, j]).astype(np.float32)
        y[t] = acc
    if cfg.shared_intermediate:
        y = (y + shared_out(cfg, w, x, mode)).astype(np.float32)
    return dict(y_f32=y, y_bf16=bf16_bits(y), ids=ids, weights=wts)


def gemma_route(rc, rw, x_bits):
    """Router::forward of gemma4.rs:716-736 (rc / rw: oracle.GemmaRouterConfig /
    GemmaRouterWeights): rms_norm in f32 with weight f32(scale) * H^-1/2,
    quantized projection in f32, top-k (score desc, id asc), softmax over
    the k, * per_expert_scale.  Returns (ids [T, K], weights [T, K], scores)."""
    H, E, K = rc.hidden, rc.num_experts, rc.top_k
    x = bf16_val(x_bits).reshape(-1, H).astype(np.float32)
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True)
    inv = (1.0 / np.sqrt(ms + rc.eps)).astype(np.float32)
    weff = (bf16_val(rw.scale) * np.float32(H ** -0.5)).astype(np.float32)
    xn = ((x * inv).astype(np.float32) * weff).astype(np.float32)
    pd = dequantize(rw.proj_w, rw.proj_s, rw.proj_b, rc.group_size, rc.bits).astype(np.float64)
    scores = (xn.astype(np.float64) @ pd.T).astype(np.float32)
    order = np.lexsort((np.broadcast_to(np.arange(E), scores.shape), -scores), axis=-1)
    ids = order[:, :K].astype(np.int32)
    picked = np.take_along_axis(scores, ids, -1).astype(np.float32)
    ex = np.exp((picked - picked.max(-1, keepdims=True)).astype(np.float32)).astype(np.float32)
    wts = (ex / ex.sum(-1, keepdims=True)).astype(np.float32) * bf16_val(rw.per_expert_scale)[ids]
    return ids, wts.astype(np.float32), scores
