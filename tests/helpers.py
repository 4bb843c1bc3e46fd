"""Shared helpers for the tests: moving oracle (numpy) layers to the device
and the parity metrics with their tolerances."""
from __future__ import annotations

import numpy as np

# Block-output tolerance (bf16): max abs error and relative L2 error.
MAX_ABS_TOL = 2e-2
REL_L2_TOL = 5e-3


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bf16_np_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def t_bf16(a, device="cuda"):
    """numpy uint16 (bf16 bits) -> torch bfloat16 on device."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint16).view(np.int16)).view(torch.bfloat16).to(device)


def t_u32(a, device="cuda"):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(device)


def to_numpy_bf16(t) -> np.ndarray:
    """torch bfloat16 -> numpy uint16 bits."""
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def device_weights(mw, device="cuda"):
    """oracle.MoeWeights -> senmoe.MoeWeights on the device."""
    import senmoe
    sl = lambda w, s, b: senmoe.SwitchLinear(t_u32(w, device), t_bf16(s, device), t_bf16(b, device))
    out = senmoe.MoeWeights(
        router_weight=None if mw.router_w is None else t_bf16(mw.router_w, device),
        gate_proj=sl(mw.gate_w, mw.gate_s, mw.gate_b),
        up_proj=sl(mw.up_w, mw.up_s, mw.up_b),
        down_proj=sl(mw.down_w, mw.down_s, mw.down_b),
    )
    if mw.sh_gate_w is not None:
        out.shared_gate_proj = sl(mw.sh_gate_w, mw.sh_gate_s, mw.sh_gate_b)
        out.shared_up_proj = sl(mw.sh_up_w, mw.sh_up_s, mw.sh_up_b)
        out.shared_down_proj = sl(mw.sh_down_w, mw.sh_down_s, mw.sh_down_b)
    if mw.sh_gate_vec is not None:
        out.shared_gate_vector = t_bf16(mw.sh_gate_vec, device)
    return out


def moe_args(cfg, expert_path=0):
    """oracle.MoeConfig -> senmoe.MoeArgs."""
    import senmoe
    return senmoe.MoeArgs(expert_path=expert_path, hidden_size=cfg.hidden, moe_intermediate_size=cfg.intermediate,
                          n_routed_experts=cfg.num_experts, num_experts_per_tok=cfg.top_k,
                          n_shared_experts=(cfg.shared_intermediate // cfg.intermediate) if cfg.shared_intermediate else 0,
                          norm_topk_prob=cfg.norm_topk_prob, routed_scaling_factor=cfg.routed_scaling_factor,
                          bits=cfg.bits, group_size=cfg.group_size, shared_gate=cfg.shared_gate,
                          activation=getattr(cfg, "activation", 0))


def topk_match_except_ties(ids_gpu, ids_ref, scores_ref, ulp_rel=2.0 ** -7):
    """True when every token's top-k SET matches, except tokens whose
    differing experts sit within one bf16 ulp of the k-th reference score
    (an exact or near router tie).  Returns (ok, n_tie_tokens)."""
    ids_gpu = np.asarray(ids_gpu)
    ids_ref = np.asarray(ids_ref)
    ties = 0
    for t in range(ids_ref.shape[0]):
        a, b = set(ids_gpu[t].tolist()), set(ids_ref[t].tolist())
        if a == b:
            continue
        kth = scores_ref[t, ids_ref[t, -1]]
        diff = a.symmetric_difference(b)
        if all(abs(scores_ref[t, e] - kth) <= ulp_rel * abs(kth) for e in diff):
            ties += 1
            continue
        return False, ties
    return True, ties


def fixture_layer(d):
    """(oracle.MoeConfig, oracle.MoeWeights) of a tests/golden/moe_block_small_*.npz fixture."""
    from oracle import oracle as O

    H, I, E, K, bits, g, norm, shared, sgate = (int(v) for v in d["cfg"])
    cfg = O.MoeConfig(hidden=H, intermediate=I, num_experts=E, top_k=K, bits=bits, group_size=g,
                      norm_topk_prob=bool(norm), routed_scaling_factor=float(d["routed_scaling_factor"]),
                      shared_intermediate=shared, shared_gate=bool(sgate))
    w = O.MoeWeights(d["router_w"], d["gate_w"], d["gate_s"], d["gate_b"], d["up_w"], d["up_s"], d["up_b"],
                     d["down_w"], d["down_s"], d["down_b"])
    if shared:
        for k in ("sh_gate_w", "sh_gate_s", "sh_gate_b", "sh_up_w", "sh_up_s", "sh_up_b", "sh_down_w",
                  "sh_down_s", "sh_down_b", "sh_gate_vec"):
            setattr(w, k, d[k])
    return cfg, w


def routing_mismatches(ids_gpu, ids_ref, scores_ref, ulp_rel=2.0 ** -7):
    """Tokens whose ordered top-k ids differ between the GPU and the oracle,
    and whether every one of them is explained by a router tie: a differing
    expert of the top-k SET within one bf16 ulp of the k-th reference score,
    or (same set, other order) slot pairs whose reference scores lie within
    one bf16 ulp of each other.  Returns (mismatched token indices, all_ties)."""
    ids_gpu = np.asarray(ids_gpu)
    ids_ref = np.asarray(ids_ref)
    bad = np.nonzero((ids_gpu != ids_ref).any(axis=1))[0]
    for t in bad:
        a, b = ids_gpu[t].tolist(), ids_ref[t].tolist()
        if set(a) != set(b):
            kth = scores_ref[t, b[-1]]
            if not all(abs(scores_ref[t, e] - kth) <= ulp_rel * abs(kth) for e in set(a) ^ set(b)):
                return bad, False
        else:
            for ea, eb in zip(a, b):
                if ea != eb and abs(scores_ref[t, ea] - scores_ref[t, eb]) > ulp_rel * max(abs(scores_ref[t, eb]),
                                                                                           1e-30):
                    return bad, False
    return bad, True


def max_dropped(num_tokens: int) -> int:
    """Tokens a parity check may leave out for router ties: 1 % of T, at least one."""
    return max(1, num_tokens // 100)
