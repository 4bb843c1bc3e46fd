"""GPU parity of the Gemma-4 MoE pieces through the C ABI against the oracle:
Router::forward (gemma4.rs:716-736) and Experts::forward with GeGLU experts
(gemma4.rs:809-848).

Tolerances: router top-k sets identical except at near-ties of the fp32
scores (the GPU sums the projection in fp32, the oracle in fp64), router
weights within 2e-5 absolute; expert outputs max abs <= 2e-2 and relative
L2 <= 5e-3 against the oracle's fp32 result."""
import numpy as np
import pytest

from helpers import (MAX_ABS_TOL, REL_L2_TOL, bf16_np_to_f32, device_weights, moe_args, rel_l2, t_bf16, t_u32,
                     to_numpy_bf16, topk_match_except_ties)
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def senmoe():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import senmoe as s
    s.lib()
    return s


def gpu_router(senmoe, rc, rw):
    w = senmoe.GemmaRouterWeights(senmoe.SwitchLinear(t_u32(rw.proj_w), t_bf16(rw.proj_s), t_bf16(rw.proj_b)),
                                  t_bf16(rw.scale), t_bf16(rw.per_expert_scale))
    return senmoe.GemmaRouter(rc.hidden, rc.num_experts, rc.top_k, w, rms_norm_eps=rc.eps, bits=rc.bits,
                              group_size=rc.group_size)


def check_router(ids, w, rc, rw, x):
    ids_r, w_r, sc_r = O.gemma_router(rc, rw, x)
    ok, ties = topk_match_except_ties(ids, ids_r, sc_r, ulp_rel=1e-5)
    assert ok, "top-k ids differ beyond near-ties"
    same = (np.sort(ids, 1) == np.sort(ids_r, 1)).all(1)
    # same set: compare the weights expert by expert
    for t in np.nonzero(same)[0]:
        got = dict(zip(ids[t].tolist(), w[t].tolist()))
        ref = dict(zip(ids_r[t].tolist(), w_r[t].tolist()))
        for e in ref:
            assert abs(got[e] - ref[e]) <= 2e-5, (t, e, got[e], ref[e])
    return ids_r, w_r


@pytest.mark.parametrize("T", [1, 7, 64])
@pytest.mark.parametrize("bits", [8, 4])
def test_gemma_router_vs_oracle(senmoe, T, bits):
    """The 26B-A4B router shape (H=2816, E=128, K=8; 8-bit projection in the
    checkpoint, 4-bit also accepted)."""
    rc = O.GemmaRouterConfig(hidden=2816, num_experts=128, top_k=8, bits=bits)
    rw = O.make_gemma_router(rc, seed=3 + bits)
    x = O.make_tokens(T, rc.hidden, seed=T)
    r = gpu_router(senmoe, rc, rw)
    ids, w = r.forward(t_bf16(x))
    check_router(ids.cpu().numpy(), w.cpu().numpy(), rc, rw, x)


def test_gemma_router_shapes_and_errors(senmoe):
    import torch
    rc = O.GemmaRouterConfig(hidden=256, num_experts=16, top_k=4)
    rw = O.make_gemma_router(rc, seed=1)
    r = gpu_router(senmoe, rc, rw)
    x = O.make_tokens(6, rc.hidden, seed=2).reshape(2, 3, rc.hidden)
    ids, w = r.forward(t_bf16(x))
    assert ids.shape == (2, 3, 4) and w.shape == (2, 3, 4)
    check_router(ids.reshape(-1, 4).cpu().numpy(), w.reshape(-1, 4).cpu().numpy(), rc, rw, x.reshape(-1, rc.hidden))
    empty = r.forward(torch.empty(0, rc.hidden, dtype=torch.bfloat16, device="cuda"))
    assert empty[0].shape == (0, 4)
    bad = senmoe.GemmaRouter(rc.hidden, rc.num_experts, 17, r.weights)  # top_k beyond the supported 16
    with pytest.raises(senmoe.SenMoeError):
        bad.forward(t_bf16(x))


@pytest.mark.parametrize("path", ["gemv", "tc", "mma"])
def test_experts_forward_geglu_vs_oracle(senmoe, path):
    """Experts::forward with GeGLU experts on given routing, on each expert
    path (a shape all three support)."""
    cfg = O.MoeConfig(hidden=512, intermediate=256, num_experts=16, top_k=4, bits=4, activation=1)
    mw = O.make_layer(cfg, seed=31)
    rc = O.GemmaRouterConfig(hidden=512, num_experts=16, top_k=4)
    rw = O.make_gemma_router(rc, seed=32)
    T = {"gemv": 5, "mma": 24, "tc": 200}[path]
    x = O.make_tokens(T, cfg.hidden, seed=33)
    ids, w, _ = O.gemma_router(rc, rw, x)
    mw.router_w = None
    args = moe_args(cfg, {"gemv": 1, "tc": 2, "mma": 3}[path])
    blk = senmoe.DeepseekMoe(args, device_weights(mw), max_tokens=T)
    assert blk.expert_path(T) == {"gemv": 1, "tc": 2, "mma": 3}[path]
    import torch
    y = blk.experts_forward(t_bf16(x), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    blk.check()
    blk.close()
    got = bf16_np_to_f32(to_numpy_bf16(y))
    ref, _ = O.experts_forward(cfg, mw, x, ids, w)
    assert np.abs(got - ref).max() <= MAX_ABS_TOL
    assert rel_l2(got, ref) <= REL_L2_TOL


def test_gemma_moe_branch_26b_shape(senmoe):
    """The routed branch at the 26B-A4B shape (H=2816, E=128, K=8, I=704,
    4-bit experts, 8-bit router): GPU router then GPU experts against the
    oracle's router then experts.  I=704 is not a multiple of 128, so the
    experts run on the CUDA-core GEMV path."""
    import torch
    rc = O.GemmaRouterConfig(hidden=2816, num_experts=128, top_k=8)
    rw = O.make_gemma_router(rc, seed=41)
    cfg = O.MoeConfig(hidden=2816, intermediate=704, num_experts=128, top_k=8, bits=4, activation=1)
    mw = O.make_layer(cfg, seed=42)
    x = O.make_tokens(4, cfg.hidden, seed=43)
    r = gpu_router(senmoe, rc, rw)
    ids, w = r.forward(t_bf16(x))
    ids_r, w_r = check_router(ids.cpu().numpy(), w.cpu().numpy(), rc, rw, x)
    mw.router_w = None
    blk = senmoe.DeepseekMoe(moe_args(cfg), device_weights(mw), max_tokens=4)
    y = blk.experts_forward(t_bf16(x), ids, w)
    blk.check()
    blk.close()
    got = bf16_np_to_f32(to_numpy_bf16(y))
    same = (np.sort(ids.cpu().numpy(), 1) == np.sort(ids_r, 1)).all(1)
    ref, _ = O.experts_forward(cfg, mw, x, ids_r, w_r)
    assert np.abs(got[same] - ref[same]).max() <= MAX_ABS_TOL
    assert rel_l2(got[same], ref[same]) <= REL_L2_TOL


def test_experts_forward_without_router_rejects_forward(senmoe):
    import torch
    cfg = O.MoeConfig(hidden=256, intermediate=128, num_experts=8, top_k=2, bits=4)
    mw = O.make_layer(cfg, seed=5)
    mw.router_w = None
    blk = senmoe.DeepseekMoe(moe_args(cfg), device_weights(mw), max_tokens=4)
    with pytest.raises(senmoe.SenMoeError):
        blk.forward(torch.zeros(2, cfg.hidden, dtype=torch.bfloat16, device="cuda"))
    bad = torch.tensor([[0, 9], [1, 2]], dtype=torch.int32, device="cuda")  # expert 9 >= E
    blk.experts_forward(torch.zeros(2, cfg.hidden, dtype=torch.bfloat16, device="cuda"), bad,
                        torch.ones(2, 2, dtype=torch.float32, device="cuda"))
    with pytest.raises(senmoe.SenMoeError):
        blk.check()
    blk.close()
