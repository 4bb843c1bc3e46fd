"""GPU parity of the whole block (DeepseekMoe::forward,
src/engine/mlx_lm/models/deepseek_v2.rs:520-553) with the oracle's MLX
rounding mode, through the C ABI.

Tolerances (bf16 block outputs): max abs error <= 2e-2 and relative L2 error
<= 5e-3; top-k ids identical except at router ties; dispatch bit-exact."""
import os

import numpy as np
import pytest

from helpers import (MAX_ABS_TOL, REL_L2_TOL, bf16_np_to_f32, device_weights, fixture_layer, max_dropped, moe_args,
                     rel_l2, routing_mismatches, t_bf16, to_numpy_bf16, topk_match_except_ties)
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def senmoe():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import senmoe as s
    s.lib()
    return s


PATHS = {"gemv": 1, "tc": 2, "mma": 3}


def run_block(senmoe, cfg, mw, x_bits, max_tokens=None, path=0, mma_form=0):
    import torch
    T = x_bits.shape[0]
    args = moe_args(cfg, path)
    args.mma_form = mma_form
    blk = senmoe.DeepseekMoe(args, device_weights(mw), max_tokens=max_tokens or max(T, 1))
    if path:
        assert blk.expert_path(T) == path, "the forced expert path is not the one that runs"
    dbg = dict(topk_ids=torch.empty((T, cfg.top_k), dtype=torch.int32, device="cuda"),
               topk_weights=torch.empty((T, cfg.top_k), dtype=torch.float32, device="cuda"),
               perm=torch.empty(T * cfg.top_k, dtype=torch.int32, device="cuda"),
               offsets=torch.empty(cfg.num_experts + 1, dtype=torch.int32, device="cuda"))
    y = blk.forward(t_bf16(x_bits), debug=dbg)
    blk.check()
    out = dict(y=bf16_np_to_f32(to_numpy_bf16(y)), **{k: v.cpu().numpy() for k, v in dbg.items()})
    blk.close()
    return out


def check_against_oracle(cfg, mw, x, got):
    """Top-k ids equal except router ties (each mismatching token must be a
    tie, and at most 1 % of the tokens may mismatch), dispatch bit-exact
    when nothing mismatches, block outputs of the other tokens within the
    tolerance."""
    ref = O.moe_forward(cfg, mw, x, mode=0)
    _, _, scores = O.router(cfg, mw, x)
    ok, ties = topk_match_except_ties(got["topk_ids"], ref["ids"], scores)
    assert ok, "top-k ids differ beyond router ties"
    bad, all_ties = routing_mismatches(got["topk_ids"], ref["ids"], scores)
    assert all_ties, f"top-k order differs beyond router ties (tokens {bad.tolist()[:8]})"
    assert bad.size <= max_dropped(x.shape[0]), f"{bad.size} of {x.shape[0]} tokens differ in routing"
    same = (got["topk_ids"] == ref["ids"]).all(axis=1)
    if bad.size == 0:
        # dispatch is a pure function of the ids: bit-exact
        np.testing.assert_array_equal(got["perm"], ref["perm"])
        np.testing.assert_array_equal(got["offsets"], ref["offsets"])
    y, yr = got["y"][same], ref["y_f32"][same]
    err = np.abs(y - yr).max() if y.size else 0.0
    r = rel_l2(y, yr) if y.size else 0.0
    assert err <= MAX_ABS_TOL, f"max abs error {err}"
    assert r <= REL_L2_TOL, f"relative L2 error {r}"
    return err, r


@pytest.mark.parametrize("bits", [4, 8])
def test_small_block_vs_golden_fixture(senmoe, bits):
    d = np.load(os.path.join(GOLD, f"moe_block_small_{bits}bit.npz"))
    cfg, mw = fixture_layer(d)
    got = run_block(senmoe, cfg, mw, d["x"])
    np.testing.assert_array_equal(got["topk_ids"], d["ids"])
    assert np.abs(got["y"] - d["y_f32"]).max() <= MAX_ABS_TOL
    assert rel_l2(got["y"], d["y_f32"]) <= REL_L2_TOL


@pytest.fixture(scope="module")
def config0_layer():
    """H=2048, E=128, K=8, I=768, 4-bit g64, seed 0."""
    cfg = O.MoeConfig()
    return cfg, O.make_layer(cfg, seed=0)


@pytest.mark.parametrize("path", ["gemv", "tc", "mma"])
@pytest.mark.parametrize("T", [1, 8, 16, 64])
def test_config0_block_vs_oracle(senmoe, config0_layer, T, path):
    cfg, mw = config0_layer
    x = O.make_tokens(T, cfg.hidden, seed=T)
    got = run_block(senmoe, cfg, mw, x, path=PATHS[path])
    check_against_oracle(cfg, mw, x, got)


@pytest.mark.parametrize("T", [256, 1024, 2048])
def test_config0_prefill_tensor_core_vs_oracle(senmoe, config0_layer, T):
    """Prefill-size batches on the tcgen05 path: 16, 64 and 128 tokens per
    expert, i.e. the 16-, 64- and 128-slot tiles (the last with the staged
    gate/up epilogue and the single-issuer down kernel)."""
    cfg, mw = config0_layer
    x = O.make_tokens(T, cfg.hidden, seed=100 + T)
    got = run_block(senmoe, cfg, mw, x, path=PATHS["tc"])
    check_against_oracle(cfg, mw, x, got)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T", [3, 40, 600, 3000])
def test_tensor_core_tiles_vs_oracle(senmoe, bits, T):
    """Every token-tile width (16..256) and ragged expert groups, both code widths,
    on a small layer so the oracle stays fast (H=256, I=256, E=16, K=4)."""
    cfg = O.MoeConfig(hidden=256, intermediate=256, num_experts=16, top_k=4, bits=bits)
    mw = O.make_layer(cfg, seed=20 + bits)
    x = O.make_tokens(T, cfg.hidden, seed=T + bits)
    got = run_block(senmoe, cfg, mw, x, path=PATHS["tc"])
    check_against_oracle(cfg, mw, x, got)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T", [3, 40, 200])
@pytest.mark.parametrize("form", [0, 1, 2])
def test_warp_mma_tiles_vs_oracle(senmoe, bits, T, form):
    """Warp-MMA decode kernel at each slot-tile width (8, 16, 32 slots: about 1,
    10 and 50 tokens per expert, the last in several slot chunks per expert),
    both code widths, on a small layer (H=256, I=256, E=16, K=4); 4-bit at 8
    and 16 slots takes the group-scaled form (at 8 slots the two-CTA kernel)
    unless form 1 (dequantise) or 2 (one CTA per SM) is forced."""
    cfg = O.MoeConfig(hidden=256, intermediate=256, num_experts=16, top_k=4, bits=bits)
    mw = O.make_layer(cfg, seed=40 + bits)
    x = O.make_tokens(T, cfg.hidden, seed=T + 7 * bits)
    got = run_block(senmoe, cfg, mw, x, path=PATHS["mma"], mma_form=form)
    check_against_oracle(cfg, mw, x, got)


@pytest.mark.parametrize("T", [5, 60])
@pytest.mark.parametrize("form", [0, 2])
def test_warp_mma_group_scaled_wide_scales(senmoe, T, form):
    """Group-scaled 4-bit form with scales beyond the dequantising form's fp16
    fast range (|s| > 0.0624 for ~6 % of the groups) and activations up to
    ~16 (h up to ~7e3): the fp32 post-scale has no such limit."""
    cfg = O.MoeConfig(hidden=512, intermediate=256, num_experts=16, top_k=4, bits=4)
    mw = O.make_layer(cfg, seed=77)
    rng = np.random.default_rng(5)
    for name in ("gate_s", "up_s", "down_s"):
        s = O.bf16_to_f32(getattr(mw, name))
        setattr(mw, name, O.f32_to_bf16((s * rng.uniform(3.0, 10.0, s.shape)).astype(np.float32)))
    x = O.bf16_to_f32(O.make_tokens(T, cfg.hidden, seed=T))
    x = x * rng.choice([1.0, 4.0], size=x.shape).astype(np.float32)
    x_bits = O.f32_to_bf16(x.astype(np.float32))
    got = run_block(senmoe, cfg, mw, x_bits, path=PATHS["mma"], mma_form=form)
    ref = O.moe_forward(cfg, mw, x_bits, mode=0)
    same = (got["topk_ids"] == ref["ids"]).all(axis=1)
    y, yr = got["y"][same], ref["y_f32"][same]
    scale = max(1.0, float(np.abs(yr).max()))
    assert np.abs(y - yr).max() <= MAX_ABS_TOL * scale
    assert rel_l2(y, yr) <= REL_L2_TOL


@pytest.mark.parametrize("T", [32, 64])
def test_warp_mma_down_row_pairs_equal_single_rows(senmoe, config0_layer, T):
    """Group-scaled down at 8-slot tiles in 256-row tiles (two 128-row blocks
    per warp: forms 0 and 2 once the expected tiles give every SM five)
    against 128-row tiles (form 3), config 0's layer at decode batches: every
    output is the same fp32 chain in both tilings, so the block outputs are
    bit-identical; the pairs also against the oracle."""
    cfg, mw = config0_layer
    x = O.make_tokens(T, cfg.hidden, seed=500 + T)
    single = run_block(senmoe, cfg, mw, x, path=PATHS["mma"], mma_form=3)
    pair = run_block(senmoe, cfg, mw, x, path=PATHS["mma"], mma_form=2)
    auto = run_block(senmoe, cfg, mw, x, path=PATHS["mma"], mma_form=0)
    np.testing.assert_array_equal(pair["topk_ids"], single["topk_ids"])
    np.testing.assert_array_equal(pair["y"], single["y"])
    np.testing.assert_array_equal(auto["y"], single["y"])
    check_against_oracle(cfg, mw, x, pair)


@pytest.mark.parametrize("path", ["gemv", "tc", "mma"])
def test_block_8bit_shared_gated_large_e(senmoe, path):
    """Config-3-like: E=512, K=10, I=512, sigmoid-gated shared expert (I_s=512)."""
    cfg = O.MoeConfig(hidden=2048, intermediate=512, num_experts=512, top_k=10, bits=4,
                      shared_intermediate=512, shared_gate=True)
    mw = O.make_layer(cfg, seed=3)
    x = O.make_tokens(24, cfg.hidden, seed=5)
    got = run_block(senmoe, cfg, mw, x, path=PATHS[path])
    check_against_oracle(cfg, mw, x, got)


def test_prefill_router_large_e(senmoe):
    """Prefill-size batch at E=512 (config 3 shape, gated shared expert): the
    tensor-core router runs its four 128-expert chunks, then the tcgen05 path."""
    cfg = O.MoeConfig(hidden=2048, intermediate=512, num_experts=512, top_k=10, bits=4,
                      shared_intermediate=512, shared_gate=True)
    mw = O.make_layer(cfg, seed=13, router_std=1.0 / np.sqrt(2048))
    x = O.make_tokens(512, cfg.hidden, seed=14)
    got = run_block(senmoe, cfg, mw, x)
    check_against_oracle(cfg, mw, x, got)


def test_prefill_router_chunk_split_equals_fused(senmoe):
    """E=512 prefill router: below one 32-token tile per SM (2048 tokens) each
    CTA takes one 128-expert chunk and a top-k launch follows; from one tile
    per SM one CTA runs all chunks and its own top-k.  Routing is per token,
    so the first 2048 tokens get the same ids and weights both ways, bit for
    bit, and the ids match the oracle except at router ties."""
    import torch
    cfg = O.MoeConfig(hidden=2048, intermediate=512, num_experts=512, top_k=10, bits=4)
    mw = O.make_layer(cfg, seed=15, router_std=1.0 / np.sqrt(2048))
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    x = O.make_tokens(32 * sms + 64, cfg.hidden, seed=16)
    big = run_block(senmoe, cfg, mw, x)
    small = run_block(senmoe, cfg, mw, x[:2048])
    np.testing.assert_array_equal(small["topk_ids"], big["topk_ids"][:2048])
    np.testing.assert_array_equal(small["topk_weights"], big["topk_weights"][:2048])
    ids_ref, _, scores = O.router(cfg, mw, x[:64])
    ok, _ = topk_match_except_ties(small["topk_ids"][:64], ids_ref, scores)
    assert ok, "top-k ids differ from the oracle beyond router ties"


@pytest.mark.parametrize("path", ["gemv", "tc", "mma"])
def test_block_8bit_skewed(senmoe, path):
    """Config-4-like: 8-bit weights, Zipf-biased router (many tokens on few experts)."""
    cfg = O.MoeConfig(hidden=2048, intermediate=768, num_experts=128, top_k=8, bits=8)
    mw = O.make_layer(cfg, seed=4)
    bias = (1.0 / np.arange(1, 129) ** 1.2).astype(np.float32)
    # fold a per-expert offset into the router: x gets a constant column, Wg that column's weight
    rw = O.bf16_to_f32(mw.router_w)
    rw[:, 0] += 3.0 * bias / max(bias.max(), 1e-9)
    mw.router_w = O.f32_to_bf16(rw)
    x = O.make_tokens(96, cfg.hidden, seed=8)
    xf = O.bf16_to_f32(x)
    xf[:, 0] = 4.0
    x = O.f32_to_bf16(xf)
    got = run_block(senmoe, cfg, mw, x, path=PATHS[path])
    counts = np.diff(got["offsets"])
    assert counts.max() > 4 * counts[counts > 0].mean()  # skew present
    check_against_oracle(cfg, mw, x, got)


@pytest.mark.parametrize("path", ["gemv", "tc", "mma"])
def test_many_tokens_multi_chunk_dispatch(senmoe, path):
    """T*K > 2048 pairs takes the three-kernel dispatch; small H/I keep the oracle fast."""
    cfg = O.MoeConfig(hidden=256, intermediate=256, num_experts=64, top_k=8, bits=4)
    mw = O.make_layer(cfg, seed=6)
    x = O.make_tokens(2000, cfg.hidden, seed=9)
    got = run_block(senmoe, cfg, mw, x, path=PATHS[path])
    check_against_oracle(cfg, mw, x, got)


def test_scaling_factor_and_geglu_free_path(senmoe):
    cfg = O.MoeConfig(hidden=512, intermediate=256, num_experts=32, top_k=4, bits=4, norm_topk_prob=False,
                      routed_scaling_factor=2.5)
    mw = O.make_layer(cfg, seed=12)
    x = O.make_tokens(40, cfg.hidden, seed=1)
    got = run_block(senmoe, cfg, mw, x)
    check_against_oracle(cfg, mw, x, got)


def test_deterministic_and_stream_ordered(senmoe, config0_layer):
    import torch
    cfg, mw = config0_layer
    blk = senmoe.DeepseekMoe(moe_args(cfg), device_weights(mw), max_tokens=64)
    x = t_bf16(O.make_tokens(64, cfg.hidden, seed=3))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        a = blk.forward(x, stream=s)
        b = blk.forward(x, stream=s)
    s.synchronize()
    assert torch.equal(a, b)
    blk.check()
    blk.close()


def test_zero_tokens_and_max_tokens(senmoe, config0_layer):
    import torch
    cfg, mw = config0_layer
    blk = senmoe.DeepseekMoe(moe_args(cfg), device_weights(mw), max_tokens=4)
    y = blk.forward(torch.empty(0, cfg.hidden, dtype=torch.bfloat16, device="cuda"))
    assert y.shape == (0, cfg.hidden)
    with pytest.raises(senmoe.SenMoeError):
        blk.forward(torch.zeros(5, cfg.hidden, dtype=torch.bfloat16, device="cuda"))
    blk.close()


def test_cuda_graph_capture_of_forward(senmoe, config0_layer):
    import torch
    cfg, mw = config0_layer
    blk = senmoe.DeepseekMoe(moe_args(cfg), device_weights(mw), max_tokens=8)
    x = t_bf16(O.make_tokens(8, cfg.hidden, seed=21))
    y = torch.empty_like(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blk.forward(x, out=y, stream=s)  # warm-up (sets kernel attributes)
    s.synchronize()
    ref = y.clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        blk.forward(x, out=y, stream=s)
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    del g
    blk.close()


def test_expert_slot_capacity_overflow_is_reported(senmoe):
    """An expert-slot capacity below the pairs a call sends to the rank's
    experts: the kernels skip the excess and check() reports a device error
    (the context stays usable); a capped layer without expert parallelism is
    refused on the host."""
    from dataclasses import replace

    import torch
    cfg = O.MoeConfig(hidden=256, intermediate=256, num_experts=16, top_k=4, bits=4)
    mw = O.make_layer(cfg, seed=31)
    args = replace(moe_args(cfg, PATHS["tc"]), expert_slots=32)
    x = t_bf16(O.make_tokens(40, cfg.hidden, seed=2))
    blk = senmoe.DeepseekMoe(args, device_weights(mw), max_tokens=64)
    with pytest.raises(senmoe.SenMoeError) as e:
        blk.forward(x)  # 160 pairs, capacity 32, one GPU
    assert e.value.status == senmoe.ERR_UNSUPPORTED
    blk.forward(x[:8])  # 32 pairs fit: runs
    blk.check()
    blk.connect_peers(0, [blk.peer_info()])  # expert parallelism of one rank
    blk.forward(x)
    with pytest.raises(senmoe.SenMoeError) as e:
        blk.check()
    assert e.value.status == senmoe.ERR_DEVICE and "capacity" in str(e.value)
    y = blk.forward(x[:8])  # the context stays usable
    blk.check()
    assert torch.isfinite(y.float()).all()
    blk.close()


@pytest.mark.parametrize("activation", [0, 1])
def test_single_token_fused_layer_equals_gemv_path(senmoe, config0_layer, activation):
    """One token on one GPU runs the whole block in one persistent launch
    (router, top-k, both expert products and the combine); its output equals
    the CUDA-core GEMV path's bit for bit, plain and with the fused residual,
    eagerly and through a CUDA-graph stack, and the oracle within the block
    tolerance."""
    import torch
    cfg, mw = config0_layer
    cfg = O.MoeConfig(**{**cfg.__dict__, "activation": activation}) if activation else cfg
    fused = senmoe.DeepseekMoe(moe_args(cfg, 0), device_weights(mw), max_tokens=1)
    gemv = senmoe.DeepseekMoe(moe_args(cfg, PATHS["gemv"]), device_weights(mw), max_tokens=1)
    assert fused.expert_path(1) == senmoe.PATH_SINGLE_TOKEN and gemv.expert_path(1) == PATHS["gemv"]
    for seed in range(6):
        x = O.make_tokens(1, cfg.hidden, seed=300 + seed)
        xt = t_bf16(x)
        y1, y2 = fused.forward(xt), gemv.forward(xt)
        r1, r2 = fused.forward_residual(xt), gemv.forward_residual(xt)
        fused.check()
        gemv.check()
        assert torch.equal(y1, y2), f"seed {seed}: fused single-token block differs from the GEMV path"
        assert torch.equal(r1, r2), f"seed {seed}: fused residual differs from the GEMV path"
        if seed == 0:  # the GEMV path it equals, against the oracle (ids, dispatch, tolerance)
            check_against_oracle(cfg, mw, x, run_block(senmoe, cfg, mw, x, path=PATHS["gemv"]))
    # the same through a two-layer graph-captured stack (replays equal the eager chain)
    stack = senmoe.MoeStack([fused, fused], max_tokens=1, use_graph=True)
    x = t_bf16(O.make_tokens(1, cfg.hidden, seed=399))
    h = fused.forward_residual(fused.forward_residual(x))
    for _ in range(3):
        assert torch.equal(stack.forward(x), h), "graph replay of the single-token block differs from eager"
    stack.release()
    fused.close()
    gemv.close()
