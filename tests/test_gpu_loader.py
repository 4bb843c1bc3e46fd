"""Checkpoint loader end to end on the GPU: synthetic MLX checkpoints (the
reference's tensor names) loaded by senmoe.loader run the block / the Gemma
router and experts with the same results as the oracle on the same arrays."""
import numpy as np
import pytest

from helpers import MAX_ABS_TOL, REL_L2_TOL, bf16_np_to_f32, rel_l2, t_bf16, to_numpy_bf16
from oracle import oracle as O
from test_loader import deepseek_checkpoint, gemma_checkpoint, small_cfg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def senmoe():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import senmoe as s
    s.lib()
    return s


def test_deepseek_checkpoint_forward(senmoe, tmp_path):
    from senmoe import loader
    cfg = small_cfg()
    mw1, mw2 = O.make_layer(cfg, seed=11), O.make_layer(cfg, seed=12)
    deepseek_checkpoint(str(tmp_path), cfg, mw1, mw2)
    x = O.make_tokens(9, cfg.hidden, seed=13)
    for g, mw in zip(loader.load_deepseek_moe(str(tmp_path)), (mw1, mw2)):
        blk = senmoe.DeepseekMoe(g.args, g.weights, max_tokens=9)
        y = bf16_np_to_f32(to_numpy_bf16(blk.forward(t_bf16(x))))
        blk.check()
        blk.close()
        ref = O.moe_forward(cfg, mw, x)["y_f32"]
        assert np.abs(y - ref).max() <= MAX_ABS_TOL and rel_l2(y, ref) <= REL_L2_TOL


def test_gemma_checkpoint_router_and_experts(senmoe, tmp_path):
    from senmoe import loader
    cfg = O.MoeConfig(hidden=128, intermediate=64, num_experts=8, top_k=2, bits=4, activation=1)
    mw = O.make_layer(cfg, seed=15)
    rc = O.GemmaRouterConfig(hidden=128, num_experts=8, top_k=2, bits=8)
    rw = O.make_gemma_router(rc, seed=16)
    gemma_checkpoint(str(tmp_path), cfg, mw, rw, 8)
    (g,) = loader.load_gemma4_moe(str(tmp_path))
    x = O.make_tokens(6, cfg.hidden, seed=17)
    r = senmoe.GemmaRouter(g.args.hidden_size, g.args.n_routed_experts, g.args.num_experts_per_tok, g.router,
                           rms_norm_eps=g.rms_norm_eps, bits=g.router_bits)
    ids, w = r.forward(t_bf16(x))
    ids_r, w_r, _ = O.gemma_router(rc, rw, x)
    np.testing.assert_array_equal(np.sort(ids.cpu().numpy(), 1), np.sort(ids_r, 1))
    blk = senmoe.DeepseekMoe(g.args, g.weights, max_tokens=6)
    y = bf16_np_to_f32(to_numpy_bf16(blk.experts_forward(t_bf16(x), ids, w)))
    blk.check()
    blk.close()
    ref, _ = O.experts_forward(cfg, mw, x, ids_r, w_r)
    assert np.abs(y - ref).max() <= MAX_ABS_TOL and rel_l2(y, ref) <= REL_L2_TOL
