"""CPU tests of the expert-parallel host logic, with world_size-2 gloo ranks:
the expert partition, weight sharding, the peer-table exchange, and the
decomposition the GPU path implements (rows computed by their owner, combined
by every rank in slot order), checked bit-exactly against the one-device
restatement."""
import os

import numpy as np
import pytest
import torch

from ep_workers import GOLD, spawn_ranks
from helpers import fixture_layer
from oracle import numpy_ref as N


def test_expert_bounds_tile_the_experts():
    from senmoe import SenMoeError, ep

    for E in (8, 128, 512):
        for G in (1, 2, 4, 8):
            b = ep.expert_bounds(E, G)
            assert b[0] == 0 and b[-1] == E and len(b) == G + 1
            sizes = np.diff(b)
            assert sizes.min() >= 1 and sizes.max() - sizes.min() <= 1
    assert ep.expert_bounds(10, 3) == [0, 3, 6, 10]
    with pytest.raises(SenMoeError):
        ep.expert_bounds(4, 9)
    with pytest.raises(SenMoeError):
        ep.expert_bounds(2, 4)


def test_shard_weights_are_views_of_the_rank_experts():
    import senmoe
    from senmoe import ep

    E, I, H = 8, 4, 64

    def sl():
        return senmoe.SwitchLinear(torch.arange(E * I * 8, dtype=torch.int32).reshape(E, I, 8),
                                   torch.zeros(E, I, 1, dtype=torch.bfloat16), torch.ones(E, I, 1, dtype=torch.bfloat16))

    w = senmoe.MoeWeights(torch.zeros(E, H, dtype=torch.bfloat16), sl(), sl(), sl())
    s = ep.shard_weights(w, 2, 6)
    assert s.router_weight is w.router_weight
    for name in ("gate_proj", "up_proj", "down_proj"):
        full, part = getattr(w, name), getattr(s, name)
        assert part.weight.shape[0] == 4 and part.weight.is_contiguous()
        assert part.weight.data_ptr() == full.weight[2].data_ptr()
        assert torch.equal(part.weight, full.weight[2:6])


def test_peer_table_exchange_gloo():
    res = spawn_ranks("exchange", 2, 3)
    for rank, layers in enumerate(res):
        assert len(layers) == 3
        for i, (r, infos) in enumerate(layers):
            assert r == rank
            assert infos == [f"r0l{i}", f"r1l{i}"]  # rank order, same layer index


def test_peer_table_exchange_rejects_layer_count_mismatch():
    with pytest.raises(AssertionError, match="offered"):
        spawn_ranks("exchange", 2, 2, 1)


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("bits", [4, 8])
def test_expert_parallel_decomposition_is_exact(bits, world):
    """At 3 ranks the fixture's 8 experts split 2/3/3 and its 5 tokens 1/2/2:
    uneven expert blocks and uneven token-owned combine blocks."""
    d = np.load(os.path.join(GOLD, f"moe_block_small_{bits}bit.npz"))
    cfg, w = fixture_layer(d)
    ref = N.moe_forward(cfg, w, d["x"])["y_f32"]
    ys = spawn_ranks("decomposition", world, bits)
    for y in ys:
        np.testing.assert_array_equal(y, ref)  # same rows, same slot order, same fp32 sums
    np.testing.assert_allclose(ys[0], d["y_f32"], rtol=0, atol=1e-4)
