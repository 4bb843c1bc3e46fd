"""CPU tests of the oracle (the parity checker) against the golden fixtures.

The C oracle (oracle/moe_oracle.c) and the numpy restatement
(oracle/numpy_ref.py) are written separately; the fixtures come from the
numpy one.  The reference's own known-answer test is
src/engine/mlx_lm/utils/moe.rs:89-146.
"""
import os

import numpy as np
import pytest

from oracle import numpy_ref as N
from oracle import oracle as O
from helpers import bf16_np_to_f32, fixture_layer

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_kat_inputs_follow_reference_formulas():
    d = np.load(os.path.join(GOLD, "gather_qmm_kat.npz"))
    i = np.arange(4 * 32 * 64)
    np.testing.assert_array_equal(d["w_float"].ravel(), ((i % 7).astype(np.float32) - 3.0) * np.float32(0.05))
    xf = ((np.arange(3 * 64) % 5).astype(np.float32) - 2.0) * np.float32(0.1)
    np.testing.assert_array_equal(d["x"].ravel(), N.bf16_bits(xf))
    np.testing.assert_array_equal(d["inds"].ravel(), [0, 1, 2, 3, 1, 0])


def test_kat_quantizer_c_matches_fixture():
    d = np.load(os.path.join(GOLD, "gather_qmm_kat.npz"))
    wq, s, b = O.quantize(d["w_float"], 64, 4)
    np.testing.assert_array_equal(wq, d["wq"])
    np.testing.assert_array_equal(s, d["scales"])
    np.testing.assert_array_equal(b, d["biases"])


def test_kat_gather_qmm_matches_reference_check():
    """moe.rs:118-144: every (m, k) pair within 1e-2 of dequantize+matmul."""
    d = np.load(os.path.join(GOLD, "gather_qmm_kat.npz"))
    y = O.gather_qmm(d["x"], d["wq"], d["scales"], d["biases"], d["inds"], 64, 4).reshape(3, 2, 32)
    np.testing.assert_array_equal(y, d["y_bf16"])  # C oracle == numpy restatement, bit for bit
    assert np.abs(bf16_np_to_f32(y) - d["expected_f64"]).max() < 1e-2
    # dequantisation itself reproduces the fixture's float64 products
    wd = O.dequantize(d["wq"], d["scales"], d["biases"], 64, 4)
    ref = np.stack([[wd[d["inds"][m, k]].astype(np.float64) @ bf16_np_to_f32(d["x"][m]) for k in range(2)]
                    for m in range(3)])
    np.testing.assert_allclose(ref, d["expected_f64"], rtol=0, atol=1e-12)


@pytest.mark.parametrize("bits", [4, 8])
def test_small_block_c_oracle_matches_fixture(bits):
    d = np.load(os.path.join(GOLD, f"moe_block_small_{bits}bit.npz"))
    cfg, w = fixture_layer(d)
    r = O.moe_forward(cfg, w, d["x"], mode=0)
    np.testing.assert_array_equal(r["ids"], d["ids"])
    np.testing.assert_allclose(r["weights"], d["weights"], rtol=1e-6, atol=0)
    # identical rounding model; only fp summation order may differ
    np.testing.assert_allclose(r["y_f32"], d["y_f32"], rtol=0, atol=1e-4)


def test_dispatch_is_stable_counting_sort():
    rng = np.random.default_rng(7)
    T, K, E = 37, 4, 16
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    perm, offs, inv = O.dispatch(ids, E)
    flat = ids.ravel()
    np.testing.assert_array_equal(perm, np.argsort(flat, kind="stable"))
    np.testing.assert_array_equal(offs, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]))
    np.testing.assert_array_equal(inv[perm], np.arange(T * K))


def test_dispatch_rejects_bad_index():
    with pytest.raises(RuntimeError):
        O.dispatch(np.array([[0, 5]], dtype=np.int32), 4)


def test_router_tie_break_lowest_id():
    # all-zero router weights -> all logits 0 -> uniform scores: top-k must be 0..K-1
    cfg = O.MoeConfig(hidden=256, intermediate=64, num_experts=16, top_k=4)
    w = O.make_layer(cfg, seed=3)
    w.router_w = np.zeros_like(w.router_w)
    ids, wts, scores = O.router(cfg, w, O.make_tokens(3, 256))
    np.testing.assert_array_equal(ids, np.tile(np.arange(4), (3, 1)))
    np.testing.assert_allclose(wts, 0.25, rtol=1e-6)


def test_mlx_mode_close_to_fp32_mode():
    cfg = O.MoeConfig(hidden=256, intermediate=128, num_experts=16, top_k=4)
    w = O.make_layer(cfg, seed=11)
    x = O.make_tokens(9, 256, seed=2)
    a, b = O.moe_forward(cfg, w, x, mode=0), O.moe_forward(cfg, w, x, mode=1)
    same = (a["ids"] == b["ids"]).all(axis=1)
    assert same.mean() > 0.5
    d = a["y_f32"][same] - b["y_f32"][same]
    assert np.linalg.norm(d) / np.linalg.norm(b["y_f32"][same]) < 2e-2


def test_zero_tokens():
    cfg = O.MoeConfig(hidden=256, intermediate=64, num_experts=8, top_k=2)
    w = O.make_layer(cfg, seed=1)
    r = O.moe_forward(cfg, w, np.zeros((0, 256), dtype=np.uint16))
    assert r["y_f32"].shape == (0, 256)


def test_seeded_generator_is_reproducible():
    a = O.normal(5, (1000,), 1.0)
    O.set_threads(1)
    b = O.normal(5, (1000,), 1.0)
    O.set_threads(os.cpu_count() or 1)
    np.testing.assert_array_equal(a, b)
    assert abs(a.mean()) < 0.1 and abs(a.std() - 1.0) < 0.1


def test_gemma_router_c_matches_numpy():
    """Router::forward (gemma4.rs:716-736): the C oracle and the numpy
    restatement pick the same experts and agree on the weights."""
    rc = O.GemmaRouterConfig(hidden=256, num_experts=32, top_k=6)
    rw = O.make_gemma_router(rc, seed=4)
    x = O.make_tokens(16, rc.hidden, seed=8)
    ids, w, sc = O.gemma_router(rc, rw, x)
    ids_n, w_n, sc_n = N.gemma_route(rc, rw, x)
    np.testing.assert_allclose(sc, sc_n, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(ids, ids_n)
    np.testing.assert_allclose(w, w_n, rtol=1e-5, atol=1e-6)
    # softmax over the k picks only, then the per-expert scale
    pes = O.bf16_to_f32(rw.per_expert_scale)
    np.testing.assert_allclose((w / pes[ids]).sum(-1), 1.0, rtol=1e-5)


def test_experts_forward_geglu_c_matches_numpy():
    """Experts::forward (gemma4.rs:842-848) with GeGLU on given routing: the C
    oracle and the numpy restatement agree."""
    cfg = O.MoeConfig(hidden=128, intermediate=64, num_experts=8, top_k=3, bits=4, activation=1)
    mw = O.make_layer(cfg, seed=21)
    rc = O.GemmaRouterConfig(hidden=128, num_experts=8, top_k=3)
    rw = O.make_gemma_router(rc, seed=22)
    x = O.make_tokens(6, cfg.hidden, seed=23)
    ids, w, _ = O.gemma_router(rc, rw, x)
    y, _ = O.experts_forward(cfg, mw, x, ids, w)
    ref = N.moe_forward(cfg, mw, x, ids=ids, wts=w)
    np.testing.assert_allclose(y, ref["y_f32"], rtol=2e-3, atol=2e-5)
