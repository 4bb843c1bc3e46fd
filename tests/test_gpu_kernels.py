"""GPU parity of the stage entry points (gather_qmm, router, dispatch) with
the oracle, through the C ABI.  Integer / index outputs are compared bit for
bit; bf16 outputs within one bf16 ulp-scale tolerance."""
import os

import numpy as np
import pytest

from helpers import bf16_np_to_f32, t_bf16, t_u32, to_numpy_bf16, topk_match_except_ties
from oracle import oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def senmoe(torch_cuda):
    import senmoe as s
    s.lib()  # raises if the library is missing: no fallback
    return s


def test_gather_qmm_reference_known_answer(senmoe, torch_cuda):
    """src/engine/mlx_lm/utils/moe.rs:89-146 through the C ABI: output shape
    [M, K, 1, out] and each pair within 1e-2 of dequantize + matmul."""
    d = np.load(os.path.join(GOLD, "gather_qmm_kat.npz"))
    x = t_bf16(d["x"]).reshape(3, 1, 1, 64)
    y = senmoe.gather_qmm(x, t_u32(d["wq"]), t_bf16(d["scales"]), t_bf16(d["biases"]),
                          torch_cuda.from_numpy(d["inds"]).cuda(), True, 64, 4, False)
    torch_cuda.cuda.synchronize()
    assert tuple(y.shape) == (3, 2, 1, 32)
    got = bf16_np_to_f32(to_numpy_bf16(y)).reshape(3, 2, 32)
    assert np.abs(got - d["expected_f64"]).max() < 1e-2
    # and matches the oracle's bf16 result to within one bf16 ulp
    ref = bf16_np_to_f32(d["y_bf16"])
    assert np.all(np.abs(got - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-6)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("in_f,out_f", [(2048, 768), (768, 2048), (512, 96), (128, 32)])
def test_gather_qmm_random_vs_oracle(senmoe, torch_cuda, bits, in_f, out_f):
    E, M, K = 6, 5, 3
    rng = np.random.default_rng(in_f + out_f + bits)
    wq, s, b = O.quantize(O.normal(in_f * 7 + bits, (E, out_f, in_f), 0.02), 64, bits)
    x = O.make_tokens(M, in_f, seed=bits)
    idx = rng.integers(0, E, size=(M, K)).astype(np.int32)
    ref = bf16_np_to_f32(O.gather_qmm(x, wq, s, b, idx, 64, bits)).reshape(M, K, out_f)
    y = senmoe.gather_qmm(t_bf16(x).reshape(M, 1, 1, in_f), t_u32(wq), t_bf16(s), t_bf16(b),
                          torch_cuda.from_numpy(idx).cuda(), True, 64, bits)
    got = bf16_np_to_f32(to_numpy_bf16(y)).reshape(M, K, out_f)
    # fp32 accumulation in a different order: at most one bf16 rounding step apart
    assert np.all(np.abs(got - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-5)
    # per-pair form (x has one row per index, SwitchGlu's down call)
    xp = O.make_tokens(M * K, in_f, seed=bits + 1)
    refp = bf16_np_to_f32(O.gather_qmm(xp, wq, s, b, idx, 64, bits)).reshape(M, K, out_f)
    yp = senmoe.gather_qmm(t_bf16(xp).reshape(M, K, 1, in_f), t_u32(wq), t_bf16(s), t_bf16(b),
                           torch_cuda.from_numpy(idx).cuda(), True, 64, bits)
    gotp = bf16_np_to_f32(to_numpy_bf16(yp)).reshape(M, K, out_f)
    assert np.all(np.abs(gotp - refp) <= 2.0 ** -7 * np.abs(refp) + 1e-5)


@pytest.mark.parametrize("T,E,K", [(1, 128, 8), (16, 128, 8), (64, 128, 8), (300, 512, 10), (7, 8, 8)])
def test_router_vs_oracle(senmoe, torch_cuda, T, E, K):
    cfg = O.MoeConfig(hidden=2048, intermediate=64, num_experts=E, top_k=K)
    rw = O.f32_to_bf16(O.normal(100 + E, (E, 2048), 0.02))
    w = O.MoeWeights(rw, *([None] * 9))
    x = O.make_tokens(T, 2048, seed=T)
    ids_r, w_r, sc_r = O.router(cfg, w, x)
    ids, wts = senmoe.router(t_bf16(x), t_bf16(rw), K, True, 1.0)
    ids, wts = ids.cpu().numpy(), wts.cpu().numpy()
    ok, ties = topk_match_except_ties(ids, ids_r, sc_r)
    assert ok
    same = (ids == ids_r).all(axis=1)
    assert same.mean() >= 0.9
    np.testing.assert_allclose(wts[same], w_r[same], rtol=2e-6, atol=0)


def test_router_scaling_and_no_renorm(senmoe, torch_cuda):
    cfg = O.MoeConfig(hidden=256, intermediate=64, num_experts=64, top_k=6, norm_topk_prob=False,
                      routed_scaling_factor=2.5)
    rw = O.f32_to_bf16(O.normal(9, (64, 256), 0.06))
    w = O.MoeWeights(rw, *([None] * 9))
    x = O.make_tokens(33, 256, seed=4)
    ids_r, w_r, sc_r = O.router(cfg, w, x)
    ids, wts = senmoe.router(t_bf16(x), t_bf16(rw), 6, False, 2.5)
    ids, wts = ids.cpu().numpy(), wts.cpu().numpy()
    same = (ids == ids_r).all(axis=1)
    assert same.mean() >= 0.9
    np.testing.assert_allclose(wts[same], w_r[same], rtol=2e-6, atol=0)


def test_router_exact_ties_pick_lowest_ids(senmoe, torch_cuda):
    import torch
    x = torch.randn(5, 256, device="cuda").to(torch.bfloat16)
    rw = torch.zeros(32, 256, dtype=torch.bfloat16, device="cuda")
    ids, wts = senmoe.router(x, rw, 4, True, 1.0)
    np.testing.assert_array_equal(ids.cpu().numpy(), np.tile(np.arange(4), (5, 1)))
    np.testing.assert_allclose(wts.cpu().numpy(), 0.25, rtol=1e-6)


@pytest.mark.parametrize("T,K,E,skew", [(1, 8, 128, False), (64, 8, 128, False), (256, 8, 128, True),
                                        (4096, 8, 128, False), (2048, 10, 512, True), (3, 4, 4, False)])
def test_dispatch_bit_exact(senmoe, torch_cuda, T, K, E, skew):
    rng = np.random.default_rng(T * K + E)
    p = None
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** 1.2
        p = p / p.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    perm_r, offs_r, inv_r = O.dispatch(ids, E)
    perm, inv, offs, active = senmoe.dispatch(torch_cuda.from_numpy(ids).cuda(), E)
    np.testing.assert_array_equal(perm.cpu().numpy(), perm_r)
    np.testing.assert_array_equal(inv.cpu().numpy(), inv_r)
    np.testing.assert_array_equal(offs.cpu().numpy(), offs_r)
    np.testing.assert_array_equal(active.cpu().numpy(), np.nonzero(np.diff(offs_r))[0])


def test_dispatch_all_pairs_one_expert(senmoe, torch_cuda):
    ids = np.full((1500, 1), 3, dtype=np.int32)
    perm, inv, offs, active = senmoe.dispatch(torch_cuda.from_numpy(ids).cuda(), 8)
    np.testing.assert_array_equal(perm.cpu().numpy(), np.arange(1500))
    np.testing.assert_array_equal(offs.cpu().numpy(), [0, 0, 0, 0, 1500, 1500, 1500, 1500, 1500])
    np.testing.assert_array_equal(active.cpu().numpy(), [3])


def test_dispatch_reports_bad_id_without_fault(senmoe, torch_cuda):
    ids = np.array([[0, 1], [9, 2]], dtype=np.int32)  # 9 is outside [0, 4)
    with pytest.raises(senmoe.SenMoeError):
        senmoe.dispatch(torch_cuda.from_numpy(ids).cuda(), 4)
    # the context is still usable
    perm, _, _, _ = senmoe.dispatch(torch_cuda.from_numpy(np.array([[1, 0]], dtype=np.int32)).cuda(), 4)
    np.testing.assert_array_equal(perm.cpu().numpy(), [1, 0])


def test_gather_qmm_skips_bad_index_without_fault(senmoe, torch_cuda):
    import torch
    wq, s, b = O.quantize(O.normal(1, (2, 32, 64), 0.02), 64, 4)
    x = torch.zeros(1, 1, 1, 64, dtype=torch.bfloat16, device="cuda")
    idx = torch.tensor([[0, 5]], dtype=torch.int32, device="cuda")
    y = senmoe.gather_qmm(x, t_u32(wq), t_bf16(s), t_bf16(b), idx)  # expert 5 of 2: skipped, no fault
    torch.cuda.synchronize()
    assert y.shape == (1, 2, 1, 32)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("T,in_f,out_f", [(1, 2048, 3072), (16, 2048, 512), (5, 768, 2048)])
def test_quantized_linear_vs_oracle(senmoe, torch_cuda, bits, T, in_f, out_f):
    """nn::QuantizedLinear without bias (the projections beside the block,
    deepseek_v2.rs:213, :382): the oracle's gather_qmm with one expert."""
    wq, s, b = O.quantize(O.normal(in_f + out_f + bits, (1, out_f, in_f), 0.02), 64, bits)
    x = O.make_tokens(T, in_f, seed=T + bits)
    ref = bf16_np_to_f32(O.gather_qmm(x, wq, s, b, np.zeros((T, 1), np.int32), 64, bits)).reshape(T, out_f)
    y = senmoe.quantized_linear(t_bf16(x), t_u32(wq[0]), t_bf16(s[0]), t_bf16(b[0]), 64, bits)
    assert y.shape == (T, out_f)
    got = bf16_np_to_f32(to_numpy_bf16(y))
    assert np.all(np.abs(got - ref) <= 2.0 ** -7 * np.abs(ref) + 1e-5)


def test_epilogue_sigmoid_fast_form_is_bit_identical(senmoe, torch_cuda):
    """The expert epilogues' sigmoid (intrinsics away from bf16 rounding
    midpoints, the exact form near them) rounds to the same bf16 value as
    bf16(1 / (1 + expf(-g))) for every bf16 gate value g."""
    import ctypes as C
    torch_cuda.cuda.set_device(0)
    mism, exact = C.c_int64(-1), C.c_int64(-1)
    senmoe._check(senmoe.lib().senmoe_selftest_sigmoid(C.byref(mism), C.byref(exact)))
    assert mism.value == 0
    # the exact form: |g| >= 16 (about half of all bf16 patterns) and the
    # inputs whose fast value sits near a midpoint
    assert 0 < exact.value < 65536
