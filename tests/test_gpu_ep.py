"""Expert parallelism on 2 or more B200s of one box: one spawned process per
GPU, experts split in contiguous blocks, the combine reading every row from
its owner GPU.  Every rank must return the same output, repeatably, equal bit
for bit to the one-GPU layer's (same kernels, same expert rows, same slot
order and fp32 sums) and within the parity tolerance of the oracle.  Skipped
with fewer than 2 GPUs."""
import os

import pytest
import torch

from ep_workers import spawn_ranks
from helpers import MAX_ABS_TOL

pytestmark = pytest.mark.gpu


# world sizes to run (SENMOE_EP_WORLDS="8" runs only the 8-rank cases)
WORLDS = [int(w) for w in os.environ.get("SENMOE_EP_WORLDS", "2,4,8").split(",")]


def _ngpu() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


CASES = {
    # H, I, E, K, bits, Ts, shared, seed, expert_path
    "config0": (2048, 768, 128, 8, 4, [1, 8, 64, 256], 0, 3, 0),
    # 5000 tokens: the router takes more than one wave of CTAs, so each rank
    # routes its own token block and the routing rows are exchanged
    "shared8": (256, 256, 16, 4, 8, [3, 40, 600, 5000], 256, 5, 0),
    "config0_tc": (2048, 768, 128, 8, 4, [16, 512], 0, 7, 2),
    # 8-bit, skewed router, 2048 pairs at 16 per expert: the warp-MMA path
    # with the loaded experts split off to the tcgen05 GEMM (second stream)
    "skew8": (512, 256, 128, 8, 8, [256], 0, 11, 0, True),
}


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("case", sorted(CASES))
def test_expert_parallel_matches_one_gpu(world, case):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    H, I, E, K, bits, Ts, shared, seed, path, *skew = CASES[case]
    res = spawn_ranks("ep_forward", world, H, I, E, K, bits, Ts, shared, seed, path, bool(skew and skew[0]),
                      timeout=600)
    for rank, out in enumerate(res):
        assert out["stack_repeat"], f"rank {rank}: graph replays of the EP stack differ"
        assert out["stack_digest"] == res[0]["stack_digest"], f"rank {rank}: EP stack output differs across ranks"
        if out["stack_same_kernels"]:
            assert out["stack_max_abs"] == 0.0, f"rank {rank}: EP stack differs from the one-GPU stack"
        else:
            assert out["stack_max_abs"] <= MAX_ABS_TOL, f"rank {rank}: EP stack {out['stack_max_abs']} from one GPU"
        for T in Ts:
            r = out[T]
            assert r["repeat"], f"rank {rank} T={T}: two EP calls differ"
            assert r["digest"] == res[0][T]["digest"], f"rank {rank} T={T}: ranks disagree"
            # bit-identical to one GPU whenever both take the same kernels (the
            # rank may pick the warp-MMA kernel's two-CTA form, holding fewer experts)
            if r["same_kernels"]:
                assert r["exact"], f"rank {rank} T={T}: EP output differs from one GPU (max abs {r['max_abs']})"
            else:
                assert r["max_abs"] <= MAX_ABS_TOL and r["rel_l2"] <= 1e-3, f"rank {rank} T={T}: {r}"
            assert r["max_abs_oracle"] <= MAX_ABS_TOL, f"rank {rank} T={T}: {r['max_abs_oracle']} vs oracle"


TOKEN_CASES = {
    # H, I, E, K, bits, shared, seed, expert_path
    "config0": (2048, 768, 128, 8, 4, 0, 13, 0),
    "shared8_tc": (256, 256, 16, 4, 8, 256, 15, 2),
}


def token_counts(world):
    """Per case every rank's token count: equal small blocks, uneven blocks,
    one rank without tokens, and prefill-size blocks (each case keeps the
    same router kernel on the rank and on one GPU, so results are exact)."""
    return [[16] * world, [8 + 7 * r for r in range(world)], [0] + [24] * (world - 1), [600] * world]


@pytest.mark.parametrize("world", WORLDS)
@pytest.mark.parametrize("case", sorted(TOKEN_CASES))
def test_token_local_expert_parallel_matches_one_gpu(world, case):
    """Token-local expert parallelism (each rank its own tokens; the prefill
    form): every rank's output equals bit for bit what one GPU returns for
    those tokens when it runs all ranks' tokens, on every call, and through a
    graph-captured residual stack."""
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    H, I, E, K, bits, shared, seed, path = TOKEN_CASES[case]
    counts = token_counts(world)
    res = spawn_ranks("ep_tokens_forward", world, H, I, E, K, bits, counts, shared, seed, path, timeout=600)
    for rank, out in enumerate(res):
        assert out["stack_repeat"], f"rank {rank}: graph replays of the token-local stack differ"
        if out["stack_same_kernels"]:
            assert out["stack_exact"], f"rank {rank}: token-local stack differs from the one-GPU stack"
        else:
            assert out["stack_max_abs"] <= MAX_ABS_TOL, f"rank {rank}: stack {out['stack_max_abs']} from one GPU"
        for ci in range(len(counts)):
            r = out[ci]
            assert r["repeat"], f"rank {rank} case {counts[ci]}: two calls differ"
            if r["same_kernels"]:
                assert r["exact"], f"rank {rank} case {counts[ci]}: differs from one GPU (max abs {r['max_abs_full']})"
            else:
                assert r["max_abs_full"] <= MAX_ABS_TOL, f"rank {rank} case {counts[ci]}: {r['max_abs_full']}"
            assert r["max_abs_oracle"] <= MAX_ABS_TOL, f"rank {rank} case {counts[ci]}: {r['max_abs_oracle']}"


def test_missing_rank_times_out_with_status():
    if _ngpu() < 2:
        pytest.skip("needs 2 GPUs")
    res = spawn_ranks("ep_missing_rank", 2, 256, 256, 16, 4, 4, 8, 11, timeout=300)
    assert res[0] == "status 4", res  # SENMOE_ERR_TIMEOUT
    assert res[1] == "ok", res
