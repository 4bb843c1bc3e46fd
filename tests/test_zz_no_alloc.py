"""The allocation-free forward (senmoe_moe_forward_noalloc) against the layer
forward (senmoe_layer_forward), through the C ABI.

That entry point exists for callers that cannot allocate device memory when
they run a MoE forward -- code inside an open CUDA stream capture, serving
loops whose HBM another allocator has fully reserved, plugin hosts that forbid
device allocation on the hot path.  It keeps all scratch in one fixed device
array inside the library, so this test checks that its output matches the
allocating path on two calls in a row (the second call sees the first call's
leftover scratch) and that it refuses token counts beyond that array.

The file name sorts last so a run that stops at the first failure has already
run every other test; the test also passes alone in a fresh process.
"""
import ctypes as C
import math

import pytest

from helpers import MAX_ABS_TOL, REL_L2_TOL

pytestmark = pytest.mark.gpu

H, E, K, I = 2048, 128, 8, 768


def _weights(torch, senmoe, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def proj(rows, cols):
        w = torch.randint(-2**31, 2**31 - 1, (E, rows, cols // 8), generator=g, device=dev, dtype=torch.int32)
        s = (torch.rand((E, rows, cols // 64), generator=g, device=dev) * 0.002 + 0.006)
        b = -(s * 7.5)
        return senmoe.SwitchLinear(w, s.to(torch.bfloat16), b.to(torch.bfloat16))

    rw = (torch.randn((E, H), generator=g, device=dev) / math.sqrt(H)).to(torch.bfloat16)
    return senmoe.MoeWeights(router_weight=rw, gate_proj=proj(I, H), up_proj=proj(I, H), down_proj=proj(H, I))


def test_noalloc_forward_matches_layer_forward_twice():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import senmoe
    L = senmoe.lib()
    dev = torch.device("cuda", 0)
    args = senmoe.MoeArgs(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, num_experts_per_tok=K)
    wts = _weights(torch, senmoe, dev, seed=7)
    blk = senmoe.DeepseekMoe(args, wts, max_tokens=64, device=0)
    stream = torch.cuda.current_stream().cuda_stream
    for call, T in enumerate((64, 17)):
        x = torch.randn((T, H), device=dev, generator=torch.Generator(device=dev).manual_seed(call)).to(torch.bfloat16)
        ref = blk.forward(x)
        y = torch.full_like(x, float("nan"))
        rc = L.senmoe_moe_forward_noalloc(C.byref(blk._cfg), C.byref(blk._wt), x.data_ptr(), T, y.data_ptr(),
                                          stream)
        assert rc == senmoe.OK, L.senmoe_last_error().decode()
        torch.cuda.synchronize()
        a, b = y.float(), ref.float()
        assert torch.isfinite(a).all()
        err = (a - b).abs().max().item()
        rel = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
        assert err <= MAX_ABS_TOL and rel <= REL_L2_TOL, f"call {call}: max abs {err}, rel L2 {rel}"
    blk.close()


def noalloc_limit(h, e, k, i, shared=0, array_bytes=4 << 20):
    """Largest token count whose scratch fits the fixed array: the sum of the
    pieces the header lists, each rounded up to 256 bytes."""
    def need(t):
        p = t * k
        pieces = [t * e * 4, p * 4, p * 4, p * 4, p * 4, (e + 1) * 4, e * 4, 4, 4, -(-p // 1024) * e * 4,
                  p * i * 2, p * h * 2]
        if shared:
            pieces += [t * shared * 2, t * h * 2, t * 4, t * 4]
        return sum(-(-s // 256) * 256 for s in pieces)
    t = 0
    while need(t + 1) <= array_bytes:
        t += 1
    return t


def test_noalloc_limit_is_the_documented_one():
    assert noalloc_limit(H, E, K, I) == 91
    assert noalloc_limit(2048, 512, 10, 512, shared=512) == 71


def test_noalloc_forward_at_and_above_its_limit():
    """The largest token count that fits the array runs and matches the layer
    forward; one token more is refused before any GPU work."""
    import torch
    import senmoe
    L = senmoe.lib()
    dev = torch.device("cuda", 0)
    args = senmoe.MoeArgs(hidden_size=H, moe_intermediate_size=I, n_routed_experts=E, num_experts_per_tok=K)
    wts = _weights(torch, senmoe, dev, seed=8)
    blk = senmoe.DeepseekMoe(args, wts, max_tokens=4096, device=0)
    stream = torch.cuda.current_stream().cuda_stream
    top = noalloc_limit(H, E, K, I)
    # buffers hold 4096 rows, so even a refused size would stay inside them
    x = torch.randn((4096, H), device=dev, generator=torch.Generator(device=dev).manual_seed(3)).to(torch.bfloat16)
    y = torch.full_like(x, float("nan"))
    rc = L.senmoe_moe_forward_noalloc(C.byref(blk._cfg), C.byref(blk._wt), x.data_ptr(), top, y.data_ptr(), stream)
    assert rc == senmoe.OK, L.senmoe_last_error().decode()
    ref = blk.forward(x[:top])
    torch.cuda.synchronize()
    a, b = y[:top].float(), ref.float()
    err = (a - b).abs().max().item()
    rel = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
    assert err <= MAX_ABS_TOL and rel <= REL_L2_TOL, f"{top} tokens: max abs {err}, rel L2 {rel}"
    assert torch.isnan(y[top].float()).all(), "the call wrote past its num_tokens rows"
    for T in (top + 1, 4096):
        rc = L.senmoe_moe_forward_noalloc(C.byref(blk._cfg), C.byref(blk._wt), x.data_ptr(), T, y.data_ptr(), stream)
        assert rc == senmoe.ERR_BAD_ARG
        assert "scratch" in L.senmoe_last_error().decode()
    blk.close()
