// common.cuh -- device helpers shared by the senmoe kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "senmoe kernels are written for sm_100a (B200) only"
#endif

namespace senmoe {

// Bounded waits: give up after this many SM clock cycles (~2 s at <= 2 GHz).
// The spin measures time with clock64 (an SM-local counter, cheap to read);
// %globaltimer is a much slower read and would add its latency to every
// handoff that is not ready on the first try.
constexpr long long kWaitLimitCycles = 4000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }

// ----------------------------------------------------------- mbarrier + TMA
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a phase (acquire on success): lets a consumer ask
// early whether its next stage has landed, hiding the barrier round trip.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes (or about kWaitSleepNs passes) instead of
// returning at once, so waiting warps do not spin through issue slots that
// working warps need.
constexpr uint32_t kWaitSleepNs = 20000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kWaitSleepNs)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete, for at most
// kWaitLimitCycles.  On timeout records kDevWaitTimeout and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared (no multicast), completion on `bar` by bytes.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 8-byte asynchronous global -> shared copy (both addresses 8-byte aligned).
__device__ __forceinline__ void cp_async_8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
// 4-byte asynchronous global -> shared copy (both addresses 4-byte aligned).
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// Arrival on `bar` once all of this thread's earlier cp.async copies have
// landed; counts as one of the barrier's expected arrivals (.noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch: wait for the upstream grid's memory to be
// visible / let the downstream grid start its prologue.  No-ops when the
// launch did not opt in.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ warps
// One lane of the (converged) warp, chosen by elect.sync: true on it only.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Activations with MLX's per-op bf16 rounding (nn::silu = x * sigmoid(x),
// then the product with `up`, deepseek_v2.rs:472-474).
__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }
// bf16(sigmoid_f(g)), bit for bit, at a fraction of the cost.  The intrinsic
// form s' = __fdividef(1, 1 + __expf(-g)) differs from sigmoid_f(g) by at
// most 53 fp32 units in the last place for |g| < 16, from the documented
// bounds: __expf 2 + floor(1.173 |x|) ulp, expf 2 ulp, the two roundings of
// 1 + e, __fdividef 2 ulp, IEEE division 0.5 ulp.  So where s' lies more than
// 64 units from a bf16 rounding midpoint (its low 16 bits outside
// 0x8000 +- 64), both round to the same bf16 value; elsewhere (about 0.2 % of
// the values) and for |g| >= 16 the exact form runs.  senmoe_selftest_sigmoid
// checks every bf16 input on the device.
__device__ __forceinline__ float sigmoid_fast(float g) { return __fdividef(1.0f, 1.0f + __expf(-g)); }
__device__ __forceinline__ bool sigmoid_fast_ok(float g, float sf) {
  return fabsf(g) < 16.0f && (__float_as_uint(sf) & 0xffffu) - 0x7fc0u > 0x80u;
}
__device__ __forceinline__ float sigmoid_bf16(float g) {
  const float sf = sigmoid_fast(g);
  return round_bf16(sigmoid_fast_ok(g, sf) ? sf : sigmoid_f(g));
}
__device__ __forceinline__ float act_swiglu_mlx(float g, float u) {
  const float sg = sigmoid_bf16(g);
  const float a = round_bf16(g * sg);
  return round_bf16(a * u);
}
// act_swiglu_mlx of N (gate, up) pairs: the N fast sigmoids run first as
// straight-line chains that interleave, then the exact form for the few
// that need it, so its rare branch does not split the chains.
template <int N>
__device__ __forceinline__ void act_swiglu_mlx_n(const float (&g)[N], const float (&u)[N], float (&h)[N]) {
  float s[N];
  uint32_t slow = 0;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    s[j] = sigmoid_fast(g[j]);
    slow |= sigmoid_fast_ok(g[j], s[j]) ? 0u : 1u << j;
  }
  if (slow) {
#pragma unroll
    for (int j = 0; j < N; ++j)
      if (slow & (1u << j)) s[j] = sigmoid_f(g[j]);
  }
#pragma unroll
  for (int j = 0; j < N; ++j) h[j] = round_bf16(round_bf16(g[j] * round_bf16(s[j])) * u[j]);
}
// gelu_approximate (tanh form) then the product, each rounded to bf16.
__device__ __forceinline__ float act_geglu_mlx(float g, float u) {
  const float c = 0.7978845608028654f;  // sqrt(2/pi)
  const float a = round_bf16(0.5f * g * (1.0f + tanhf(c * (g + 0.044715f * g * g * g))));
  return round_bf16(a * u);
}


// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}


// Bounded wait that also gives up as soon as another role of the CTA has.
// Warp-wide callers combine the result with __all_sync so that every lane
// takes the same branch (they arrive per warp and issue .sync.aligned ops).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      record_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

}  // namespace senmoe
