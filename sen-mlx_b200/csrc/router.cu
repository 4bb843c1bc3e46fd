// router.cu -- the MoE router: gate GEMV/GEMM, softmax, top-k, renorm.
//
// Restates the router half of DeepseekMoe::forward
// (src/engine/mlx_lm/models/deepseek_v2.rs:526-543):
//   logits = bf16(x . Wg^T)                 nn::Linear on bf16 -> bf16
//   scores = bf16(softmax_fp32(logits))     softmax_axis(.., precise=true)
//   top-k over scores                       argpartition(-scores, k)[:k]
//   w = scores[top-k]; if norm: w = f32(w) / (f32(bf16(sum w)) + 1e-20f)
//   if routed_scaling_factor != 1: w *= routed_scaling_factor
// MLX leaves the order inside the k unspecified; slots here are ordered by
// score descending, then expert id ascending, which also fixes tie-breaking.

#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace senmoe {

namespace {
constexpr int kRouterWarps = 4;        // experts per CTA (one per warp)
constexpr int kRouterTokTile = 16;     // tokens per CTA (x tile in shared memory)
constexpr int kTopkWarps = 4;          // tokens per CTA in the top-k kernel
constexpr int kMaxTopK = 16;
}  // namespace

// Each warp owns one expert row (held in registers as packed bf16; lane l
// holds columns 256 i + 8 l .. +8), each CTA a tile of tokens staged in shared
// memory; one fp32 dot per (token, expert), reduced by warp shuffles.
template <int VPL>  // 16-byte vectors per lane = ceil(H / 256)
__global__ void __launch_bounds__(kRouterWarps * 32) router_logits_kernel(RouterArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ __align__(8) uint64_t bar;
  uint4* xs = reinterpret_cast<uint4*>(smem);  // [tile][H/8]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x * kRouterWarps + warp;
  const int t0 = blockIdx.y * kRouterTokTile;
  const int nt = min(kRouterTokTile, a.num_tokens - t0);
  const int vec_per_row = a.hidden / 8;

  // The router weights do not depend on the previous kernel: load them before
  // waiting for it (programmatic dependent launch).
  float wv[VPL][8];
  const uint4* wrow = reinterpret_cast<const uint4*>(a.weight + static_cast<size_t>(e < a.num_experts ? e : 0) *
                                                                    a.hidden);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint4 v = (32 * i + lane < vec_per_row) ? wrow[32 * i + lane] : make_uint4(0, 0, 0, 0);
    wv[i][0] = bf16_lo(v.x); wv[i][1] = bf16_hi(v.x); wv[i][2] = bf16_lo(v.y); wv[i][3] = bf16_hi(v.y);
    wv[i][4] = bf16_lo(v.z); wv[i][5] = bf16_hi(v.z); wv[i][6] = bf16_lo(v.w); wv[i][7] = bf16_hi(v.w);
  }
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  // the token tile is one contiguous range of x: a single bulk copy
  if (threadIdx.x == 0) {
    const uint32_t bytes = static_cast<uint32_t>(nt) * a.hidden * 2;
    mbar_arrive_expect_tx(&bar, bytes);
    bulk_g2s(xs, a.x + static_cast<size_t>(t0) * a.hidden, bytes, &bar, policy_evict_last());
  }
  if (!mbar_wait(&bar, 0, nullptr)) return;
  if (e >= a.num_experts) return;
  for (int t = 0; t < nt; ++t) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (32 * i + lane >= vec_per_row) break;
      const uint4 v = xs[t * vec_per_row + 32 * i + lane];
      acc = fmaf(bf16_lo(v.x), wv[i][0], acc); acc = fmaf(bf16_hi(v.x), wv[i][1], acc);
      acc = fmaf(bf16_lo(v.y), wv[i][2], acc); acc = fmaf(bf16_hi(v.y), wv[i][3], acc);
      acc = fmaf(bf16_lo(v.z), wv[i][4], acc); acc = fmaf(bf16_hi(v.z), wv[i][5], acc);
      acc = fmaf(bf16_lo(v.w), wv[i][6], acc); acc = fmaf(bf16_hi(v.w), wv[i][7], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0)
      a.logits[static_cast<size_t>(t0 + t) * a.num_experts + e] = a.round_logits ? round_bf16(acc) : acc;
  }
}

// One warp per token: softmax over E (fp32), scores rounded to bf16, K rounds
// of warp arg-max (score desc, id asc), then renorm / scaling in fp32.
// Softmax, top-k and renormalisation of token t's logits, by one warp.
// Logits are read with ld.global.cg (the fused router reads rows that other
// CTAs of its grid wrote).
template <int EPL>  // experts per lane = ceil(E / 32)
__device__ __forceinline__ void topk_token(const RouterArgs& a, int t, int lane) {
  const float* lg = a.logits + static_cast<size_t>(t) * a.num_experts;
  float p[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < a.num_experts ? __ldcg(lg + e) : -INFINITY;
    m = fmaxf(m, p[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < a.num_experts ? expf(p[j] - m) : 0.f;
    sum += p[j];
  }
  sum = warp_sum(sum);
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < a.num_experts ? round_bf16(p[j] / sum) : -1.0f;
  }

  // K rounds of a warp-wide max over packed keys: bf16 score bits (scores are
  // non-negative, so their bit patterns order like the values) above the
  // inverted expert id, so the max picks the highest score and, on ties, the
  // lowest id -- one redux.sync per round.
  uint32_t key[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    key[j] = e < a.num_experts ? (static_cast<uint32_t>(f32_to_bf16_bits(p[j])) << 16) | (0xffffu - e) : 0u;
  }
  float sel_w[kMaxTopK];
  int sel_e[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) {
    if (k >= a.top_k) break;
    uint32_t best = 0;
#pragma unroll
    for (int j = 0; j < EPL; ++j) best = max(best, key[j]);
    best = __reduce_max_sync(0xffffffffu, best);
    const int be = 0xffff - static_cast<int>(best & 0xffffu);
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (key[j] == best) key[j] = 0u;  // unique: the id is part of the key
    sel_w[k] = bf16_bits_to_f32(static_cast<uint16_t>(best >> 16));
    sel_e[k] = be;
  }
  if (lane == 0) {
    if (a.norm_topk_prob) {
      float s = 0.f;
      for (int k = 0; k < a.top_k; ++k) s += sel_w[k];
      const float den = round_bf16(s) + 1e-20f;
      for (int k = 0; k < a.top_k; ++k) sel_w[k] = sel_w[k] / den;
    }
    if (fabsf(a.routed_scaling_factor - 1.0f) > 1.1920929e-7f)
      for (int k = 0; k < a.top_k; ++k) sel_w[k] *= a.routed_scaling_factor;
    for (int k = 0; k < a.top_k; ++k) {
      a.topk_ids[static_cast<size_t>(t) * a.top_k + k] = sel_e[k];
      a.topk_weights[static_cast<size_t>(t) * a.top_k + k] = sel_w[k];
    }
  }
}

template <int EPL>
__global__ void __launch_bounds__(kTopkWarps * 32) router_topk_kernel(RouterArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * kTopkWarps + warp;
  pdl_wait();
  pdl_launch_dependents();
  if (t >= a.num_tokens) return;
  topk_token<EPL>(a, t, lane);
}

__global__ void sigmoid_inplace_kernel(float* v, int n) {
  pdl_wait();
  pdl_launch_dependents();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = 1.0f / (1.0f + expf(-v[i]));
}

bool router_supported(int hidden, int num_experts, int top_k) {
  return hidden > 0 && hidden % 8 == 0 && hidden <= 4096 && num_experts >= 1 && num_experts <= 512 &&
         top_k >= 1 && top_k <= kMaxTopK && top_k <= num_experts;
}

cudaError_t launch_router_logits(const RouterArgs& a, cudaStream_t st) {
  if (a.num_tokens == 0) return cudaSuccess;
  const int v = (a.hidden + 255) / 256;
  const int vpl = v <= 2 ? v : v <= 4 ? 4 : v <= 8 ? 8 : v <= 12 ? 12 : 16;
  const size_t smem = static_cast<size_t>(kRouterTokTile) * a.hidden * 2;
  dim3 grid((a.num_experts + kRouterWarps - 1) / kRouterWarps, (a.num_tokens + kRouterTokTile - 1) / kRouterTokTile);
#define SENMOE_RL_CASE(V)                                                                                  \
  if (vpl == V) {                                                                                          \
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(router_logits_kernel<V>), smem);      \
    if (e != cudaSuccess) return e;                                                                        \
    return launch_pdl(router_logits_kernel<V>, grid, dim3(kRouterWarps * 32), smem, st, a);               \
  }
  SENMOE_RL_CASE(1) SENMOE_RL_CASE(2) SENMOE_RL_CASE(4) SENMOE_RL_CASE(8) SENMOE_RL_CASE(12) SENMOE_RL_CASE(16)
#undef SENMOE_RL_CASE
  return cudaErrorNotSupported;
}

cudaError_t launch_router_topk(const RouterArgs& a, cudaStream_t st) {
  if (a.num_tokens == 0) return cudaSuccess;
  const int epl = (a.num_experts + 31) / 32;
  dim3 grid((a.num_tokens + kTopkWarps - 1) / kTopkWarps);
#define SENMOE_TK_CASE(V) \
  if (epl <= V) return launch_pdl(router_topk_kernel<V>, grid, dim3(kTopkWarps * 32), 0, st, a);
  SENMOE_TK_CASE(1) SENMOE_TK_CASE(2) SENMOE_TK_CASE(4) SENMOE_TK_CASE(8) SENMOE_TK_CASE(16)
#undef SENMOE_TK_CASE
  return cudaErrorNotSupported;
}

cudaError_t launch_sigmoid_inplace(float* v, int n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return launch_pdl(sigmoid_inplace_kernel, dim3((n + 255) / 256), dim3(256), 0, st, v, n);
}

}  // namespace senmoe
