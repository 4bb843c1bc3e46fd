// router_core.cuh -- the router arithmetic shared by the router kernels and
// the single-token fused layer kernel (same code, so the same bits): the
// per-lane logit dot product and the per-token softmax / top-k.
#pragma once

#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace senmoe {

constexpr int kMaxTopK = 16;

// Lane `lane`'s share of one router weight row (bf16 [hidden]) as fp32:
// 16-byte vectors 32 i + lane, i < VPL.
template <int VPL>
__device__ __forceinline__ void router_load_wrow(const uint16_t* wrow16, int lane, int vec_per_row, float (&wv)[VPL][8]) {
  const uint4* wrow = reinterpret_cast<const uint4*>(wrow16);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint4 v = (32 * i + lane < vec_per_row) ? wrow[32 * i + lane] : make_uint4(0, 0, 0, 0);
    wv[i][0] = bf16_lo(v.x); wv[i][1] = bf16_hi(v.x); wv[i][2] = bf16_lo(v.y); wv[i][3] = bf16_hi(v.y);
    wv[i][4] = bf16_lo(v.z); wv[i][5] = bf16_hi(v.z); wv[i][6] = bf16_lo(v.w); wv[i][7] = bf16_hi(v.w);
  }
}

// The lane's partial of x . w (fp32 fma chain over its vectors); the logit
// is the warp sum of the partials.
template <int VPL>
__device__ __forceinline__ float router_dot_lane(const float (&wv)[VPL][8], const uint4* xrow, int lane, int vec_per_row) {
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (32 * i + lane >= vec_per_row) break;
    const uint4 v = xrow[32 * i + lane];
    acc = fmaf(bf16_lo(v.x), wv[i][0], acc); acc = fmaf(bf16_hi(v.x), wv[i][1], acc);
    acc = fmaf(bf16_lo(v.y), wv[i][2], acc); acc = fmaf(bf16_hi(v.y), wv[i][3], acc);
    acc = fmaf(bf16_lo(v.z), wv[i][4], acc); acc = fmaf(bf16_hi(v.z), wv[i][5], acc);
    acc = fmaf(bf16_lo(v.w), wv[i][6], acc); acc = fmaf(bf16_hi(v.w), wv[i][7], acc);
  }
  return acc;
}

// One warp per token: softmax over E (fp32), scores rounded to bf16, K rounds
// of warp arg-max (score desc, id asc), then renorm / scaling in fp32.
// lg is token t's logits row, in global memory (kShared false) or shared.
template <int EPL, bool kShared>  // experts per lane = ceil(E / 32)
__device__ __forceinline__ void topk_row(const RouterArgs& a, const float* lg, int t, int lane) {
  float p[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < a.num_experts ? (kShared ? lg[e] : __ldcg(lg + e)) : -INFINITY;
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

}  // namespace senmoe
