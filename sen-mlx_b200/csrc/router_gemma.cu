// router_gemma.cu -- the Gemma-4 MoE router (Router::forward,
// src/engine/mlx_lm/models/gemma4.rs:716-736):
//   w      = f32(scale) * H^-1/2            (bf16 param x array!(f32) -> f32)
//   normed = rms_norm(x, w, eps)            x bf16, w f32 -> f32:
//            x * 1 / sqrt(mean(x^2) + eps), then * w
//   scores = proj(normed)                   affine-quantized [E, H] linear
//                                           (8-bit in the checkpoint), f32
//   ids    = top-k of scores                (score desc, id asc; the order is
//                                           unspecified in MLX's argpartition)
//   w_k    = softmax_fp32(scores[ids]) * f32(per_expert_scale[ids])
//
// One CTA per token: the block reduces sum(x^2), stages the normed row in
// shared memory, each warp dots expert rows of the quantized projection
// (codes dequantised as q * scale + bias in fp32), and warp 0 picks the top k,
// normalises over them and applies the per-expert scale.  At decode sizes the
// launch is bound by reading the projection (E x H bytes at 8 bits) per
// token; it is a few microseconds next to the expert products.

#include "common.cuh"
#include "kernels.h"

namespace senmoe {
namespace {

constexpr int kGrThreads = 256;
constexpr int kGrWarps = kGrThreads / 32;
constexpr int kGrMaxK = 16;

template <int BITS>
__global__ void __launch_bounds__(kGrThreads) gemma_router_kernel(GemmaRouterArgs a) {
  extern __shared__ float sm[];
  float* s_x = sm;                   // normed row [H]
  float* s_sc = sm + a.hidden;       // scores [E]
  __shared__ float s_part[kGrWarps];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int H = a.hidden, E = a.num_experts, K = a.top_k;
  const uint16_t* xr = a.x + static_cast<size_t>(t) * H;

  // ---- rms norm (fp32), weight f32(scale) * H^-1/2
  float ss = 0.f;
  for (int h = tid; h < H; h += kGrThreads) {
    const float v = bf16_bits_to_f32(xr[h]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) s_part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kGrWarps; ++w) tot += s_part[w];
  const float inv = 1.0f / sqrtf(tot / static_cast<float>(H) + a.eps);
  const float root = a.root;
  for (int h = tid; h < H; h += kGrThreads)
    s_x[h] = (bf16_bits_to_f32(xr[h]) * inv) * (bf16_bits_to_f32(a.scale[h]) * root);
  __syncthreads();

  // ---- scores: warp w takes experts w, w + 8, ...; lane-strided packed words
  constexpr int kPer = 32 / BITS;                  // codes per word
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  const int words = H / kPer, groups = H / a.group_size;
  const int words_per_group = a.group_size / kPer;
  for (int e = warp; e < E; e += kGrWarps) {
    const uint32_t* row = a.proj_w + static_cast<size_t>(e) * words;
    const uint16_t* srow = a.proj_s + static_cast<size_t>(e) * groups;
    const uint16_t* brow = a.proj_b + static_cast<size_t>(e) * groups;
    float acc = 0.f;
    for (int j = lane; j < words; j += 32) {
      const uint32_t w = __ldg(row + j);
      const int gi = j / words_per_group;
      const float s = bf16_bits_to_f32(__ldg(srow + gi)), b = bf16_bits_to_f32(__ldg(brow + gi));
      const float* xc = s_x + j * kPer;
#pragma unroll
      for (int i = 0; i < kPer; ++i) acc = fmaf(fmaf(static_cast<float>((w >> (BITS * i)) & kMask), s, b), xc[i], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) s_sc[e] = acc;
  }
  __syncthreads();

  // ---- top-k (score desc, id asc), softmax over the k, per-expert scale
  if (warp != 0) return;
  int ids[kGrMaxK];
  float val[kGrMaxK];
  for (int j = 0; j < K; ++j) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = s_sc[e];
      if (v > best || (v == best && e < bid)) {  // -inf marks a taken expert
        best = v;
        bid = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
      if (ov > best || (ov == best && oi < bid)) {
        best = ov;
        bid = oi;
      }
    }
    if (bid >= E) bid = j;  // every remaining score was -inf (or NaN): keep the ids valid
    ids[j] = bid;
    val[j] = best;
    __syncwarp();
    if (lane == 0) s_sc[bid] = -INFINITY;
    __syncwarp();
  }
  if (lane == 0) {
    float sum = 0.f;
    float ex[kGrMaxK];
    for (int j = 0; j < K; ++j) {
      ex[j] = expf(val[j] - val[0]);
      sum += ex[j];
    }
    for (int j = 0; j < K; ++j) {
      a.topk_ids[static_cast<size_t>(t) * K + j] = ids[j];
      a.topk_weights[static_cast<size_t>(t) * K + j] =
          (ex[j] / sum) * bf16_bits_to_f32(a.per_expert_scale[ids[j]]);
    }
  }
}

}  // namespace

bool gemma_router_supported(int hidden, int num_experts, int top_k, int bits, int group_size) {
  return (bits == 4 || bits == 8) && group_size > 0 && group_size % (32 / bits) == 0 && hidden > 0 &&
         hidden % group_size == 0 && num_experts > 0 && top_k > 0 && top_k <= kGrMaxK && top_k <= num_experts &&
         size_t(hidden + num_experts) * 4 <= 200 * 1024;
}

cudaError_t launch_gemma_router(const GemmaRouterArgs& a, cudaStream_t st) {
  const size_t smem = size_t(a.hidden + a.num_experts) * 4;
  if (a.bits == 8) {
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemma_router_kernel<8>), smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(gemma_router_kernel<8>, dim3(a.num_tokens), dim3(kGrThreads), smem, st, a);
  }
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(gemma_router_kernel<4>), smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(gemma_router_kernel<4>, dim3(a.num_tokens), dim3(kGrThreads), smem, st, a);
}

}  // namespace senmoe
