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
#include "dispatch_body.cuh"
#include "router_core.cuh"

namespace senmoe {

namespace {
constexpr int kRouterWarps = 4;        // experts per CTA (one per warp)
constexpr int kRouterTokTile = 4;      // tokens per CTA (x tile in shared memory): short serial
                                       // work per warp, E/4 x T/4 CTAs
static_assert(kRouterTokTile <= kRouterWarps, "fused top-k runs one warp per token of a tile");
constexpr int kTopkWarps = 4;          // tokens per CTA in the top-k kernel
}  // namespace

// top-k of token t for any E <= 512 (logits row in global memory).
__device__ __forceinline__ void topk_any(const RouterArgs& a, int t, int lane) {
  const float* lg = a.logits + static_cast<size_t>(t) * a.num_experts;
  const int epl = (a.num_experts + 31) / 32;
  if (epl <= 1) topk_row<1, false>(a, lg, t, lane);
  else if (epl <= 2) topk_row<2, false>(a, lg, t, lane);
  else if (epl <= 4) topk_row<4, false>(a, lg, t, lane);
  else if (epl <= 8) topk_row<8, false>(a, lg, t, lane);
  else topk_row<16, false>(a, lg, t, lane);
}

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
  router_load_wrow<VPL>(a.weight + static_cast<size_t>(e < a.num_experts ? e : 0) * a.hidden, lane, vec_per_row, wv);
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
  const bool ok = mbar_wait(&bar, 0, a.err);
  if (ok && e < a.num_experts) {
    for (int t = 0; t < nt; ++t) {
      float acc = router_dot_lane<VPL>(wv, xs + t * vec_per_row, lane, vec_per_row);
      acc = warp_sum(acc);
      if (lane == 0)
        a.logits[static_cast<size_t>(t0 + t) * a.num_experts + e] = a.round_logits ? round_bf16(acc) : acc;
    }
  }
  if (!a.tile_cnt) return;

  // ---- fused top-k: the last CTA to finish this token tile (one warp per token)
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&a.tile_cnt[blockIdx.y], 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) a.tile_cnt[blockIdx.y] = 0;  // ready for the next call
  __threadfence();
  if (warp < nt) topk_any(a, t0 + warp, lane);
}

template <int EPL>
__global__ void __launch_bounds__(kTopkWarps * 32) router_topk_kernel(RouterArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * kTopkWarps + warp;
  pdl_wait();
  pdl_launch_dependents();
  if (t >= a.num_tokens) return;
  topk_row<EPL, false>(a, a.logits + static_cast<size_t>(t) * a.num_experts, t, lane);
}

// ------------------------------------------- prefill router (tensor cores)
// For prefill-size batches: CTA = 32 tokens x all experts.  x and Wg stream
// through a ring of 64-column stages by TMA (2-D tensor maps, SWIZZLE_128B,
// no multicast), warps take bf16 m16n8k16 MMA fragments from the stages with
// ldmatrix (products exact in fp32, fp32 accumulation), the bf16-rounded
// logits stay in shared memory, and the same CTA runs softmax / top-k for its
// tokens.  Experts come in chunks of 128 (E <= 512).  SPLIT (more than one
// chunk, fewer 32-token tiles than SMs): CTA (tile, chunk) computes one chunk,
// writes its logits to global memory, and router_topk_kernel follows; every
// CTA otherwise streams all of Wg (2 MB at 512 experts) and only
// T / 32 SMs work.  Same logits, same top-k code: same results.
namespace {
constexpr int kRtTok = kRouterTcTokensPerCta, kRtExp = 128, kRtStages = 8;
constexpr int kRtCompute = 8;                     // 2 token halves x 4 expert quarters
constexpr int kRtThreads = (kRtCompute + 1) * 32; // + one TMA warp
constexpr uint32_t kRtXBytes = kRtTok * 128, kRtWBytes = kRtExp * 128;
constexpr uint32_t kRtStageBytes = kRtXBytes + kRtWBytes;  // 20 KB

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
}  // namespace

size_t router_tc_smem_bytes(int num_experts, bool split) {
  return 1024 + size_t(kRtStages) * kRtStageBytes + (split ? 0 : size_t(kRtTok) * num_experts * 4);
}

template <int EPL, bool SPLIT>
__global__ void __launch_bounds__(kRtThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tX, const __grid_constant__ CUtensorMap tW, RouterArgs a) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_logits = reinterpret_cast<float*>(smem + kRtStages * kRtStageBytes);  // [kRtTok][E]
  __shared__ __align__(8) uint64_t bar_full[kRtStages], bar_empty[kRtStages];
  __shared__ int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtTok;
  const int nk = a.hidden / 64;
  const int c_begin = SPLIT ? static_cast<int>(blockIdx.y) : 0;
  const int c_end = SPLIT ? c_begin + 1 : (a.num_experts + kRtExp - 1) / kRtExp;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kRtStages; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], kRtCompute);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  pdl_wait();  // x comes from the previous kernel
  pdl_launch_dependents();

  if (warp == kRtCompute) {
    // ---------------------------------------------------- TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int c = c_begin; c < c_end && ok; ++c)
        for (int k = 0; k < nk; ++k, ++it) {
          const int slot = it % kRtStages, ph = (it / kRtStages) & 1;
          if (!(ok = wait_or_abort(&bar_empty[slot], ph ^ 1, &s_abort, a.err))) break;
          unsigned char* st = smem + slot * kRtStageBytes;
          mbar_arrive_expect_tx(&bar_full[slot], kRtStageBytes);
          tma_load_2d(st, &tX, k * 64, t0, &bar_full[slot]);
          tma_load_2d(st + kRtXBytes, &tW, k * 64, c * kRtExp, &bar_full[slot]);
        }
      int never = 0;  // the last stages must land before the CTA exits
      for (int k = (it > kRtStages ? it - kRtStages : 0); k < it; ++k)
        wait_or_abort(&bar_full[k % kRtStages], (k / kRtStages) & 1, &never, nullptr);
    }
    return;
  }

  // ------------------------------------------------------ compute warps
  const int mi = warp & 1, nq = warp >> 1;  // tokens 16 mi .. +16, experts 32 nq .. +32 of a chunk
  const uint32_t base = smem_u32(smem);
  int it = 0;
  bool ok = true;
  for (int c = c_begin; c < c_end && ok; ++c) {
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
    for (int k = 0; k < nk; ++k, ++it) {
      const int slot = it % kRtStages, ph = (it / kRtStages) & 1;
      ok = __all_sync(0xffffffffu, wait_or_abort(&bar_full[slot], ph, &s_abort, a.err));
      if (!ok) break;
      const uint32_t xs = base + slot * kRtStageBytes, ws = xs + kRtXBytes;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {  // four k16 steps of the 64-column stage
        // A: rows 16 mi + (l & 7) + 8 ((l >> 3) & 1), 16-byte chunk 2 ks + (l >> 4)
        uint32_t af[4];
        {
          const int row = 16 * mi + (lane & 7) + 8 * ((lane >> 3) & 1), ch = 2 * ks + (lane >> 4);
          ldsm_x4(xs + row * 128 + ((ch ^ (row & 7)) << 4), af);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // two ldmatrix.x4 = four n-tiles of 8 experts
          // matrix j = lane >> 3: n-tile 2h + (j >> 1), k half j & 1
          const int j = lane >> 3;
          const int row = 32 * nq + 8 * (2 * h + (j >> 1)) + (lane & 7), ch = 2 * ks + (j & 1);
          uint32_t bfr[4];
          ldsm_x4(ws + row * 128 + ((ch ^ (row & 7)) << 4), bfr);
          mma_bf16(acc[2 * h], af, bfr[0], bfr[1]);
          mma_bf16(acc[2 * h + 1], af, bfr[2], bfr[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_empty[slot]);
    }
    if (!ok) break;
    // bf16-rounded logits of this chunk -> shared [token][expert]
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 16 * mi + g + 8 * (i >> 1), e = c * kRtExp + 32 * nq + 8 * j + 2 * tq + (i & 1);
        const float v = a.round_logits ? round_bf16(acc[j][i]) : acc[j][i];
        if constexpr (SPLIT) {
          if (e < a.num_experts && t0 + tok < a.num_tokens)
            a.logits[static_cast<size_t>(t0 + tok) * a.num_experts + e] = v;
        } else {
          if (e < a.num_experts) s_logits[tok * a.num_experts + e] = v;
        }
      }
  }
  if constexpr (SPLIT) return;  // router_topk_kernel follows
  ok = __all_sync(0xffffffffu, ok);
  // all compute warps' logits are in place (named barrier: the TMA warp has left)
  asm volatile("bar.sync 1, %0;" ::"r"(kRtCompute * 32) : "memory");
  if (!ok) return;
  for (int tl = warp; tl < kRtTok; tl += kRtCompute) {
    const int tok = t0 + tl;
    if (tok < a.num_tokens) topk_row<EPL, true>(a, s_logits + tl * a.num_experts, tok, lane);
  }
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

// Small batches: the top-k of every token and the whole single-chunk dispatch
// in one CTA (one launch instead of two).  Warp w takes tokens w, w + 32, ...;
// after the block barrier the dispatch reads the ids with ld.global.cg, which
// sees this CTA's writes.
template <int EPL>
__global__ void __launch_bounds__(dispatch_detail::kThreads) router_topk_dispatch_kernel(RouterArgs a, DispatchArgs d) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm_disp[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = warp; t < a.num_tokens; t += dispatch_detail::kWarps)
    topk_row<EPL, false>(a, a.logits + static_cast<size_t>(t) * a.num_experts, t, lane);
  __syncthreads();
  dispatch_detail::dispatch_single_body(d, sm_disp);
}

// Up to 8 tokens and 128 pairs: the same in one CTA of 8 warps, the
// dispatch by one warp (no block-wide scans or barriers).
template <int EPL>
__global__ void __launch_bounds__(kTopkDispatchMaxTokens * 32)
    router_topk_dispatch_small_kernel(RouterArgs a, DispatchArgs d) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int sm_small[];  // [E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp < a.num_tokens) topk_row<EPL, false>(a, a.logits + static_cast<size_t>(warp) * a.num_experts, warp, lane);
  __syncthreads();
  if (warp == 0) dispatch_detail::dispatch_warp_body(d, sm_small, lane);
}

bool router_topk_dispatch_supported(int num_tokens, int num_pairs, int num_experts) {
  return num_tokens > 0 && num_tokens <= kTopkDispatchMaxTokens && num_pairs <= dispatch_detail::kThreads * 2 &&
         num_experts <= 512;
}

cudaError_t launch_router_topk_dispatch(const RouterArgs& a, const DispatchArgs& d, cudaStream_t st) {
  if (!router_topk_dispatch_supported(a.num_tokens, d.num_pairs, a.num_experts)) return cudaErrorNotSupported;
  const int epl = (a.num_experts + 31) / 32;
  if (d.num_pairs <= dispatch_detail::kWarpDispatchMaxPairs) {
    const size_t smem_small = static_cast<size_t>(d.num_experts) * 4;
#define SENMOE_TDS_CASE(V)                                                                                  \
  if (epl <= V)                                                                                            \
    return launch_pdl(router_topk_dispatch_small_kernel<V>, dim3(1), dim3(kTopkDispatchMaxTokens * 32), smem_small, \
                      st, a, d);
    SENMOE_TDS_CASE(1) SENMOE_TDS_CASE(2) SENMOE_TDS_CASE(4) SENMOE_TDS_CASE(8) SENMOE_TDS_CASE(16)
#undef SENMOE_TDS_CASE
    return cudaErrorNotSupported;
  }
  const size_t smem = dispatch_smem_bytes(d.num_experts);
#define SENMOE_TD_CASE(V)                                                                                   \
  if (epl <= V) {                                                                                         \
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(router_topk_dispatch_kernel<V>), smem); \
    if (e != cudaSuccess) return e;                                                                       \
    return launch_pdl(router_topk_dispatch_kernel<V>, dim3(1), dim3(dispatch_detail::kThreads), smem, st, a, d); \
  }
  SENMOE_TD_CASE(1) SENMOE_TD_CASE(2) SENMOE_TD_CASE(4) SENMOE_TD_CASE(8) SENMOE_TD_CASE(16)
#undef SENMOE_TD_CASE
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

// Every bf16 input of sigmoid_bf16 (NaNs aside) against the exact form:
// counts[0] mismatches, counts[1] inputs that took the exact form.
__global__ void selftest_sigmoid_kernel(unsigned int* counts) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536u || ((i & 0x7f80u) == 0x7f80u && (i & 0x7fu) != 0)) return;
  const float g = __uint_as_float(i << 16);
  if (__float_as_uint(sigmoid_bf16(g)) != __float_as_uint(round_bf16(sigmoid_f(g)))) atomicAdd(&counts[0], 1u);
  if (!sigmoid_fast_ok(g, sigmoid_fast(g))) atomicAdd(&counts[1], 1u);
}

cudaError_t selftest_sigmoid(int64_t* mismatches, int64_t* exact_form) {
  unsigned int* d = nullptr;
  unsigned int h[2] = {0, 0};
  cudaError_t e = cudaMalloc(&d, sizeof(h));
  if (e != cudaSuccess) return e;
  if ((e = cudaMemset(d, 0, sizeof(h))) == cudaSuccess) {
    selftest_sigmoid_kernel<<<256, 256>>>(d);
    if ((e = cudaGetLastError()) == cudaSuccess) e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  }
  cudaFree(d);
  *mismatches = h[0];
  *exact_form = h[1];
  return e;
}

cudaError_t launch_sigmoid_inplace(float* v, int n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  return launch_pdl(sigmoid_inplace_kernel, dim3((n + 255) / 256), dim3(256), 0, st, v, n);
}

bool router_tc_supported(int hidden, int num_experts, int top_k) {
  return router_supported(hidden, num_experts, top_k) && hidden % 64 == 0 && num_experts <= 512;
}

cudaError_t launch_router_tc(const CUtensorMap& tX, const CUtensorMap& tW, const RouterArgs& a, cudaStream_t st) {
  if (a.num_tokens == 0) return cudaSuccess;
  if (!router_tc_supported(a.hidden, a.num_experts, a.top_k)) return cudaErrorNotSupported;
  const int epl = (a.num_experts + 31) / 32;
  const int tiles = (a.num_tokens + kRtTok - 1) / kRtTok, nchunk = (a.num_experts + kRtExp - 1) / kRtExp;
  int sms = 0, dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (nchunk > 1 && tiles < sms) {
    // one chunk per CTA, logits through global memory, then the top-k launch
    const size_t smem = router_tc_smem_bytes(a.num_experts, true);
    auto kern = router_tc_kernel<1, true>;
    if ((e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) != cudaSuccess) return e;
    if ((e = launch_pdl(kern, dim3(tiles, nchunk), dim3(kRtThreads), smem, st, tX, tW, a)) != cudaSuccess) return e;
    return launch_router_topk(a, st);
  }
  const size_t smem = router_tc_smem_bytes(a.num_experts, false);
  const dim3 grid(tiles);
#define SENMOE_RT_CASE(V)                                                                              \
  if (epl <= V) {                                                                                    \
    e = ensure_dynamic_smem(reinterpret_cast<const void*>(router_tc_kernel<V, false>), smem);          \
    if (e != cudaSuccess) return e;                                                                  \
    return launch_pdl(router_tc_kernel<V, false>, grid, dim3(kRtThreads), smem, st, tX, tW, a);      \
  }
  SENMOE_RT_CASE(1) SENMOE_RT_CASE(2) SENMOE_RT_CASE(4) SENMOE_RT_CASE(8) SENMOE_RT_CASE(16)
#undef SENMOE_RT_CASE
  return cudaErrorNotSupported;
}

}  // namespace senmoe
