// layer_single.cu -- the whole MoE block for one token in one launch
// (decode at batch 1: DeepseekMoe::forward, deepseek_v2.rs:520-553, with the
// residual add of DecoderLayer::forward, :613-620).
//
// At one token the block is a chain of tiny dependent steps (router logits,
// top-k, dispatch, gather, two expert products, combine), each a few
// kilobytes of work, while the expert weights (14 MB at config 1) want the
// whole GPU streaming at once.  One persistent grid of one CTA per SM runs:
//   A. router logits: warp w of the grid computes expert w's logit (the
//      router kernel's arithmetic, router_core.cuh);
//   -- grid barrier --
//   B. every CTA takes the token's top-k itself (router_core.cuh topk_row,
//      into shared memory; CTA 0 also writes it out) and at once issues bulk
//      copies (cp.async.bulk, no multicast) of all the weights it will use:
//      its block of gate/up rows of one selected expert and its block of
//      down rows of every selected expert, so the ~21 MB of the layer are in
//      flight together;
//   C. gate/up rows + SwiGLU/GeGLU into h [K, I] (bf16, global);
//   -- grid barrier --
//   D. for its down rows, each warp computes the row of every selected
//      expert and combines them in top-k order with the weights (+ the
//      residual): y needs no further pass.
// The row arithmetic is the CUDA-core GEMV's (gemv_core.cuh) and the combine
// sums in the combine kernel's order, so the output equals the layer's
// CUDA-core GEMV path bit for bit.
//
// The grid barrier is a flip-bit counter (CTA 0 adds 2^31 - (G - 1), the
// others 1: the high bit flips once per barrier and the low bits return to
// zero), so it needs no reset between calls or graph replays.  Every wait is
// bounded; a timeout records kDevWaitTimeout and the kernel finishes with an
// undefined y.  The dependent launch is triggered only after the first
// barrier, when every CTA of the grid is resident.

#include "common.cuh"
#include "gemv_core.cuh"
#include "kernels.h"
#include "router_core.cuh"

namespace senmoe {
namespace {

constexpr int kSingleWarps = 16;  // 4 per scheduler: the row arithmetic needs the latency hiding
constexpr int kSingleThreads = kSingleWarps * 32;

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// All CTAs of the grid; false after a timeout (recorded in *err).
__device__ __forceinline__ bool grid_barrier(unsigned int* bar, int* err, int* s_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int nb = gridDim.x;
    const unsigned int inc = blockIdx.x == 0 ? 0x80000000u - (nb - 1u) : 1u;
    __threadfence();  // this CTA's global writes before its arrival
    const unsigned int old = atomicAdd(bar, inc);
    const long long t0 = clock64();
    int ok = 1;
    while (((ld_acquire_gpu(bar) ^ old) & 0x80000000u) == 0u) {
      if (clock64() - t0 > kWaitLimitCycles) {
        record_error(err, kDevWaitTimeout);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    *s_flag = ok;
  }
  __syncthreads();
  return *s_flag != 0;
}

// Rows [lo, hi) of an even split of n rows (in units of `unit` rows) over `parts` parts.
__device__ __forceinline__ void split_rows(int n, int unit, int parts, int part, int& lo, int& hi) {
  const int units = n / unit;
  lo = static_cast<int>(static_cast<long long>(units) * part / parts) * unit;
  hi = static_cast<int>(static_cast<long long>(units) * (part + 1) / parts) * unit;
}

}  // namespace

template <int BITS, int WPL_GU, int WPL_D, int EPL>
__global__ void __launch_bounds__(kSingleThreads, 1) single_token_kernel(SingleTokenArgs a) {
  constexpr int CPW = Codes<BITS>::kPerWord;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bar_c, bar_d;
  __shared__ int s_ids[kMaxTopK];
  __shared__ float s_w[kMaxTopK];
  __shared__ int s_flag;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int H = a.hidden, I = a.inter, E = a.num_experts, K = a.top_k;
  const int G = gridDim.x, cta = blockIdx.x;
  const int wg = H * BITS / 32, gh = H / 64;  // gate/up: words / groups per row
  const int wd = I * BITS / 32, gi = I / 64;  // down

  if (threadIdx.x == 0) {
    mbar_init(&bar_c, 1);
    mbar_init(&bar_d, 1);
    fence_mbar_init();
  }
  pdl_wait();  // x and the residual come from the previous kernel

  // ---- A. router logits, one expert per warp of the grid, spread over the
  // CTAs first (expert e on CTA e mod G) so each SM loads only a few rows
  {
    const int vec = H / 8;
    for (int e = warp * G + cta; e < E; e += G * kSingleWarps) {
      // H / 256 16-byte vectors per lane: WPL_GU at 4 bits (H / 8 words of 8 codes)
      float wv[WPL_GU][8];
      router_load_wrow<WPL_GU>(a.router_weight + static_cast<size_t>(e) * H, lane, vec, wv);
      float acc = router_dot_lane<WPL_GU>(wv, reinterpret_cast<const uint4*>(a.x), lane, vec);
      acc = warp_sum(acc);
      if (lane == 0) a.logits[e] = round_bf16(acc);
    }
  }
  if (!grid_barrier(a.grid_bar, a.err, &s_flag)) return;
  pdl_launch_dependents();

  // ---- B. top-k of the token (every CTA), then this CTA's weight copies
  if (warp == 0) {
    RouterArgs ra{};
    ra.num_experts = E;
    ra.top_k = K;
    ra.norm_topk_prob = a.norm_topk_prob;
    ra.routed_scaling_factor = a.routed_scaling_factor;
    ra.topk_ids = s_ids;
    ra.topk_weights = s_w;
    topk_row<EPL, false>(ra, a.logits, 0, lane);
  }
  __syncthreads();
  if (cta == 0 && threadIdx.x < K) {
    a.topk_ids[threadIdx.x] = s_ids[threadIdx.x];
    a.topk_weights[threadIdx.x] = s_w[threadIdx.x];
  }
  // gate/up: CTA cta serves selected expert kc = cta * K / G (the CTAs of
  // one expert are consecutive), rows of an even split among those CTAs;
  // down: rows of an even split of H over all CTAs, for every expert
  const int kc = static_cast<int>(static_cast<long long>(cta) * K / G);
  const int c_first = static_cast<int>((static_cast<long long>(kc) * G + K - 1) / K);       // first CTA of kc
  const int c_last = static_cast<int>((static_cast<long long>(kc + 1) * G + K - 1) / K);    // one past
  int rc0, rc1;
  split_rows(I, a.unit_c, c_last - c_first, cta - c_first, rc0, rc1);
  int rd0, rd1;
  split_rows(H, a.unit_d, G, cta, rd0, rd1);
  const int nrc = rc1 - rc0, nrd = rd1 - rd0;
  // shared memory: [proj][nrc][wg] codes, [proj][nrc][gh] scales, biases;
  // then [K][nrd][wd] down codes, [K][nrd][gi] scales, biases
  uint32_t* sc_w = reinterpret_cast<uint32_t*>(smem);
  uint16_t* sc_s = reinterpret_cast<uint16_t*>(sc_w + 2 * a.rows_c * wg);
  uint16_t* sc_b = sc_s + 2 * a.rows_c * gh;
  uint32_t* sd_w = reinterpret_cast<uint32_t*>(smem + a.smem_c);
  uint16_t* sd_s = reinterpret_cast<uint16_t*>(sd_w + K * a.rows_d * wd);
  uint16_t* sd_b = sd_s + K * a.rows_d * gi;
  // the expected bytes first (one thread), then one bulk copy per thread:
  // threads 0-5 the gate/up rows (projection, array), 32.. the down rows
  // (expert, array), so the ~30 copies issue in parallel
  const uint32_t cw = static_cast<uint32_t>(nrc) * wg * 4u, cs = static_cast<uint32_t>(nrc) * gh * 2u;
  const uint32_t dw = static_cast<uint32_t>(nrd) * wd * 4u, ds = static_cast<uint32_t>(nrd) * gi * 2u;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bar_c, nrc > 0 ? 2u * (cw + 2u * cs) : 0u);
    mbar_arrive_expect_tx(&bar_d, nrd > 0 ? static_cast<uint32_t>(K) * (dw + 2u * ds) : 0u);
  }
  __syncthreads();
  {
    const int t = threadIdx.x;
    if (t < 6 && nrc > 0) {
      const int p = t / 3, which = t % 3;
      const size_t row = static_cast<size_t>(s_ids[kc]) * I + rc0;
      const uint64_t pol = policy_evict_first();
      if (which == 0) bulk_g2s(sc_w + p * a.rows_c * wg, a.w[p] + row * wg, cw, &bar_c, pol);
      else if (which == 1) bulk_g2s(sc_s + p * a.rows_c * gh, a.s[p] + row * gh, cs, &bar_c, pol);
      else bulk_g2s(sc_b + p * a.rows_c * gh, a.b[p] + row * gh, cs, &bar_c, pol);
    } else if (t >= 32 && t < 32 + 3 * K && nrd > 0) {
      const int k = (t - 32) / 3, which = (t - 32) % 3;
      const size_t row = static_cast<size_t>(s_ids[k]) * H + rd0;
      const uint64_t pol = policy_evict_first();
      if (which == 0) bulk_g2s(sd_w + k * a.rows_d * wd, a.w[2] + row * wd, dw, &bar_d, pol);
      else if (which == 1) bulk_g2s(sd_s + k * a.rows_d * gi, a.s[2] + row * gi, ds, &bar_d, pol);
      else bulk_g2s(sd_b + k * a.rows_d * gi, a.b[2] + row * gi, ds, &bar_d, pol);
    }
  }

  // ---- C. gate/up rows of expert s_ids[kc] + activation -> h[kc]
  bool ok = mbar_wait(&bar_c, 0, a.err);
  if (ok && nrc > 0) {
    float xv[WPL_GU][CPW], xs[WPL_GU];
    load_x_slice<BITS, WPL_GU>(a.x, lane, wg, xv, xs);
    // two rows per step (four independent dot products in flight)
    auto gate_up = [&](int r, float& g, float& u) {
      g = row_partial<BITS, WPL_GU>(sc_w + static_cast<size_t>(r) * wg, sc_s + r * gh, sc_b + r * gh, lane, wg, xv,
                                    xs);
      u = row_partial<BITS, WPL_GU>(sc_w + static_cast<size_t>(a.rows_c + r) * wg, sc_s + (a.rows_c + r) * gh,
                                    sc_b + (a.rows_c + r) * gh, lane, wg, xv, xs);
    };
    auto emit = [&](int r, float g, float u) {
      g = warp_sum(g);
      u = warp_sum(u);
      if (lane == 0) {
        const float gg = round_bf16(g), uu = round_bf16(u);
        const float hv = a.act == 0 ? act_swiglu_mlx(gg, uu) : act_geglu_mlx(gg, uu);
        a.h[static_cast<size_t>(kc) * I + rc0 + r] = f32_to_bf16_bits(hv);
      }
    };
    for (int r = warp; r < nrc; r += 2 * kSingleWarps) {
      const int r2 = r + kSingleWarps;
      float g0, u0, g1 = 0.f, u1 = 0.f;
      gate_up(r, g0, u0);
      if (r2 < nrc) gate_up(r2, g1, u1);
      emit(r, g0, u0);
      if (r2 < nrc) emit(r2, g1, u1);
    }
  }
  if (!ok) {  // copies may still land: one more bounded wait before leaving
    mbar_wait(&bar_c, 0, nullptr);
    mbar_wait(&bar_d, 0, nullptr);
    return;
  }
  if (!grid_barrier(a.grid_bar, a.err, &s_flag)) {
    mbar_wait(&bar_d, 0, nullptr);
    return;
  }

  // ---- D. down rows of every selected expert, combined in top-k order;
  // h [K, I] is staged in shared memory once (each row reads all of it)
  uint16_t* sh_h = reinterpret_cast<uint16_t*>(smem + a.smem_c + a.smem_d);
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.h);
    uint4* dst = reinterpret_cast<uint4*>(sh_h);
    for (int i = threadIdx.x; i < K * I / 8; i += kSingleThreads) dst[i] = __ldcg(src + i);
  }
  __syncthreads();
  ok = mbar_wait(&bar_d, 0, a.err);
  if (!ok) {
    mbar_wait(&bar_d, 0, nullptr);
    return;
  }
  auto down_row = [&](int k, int r) {
    float xv[WPL_D][CPW], xs[WPL_D];
    load_x_slice<BITS, WPL_D>(sh_h + k * I, lane, wd, xv, xs);
    return row_partial<BITS, WPL_D>(sd_w + static_cast<size_t>(k * a.rows_d + r) * wd, sd_s + (k * a.rows_d + r) * gi,
                                    sd_b + (k * a.rows_d + r) * gi, lane, wd, xv, xs);
  };
  for (int r = warp; r < nrd; r += kSingleWarps) {
    float acc = 0.f;
    // two experts' rows per step, summed into acc in top-k order
    for (int k = 0; k < K; k += 2) {
      float v0 = down_row(k, r), v1 = k + 1 < K ? down_row(k + 1, r) : 0.f;
      v0 = warp_sum(v0);
      v1 = warp_sum(v1);
      const float d0 = bf16_bits_to_f32(f32_to_bf16_bits(v0));  // d as the down kernel stores it
      acc += d0 * s_w[k];                                        // the combine kernel's expression
      if (k + 1 < K) {
        const float d1 = bf16_bits_to_f32(f32_to_bf16_bits(v1));
        acc += d1 * s_w[k + 1];
      }
    }
    if (lane == 0) {
      if (a.residual) acc += bf16_bits_to_f32(a.residual[rd0 + r]);
      a.y[rd0 + r] = f32_to_bf16_bits(acc);
    }
  }
}

// ------------------------------------------------------------- host side
namespace {
int single_wpl(int words) {
  const int wpl = (words + 31) / 32;
  return wpl;
}
int gcd_int(int x, int y) { return y == 0 ? x : gcd_int(y, x % y); }
}  // namespace

bool single_token_plan(SingleTokenArgs& a, int sms) {
  const int H = a.hidden, I = a.inter, K = a.top_k, bits = a.bits;
  if (bits != 4 || K < 1 || K > kMaxTopK || K > sms || a.num_experts > 512 || H > 4096) return false;
  if (H % 64 || I % 64) return false;
  const int wg = H * bits / 32, wd = I * bits / 32;
  if (single_wpl(wg) != 8 || (single_wpl(wd) != 3 && single_wpl(wd) != 2)) return false;
  // bulk copies start and end on 16-byte boundaries: codes rows are (H or I
  // x bits / 8) bytes, scale / bias rows H / 32 or I / 32 bytes
  if ((wg * 4) % 16 || (wd * 4) % 16) return false;
  a.unit_c = 16 / gcd_int(16, H / 32);
  a.unit_d = 16 / gcd_int(16, I / 32);
  if (I % a.unit_c || H % a.unit_d) return false;
  if ((static_cast<long long>(I) * (H / 32)) % 16) return false;  // one expert's scale rows: whole 16-byte units
  // the most rows a CTA takes: its expert's share of I, its share of H
  const int ctas_per_expert = sms / K;  // at least, per expert
  a.rows_c = ((I / a.unit_c + ctas_per_expert - 1) / ctas_per_expert) * a.unit_c;
  a.rows_d = ((H / a.unit_d + sms - 1) / sms) * a.unit_d;
  const size_t smem_c = (static_cast<size_t>(2) * a.rows_c * (wg * 4 + 2 * (H / 64) * 2) + 127) / 128 * 128;
  const size_t smem_d = (static_cast<size_t>(K) * a.rows_d * (wd * 4 + 2 * (I / 64) * 2) + 127) / 128 * 128;
  const size_t smem_h = static_cast<size_t>(K) * I * 2;  // h staged for the down rows
  if (I % 8) return false;
  a.smem_c = static_cast<int>(smem_c);
  a.smem_d = static_cast<int>(smem_d);
  a.smem = static_cast<int>(smem_c + smem_d + smem_h);
  return a.smem <= 200 * 1024;
}

cudaError_t launch_single_token_layer(const SingleTokenArgs& a, int sms, cudaStream_t st) {
  const int epl = (a.num_experts + 31) / 32;
  const int wpl_d = single_wpl(a.inter * a.bits / 32);
#define SENMOE_ST_CASE(WD, V)                                                                       \
  if (wpl_d == WD && epl <= V) {                                                                   \
    auto kern = single_token_kernel<4, 8, WD, V>;                                                  \
    cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), a.smem);             \
    if (e != cudaSuccess) return e;                                                                \
    return launch_pdl(kern, dim3(sms), dim3(kSingleThreads), a.smem, st, a);                        \
  }
  SENMOE_ST_CASE(3, 4) SENMOE_ST_CASE(3, 16) SENMOE_ST_CASE(2, 4) SENMOE_ST_CASE(2, 16)
#undef SENMOE_ST_CASE
  return cudaErrorNotSupported;
}

}  // namespace senmoe
