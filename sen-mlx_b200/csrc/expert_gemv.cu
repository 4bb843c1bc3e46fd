// expert_gemv.cu -- grouped affine-quantized dequant-GEMV for decode-size
// batches, plus the weighted combine.
//
// Replaces the per-(token, slot) MLX gather_qmm calls of SwitchGlu::forward
// (src/engine/mlx_lm/models/deepseek_v2.rs:466-478, utils/moe.rs:33-77) when
// few tokens land on each expert.  Only the experts that received tokens are
// touched: CTA (blockIdx.x = a, blockIdx.y = rb) handles rows
// [rb*RB, rb*RB + RB) of the a-th active expert.  Its packed words, scales and
// biases (one contiguous range per tensor in MLX layout) arrive in shared
// memory by 1-D TMA bulk copies (cp.async.bulk, no multicast) completing on one
// mbarrier; weights are streamed once (L2 evict-first).
//
// Per warp, lane l owns packed words l, l+32, l+64, ... of every row, so a
// warp's shared-memory word loads are conflict-free and its x loads (one
// 16-byte vector of 8 bf16 per word) are coalesced.  Dequantisation uses the
// bf16 magic-number trick: (w >> 4k) & 0x000F000F | 0x43004300 holds two bf16
// values 128 + q, so sum((128+q) x) - 128 sum(x) = sum(q x) and per word
//   acc += scale * sum((128+q) x) + (bias - 128 scale) * sum(x)
// which is MLX qmv's scale*sum(q x) + bias*sum(x) factorisation in fp32.
// 8-bit codes use the fp32 magic 2^23 + q built with one byte permute.
// Row results are reduced with warp shuffles.

#include "common.cuh"
#include "gemv_core.cuh"
#include "kernels.h"

namespace senmoe {

namespace {

constexpr int kGemvWarps = 4;
constexpr int kGemvThreads = kGemvWarps * 32;

}  // namespace

// NPROJ = 2: gate and up rows of the same expert, fused with the activation
// (SwiGLU / GeGLU with MLX's bf16 rounding); NPROJ = 1: a plain projection
// (the down projection, the shared expert's down, gather_qmm).
template <int BITS, int WPL, int NPROJ>
__global__ void __launch_bounds__(kGemvThreads) qgemv_kernel(QGemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bar;
  constexpr int CPW = Codes<BITS>::kPerWord;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int words_per_row = a.kdim * BITS / 32;  // <= WPL * 32
  const int groups = a.kdim / 64;

  pdl_wait();  // the active list / offsets come from the dispatch kernel
  pdl_launch_dependents();
  // ---- which expert / slots does this CTA serve?
  int expert, s_begin, s_end, s_local0 = 0;  // slot s is row s - s_local0 of out (and of x by slot)
  if (a.mode == kItemsGrouped) {
    if (blockIdx.x >= static_cast<unsigned>(*a.active_count)) return;
    expert = a.active[blockIdx.x];
    s_begin = a.offsets[expert];
    s_end = a.offsets[expert + 1];
    s_local0 = a.offsets[a.expert_begin];  // this rank's first slot (0 on one GPU)
    expert -= a.expert_begin;
  } else {  // kItemsGather: one index per CTA row (no index list: expert 0, a dense linear)
    const uint32_t e = a.gather_idx ? a.gather_idx[blockIdx.x] : 0u;
    if (e >= static_cast<uint32_t>(a.num_experts)) {
      if (threadIdx.x == 0) record_error(a.err, kDevBadExpert);
      return;
    }
    expert = static_cast<int>(e);
    s_begin = blockIdx.x;
    s_end = s_begin + 1;
  }
  const int row0 = blockIdx.y * a.rows_per_cta;
  const int nrows = min(a.rows_per_cta, a.rows - row0);
  if (nrows <= 0) return;

  // ---- shared-memory carve-up: [proj][words], then [proj][scales], [proj][biases]
  uint32_t* sw = reinterpret_cast<uint32_t*>(smem);
  const size_t w_elems = static_cast<size_t>(a.rows_per_cta) * words_per_row;
  uint16_t* ss = reinterpret_cast<uint16_t*>(sw + NPROJ * w_elems);
  const size_t sb_elems = static_cast<size_t>(a.rows_per_cta) * groups;
  uint16_t* sb = ss + NPROJ * sb_elems;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t wbytes = static_cast<uint32_t>(nrows) * words_per_row * 4u;
    const uint32_t sbytes = static_cast<uint32_t>(nrows) * groups * 2u;
    mbar_arrive_expect_tx(&bar, NPROJ * (wbytes + 2u * sbytes));
    const uint64_t pol = policy_evict_first();
#pragma unroll
    for (int p = 0; p < NPROJ; ++p) {
      const size_t wrow = static_cast<size_t>(expert) * a.rows + row0;
      bulk_g2s(sw + p * w_elems, a.w[p] + wrow * words_per_row, wbytes, &bar, pol);
      bulk_g2s(ss + p * sb_elems, a.s[p] + wrow * groups, sbytes, &bar, pol);
      bulk_g2s(sb + p * sb_elems, a.b[p] + wrow * groups, sbytes, &bar, pol);
    }
  }
  const bool ready = mbar_wait(&bar, 0, a.err);
  if (!ready) {
    // Copies may still be landing: give them one more bounded wait before
    // the CTA releases its shared memory.
    mbar_wait(&bar, 0, nullptr);
    return;
  }

  for (int s = s_begin; s < s_end; ++s) {
    const int token =
        (a.mode == kItemsGather) ? static_cast<int>(s / a.rep) : (a.x_by_slot ? s - s_local0 : a.perm[s] / a.k_div);
    float xv[WPL][CPW], xs[WPL];
    load_x_slice<BITS, WPL>(a.x + static_cast<size_t>(token) * a.kdim, lane, words_per_row, xv, xs);
    uint16_t* out = a.out + static_cast<size_t>(s - s_local0) * a.out_stride + row0;
    for (int r = warp; r < nrows; r += kGemvWarps) {
      float v0 = row_partial<BITS, WPL>(sw + static_cast<size_t>(r) * words_per_row, ss + r * groups,
                                        sb + r * groups, lane, words_per_row, xv, xs);
      v0 = warp_sum(v0);
      if constexpr (NPROJ == 2) {
        float v1 = row_partial<BITS, WPL>(sw + w_elems + static_cast<size_t>(r) * words_per_row,
                                          ss + sb_elems + r * groups, sb + sb_elems + r * groups, lane, words_per_row, xv, xs);
        v1 = warp_sum(v1);
        if (lane == 0) {
          const float g = round_bf16(v0), u = round_bf16(v1);
          const float h = (a.act == 0) ? act_swiglu_mlx(g, u) : act_geglu_mlx(g, u);
          out[r] = f32_to_bf16_bits(h);
        }
      } else {
        if (lane == 0) out[r] = f32_to_bf16_bits(v0);
      }
    }
  }
}

// y[t, :] = bf16( sum_j f32(d[inv[t*K + j], :]) * w[t, j]  (+ gate_t * shared[t, :]) )
// in slot order j = 0..K-1 with fp32 accumulation (deepseek_v2.rs:546-552).
// KMAX: compile-time bound on top_k (8 or 16) sizing the per-thread slot and
// row arrays, so that the register budget allows several CTAs per SM.
template <int KMAX>
__global__ void __launch_bounds__(256, KMAX <= 8 ? 4 : 2) combine_kernel(CombineArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= a.hidden) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  // all slot indices and weights first, then all rows, so the loads overlap;
  // the sum still runs in slot order j = 0..K-1
  constexpr int kMaxK = KMAX;
  int slot[kMaxK];
  float wj[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    if (j < a.top_k) {
      slot[j] = a.inverse[t * a.top_k + j];
      wj[j] = a.weights[t * a.top_k + j];
    }
  }
  uint4 rows[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j)
    if (j < a.top_k && slot[j] >= 0)  // slot < 0: expert held by another rank
      rows[j] = *reinterpret_cast<const uint4*>(a.d + static_cast<size_t>(slot[j]) * a.hidden + col);
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    if (j < a.top_k && slot[j] >= 0) {
      const uint4 v = rows[j];
      const float w = wj[j];
      acc[0] += bf16_lo(v.x) * w; acc[1] += bf16_hi(v.x) * w;
      acc[2] += bf16_lo(v.y) * w; acc[3] += bf16_hi(v.y) * w;
      acc[4] += bf16_lo(v.z) * w; acc[5] += bf16_hi(v.z) * w;
      acc[6] += bf16_lo(v.w) * w; acc[7] += bf16_hi(v.w) * w;
    }
  }
  if (a.shared_out) {
    const float g = a.shared_gate ? a.shared_gate[t] : 1.0f;
    const uint4 v =
        *reinterpret_cast<const uint4*>(a.shared_out + static_cast<size_t>(t - a.shared_row0) * a.hidden + col);
    acc[0] += g * bf16_lo(v.x); acc[1] += g * bf16_hi(v.x);
    acc[2] += g * bf16_lo(v.y); acc[3] += g * bf16_hi(v.y);
    acc[4] += g * bf16_lo(v.z); acc[5] += g * bf16_hi(v.z);
    acc[6] += g * bf16_lo(v.w); acc[7] += g * bf16_hi(v.w);
  }
  if (a.residual) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.residual + static_cast<size_t>(t) * a.hidden + col);
    acc[0] += bf16_lo(v.x); acc[1] += bf16_hi(v.x); acc[2] += bf16_lo(v.y); acc[3] += bf16_hi(v.y);
    acc[4] += bf16_lo(v.z); acc[5] += bf16_hi(v.z); acc[6] += bf16_lo(v.w); acc[7] += bf16_hi(v.w);
  }
  if (a.y_f32) {
    float4* yf = reinterpret_cast<float4*>(a.y_f32 + static_cast<size_t>(t) * a.hidden + col);
    yf[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    yf[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
  uint4 o;
  o.x = uint32_t(f32_to_bf16_bits(acc[0])) | (uint32_t(f32_to_bf16_bits(acc[1])) << 16);
  o.y = uint32_t(f32_to_bf16_bits(acc[2])) | (uint32_t(f32_to_bf16_bits(acc[3])) << 16);
  o.z = uint32_t(f32_to_bf16_bits(acc[4])) | (uint32_t(f32_to_bf16_bits(acc[5])) << 16);
  o.w = uint32_t(f32_to_bf16_bits(acc[6])) | (uint32_t(f32_to_bf16_bits(acc[7])) << 16);
  *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(t) * a.hidden + col) = o;
}

// ------------------------------------------------------------- launchers
size_t qgemv_smem_bytes(int nproj, int rows_per_cta, int kdim, int bits) {
  const size_t words = static_cast<size_t>(kdim) * bits / 32;
  const size_t groups = kdim / 64;
  return static_cast<size_t>(nproj) * rows_per_cta * (words * 4 + 2 * groups * 2);
}

template <int BITS, int WPL, int NPROJ>
static cudaError_t launch_qgemv_t(const QGemvArgs& a, int num_items, cudaStream_t st) {
  const size_t smem = qgemv_smem_bytes(NPROJ, a.rows_per_cta, a.kdim, BITS);
  auto kern = qgemv_kernel<BITS, WPL, NPROJ>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  if (num_items == 0) return cudaSuccess;
  dim3 grid(num_items, (a.rows + a.rows_per_cta - 1) / a.rows_per_cta);
  return launch_pdl(kern, grid, dim3(kGemvThreads), smem, st, a);
}

// Words per lane WPL = ceil(kdim * bits / 32 / 32) selects the instance;
// kdim must be a multiple of 64 (one quantization group) and WPL <= 16.
static int qgemv_wpl(int kdim, int bits) {
  const int words = kdim * bits / 32;
  const int wpl = (words + 31) / 32;
  if (wpl <= 4) return wpl;
  if (wpl <= 6) return 6;
  if (wpl <= 8) return 8;
  if (wpl <= 12) return 12;
  return wpl <= 16 ? 16 : -1;
}

cudaError_t launch_qgemv(const QGemvArgs& a, int nproj, int bits, int num_items, cudaStream_t st) {
  const int wpl = qgemv_wpl(a.kdim, bits);
#define SENMOE_QGEMV_CASE(B, W)                                                      \
  if (bits == B && wpl == W)                                                         \
    return nproj == 2 ? launch_qgemv_t<B, W, 2>(a, num_items, st) : launch_qgemv_t<B, W, 1>(a, num_items, st);
  SENMOE_QGEMV_CASE(4, 1) SENMOE_QGEMV_CASE(4, 2) SENMOE_QGEMV_CASE(4, 3) SENMOE_QGEMV_CASE(4, 4)
  SENMOE_QGEMV_CASE(4, 6) SENMOE_QGEMV_CASE(4, 8) SENMOE_QGEMV_CASE(4, 12) SENMOE_QGEMV_CASE(4, 16)
  SENMOE_QGEMV_CASE(8, 1) SENMOE_QGEMV_CASE(8, 2) SENMOE_QGEMV_CASE(8, 3) SENMOE_QGEMV_CASE(8, 4)
  SENMOE_QGEMV_CASE(8, 6) SENMOE_QGEMV_CASE(8, 8) SENMOE_QGEMV_CASE(8, 12) SENMOE_QGEMV_CASE(8, 16)
#undef SENMOE_QGEMV_CASE
  return cudaErrorNotSupported;
}

bool qgemv_supported(int kdim, int bits) {
  return kdim > 0 && kdim % 64 == 0 && (bits == 4 || bits == 8) && qgemv_wpl(kdim, bits) > 0;
}

cudaError_t launch_combine(const CombineArgs& a, int num_tokens, cudaStream_t st) {
  if (num_tokens == 0) return cudaSuccess;
  // small batches: narrow CTAs, so a token's row spreads over several SMs
  const int threads = num_tokens < 256 ? 64 : 256;
  dim3 grid((a.hidden / 8 + threads - 1) / threads, num_tokens);
  if (a.top_k <= 8) return launch_pdl(combine_kernel<8>, grid, dim3(threads), 0, st, a);
  return launch_pdl(combine_kernel<16>, grid, dim3(threads), 0, st, a);
}

}  // namespace senmoe
