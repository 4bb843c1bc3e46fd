// expert_tc.cu -- grouped affine-quantized expert GEMM on the 5th-generation
// tensor cores (tcgen05 + TMEM), for batches that put more than a couple of
// tokens on each expert (prefill, and larger decode batches).
//
// Same contraction as the reference's SwitchGlu gather_qmm calls
// (src/engine/mlx_lm/models/deepseek_v2.rs:466-478, utils/moe.rs:33-77), with
// tokens grouped by expert (dispatch.cu).  Orientation: the weights are the
// M side (128 output rows per tile, K-major as MLX stores them) and the
// expert's tokens the N side (BN per tile, K-major rows of the slot-ordered
// activations), so one accumulator tile is D[128 rows, BN slots] in TMEM.
//
// Operands are fp16: codes dequantise to w = q * scale + bias in fp16 (11-bit
// mantissa; q * scale + bias of bf16 scale/bias is nearly always exact there),
// activations are bf16 values converted exactly to fp16, accumulation is fp32.
// A bf16 operand path would round every dequantised weight to 8 bits and move
// block outputs ~5e-3 (relative L2) away from MLX's fp32 qmv arithmetic, which
// the reference always runs (M = 1 per (token, slot)); fp16 keeps it ~1e-4.
// Activations must stay inside fp16 range (|v| < 65504); a value outside it
// records kDevFp16Range (the CUDA-core GEMV path has no such limit).
//
// One CTA computes one (expert, 128-row block, BN-slot block) tile, for one
// projection (down) or two sharing the activation tile (gate and up, whose
// epilogue applies SwiGLU/GeGLU with MLX's bf16 rounding and stores h as fp16
// for the down GEMM's B operand).  Warp roles:
//   warp 0     TMA producer: packed codes (2-D tensor map, no swizzle), the
//              activation tile (2-D tensor map, SWIZZLE_128B), and once per
//              tile the rows' scales and biases (1-D bulk copies).  No
//              multicast anywhere.
//   warp 1     TMEM owner; one lane issues tcgen05.mma (kind::f16, bf16 x
//              bf16 -> fp32, M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2-9  dequantise each 64-column k-block of codes to fp16
//              (w = q * scale + bias, one rounding) into SWIZZLE_128B K-major
//              tiles, then run the TMEM epilogue.
// Every mbarrier wait is bounded; a timeout sets a CTA-wide abort flag, every
// role drains and the CTA frees its TMEM and returns.

#include <cuda.h>

#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.h"

namespace senmoe {
namespace {

constexpr int kTcThreads = 320;
constexpr int kDqThreads = 256;
constexpr int BM = 128;  // weight rows per tile
constexpr int BK = 64;   // one quantization group per k-block

// ------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  // start address >> 4, LBO 16 B (unused for swizzled K-major), SBO 1024 B
  // (8 rows x 128 B), descriptor version 1, layout SWIZZLE_128B.
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

template <int N>
__device__ __forceinline__ constexpr uint32_t idesc_f16_f32() {
  // D fp32 (bits 4-5 = 1), A and B fp16 (format 0), both K-major, N >> 3, M >> 4.
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait that also gives up as soon as another role of the CTA has.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      record_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

// ------------------------------------------------------- dequantisation
// 8 consecutive 4-bit codes (one u32) -> 8 fp16 w = q * s + b, in order.
__device__ __forceinline__ uint4 dequant8_u4(uint32_t w, __half2 s2, __half2 b2) {
  const __half2 k1024 = __floats2half2_rn(1024.0f, 1024.0f);
  uint32_t v[4];
  v[0] = (w & 0x000F000Fu) | 0x64006400u;          // codes 0, 4 as fp16 1024 + q
  v[1] = ((w >> 4) & 0x000F000Fu) | 0x64006400u;   // 1, 5
  v[2] = ((w >> 8) & 0x000F000Fu) | 0x64006400u;   // 2, 6
  v[3] = ((w >> 12) & 0x000F000Fu) | 0x64006400u;  // 3, 7
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 q = __hsub2(*reinterpret_cast<__half2*>(&v[i]), k1024);  // exact
    __half2 r = __hfma2(q, s2, b2);                                 // one rounding
    o[i] = *reinterpret_cast<uint32_t*>(&r);
  }
  // (0,4),(1,5),(2,6),(3,7) -> (0,1),(2,3),(4,5),(6,7)
  return make_uint4(__byte_perm(o[0], o[1], 0x5410), __byte_perm(o[2], o[3], 0x5410),
                    __byte_perm(o[0], o[1], 0x7632), __byte_perm(o[2], o[3], 0x7632));
}

// 4 consecutive 8-bit codes (one u32) -> 4 fp16 (two u32), w = q * s + b.
__device__ __forceinline__ uint2 dequant4_u8(uint32_t w, float s, float b) {
  float f[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    f[k] = fmaf(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540 + k)) - 8388608.0f, s, b);
  __half2 lo = __floats2half2_rn(f[0], f[1]);
  __half2 hi = __floats2half2_rn(f[2], f[3]);
  return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// Shared-memory byte offset of 16-byte chunk `c` (0..7) of row `r` in a
// [rows x 64] 16-bit SWIZZLE_128B K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return static_cast<uint32_t>(r) * 128u + (static_cast<uint32_t>(c ^ (r & 7)) << 4);
}

// Stage counts per tile shape: activation (B) stages, packed-code stages.
template <int BN> struct TcStages {
  static constexpr int kB = BN >= 128 ? 2 : 4;
  static constexpr int kP = BN >= 128 ? 4 : 6;
  static constexpr int kA = 2;
};

}  // namespace

template <int BITS, int NPROJ, int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB, TcGemmArgs a) {
  constexpr int SA = TcStages<BN>::kA, SB = TcStages<BN>::kB, SP = TcStages<BN>::kP;
  constexpr int WK = BK * BITS / 32;                 // packed words per row per k-block
  constexpr uint32_t kABytes = BM * BK * 2;          // one fp16 A tile (16 KB)
  constexpr uint32_t kBBytes = BN * BK * 2;          // one activation tile
  constexpr uint32_t kPBytes = BM * WK * 4;          // one projection's packed k-block
  constexpr int kCols = (NPROJ * BN) <= 32 ? 32 : (NPROJ * BN) <= 64 ? 64 : (NPROJ * BN) <= 128 ? 128
                        : (NPROJ * BN) <= 256 ? 256 : 512;
  constexpr uint32_t kIdesc = idesc_f16_f32<BN>();

  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar_pfull[SP], bar_pempty[SP], bar_afull[SA], bar_aempty[SA], bar_bfull[SB],
      bar_bempty[SB], bar_sb, bar_acc, bar_drain;
  __shared__ uint32_t s_tmem;
  __shared__ int s_tile[4];  // local expert, first weight row, first slot, valid slots (-1: no tile)
  __shared__ volatile int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int groups = a.kdim / BK, ktiles = a.kdim / BK;

  // ---- carve dynamic shared memory (1024-byte aligned for SWIZZLE_128B)
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  unsigned char* sA = base;                                   // [SA][NPROJ][16 KB]
  unsigned char* sB = sA + SA * NPROJ * kABytes;              // [SB][BN*128]
  unsigned char* sP = sB + SB * kBBytes;                      // [SP][NPROJ][kPBytes]
  uint16_t* sSB = reinterpret_cast<uint16_t*>(sP + SP * NPROJ * kPBytes);  // [NPROJ][2][BM*groups]

  // ---- which tile: walk the active experts (m-block fastest)
  if (tid == 0) {
    int t = blockIdx.x, found = 0;
    const int nact = *a.active_count;
    for (int i = 0; i < nact && !found; ++i) {
      const int e = a.active[i];
      const int s0 = a.offsets[e], n = a.offsets[e + 1] - s0;
      const int cnt = ((n + BN - 1) / BN) * a.m_tiles;
      if (t < cnt) {
        const int nt = t / a.m_tiles, mt = t % a.m_tiles;
        s_tile[0] = e - a.expert_begin;
        s_tile[1] = mt * BM;
        s_tile[2] = s0 + nt * BN;
        s_tile[3] = min(BN, n - nt * BN);
        found = 1;
      } else {
        t -= cnt;
      }
    }
    if (!found) s_tile[3] = -1;
    s_abort = 0;
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < SP; ++i) { mbar_init(&bar_pfull[i], 1); mbar_init(&bar_pempty[i], kDqThreads); }
    for (int i = 0; i < SA; ++i) { mbar_init(&bar_afull[i], kDqThreads); mbar_init(&bar_aempty[i], 1); }
    for (int i = 0; i < SB; ++i) { mbar_init(&bar_bfull[i], 1); mbar_init(&bar_bempty[i], 1); }
    mbar_init(&bar_sb, 1);
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_drain, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (s_tile[3] <= 0) return;  // no tile for this CTA (uniform exit before TMEM use)
  const int e_local = s_tile[0], m0 = s_tile[1], slot0 = s_tile[2], nvalid = s_tile[3];

  if (warp == 1) {  // TMEM allocation (whole warp)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int row_base = e_local * a.rows + m0;  // first packed row of this tile

  if (warp == 0) {
    // ================================================= TMA producer
    if (lane == 0) {
      const uint32_t sb_bytes = BM * groups * 2;
      mbar_arrive_expect_tx(&bar_sb, NPROJ * 2 * sb_bytes);
      const uint64_t pol = policy_evict_first();
#pragma unroll
      for (int p = 0; p < NPROJ; ++p) {
        bulk_g2s(sSB + (p * 2 + 0) * BM * groups, a.s[p] + static_cast<size_t>(row_base) * groups, sb_bytes, &bar_sb,
                 pol);
        bulk_g2s(sSB + (p * 2 + 1) * BM * groups, a.b[p] + static_cast<size_t>(row_base) * groups, sb_bytes, &bar_sb,
                 pol);
      }
      int last_p[SP], last_b[SB];  // parity of the last load issued per stage (-1: none)
#pragma unroll
      for (int i = 0; i < SP; ++i) last_p[i] = -1;
#pragma unroll
      for (int i = 0; i < SB; ++i) last_b[i] = -1;
      bool ok = true;
      for (int kt = 0; kt < ktiles; ++kt) {
        const int ps = kt % SP, pph = (kt / SP) & 1;
        if (!(ok = wait_or_abort(&bar_pempty[ps], pph ^ 1, &s_abort, a.err))) break;
        mbar_arrive_expect_tx(&bar_pfull[ps], NPROJ * kPBytes);
        tma_load_2d(sP + (ps * NPROJ + 0) * kPBytes, &tmA0, kt * WK, row_base, &bar_pfull[ps]);
        if constexpr (NPROJ == 2) tma_load_2d(sP + (ps * NPROJ + 1) * kPBytes, &tmA1, kt * WK, row_base, &bar_pfull[ps]);
        last_p[ps] = pph;
        const int bs = kt % SB, bph = (kt / SB) & 1;
        if (!(ok = wait_or_abort(&bar_bempty[bs], bph ^ 1, &s_abort, a.err))) break;
        mbar_arrive_expect_tx(&bar_bfull[bs], kBBytes);
        tma_load_2d(sB + bs * kBBytes, &tmB, kt * BK, slot0, &bar_bfull[bs]);
        last_b[bs] = bph;
      }
      if (!ok) {  // give the copies already issued a bounded chance to land before exit
        volatile int never = 0;
        wait_or_abort(&bar_sb, 0, &never, nullptr);
#pragma unroll
        for (int i = 0; i < SP; ++i)
          if (last_p[i] >= 0) wait_or_abort(&bar_pfull[i], last_p[i], &never, nullptr);
#pragma unroll
        for (int i = 0; i < SB; ++i)
          if (last_b[i] >= 0) wait_or_abort(&bar_bfull[i], last_b[i], &never, nullptr);
      }
    }
  } else if (warp == 1) {
    // ================================================= MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int kt = 0; kt < ktiles && ok; ++kt) {
        const int as = kt % SA, aph = (kt / SA) & 1;
        const int bs = kt % SB, bph = (kt / SB) & 1;
        ok = wait_or_abort(&bar_afull[as], aph, &s_abort, a.err) &&
             wait_or_abort(&bar_bfull[bs], bph, &s_abort, a.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t b_addr = smem_u32(sB + bs * kBBytes);
#pragma unroll
        for (int p = 0; p < NPROJ; ++p) {
          const uint32_t a_addr = smem_u32(sA + (as * NPROJ + p) * kABytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(tmem + p * BN, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32),
                      kIdesc, (kt | k) != 0);
        }
        umma_commit(&bar_aempty[as]);
        umma_commit(&bar_bempty[bs]);
      }
      umma_commit(ok ? &bar_acc : &bar_drain);
      if (!ok) {  // let issued MMAs finish before TMEM is released
        volatile int never = 0;
        wait_or_abort(&bar_drain, 0, &never, nullptr);
      }
    }
  } else {
    // ================================================= dequant + epilogue
    const int d = tid - 64;  // 0..255
    // Per k-block: NPROJ x 128 rows x 64 codes over 256 threads.
    // NPROJ == 2: thread -> (projection d / 128, row d % 128, all 64 codes)
    // NPROJ == 1: thread -> (row d / 2, codes [32 * (d % 2), +32))
    const int proj = NPROJ == 2 ? d / 128 : 0;
    const int row = NPROJ == 2 ? d % 128 : d / 2;
    const int half = NPROJ == 2 ? 0 : d % 2;
    constexpr int kChunks = NPROJ == 2 ? 8 : 4;  // 16-byte output chunks per thread
    bool ok = wait_or_abort(&bar_sb, 0, &s_abort, a.err);
    const uint16_t* srow = sSB + (proj * 2 + 0) * BM * groups + row * groups;
    const uint16_t* brow = sSB + (proj * 2 + 1) * BM * groups + row * groups;
    for (int kt = 0; kt < ktiles && ok; ++kt) {
      const int ps = kt % SP, pph = (kt / SP) & 1;
      const int as = kt % SA, aph = (kt / SA) & 1;
      ok = wait_or_abort(&bar_pfull[ps], pph, &s_abort, a.err) &&
           wait_or_abort(&bar_aempty[as], aph ^ 1, &s_abort, a.err);
      if (!ok) break;
      const uint16_t sb = srow[kt], bb = brow[kt];
      const uint32_t* src = reinterpret_cast<const uint32_t*>(sP + (ps * NPROJ + proj) * kPBytes) + row * WK;
      unsigned char* dst = sA + (as * NPROJ + proj) * kABytes;
      if constexpr (BITS == 4) {
        const __half2 s2 = __float2half2_rn(bf16_bits_to_f32(sb));
        const __half2 b2 = __float2half2_rn(bf16_bits_to_f32(bb));
        const uint4* src4 = reinterpret_cast<const uint4*>(src + half * 4);
#pragma unroll
        for (int q = 0; q < kChunks / 4; ++q) {
          const uint4 w = src4[q];
          const int c = half * 4 + q * 4;
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 0)) = dequant8_u4(w.x, s2, b2);
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 1)) = dequant8_u4(w.y, s2, b2);
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 2)) = dequant8_u4(w.z, s2, b2);
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 3)) = dequant8_u4(w.w, s2, b2);
        }
      } else {
        const float sf = bf16_bits_to_f32(sb), bf = bf16_bits_to_f32(bb);
        const uint4* src4 = reinterpret_cast<const uint4*>(src + half * 8);
#pragma unroll
        for (int q = 0; q < kChunks / 2; ++q) {
          const uint4 w = src4[q];  // 16 codes = 2 output chunks
          const uint2 l0 = dequant4_u8(w.x, sf, bf), l1 = dequant4_u8(w.y, sf, bf);
          const uint2 h0 = dequant4_u8(w.z, sf, bf), h1 = dequant4_u8(w.w, sf, bf);
          const int c = half * 4 + q * 2;
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 0)) = make_uint4(l0.x, l0.y, l1.x, l1.y);
          *reinterpret_cast<uint4*>(dst + sw128_offset(row, c + 1)) = make_uint4(h0.x, h0.y, h1.x, h1.y);
        }
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&bar_afull[as]);
      mbar_arrive(&bar_pempty[ps]);
    }

    // ---- epilogue: TMEM -> registers -> global (slot-major output)
    if (ok && wait_or_abort(&bar_acc, 0, &s_abort, a.err)) {
      tc_fence_after();
      const int q = warp & 3;                    // TMEM lane quarter this warp may read
      const int colhalf = (warp - 2) >> 2;       // two warps per quarter split the columns
      const int r = m0 + q * 32 + lane;          // output row of this thread
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
      constexpr int kHalf = BN / 2 < 16 ? 16 : BN / 2;
      const int c_begin = colhalf * kHalf;
      for (int c0 = c_begin; c0 < c_begin + kHalf && c0 < BN; c0 += 16) {
        if (c0 >= nvalid) break;  // uniform across the warp
        uint32_t g[16], u[16];
        tmem_ld16(lane_addr + c0, g);
        if constexpr (NPROJ == 2) tmem_ld16(lane_addr + BN + c0, u);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j >= nvalid) break;
          uint16_t bits;
          if constexpr (NPROJ == 2) {  // h = act(bf16(g), bf16(u)) (bf16 value), stored as fp16
            const float gg = round_bf16(__uint_as_float(g[j])), uu = round_bf16(__uint_as_float(u[j]));
            const float v = a.act == 0 ? act_swiglu_mlx(gg, uu) : act_geglu_mlx(gg, uu);
            if (!(fabsf(v) < 65504.0f)) record_error(a.err, kDevFp16Range);
            bits = __half_as_ushort(__float2half_rn(v));
          } else {
            bits = f32_to_bf16_bits(__uint_as_float(g[j]));
          }
          a.out[static_cast<size_t>(slot0 + c0 + j) * a.out_stride + r] = bits;
        }
      }
    }
  }

  // ---- teardown: every role is done with TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ------------------------------------------------------------- host side
size_t tc_smem_bytes(int bits, int nproj, int bn, int kdim) {
  const int groups = kdim / BK;
  const int wk = BK * bits / 32;
  const int sb = bn >= 128 ? 2 : 4, sp = bn >= 128 ? 4 : 6, sa = 2;
  return 1024 + static_cast<size_t>(sa) * nproj * BM * BK * 2 + static_cast<size_t>(sb) * bn * BK * 2 +
         static_cast<size_t>(sp) * nproj * BM * wk * 4 + static_cast<size_t>(nproj) * 2 * BM * groups * 2;
}

bool tc_supported(int rows, int kdim, int bits, int nproj, int bn) {
  return rows % BM == 0 && kdim % BK == 0 && kdim >= BK && (bits == 4 || bits == 8) &&
         tc_smem_bytes(bits, nproj, bn, kdim) <= 227 * 1024;
}

template <int BITS, int NPROJ, int BN>
static cudaError_t launch_tc_t(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                               const TcGemmArgs& a, int grid, cudaStream_t st) {
  const size_t smem = tc_smem_bytes(BITS, NPROJ, BN, a.kdim);
  auto kern = tc_gemm_kernel<BITS, NPROJ, BN>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kTcThreads, smem, st>>>(tA0, tA1, tB, a);
  return cudaGetLastError();
}

cudaError_t launch_tc_gemm(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                           const TcGemmArgs& a, int bits, int nproj, int bn, int grid, cudaStream_t st) {
  if (grid <= 0) return cudaSuccess;
#define SENMOE_TC_CASE(B, P, N) \
  if (bits == B && nproj == P && bn == N) return launch_tc_t<B, P, N>(tA0, tA1, tB, a, grid, st);
#define SENMOE_TC_BN(B, P) \
  SENMOE_TC_CASE(B, P, 16) SENMOE_TC_CASE(B, P, 32) SENMOE_TC_CASE(B, P, 64) SENMOE_TC_CASE(B, P, 128) \
  SENMOE_TC_CASE(B, P, 256)
  SENMOE_TC_BN(4, 1) SENMOE_TC_BN(4, 2) SENMOE_TC_BN(8, 1) SENMOE_TC_BN(8, 2)
#undef SENMOE_TC_BN
#undef SENMOE_TC_CASE
  return cudaErrorNotSupported;
}

}  // namespace senmoe

// ---------------------------------------------------- tensor maps, gather
#include <cudaTypedefs.h>

#include <mutex>

namespace senmoe {

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

cudaError_t make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner,
                         uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         bool swizzle128) {
  auto enc = tmap_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Slot-ordered fp16 copy of the token rows (bf16 -> fp16 is exact in range).
__global__ void gather_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm, int k_div,
                                   uint16_t* __restrict__ out, int hidden, int* err) {
  const int s = blockIdx.x;
  const int token = perm[s] / k_div;
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(token) * hidden);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(s) * hidden);
  bool range_ok = true;
  for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) {
    const uint4 v = src[i];
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float lo = bf16_lo(in[k]), hi = bf16_hi(in[k]);
      range_ok &= fabsf(lo) < 65504.0f && fabsf(hi) < 65504.0f;
      const __half2 h = __floats2half2_rn(lo, hi);
      o[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    dst[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (!range_ok) record_error(err, kDevFp16Range);
}

cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* perm, int k_div, uint16_t* x_sorted,
                               int num_slots, int hidden, int* err, cudaStream_t st) {
  if (num_slots <= 0) return cudaSuccess;
  const int threads = hidden / 8 < 256 ? ((hidden / 8 + 31) / 32) * 32 : 256;
  gather_rows_kernel<<<num_slots, threads, 0, st>>>(x, perm, k_div, x_sorted, hidden, err);
  return cudaGetLastError();
}

}  // namespace senmoe
