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
//   warp 0     producer of the packed codes (lane 0: 2-D TMA, no swizzle)
//              and, per packed stage, its rows' scales and biases (all 32
//              lanes, 4- or 8-byte cp.async into shared memory, arriving on
//              the stage's barrier).  No multicast anywhere.
//   warp 1     TMEM owner; one lane issues tcgen05.mma (kind::f16, fp16 x
//              fp16 -> fp32, M=128, N=BN, K=16) and tcgen05.commit.
//   warps 2-17 dequantise each 64-column k-block of codes to fp16
//              (w = q * scale + bias, one rounding) straight into TMEM with
//              tcgen05.st: the MMA reads its A operand from TMEM, so the
//              8x-expanded fp16 weights never cross the shared-memory port
//              (which would otherwise bound the kernel).
//   warps 18-21 epilogue (TMEM accumulators -> global), warp 22 TMA of the
//              activation tiles, warp 23 the second MMA issuer, warps 24-27
//              (gate/up at 128 slots) epilogue helpers.
// Every mbarrier wait is bounded; a timeout sets a CTA-wide abort flag, every
// role drains and the CTA frees its TMEM and returns.

#include <cuda.h>

#include <cuda_fp16.h>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"
#include "tiles.cuh"

namespace senmoe {
namespace {

constexpr int kDqWarps = 16;
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
// The same with N chosen at run time: a tile's valid slots rounded up to 16
// (M = 128 takes N = 16 .. 256 in steps of 16), so a partly filled last slot
// tile of an expert costs MMA time in proportion to its slots.
__device__ __forceinline__ uint32_t idesc_f16_f32_n(int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

// A from TMEM (row m in lane m, K pairs per 32-bit column), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

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

// ------------------------------------------------------- dequantisation
// Within every aligned block of 8 k-columns both MMA operands are stored in
// the order (0,4,1,5,2,6,3,7): it is the order in which the 4-bit codes of a
// u32 unpack two at a time, and the contraction over k does not depend on it.
// The activations are written in that order by gather_rows_kernel and by the
// gate/up epilogue (kperm8).
__device__ __forceinline__ int kperm8(int col) {
  const int j = col & 7;
  return (col & ~7) | (j < 4 ? 2 * j : 2 * (j - 4) + 1);
}

// 8 consecutive 8-bit codes (two u32) -> 8 fp16 w = q * s + b, k-permuted.
__device__ __forceinline__ uint4 dequant8_u8(uint32_t w0, uint32_t w1, float s, float b) {
  float f[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[k] = fmaf(__uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7540 + k)) - 8388608.0f, s, b);
    f[k + 4] = fmaf(__uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7540 + k)) - 8388608.0f, s, b);
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __floats2half2_rn(f[i], f[i + 4]);
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Pipeline shape per instance.  A packed-code stage holds KP k-blocks so each
// weight row contributes one full 128-byte line per load (KP = 4 at 4 bits,
// 2 at 8 bits); it lands with SWIZZLE_128B so the dequant warps' reads are
// bank-conflict free.  Decode-size token tiles get a third fp16 A stage so
// dequantisation runs ahead of the MMA round trip; TMEM holds two
// accumulators whenever they fit, so the epilogue of one tile overlaps the
// MMAs of the next.
template <int BITS, int NPROJ, int BN> struct TcShape {
  static constexpr int KP = 512 / BITS / 32;                    // k-blocks per packed stage
  // One pipeline step (an A stage and its activation stage) spans KA k-blocks
  // so that each barrier wait and commit covers 16 MMAs: every wait costs a
  // few hundred cycles even when its phase has already completed.
  static constexpr int KA = NPROJ == 2 ? 2 : (KP < 4 ? KP : 4);
  static constexpr int kACols = NPROJ * KA * 32;                // TMEM columns of one A stage
  // MMA issuers: gate/up has one per projection.  The down projection has
  // two at small BN, where one thread's issue latency bounds the rate, each
  // taking alternate K steps into its own partial sum; at BN = 128 an MMA
  // takes longer than its issue, so one issuer keeps up and its single
  // accumulator leaves TMEM room for two accumulator sets.
  static constexpr int kIss = (NPROJ == 1 && BN >= 128) ? 1 : 2;
  // TMEM (512 columns): ACC accumulator sets of kIss*BN columns (gate and up,
  // or the down projection's partial sums), then kA A stages (128 rows x 64 k
  // per k-block, two fp16 per column).
  static constexpr int kAccCols = kIss * BN;
  static constexpr int kAcc = 2 * kAccCols + 2 * kACols <= 512 ? 2 : 1;
  static constexpr int kAFit = (512 - kAcc * kAccCols) / kACols;
  static constexpr int kA = kAFit > 4 ? 4 : kAFit;              // TMEM A stages
  static constexpr int kACol0 = kAcc * kAccCols;                // first A column
  static constexpr int kCols = 512;
  // activation stages (KA tiles each): refilled only after the MMAs that read
  // them, so the ring covers an L2 round trip
  static constexpr uint32_t kBTile = BN * 64 * 2;               // one k-block of activations
  static constexpr uint32_t kBBytes = KA * kBTile;
  static constexpr int kBFit = int(65536u / kBBytes);
  static constexpr int kB = kBFit < 2 ? 2 : (kBFit > 8 ? 8 : kBFit);
  static constexpr uint32_t kPBytes = 128 * 128;                // one projection's packed stage
  // With a single accumulator (gate/up at BN = 128) the epilogue first copies
  // it into a shared-memory staging row per thread (bf16 gate/up pairs; rows
  // padded by 16 bytes so 16-byte accesses spread over the banks), releases
  // it, and evaluates the activation from there while the next tile's MMAs
  // run.  A tile's activation math takes about as long as its main loop.
  static constexpr bool kStage = NPROJ == 2 && kAcc == 1;
  static constexpr uint32_t kEStride = BN * 4 + 16;
  static constexpr uint32_t kEBytes = kStage ? 128u * kEStride : 0u;
  // each packed stage carries its rows' scales and biases: [NPROJ][scale,
  // bias][128 rows][KP bf16], copied by the producer warp's lanes
  static constexpr uint32_t kSBRow = KP * 2;
  static constexpr uint32_t kSBStage = NPROJ * 2 * 128 * kSBRow;
  // packed stages fill the rest of shared memory (at most 8); staged shapes
  // budget up to the 227 KB limit (static shared memory below 2 KB)
  static constexpr uint32_t kBudget = (kStage ? 224u : 200u) * 1024u;
  static constexpr int kPFit = int((kBudget - kB * kBBytes - kEBytes) / (NPROJ * kPBytes + kSBStage));
  static constexpr int kP = kPFit > 8 ? 8 : kPFit;
  static constexpr size_t kSmem =
      1024 + size_t(kB) * kBBytes + size_t(kP) * (NPROJ * kPBytes + kSBStage) + kEBytes;
  // Staged shapes add four helper warps that evaluate half of each staging
  // row (see kHelpWarp0).
  static constexpr int kThreads = (kStage ? 28 : 24) * 32;
};

constexpr int kMaxTilesPerCta = 64;
// warp 0: TMA of packed codes; warp 1: TMEM + MMA issuer 0; warps 2-17:
// dequant; warps 18-21: epilogue; warp 22: TMA of activation tiles; warp 23:
// MMA issuer 1.  The two TMA streams live in separate warps so the weight
// prefetch never waits behind an activation slot that only the MMA frees.
// Small-N tcgen05.mma issue is latency-bound per issuing thread, and a second
// issuer (in another warp, into its own accumulator) doubles the rate:
// issuer p takes projection p (gate/up), or alternate K steps of the down
// projection into partial sums the epilogue adds.  Dequantisation is the
// busiest role (~12 instructions per 8 codes), so it gets 16 warps.
constexpr int kEpiWarp0 = 2 + kDqWarps;
constexpr int kBWarp = kEpiWarp0 + 4;
constexpr int kMma1Warp = kBWarp + 1;
// Warps 24-27 (staged shapes only): epilogue helpers.  With the accumulator
// staged, the activation math of a tile is the kernel's longest chain (one
// warp per SM sub-partition evaluating 128 columns per row while four
// dequant warps share its issue slots); the helper of lane quarter q takes
// the upper half of the staging row of every thread of that quarter.
constexpr int kHelpWarp0 = kMma1Warp + 1;
constexpr int kHelpCol0 = 64;  // helpers evaluate slots [64, BN) of a 128-slot tile

// Scale/bias of k-block j (0 <= j < KP) from KP bf16 values held as packed u32s.
template <int KP>
__device__ __forceinline__ uint16_t pick_bf16(const uint32_t (&v)[KP / 2], int j) {
  uint32_t w = v[0];
#pragma unroll
  for (int i = 1; i < KP / 2; ++i)
    if (j / 2 == i) w = v[i];
  return static_cast<uint16_t>(j & 1 ? w >> 16 : w & 0xffffu);
}

template <int KP>
__device__ __forceinline__ void load_group_params_smem(const unsigned char* p, uint32_t (&v)[KP / 2]) {
  if constexpr (KP == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    v[0] = t.x;
    v[1] = t.y;
  } else {
    v[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

}  // namespace

// Persistent grouped GEMM: each CTA walks a strided list of (expert, 128-row
// block, BN-slot block) tiles with one continuous pipeline across them.
template <int BITS, int NPROJ, int BN>
__global__ void __launch_bounds__(TcShape<BITS, NPROJ, BN>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB, TcGemmArgs a) {
  using S = TcShape<BITS, NPROJ, BN>;
  constexpr int SA = S::kA, SB = S::kB, SP = S::kP, KP = S::KP, KA = S::KA, ACC = S::kAcc;
  constexpr uint32_t kBTile = S::kBTile, kBBytes = S::kBBytes, kPBytes = S::kPBytes;
  static_assert(S::kSmem + 2048 <= 227 * 1024, "shared memory budget");
  static_assert(SA >= 2 && SP >= 2 && KP % KA == 0, "pipeline shape");
  static_assert(S::kACol0 + SA * S::kACols <= S::kCols, "TMEM budget");
  // With rings of equal depth the A and B stages of a step free together:
  // one commit (and one barrier) per step serves both producers.
  constexpr bool kJointEmpty = SA == SB;

  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar_pfull[SP], bar_pempty[SP], bar_afull[SA], bar_aempty[SA], bar_bfull[SB],
      bar_bempty[SB], bar_accfull[ACC], bar_accempty[ACC], bar_drain[S::kIss], bar_stgfull, bar_stgempty;
  __shared__ uint32_t s_tmem;
  __shared__ int4 s_tiles[kMaxTilesPerCta];  // local expert, first weight row, first slot, valid slots
  __shared__ int s_ntiles;
  __shared__ volatile int s_abort;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int groups = a.kdim / BK, ktiles = a.kdim / BK;
  const int nsteps = ktiles / KA;  // pipeline steps per tile

  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  unsigned char* sB = base;                       // [SB][KA][BN*128]
  unsigned char* sP = sB + SB * kBBytes;          // [SP][NPROJ][16 KB]
  unsigned char* sE = sP + SP * NPROJ * kPBytes;  // [128 rows][kEStride] epilogue staging (kStage)
  unsigned char* sSB = sE + S::kEBytes;             // [SP] packed stages' scales and biases

  // ---- barriers and TMEM first: they do not depend on the previous kernel
  if (warp == 0 && lane == 0) {
    // consumer-side barriers count warps: each warp fences, syncs, and arrives once
    // packed stage full: the TMA's expect_tx arrival plus one cp.async arrival per producer lane
    for (int i = 0; i < SP; ++i) { mbar_init(&bar_pfull[i], 33); mbar_init(&bar_pempty[i], kDqWarps); }
    for (int i = 0; i < SA; ++i) { mbar_init(&bar_afull[i], kDqWarps); mbar_init(&bar_aempty[i], S::kIss); }
    for (int i = 0; i < SB; ++i) { mbar_init(&bar_bfull[i], 1); mbar_init(&bar_bempty[i], S::kIss); }
    for (int i = 0; i < ACC; ++i) { mbar_init(&bar_accfull[i], S::kIss); mbar_init(&bar_accempty[i], 4); }
    for (int i = 0; i < S::kIss; ++i) mbar_init(&bar_drain[i], 1);
    mbar_init(&bar_stgfull, 4);   // staged: the four primary epilogue warps filled the staging rows
    mbar_init(&bar_stgempty, 8);  // staged: all eight epilogue warps finished reading them
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(S::kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_wait();  // the tile list comes from the dispatch kernel's active list / offsets
  pdl_launch_dependents();

  // ---- this CTA's tiles: global tile t (m-block fastest within an expert's
  // slot block) belongs to CTA t % gridDim.x.  The packed-code ring is free
  // until the producer starts: it is the list's scratch.
  {
    const int n = list_tiles(a.active, a.active_count, a.offsets, a.expert_begin, a.m_tiles, BM, BN, true, s_tiles,
                             kMaxTilesPerCta, reinterpret_cast<int*>(sP), a.err, a.slot_cap, a.cnt_lo,
                             a.cnt_hi);
    if (tid == 0) {
      s_ntiles = n;
      s_abort = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  const int ntiles = s_ntiles;
  if (ntiles == 0) {  // no tile for this CTA: release TMEM and leave
    if (warp == 1)
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::kCols) : "memory");
    return;
  }

  if (warp == 0 || warp == kBWarp) {
    // ================================================= TMA producers
    // warp 0: packed codes (lane 0's TMA) and their scales / biases (every
    // lane, cp.async); warp kBWarp: activation tiles (lane 0)
    const bool packed = warp == 0;
    if (packed || lane == 0) {
      int last_p[SP], last_b[SB];     // parity of the last load issued per stage (-1: none)
#pragma unroll
      for (int i = 0; i < SP; ++i) last_p[i] = -1;
#pragma unroll
      for (int i = 0; i < SB; ++i) last_b[i] = -1;
      bool ok = true;
      int pi = 0, bi = 0;
      for (int ti = 0; ti < ntiles && ok; ++ti) {
        const int4 tl = s_tiles[ti];
        const int row_base = tl.x * a.rows + tl.y;
        if (packed) {
          for (int kt = 0; kt < ktiles; kt += KP) {  // packed stage: k-blocks [kt, kt + KP)
            const int ps = pi % SP, pph = (pi / SP) & 1;
            if (!(ok = __all_sync(0xffffffffu, wait_or_abort(&bar_pempty[ps], pph ^ 1, &s_abort, a.err)))) break;
            if (lane == 0) {
              mbar_arrive_expect_tx(&bar_pfull[ps], NPROJ * kPBytes);
              tma_load_2d(sP + (ps * NPROJ + 0) * kPBytes, &tmA0, (kt / KP) * 32, row_base, &bar_pfull[ps]);
              if constexpr (NPROJ == 2)
                tma_load_2d(sP + (ps * NPROJ + 1) * kPBytes, &tmA1, (kt / KP) * 32, row_base, &bar_pfull[ps]);
            }
            // the stage's scales and biases: KP bf16 per row and array, rows
            // lane, lane + 32, lane + 64, lane + 96
            const uint32_t sb0 = smem_u32(sSB + ps * S::kSBStage);
#pragma unroll
            for (int pa = 0; pa < 2 * NPROJ; ++pa) {  // array pa: scales (even) / biases (odd) of proj pa / 2
              const uint16_t* src = ((pa & 1) ? a.b[pa >> 1] : a.s[pa >> 1]) + kt;
#pragma unroll
              for (int rr = 0; rr < 4; ++rr) {
                const int r = lane + 32 * rr;
                const uint32_t dst = sb0 + (pa * 128 + r) * S::kSBRow;
                const uint16_t* g = src + static_cast<size_t>(row_base + r) * groups;
                if constexpr (S::kSBRow == 8) cp_async_8(dst, g);
                else cp_async_4(dst, g);
              }
            }
            cp_async_arrive_noinc(&bar_pfull[ps]);
            last_p[ps] = pph;
            ++pi;
          }
        } else {
          for (int st = 0; st < nsteps; ++st) {  // activation stage: k-blocks [st*KA, st*KA + KA)
            const int bs = bi % SB, bph = (bi / SB) & 1;
            if (!(ok = wait_or_abort(kJointEmpty ? &bar_aempty[bs] : &bar_bempty[bs], bph ^ 1, &s_abort, a.err)))
              break;
            mbar_arrive_expect_tx(&bar_bfull[bs], kBBytes);
#pragma unroll
            for (int kk = 0; kk < KA; ++kk)
              tma_load_2d(sB + bs * kBBytes + kk * kBTile, &tmB, (st * KA + kk) * BK, tl.z, &bar_bfull[bs]);
            last_b[bs] = bph;
            ++bi;
          }
        }
      }
      if (!ok) {  // give the copies already issued a bounded chance to land before exit
        volatile int never = 0;
#pragma unroll
        for (int i = 0; i < SP; ++i)
          if (last_p[i] >= 0) wait_or_abort(&bar_pfull[i], last_p[i], &never, nullptr);
#pragma unroll
        for (int i = 0; i < SB; ++i)
          if (last_b[i] >= 0) wait_or_abort(&bar_bfull[i], last_b[i], &never, nullptr);
      }
    }
  } else if (warp == 1 || warp == kMma1Warp) {
    // ================================================= MMA issuers
    // (a single-issuer shape leaves the second issuer warp without work; it
    // goes straight to the teardown barrier).  The whole warp walks the
    // pipeline and waits on the barriers, one elected lane issues the MMAs
    // and commits: the loop stays warp-uniform, so its descriptor arithmetic
    // is not a single diverged lane's (the issuer shares its sub-partition's
    // issue slots with six busy warps).
    if (warp == 1 || S::kIss == 2) {
      const int iss = warp == 1 ? 0 : 1;
      const bool leader = elect_one();
      bool ok = true;
      int ai = 0;  // pipeline steps issued (A and B stages advance together)
      for (int ti = 0; ti < ntiles && ok; ++ti) {
        const int ab = ti % ACC, accph = (ti / ACC) & 1;
        if (!(ok = __all_sync(0xffffffffu, wait_or_abort(&bar_accempty[ab], accph ^ 1, &s_abort, a.err)))) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * S::kAccCols + iss * BN;  // this issuer's accumulator
        // MMA width: the tile's valid slots rounded up to 16 (columns past
        // them are never read by the epilogue)
        const int n_mma = min(BN, (s_tiles[ti].w + 15) & ~15);
        const uint32_t kIdesc = idesc_f16_f32_n(n_mma < 16 ? 16 : n_mma);
        for (int st = 0; st < nsteps; ++st, ++ai) {
          const int as = ai % SA, aph = (ai / SA) & 1;
          const int bs = ai % SB, bph = (ai / SB) & 1;
          ok = __all_sync(0xffffffffu, wait_or_abort(&bar_afull[as], aph, &s_abort, a.err) &&
                                           wait_or_abort(&bar_bfull[bs], bph, &s_abort, a.err));
          if (!ok) break;
          tc_fence_after();
          const uint64_t b_desc0 = sw128_kmajor_desc(smem_u32(sB + bs * kBBytes));
          const uint32_t a_stage = tmem + S::kACol0 + as * S::kACols;
          if (leader) {
            if constexpr (NPROJ == 2) {  // projection iss, all K steps
#pragma unroll
              for (int kk = 0; kk < KA; ++kk)
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)  // K = 16 per MMA: 8 TMEM columns of A, 32 bytes of B
                  umma_f16_ts(d, a_stage + (iss * KA + kk) * 32 + k * 8, b_desc0 + ((kk * kBTile + k * 32) >> 4),
                              kIdesc, (st | kk | k) != 0);
            } else {  // K steps iss, iss + kIss, ... into this issuer's partial sum
#pragma unroll
              for (int kk = 0; kk < KA; ++kk)
#pragma unroll
                for (int k = iss; k < BK / 16; k += S::kIss)
                  umma_f16_ts(d, a_stage + kk * 32 + k * 8, b_desc0 + ((kk * kBTile + k * 32) >> 4), kIdesc,
                              (st | kk | (k - iss)) != 0);
            }
            umma_commit(&bar_aempty[as]);
            if constexpr (!kJointEmpty) umma_commit(&bar_bempty[bs]);
          }
          __syncwarp();
        }
        if (ok && leader) umma_commit(&bar_accfull[ab]);
        __syncwarp();
      }
      // all MMAs issued by the leader have completed once this fires
      if (leader) umma_commit(&bar_drain[iss]);
      __syncwarp();
      volatile int never = 0;
      wait_or_abort(&bar_drain[iss], 0, &never, nullptr);
    }
  } else if (warp < kEpiWarp0) {
    // ================================================= dequantisation -> TMEM
    // A warp may only touch its TMEM lane quarter q = warp % 4, so lane l of
    // warp w dequantises row 32 q + l.  The four warps of a quarter split the
    // row's NPROJ x 64 codes of a k-block into slices j = (w - 2) / 4 of
    // WPT packed words, stored as CPT TMEM columns (two fp16 per column).
    constexpr int W = BK * BITS / 32;           // packed words per row per k-block (8 or 16)
    constexpr int WPT = NPROJ * W / 4;          // words per slice
    constexpr int CPT = 16 * NPROJ / 2;         // TMEM columns per slice (16 or 8)
    const int q = warp & 3, j = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int proj = NPROJ == 2 ? j >> 1 : 0;
    const int slice = NPROJ == 2 ? j & 1 : j;   // slice within the projection's row
    const uint32_t lane_base =
        tmem + (static_cast<uint32_t>(q * 32) << 16) + S::kACol0 + proj * KA * 32 + slice * CPT;
    bool ok = true;
    int pi = 0, ai = 0;
    // this packed stage's scales / biases of the thread's row, from the
    // stage's copy in shared memory
    uint32_t sv[KP / 2], bv[KP / 2];
    for (int ti = 0; ti < ntiles && ok; ++ti) {
      int ps = 0;
      for (int st = 0; st < nsteps; ++st, ++ai) {
        const int kt0 = st * KA;
        if (kt0 % KP == 0) {
          ps = pi % SP;
          const int pph = (pi / SP) & 1;
          ok = __all_sync(0xffffffffu, wait_or_abort(&bar_pfull[ps], pph, &s_abort, a.err));
          if (!ok) break;
          const unsigned char* sbr = sSB + ps * S::kSBStage + (2 * proj * 128 + row) * S::kSBRow;
          load_group_params_smem<KP>(sbr, sv);
          load_group_params_smem<KP>(sbr + 128 * S::kSBRow, bv);
        }
        const int as = ai % SA, aph = (ai / SA) & 1;
        // the step's fp16 values are computed into registers first, then the
        // A stage is awaited and stored: the arithmetic overlaps the wait for
        // the MMAs that still read the stage
        const unsigned char* prow = sP + (ps * NPROJ + proj) * kPBytes + row * 128;
        uint32_t outs[KA][CPT];
#pragma unroll
        for (int kk = 0; kk < KA; ++kk) {
          uint32_t (&out)[CPT] = outs[kk];
          const int kt = kt0 + kk;
          const uint16_t sb = pick_bf16<KP>(sv, kt % KP), bb = pick_bf16<KP>(bv, kt % KP);
          // this thread's words start at word (kt % KP) * W + slice * WPT of the
          // row's 128-byte packed line, whose 16-byte chunks sit at (c ^ (row & 7))
          const int w0 = (kt % KP) * W + slice * WPT;
          uint32_t wd[WPT];
#pragma unroll
          for (int i = 0; i < WPT; i += (WPT >= 4 ? 4 : 2)) {
            const int wi = w0 + i;
            const unsigned char* src = prow + (((wi >> 2) ^ (row & 7)) << 4) + (wi & 3) * 4;
            if constexpr (WPT >= 4) {
              const uint4 v = *reinterpret_cast<const uint4*>(src);
              wd[i] = v.x; wd[i + 1] = v.y; wd[i + 2] = v.z; wd[i + 3] = v.w;
            } else {
              const uint2 v = *reinterpret_cast<const uint2*>(src);
              wd[i] = v.x; wd[i + 1] = v.y;
            }
          }
          if constexpr (BITS == 4) {  // one word (8 codes) -> four columns
            const float sf = bf16_bits_to_f32(sb);
            const __half2 b2 = __float2half2_rn(bf16_bits_to_f32(bb));
            // warp-uniform choice of the dequant form (no divergent branch)
            if (__all_sync(0xffffffffu, fabsf(sf) < 0.0624f)) {
              const __half2 s20 = __float2half2_rn(sf * 1048576.0f);
#pragma unroll
              for (int i = 0; i < WPT; ++i) {
                const uint4 v = dequant8_u4_sub20(wd[i], s20, b2);
                out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
              }
            } else if (fabsf(sf) < 0.2498f) {
              const __half2 s18 = __float2half2_rn(sf * 262144.0f);
#pragma unroll
              for (int i = 0; i < WPT; ++i) {
                const uint4 v = dequant8_u4_sub(wd[i], s18, b2);
                out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
              }
            } else {
              const __half2 s2 = __float2half2_rn(sf);
#pragma unroll
              for (int i = 0; i < WPT; ++i) {
                const uint4 v = dequant8_u4(wd[i], s2, b2);
                out[4 * i] = v.x; out[4 * i + 1] = v.y; out[4 * i + 2] = v.z; out[4 * i + 3] = v.w;
              }
            }
          } else {  // two words (8 codes) -> four columns
            const float sf = bf16_bits_to_f32(sb), bf = bf16_bits_to_f32(bb);
#pragma unroll
            for (int i = 0; i < WPT; i += 2) {
              const uint4 v = dequant8_u8(wd[i], wd[i + 1], sf, bf);
              out[2 * i] = v.x; out[2 * i + 1] = v.y; out[2 * i + 2] = v.z; out[2 * i + 3] = v.w;
            }
          }
        }
        ok = __all_sync(0xffffffffu, wait_or_abort(&bar_aempty[as], aph ^ 1, &s_abort, a.err));
        if (!ok) break;
        tc_fence_after();  // the MMAs that read this A stage have completed
#pragma unroll
        for (int kk = 0; kk < KA; ++kk) {
          const uint32_t taddr = lane_base + as * S::kACols + kk * 32;
          if constexpr (CPT == 16) tmem_st16(taddr, outs[kk]);
          else tmem_st8(taddr, outs[kk]);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_afull[as]);
        if ((kt0 + KA) % KP == 0) {  // this step finished its packed stage
          if (lane == 0) mbar_arrive(&bar_pempty[ps]);
          ++pi;
        }
      }
    }
  } else if (warp < kBWarp || warp >= kHelpWarp0) {
    // ================================================= epilogue (TMEM -> global)
    // TMEM lane quarter of this warp (warps 18..21 -> 2, 3, 0, 1); a helper
    // (warps 24..27, staged shapes only) reads the staging rows of quarter q
    const int q = warp & 3;
    const bool helper = warp >= kHelpWarp0;
    for (int ti = 0; ti < ntiles; ++ti) {
      const int ab = ti % ACC, accph = (ti / ACC) & 1;
      if (!helper) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&bar_accfull[ab], accph, &s_abort, a.err))) break;
        tc_fence_after();
      }
      const int4 tl = s_tiles[ti];
      const int r = tl.y + q * 32 + lane;  // output row of this thread
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16) + ab * S::kAccCols;
      // One 16-column chunk from fp32 bit patterns: g / u are gate / up, or
      // the two partial sums of down.
      auto emit_chunk = [&](int c0, const uint32_t (&g)[16], const uint32_t (&u)[16]) {
        // h feeds the down GEMM as its k dimension: store it k-permuted like x
        const int col = NPROJ == 2 ? kperm8(r) : r;
        uint16_t* orow = a.out + static_cast<size_t>(tl.z + c0) * a.out_stride + col;
        // h = act(bf16(g), bf16(u)) (a bf16 value, stored as fp16), or the
        // down projection's two partial sums added and rounded to bf16; bad
        // flags an h outside fp16 range
        auto value = [&](int jj, bool& bad) -> uint16_t {
          if constexpr (NPROJ == 2) {
            // staged values are bf16 already (rounded on the way into the staging row)
            const float gg = S::kStage ? __uint_as_float(g[jj]) : round_bf16(__uint_as_float(g[jj]));
            const float uu = S::kStage ? __uint_as_float(u[jj]) : round_bf16(__uint_as_float(u[jj]));
            const float v = a.act == 0 ? act_swiglu_mlx(gg, uu) : act_geglu_mlx(gg, uu);
            bad = bad || !(fabsf(v) < 65504.0f);
            return __half_as_ushort(__float2half_rn(v));
          } else if constexpr (S::kIss == 1) {  // one accumulator: the whole sum
            return f32_to_bf16_bits(__uint_as_float(g[jj]));
          } else {
            return f32_to_bf16_bits(__uint_as_float(g[jj]) + __uint_as_float(u[jj]));
          }
        };
        bool bad = false;
        if (c0 + 16 <= tl.w) {
          // a full chunk (warp-uniform): 16 independent chains that interleave,
          // where a per-column exit would run them one after another
          uint16_t bits[16];
          if (NPROJ == 2 && a.act == 0) {
#pragma unroll
            for (int j0 = 0; j0 < 16; j0 += 8) {  // two batches of 8 chains
              float gv[8], uv[8], hv[8];
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                gv[jj] = S::kStage ? __uint_as_float(g[j0 + jj]) : round_bf16(__uint_as_float(g[j0 + jj]));
                uv[jj] = S::kStage ? __uint_as_float(u[j0 + jj]) : round_bf16(__uint_as_float(u[j0 + jj]));
              }
              act_swiglu_mlx_n<8>(gv, uv, hv);
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                bad = bad || !(fabsf(hv[jj]) < 65504.0f);
                bits[j0 + jj] = __half_as_ushort(__float2half_rn(hv[jj]));
              }
            }
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) bits[jj] = value(jj, bad);
          }
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) orow[static_cast<size_t>(jj) * a.out_stride] = bits[jj];
        } else {
          // the tile's last valid slots only: columns past them hold other
          // experts' activations (or none) and are never evaluated.  Fully
          // unrolled, so g and u stay in registers (a runtime index would
          // put them in local memory).
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            if (c0 + jj < tl.w) orow[static_cast<size_t>(jj) * a.out_stride] = value(jj, bad);
        }
        if (bad) record_error(a.err, kDevFp16Range);
      };
      if constexpr (S::kStage) {
        // accumulator -> this thread's staging row as (bf16 gate, bf16 up)
        // pairs, the rounding the activation applies first; then release the
        // accumulator and evaluate from the staging row
        unsigned char* erow = sE + static_cast<uint32_t>(q * 32 + lane) * S::kEStride;
        if (!helper) {
          // the staging rows are free once all eight warps have evaluated the
          // previous tile from them
          if (ti > 0 && !__all_sync(0xffffffffu, wait_or_abort(&bar_stgempty, (ti - 1) & 1, &s_abort, a.err)))
            break;
          for (int c0 = 0; c0 < BN; c0 += 16) {
            if (c0 >= tl.w) break;  // uniform across the warp
            uint32_t g[16], u[16];
            tmem_ld16(lane_addr + c0, g);
            tmem_ld16(lane_addr + BN + c0, u);
            tmem_ld_wait();
            uint32_t pk[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              pk[jj] = uint32_t(f32_to_bf16_bits(__uint_as_float(g[jj]))) |
                       (uint32_t(f32_to_bf16_bits(__uint_as_float(u[jj]))) << 16);
            uint4* dst = reinterpret_cast<uint4*>(erow + c0 * 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&bar_accempty[ab]);
            mbar_arrive(&bar_stgfull);
          }
        } else if (!__all_sync(0xffffffffu, wait_or_abort(&bar_stgfull, ti & 1, &s_abort, a.err))) {
          break;
        }
        // primary warps slots [0, kHelpCol0), helpers [kHelpCol0, BN)
        static_assert(!S::kStage || BN == 2 * kHelpCol0, "staged shapes split a 128-slot row in halves");
        const int c_end = helper ? BN : kHelpCol0;
        for (int c0 = helper ? kHelpCol0 : 0; c0 < c_end; c0 += 16) {
          if (c0 >= tl.w) break;
          const uint4* src = reinterpret_cast<const uint4*>(erow + c0 * 4);
          uint32_t g[16], u[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = src[i];
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              g[4 * i + k] = w[k] << 16;
              u[4 * i + k] = w[k] & 0xffff0000u;
            }
          }
          emit_chunk(c0, g, u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_stgempty);
      } else {
        for (int c0 = 0; c0 < BN; c0 += 16) {
          if (c0 >= tl.w) break;  // uniform across the warp
          uint32_t g[16], u[16];
          tmem_ld16(lane_addr + c0, g);
          if constexpr (S::kIss == 2) tmem_ld16(lane_addr + BN + c0, u);
          tmem_ld_wait();
          emit_chunk(c0, g, u);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_accempty[ab]);
      }
    }
  }

  // ---- teardown: every role is done with TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::kCols) : "memory");
  }
}

// ------------------------------------------------------------- host side
size_t tc_smem_bytes(int bits, int nproj, int bn, int kdim) {
  (void)kdim;
#define SENMOE_TC_SMEM(B, P, N) \
  if (bits == B && nproj == P && bn == N) return TcShape<B, P, N>::kSmem;
#define SENMOE_TC_SMEM_BN(B, P) \
  SENMOE_TC_SMEM(B, P, 16) SENMOE_TC_SMEM(B, P, 32) SENMOE_TC_SMEM(B, P, 64) SENMOE_TC_SMEM(B, P, 128)
  SENMOE_TC_SMEM_BN(4, 1) SENMOE_TC_SMEM_BN(4, 2) SENMOE_TC_SMEM_BN(8, 1) SENMOE_TC_SMEM_BN(8, 2)
#undef SENMOE_TC_SMEM_BN
#undef SENMOE_TC_SMEM
  return ~size_t(0);
}

bool tc_supported(int rows, int kdim, int bits, int nproj, int bn) {
  const int kp = 512 / bits / 32;  // k-blocks per packed stage
  return rows % BM == 0 && kdim % (BK * kp) == 0 && (bits == 4 || bits == 8) &&
         tc_smem_bytes(bits, nproj, bn, kdim) + 2048 <= 227 * 1024;
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

template <int BITS, int NPROJ, int BN>
static cudaError_t launch_tc_t(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                               const TcGemmArgs& a, int tiles_upper, cudaStream_t st) {
  const size_t smem = TcShape<BITS, NPROJ, BN>::kSmem;
  auto kern = tc_gemm_kernel<BITS, NPROJ, BN>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  // one persistent CTA per SM, enough CTAs that none owns more than kMaxTilesPerCta tiles
  int grid = tiles_upper < sm_count() ? tiles_upper : sm_count();
  if ((tiles_upper + grid - 1) / grid > kMaxTilesPerCta) grid = (tiles_upper + kMaxTilesPerCta - 1) / kMaxTilesPerCta;
  return launch_pdl(kern, dim3(grid), dim3(TcShape<BITS, NPROJ, BN>::kThreads), smem, st, tA0, tA1, tB, a);
}

cudaError_t launch_tc_gemm(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                           const TcGemmArgs& a, int bits, int nproj, int bn, int tiles_upper, cudaStream_t st) {
  if (tiles_upper <= 0) return cudaSuccess;
#define SENMOE_TC_CASE(B, P, N) \
  if (bits == B && nproj == P && bn == N) return launch_tc_t<B, P, N>(tA0, tA1, tB, a, tiles_upper, st);
#define SENMOE_TC_BN(B, P) \
  SENMOE_TC_CASE(B, P, 16) SENMOE_TC_CASE(B, P, 32) SENMOE_TC_CASE(B, P, 64) SENMOE_TC_CASE(B, P, 128)
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

// Slot-ordered fp16 copy of the token rows (bf16 -> fp16 is exact in range),
// k-permuted within each block of 8 columns like the dequantised weights
// (kperm8), or in one of the warp-MMA kernel's orders (kperm256; kperm_g4,
// odd columns divided by 16).  Each CTA copies kGatherSlots slots.
constexpr int kGatherSlots = 4;
constexpr int kGatherCtasPerSm = 8;

// Row `token` of the gather's source: x, or its owner rank's exchange buffer.
__device__ __forceinline__ const uint16_t* gather_src_row(const uint16_t* x, int token, int hidden,
                                                          const PeerRows& pr) {
  if (pr.world == 0) return x + static_cast<size_t>(token) * hidden;
  int q = 0;
#pragma unroll
  for (int i = 1; i < kPeerRowsMax; ++i) q += (i < pr.world && token >= pr.begin[i]) ? 1 : 0;
  return pr.base[q] + static_cast<size_t>(token - pr.begin[q]) * hidden;
}

// kFilter: only the slots of experts with cnt_lo <= slots < cnt_hi (a
// separate instance, so the unfiltered gather carries no per-slot lookup)
template <bool kFilter>
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ perm, int k_div,
                                                          uint16_t* __restrict__ out, int num_slots, int hidden,
                                                          int* err, const int32_t* __restrict__ offsets, int eb,
                                                          int ee, int order, float* __restrict__ group_sums,
                                                          int32_t* __restrict__ one_group, const PeerRows pr,
                                                          int slot_cap, const int32_t* __restrict__ ids, int cnt_lo,
                                                          int cnt_hi) {
  pdl_wait();
  pdl_launch_dependents();
  if (one_group && blockIdx.x == 0 && threadIdx.x == 0) {
    // the consuming GEMMs' tile list: one group (local index 0) of num_slots slots
    one_group[0] = 0;          // offsets[0]
    one_group[1] = num_slots;  // offsets[1]
    one_group[2] = 0;          // active[0]
    one_group[3] = 1;          // active count
  }
  int lo_slot = 0, hi_slot = num_slots;
  if (offsets) {  // expert parallelism: only this rank's slots
    lo_slot = offsets[eb];
    hi_slot = offsets[ee];
  }
  // rows are local (slot - lo_slot) and the buffer holds slot_cap of them
  if (slot_cap > 0 && hi_slot - lo_slot > slot_cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_error(err, kDevSlotOverflow);
    hi_slot = lo_slot + slot_cap;
  }
  // slot s is row s - lo_slot of out (and of group_sums).  The grid strides
  // over groups of kGatherSlots slots (at most kGatherCtasPerSm CTAs per SM),
  // so a CTA's next group starts while its earlier stores drain.
  bool ok = true;
  for (int s0 = blockIdx.x * kGatherSlots; s0 < num_slots; s0 += gridDim.x * kGatherSlots) {
    const uint16_t* src[kGatherSlots];
    bool live[kGatherSlots];
#pragma unroll
    for (int j = 0; j < kGatherSlots; ++j) {
      const int s = s0 + j;
      live[j] = s < num_slots && s >= lo_slot && s < hi_slot;
      if (kFilter && live[j]) {  // only the slots of experts with cnt_lo <= slots < cnt_hi
        const int e = ids[perm[s]];
        const int c = offsets[e + 1] - offsets[e];
        live[j] = c >= cnt_lo && c < cnt_hi;
      }
      src[j] = live[j] ? gather_src_row(x, perm[s] / k_div, hidden, pr) : x;
    }
    if (order == kOrderMmaG4) {
      // kperm_g4, one thread per (slot, 64-column group): output position
      // 16 s + kappa (kappa = 8 a2 + 2 t + h) holds column
      // 8 (t + 4 (s / 2)) + (s & 1) + 2 a2 + 4 h, divided by 16 for odd s
      const int groups = hidden / 64;
      for (int it = threadIdx.x; it < kGatherSlots * groups; it += blockDim.x) {
        const int j = it / groups, G = it - j * groups, s = s0 + j;
        if (!live[j]) continue;
        const uint4* in = reinterpret_cast<const uint4*>(gather_src_row(x, perm[s] / k_div, hidden, pr) + 64 * G);
        uint32_t w[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 v = __ldcg(in + q);
          w[4 * q] = v.x; w[4 * q + 1] = v.y; w[4 * q + 2] = v.z; w[4 * q + 3] = v.w;
        }
        if (group_sums) {  // the group's sum of x (column order), in the MMA's 2^-24 units
          float sum = 0.f;
#pragma unroll
          for (int q = 0; q < 32; ++q) sum += bf16_lo(w[q]) + bf16_hi(w[q]);
          group_sums[static_cast<size_t>(s - lo_slot) * groups + G] = sum * 5.9604644775390625e-8f;  // 2^-24
        }
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(s - lo_slot) * hidden + 64 * G);
#pragma unroll
        for (int sg = 0; sg < 8; ++sg) {  // 16-byte segment: k-step sg / 2, kappa half sg % 2
          const int ks = sg >> 1, a2 = sg & 1;
          const float sc = (ks & 1) ? 0.0625f : 1.0f;
          uint32_t o[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int u0 = 8 * (t + 4 * (ks >> 1)) + (ks & 1) + 2 * a2, u1 = u0 + 4;
            const float f0 = (u0 & 1) ? bf16_hi(w[u0 >> 1]) : bf16_lo(w[u0 >> 1]);
            const float f1 = (u1 & 1) ? bf16_hi(w[u1 >> 1]) : bf16_lo(w[u1 >> 1]);
            ok &= fabsf(f0) < 65504.0f && fabsf(f1) < 65504.0f;
            const __half2 hv = __floats2half2_rn(f0 * sc, f1 * sc);
            o[t] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          dst[sg] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    } else if (order == kOrderMma) {
      // kperm256 (warp-MMA operand order): output segment sg (8 halves) of
      // stage st = sg / 32 holds, at half 2t + h, column
      // 256 st + 32 (2t + kh) + 8 b + p + 4h with sg % 32 = 16 kh + 4 b + p
      for (int sg = threadIdx.x; sg < hidden / 8; sg += blockDim.x) {
        const int st = sg >> 5, sp = sg & 31, kh = sp >> 4, b = (sp >> 2) & 3, p = sp & 3;
        const int c0 = st * 256 + 32 * kh + 8 * b + p;
        uint16_t v[kGatherSlots][8];
#pragma unroll
        for (int j = 0; j < kGatherSlots; ++j)
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            v[j][2 * t] = live[j] ? src[j][c0 + 64 * t] : 0;
            v[j][2 * t + 1] = live[j] ? src[j][c0 + 64 * t + 4] : 0;
          }
#pragma unroll
        for (int j = 0; j < kGatherSlots; ++j) {
          if (!live[j]) continue;
          uint32_t o[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float lo = bf16_bits_to_f32(v[j][2 * t]), hi = bf16_bits_to_f32(v[j][2 * t + 1]);
            ok &= fabsf(lo) < 65504.0f && fabsf(hi) < 65504.0f;
            const __half2 h = __floats2half2_rn(lo, hi);
            o[t] = *reinterpret_cast<const uint32_t*>(&h);
          }
          reinterpret_cast<uint4*>(out + static_cast<size_t>(s0 + j - lo_slot) * hidden)[sg] =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    } else {
      for (int i = threadIdx.x; i < hidden / 8; i += blockDim.x) {
        uint4 v[kGatherSlots];
#pragma unroll
        for (int j = 0; j < kGatherSlots; ++j)
          v[j] = live[j] ? reinterpret_cast<const uint4*>(src[j])[i] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int j = 0; j < kGatherSlots; ++j) {
          if (!live[j]) continue;
          const uint32_t in[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
          float f[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            f[2 * k] = bf16_lo(in[k]);
            f[2 * k + 1] = bf16_hi(in[k]);
          }
          uint32_t o[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // k-permuted pairs (k, k + 4), see kperm8
            ok &= fabsf(f[k]) < 65504.0f && fabsf(f[k + 4]) < 65504.0f;
            const __half2 h = __floats2half2_rn(f[k], f[k + 4]);
            o[k] = *reinterpret_cast<const uint32_t*>(&h);
          }
          reinterpret_cast<uint4*>(out + static_cast<size_t>(s0 + j - lo_slot) * hidden)[i] =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  if (!ok) record_error(err, kDevFp16Range);
}

cudaError_t launch_gather_rows(const uint16_t* x, const int32_t* perm, int k_div, uint16_t* x_sorted,
                               int num_slots, int hidden, int* err, cudaStream_t st,
                               const int32_t* offsets, int eb, int ee, int order, float* group_sums,
                               int32_t* one_group, const PeerRows* peer_rows, int slot_cap, const int32_t* ids,
                               int cnt_lo, int cnt_hi) {
  if (num_slots <= 0) return cudaSuccess;
  if (cnt_hi > 0 && (!ids || !offsets)) return cudaErrorInvalidValue;
  const int threads = hidden / 8 < 256 ? ((hidden / 8 + 31) / 32) * 32 : 256;
  int grid = (num_slots + kGatherSlots - 1) / kGatherSlots;
  if (grid > kGatherCtasPerSm * sm_count()) grid = kGatherCtasPerSm * sm_count();
  PeerRows pr{};
  if (peer_rows) pr = *peer_rows;
  auto kern = cnt_hi > 0 ? gather_rows_kernel<true> : gather_rows_kernel<false>;
  return launch_pdl(kern, dim3(grid), dim3(threads), 0, st, x, perm, k_div, x_sorted, num_slots, hidden, err,
                    offsets, eb, ee, order, order == kOrderMmaG4 ? group_sums : nullptr, one_group, pr, slot_cap, ids,
                    cnt_lo, cnt_hi);
}

}  // namespace senmoe
