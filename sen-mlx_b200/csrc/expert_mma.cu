// expert_mma.cu -- grouped affine-quantized expert GEMM for decode batches
// (a few tokens per expert), on warp-level tensor-core MMAs.
//
// Same contraction as the reference's SwitchGlu gather_qmm calls
// (src/engine/mlx_lm/models/deepseek_v2.rs:466-478, utils/moe.rs:33-77), with
// tokens grouped by expert (dispatch.cu).  With 1-16 tokens per expert the
// block is bound by streaming the touched experts' packed weights from HBM;
// what limits a kernel there is the instruction budget per packed word.  Here
// every lane dequantises its own words straight into mma.sync A-fragment
// registers (no shared-memory or TMEM round trip for the 4x-expanded fp16
// weights) and every warp issues its own m16n8k16 MMAs, so no single issuing
// thread or per-k-block handoff paces the pipeline.  (The tcgen05 kernel,
// expert_tc.cu, takes over when experts hold enough tokens for its 128 x N
// tiles to be worth the TMEM round trip.)
//
// Tile: one expert, 128 weight rows (gate and up together, or down), and up
// to 8*NT of the expert's slots; k streams in 256-column stages.
//   warp 16       TMA producer: per stage the packed codes (2-D tensor map,
//                 128 rows x 128 B boxes, SWIZZLE_128B) and the activation
//                 tile (fp16 [slots, k], 64-column x 8*NT-row boxes,
//                 SWIZZLE_128B), into a ring of stages.  No multicast.
//   warps 0-15    warp w computes rows 16*(w%8) .. +16 for the k-half w/8 of
//                 every stage (half of its 32-column chunks), then the two k-halves
//                 are added through shared memory and warps 0-7 run the
//                 epilogue (SwiGLU / GeGLU with MLX's bf16 rounding, or the
//                 bf16 down output).
// k order: lane t of k-half kh reads one 32-column chunk (2t + kh) of each
// 256-column stage, one 16-byte line per row, inside one quantization group;
// each packed word's code pairs (p, p+4) land in the k-pairs of the A
// fragment.  B (activations, written by gather_rows_kernel and by the gate/up
// epilogue) is stored in the matching order (kperm256), and the contraction
// does not depend on it.  Operands are fp16 (exact codes, q*s+b rounded once, bf16
// activations exact), accumulation fp32, as on the tcgen05 path.
// Every mbarrier wait is bounded; a timeout aborts the CTA cleanly.

#include <cuda.h>

#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"
#include "tiles.cuh"

namespace senmoe {
namespace {

constexpr int kRows = 128;           // weight rows per tile
constexpr int kStageCols = 256;      // k columns per stage
constexpr int kComputeWarps = 16;    // 8 row groups x 2 k-halves
// + one producer warp.  (Folding the producer into a compute warp would lift
// the 96-register cap that a 17th warp imposes, but measured slower: the
// issuing warp then waits for the slowest warp at every stage.)
constexpr int kThreads = (kComputeWarps + 1) * 32;
// The group-scaled form has four loader warps (16-19, one per scheduler):
// lane 0 of warp 16 issues the TMA copies, and each of the 128 loader lanes
// copies one weight row's scales / biases per stage, so the copy work does
// not pile onto one scheduler.  Twenty warps still leave 96 registers each.
constexpr int kLoaderWarps = 4;
constexpr int kThreadsG4 = (kComputeWarps + kLoaderWarps) * 32;
constexpr int kMaxTiles = 128;       // per CTA
constexpr int kSmemBudget = 226 * 1024;

// DP (group-scaled down): the tile is two 128-row blocks of the one
// projection, laid out as the two projections of a gate/up tile.
template <int BITS, int NPROJ, int NT, bool G4, bool DP = false>
struct MmaShape {
  static_assert(!DP || (G4 && NPROJ == 2), "row-block pairs: group-scaled, two blocks");
  static constexpr int kABoxes = BITS / 4;                   // 128-byte boxes per row per stage
  static constexpr int kABox = kRows * 128;                  // 16 KB
  static constexpr int kABytes = NPROJ * kABoxes * kABox;
  static constexpr int kBRows = 8 * NT;
  static constexpr int kBBox = kBRows * 128;                 // 64 fp16 columns x kBRows
  static constexpr int kBBytes = 4 * kBBox;
  static constexpr int kTmaBytes = kABytes + kBBytes;        // bytes the TMA copies per stage
  // group-scaled form: the stage's scales and biases, [proj][s, b][row][4 groups] bf16
  static constexpr int kSBOff = kTmaBytes;
  static constexpr int kSBBytes = G4 ? NPROJ * 2 * kRows * 8 : 0;
  // group-scaled gate/up: the stage's activation group sums, [slot][4 groups] fp32
  static constexpr int kXOff = kSBOff + kSBBytes;
  static constexpr int kXBytes = (G4 && NPROJ == 2 && !DP) ? 8 * NT * 16 : 0;
  static constexpr int kStageBytes = (kTmaBytes + kSBBytes + kXBytes + 1023) / 1024 * 1024;
  static constexpr int kRedBytes = 8 * 32 * NPROJ * NT * 4 * 4;
  static constexpr int kMisc = 4096;                         // barriers + tile list
  static constexpr int kFit = (kSmemBudget - kRedBytes - kMisc - 1024) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kRedBytes + kMisc;
  static_assert(kStages >= 2, "pipeline needs two stages");
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// MMAs of the group-scaled form: no memory operands, so the compiler may
// schedule them freely; the _z form starts from a zero accumulator.
__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                      uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}

// ---------------------------------------------------------------------------
// Group-scaled 4-bit form.  Instead of dequantising every weight to fp16, the
// MMA multiplies the raw codes and each 64-column quantization group is
// scaled afterwards in fp32, the way MLX's own quantized GEMV accumulates
//   y = sum_G ( s_G * sum_{k in G} q_k x_k  +  b_G * sum_{k in G} x_k ).
// A code goes into the A fragment as an fp16 subnormal with one AND: bits
// 0-3 of a half hold q * 2^-24, bits 4-7 hold q * 2^-20 (mma.sync multiplies
// subnormal fp16 operands exactly).  Each MMA k-step takes codes of one
// position kind only -- even k-steps the nibbles at bits 0-3 (and, from the
// word shifted right by 8, bits 8-11), odd k-steps those at bits 4-7 (12-15)
// -- and the activations of odd k-steps are stored divided by 16, so every
// product lands in units of 2^-24 and one accumulator serves the group.  The
// group sums of x come from four more MMAs per group whose A is the constant
// 2^-24 (even k-steps) or 2^-20 (odd), on the otherwise idle tensor pipe.
//
// k order inside each 64-column group (the same for every group): physical
// column u = 8 w + i (packed word w = 0..7 of the group, nibble i) is MMA
// k-step s = 2 (w / 4) + (i & 1), fragment index kappa = 2 (w % 4) + (i >> 2)
// + 8 ((i >> 1) & 1), and is stored at position 16 s + kappa; columns with
// odd u hold x / 16.  Lane t then needs words t and 4 + t of the group for
// each of its rows: one ldmatrix.x4 of the packed codes.
__device__ __forceinline__ int kperm_g4(int col) {
  const int u = col & 63, w = u >> 3, i = u & 7;
  const int s = 2 * (w >> 2) + (i & 1);
  const int kappa = 2 * (w & 3) + (i >> 2) + 8 * ((i >> 1) & 1);
  return (col & ~63) | (16 * s + kappa);
}
constexpr uint32_t kCodeLo = 0x000F000Fu;   // codes at bits 0-3 of each half: q * 2^-24
constexpr uint32_t kCodeHi = 0x00F000F0u;   // codes at bits 4-7: q * 2^-20
constexpr uint32_t kOne24 = 0x00010001u;    // fp16 2^-24 in both halves
constexpr uint32_t kOne20 = 0x00100010u;    // fp16 2^-20
constexpr float kG4Scale = 16777216.0f;     // 2^24: accumulator units back to 1

// Per (row, group) dequantisation constants.
struct GroupConst {
  __half2 s;    // scale (x 2^20 at 4 bits / 2^22 at 8 bits for the subnormal form)
  __half2 b;    // bias
  bool sub;     // subnormal form usable
};

// The subnormal form places each code at fp16 mantissa bits 4-7 (4-bit,
// value q * 2^-20) or 2-9 (8-bit, q * 2^-22); one fma with s * 2^20 (2^22)
// then gives q * s + b with a single rounding.  s * 2^20 must stay inside
// fp16 range: |s| < 0.0624 (4-bit), 0.0156 (8-bit); other groups take the
// 1024 + q form.
template <int BITS>
__device__ __forceinline__ GroupConst group_const(uint16_t sbits, uint16_t bbits) {
  const float sf = bf16_bits_to_f32(sbits);
  GroupConst c;
  c.b = __float2half2_rn(bf16_bits_to_f32(bbits));
  constexpr float kUp = BITS == 4 ? 1048576.0f : 4194304.0f;
  constexpr float kMax = BITS == 4 ? 0.0624f : 0.0156f;
  c.sub = fabsf(sf) < kMax;
  c.s = __float2half2_rn(c.sub ? sf * kUp : sf);
  return c;
}

// Code pairs (p, p+4), p = 0..3, of the 8 codes a lane holds for one row of a
// 32-column block, as fp16 q*s+b.  4-bit: one word; 8-bit: two words.
// FAST: every group of the warp takes the subnormal form (warp-uniform).
template <int BITS, bool FAST>
__device__ __forceinline__ uint4 dequant_pairs(uint32_t w0, uint32_t w1, const GroupConst& c) {
  uint32_t o[4];
  if constexpr (BITS == 4) {
    (void)w1;
    if (FAST || c.sub) {
      const uint32_t m = 0x00F000F0u;
      const uint32_t v[4] = {(w0 << 4) & m, w0 & m, (w0 >> 4) & m, (w0 >> 8) & m};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&v[p]), c.s, c.b);
        o[p] = *reinterpret_cast<const uint32_t*>(&r);
      }
      return make_uint4(o[0], o[1], o[2], o[3]);
    }
    return dequant8_u4(w0, c.s, c.b);
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      // bytes: [w0.p, w0.0, w1.p, w0.0]
      const uint32_t t = __byte_perm(w0, w1, static_cast<uint32_t>(p | ((4 + p) << 8)));
      __half2 r;
      if (FAST || c.sub) {
        const uint32_t v = (t << 2) & 0x03FC03FCu;  // q * 2^-22 in each half
        r = __hfma2(*reinterpret_cast<const __half2*>(&v), c.s, c.b);
      } else {
        const uint32_t v = (t & 0x00FF00FFu) | 0x64006400u;  // 1024 + q
        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&v), __floats2half2_rn(1024.0f, 1024.0f));
        r = __hfma2(q, c.s, c.b);
      }
      o[p] = *reinterpret_cast<const uint32_t*>(&r);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Position of feature `col` in the kperm256 order of the activation operand:
// within each 256-column stage, column 32 (2t + kh) + 8b + p + 4h (lane t of
// k-half kh, block b, code pair p, half h) is stored in 16-byte segment
// 16 kh + 4 b + p at half 2t + h, so one ldmatrix row per (block, pair)
// carries the four lanes' pairs in fragment order.
__device__ __forceinline__ int kperm256(int col) {
  const int c = col & 255, ch = c >> 5, t = ch >> 1, kh = ch & 1, b = (c >> 3) & 3, r = c & 7;
  return (col & ~255) | ((16 * kh + 4 * b + (r & 3)) << 3) | (t << 1) | (r >> 2);
}

// G4: the group-scaled 4-bit form (kperm_g4 activations); otherwise every
// weight is dequantised to fp16 (kperm256 activations).
// DP (group-scaled down, NPROJ = 2): a tile is 256 rows of the down
// projection, taken as two 128-row blocks in the places of gate and up
// (tA0 for both, the second block 128 rows on), so every warp runs two
// independent MMA chains, as in gate/up, instead of one, and the four MMAs
// of each group's activation sums serve both blocks.  Each output is the
// same fp32 chain as in a 128-row down tile, so both give the same bits.
template <int BITS, int NPROJ, int NT, bool G4, bool DP>
__global__ void __launch_bounds__(G4 ? kThreadsG4 : kThreads, 1)
    qmma_kernel(const __grid_constant__ CUtensorMap tA0, const __grid_constant__ CUtensorMap tA1,
                const __grid_constant__ CUtensorMap tB, TcGemmArgs a) {
  using S = MmaShape<BITS, NPROJ, NT, G4, DP>;
  constexpr bool kGateUp = NPROJ == 2 && !DP;  // two projections with the activation epilogue
  static_assert(!G4 || BITS == 4, "group-scaled form is 4-bit");
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sStage = smem;
  float* sRed = reinterpret_cast<float*>(smem + S::kStages * S::kStageBytes);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes + S::kRedBytes);
  uint64_t* bar_empty = bar_full + S::kStages;
  uint64_t* bar_red_full = bar_empty + S::kStages;   // [8] partner k-half partials written
  uint64_t* bar_red_empty = bar_red_full + 8;        // [8] partials consumed
  int4* s_tiles = reinterpret_cast<int4*>(bar_red_empty + 8);
  __shared__ int s_ntiles;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S::kStages; ++i) {
      // group-scaled form: + one cp.async arrival per loader lane
      mbar_init(&bar_full[i], G4 ? 1 + 32 * kLoaderWarps : 1);
      mbar_init(&bar_empty[i], kComputeWarps);
    }
    for (int i = 0; i < 8; ++i) {
      mbar_init(&bar_red_full[i], 1);
      mbar_init(&bar_red_empty[i], 1);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  pdl_wait();  // active list / offsets (dispatch) and the activation rows (gather or gate/up)
  pdl_launch_dependents();
  // the stage ring is free until the producer starts: use it as scratch
  const int nlisted = list_tiles(a.active, a.active_count, a.offsets, a.expert_begin, a.m_tiles, DP ? 2 * kRows : kRows, 8 * NT, false,
                                 s_tiles, kMaxTiles, reinterpret_cast<int*>(sStage), a.err, a.slot_cap, a.cnt_lo,
                                 a.cnt_hi);
  if (threadIdx.x == 0) s_ntiles = nlisted;
  __syncthreads();
  const int ntiles = s_ntiles;
  const int nst = a.kdim / kStageCols;

  const int groups = a.kdim / 64;
  if (warp >= kComputeWarps) {
    // ===================================================== TMA producer
    // Lane 0 of warp 16 issues the stage's TMA boxes (packed codes,
    // activations).  In the group-scaled form the loader lane l = 0..127 of
    // warps 16-19 also copies weight row l's scale / bias runs (8 bytes = 4
    // groups) of every projection with cp.async, whose completion the
    // stage's full barrier counts as one arrival per loader lane.
    const int ll = (warp - kComputeWarps) * 32 + lane;  // loader lane
    if (G4 || ll == 0) {
      int slot = 0;
      uint32_t ph = 0;
      int issued = 0;
      bool ok = true;
      for (int ti = 0; ti < ntiles && ok; ++ti) {
        const int4 tl = s_tiles[ti];
        const int arow = tl.x * a.rows + tl.y;
        const size_t sb_row0 = static_cast<size_t>(arow + ll) * groups;  // (row ll, group 0)
        for (int st = 0; st < nst; ++st, ++issued) {
          bool w = wait_or_abort(&bar_empty[slot], ph ^ 1, &s_abort, a.err);
          if constexpr (G4) w = __all_sync(0xffffffffu, w);
          if (!(ok = w)) break;
          unsigned char* base = sStage + slot * S::kStageBytes;
          if (ll == 0) {
            mbar_arrive_expect_tx(&bar_full[slot], S::kTmaBytes);
#pragma unroll
            for (int p = 0; p < NPROJ; ++p)
#pragma unroll
              for (int bx = 0; bx < S::kABoxes; ++bx)
                tma_load_2d(base + (p * S::kABoxes + bx) * S::kABox, (p && !DP) ? &tA1 : &tA0,
                            (st * S::kABoxes + bx) * 32, DP ? arow + p * kRows : arow, &bar_full[slot]);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              tma_load_2d(base + S::kABytes + j * S::kBBox, &tB, st * kStageCols + j * 64, tl.z, &bar_full[slot]);
          }
          if constexpr (G4) {
            static_assert(32 * kLoaderWarps == kRows, "one loader lane per weight row");
            const uint32_t dst = smem_u32(base + S::kSBOff) + ll * 8;
#pragma unroll
            for (int pa = 0; pa < 2 * NPROJ; ++pa) {  // array pa: scales (even) / biases (odd) of proj pa / 2
              if constexpr (DP)  // block pa / 2: rows 128 (pa / 2) on, of the one projection
                cp_async_8(dst + pa * kRows * 8,
                           ((pa & 1) ? a.b[0] : a.s[0]) + sb_row0 + static_cast<size_t>(pa >> 1) * kRows * groups + 4 * st);
              else
                cp_async_8(dst + pa * kRows * 8, ((pa & 1) ? a.b[pa >> 1] : a.s[pa >> 1]) + sb_row0 + 4 * st);
            }
            if constexpr (kGateUp) {
              // the group sums of the stage's 4 groups: 16 bytes per slot,
              // two 8-byte halves per loader lane (rows past the valid slots
              // exist: the buffer has 16 spare rows)
              if (ll < 16 * NT) {
                const int sl = ll >> 1, half = ll & 1;
                cp_async_8(smem_u32(base + S::kXOff) + sl * 16 + half * 8,
                           a.xsum + static_cast<size_t>(tl.z + sl) * groups + 4 * st + 2 * half);
              }
            }
            cp_async_arrive_noinc(&bar_full[slot]);
          }
          if (++slot == S::kStages) { slot = 0; ph ^= 1; }
        }
      }
      // drain: the copies of the last stages must land before the CTA may
      // exit, consumed or not (bounded; each slot's latest use only)
      int never = 0;
      for (int k = (issued > S::kStages ? issued - S::kStages : 0); k < issued; ++k)
        wait_or_abort(&bar_full[k % S::kStages], (k / S::kStages) & 1, &never, nullptr);
    }
    return;
  }

  // ======================================================= compute warps
  const int rg = warp & 7, kh = warp >> 3;
  const int g = lane >> 2, t = lane & 3;
  int slot = 0;
  uint32_t ph = 0;
  bool ok = true;
  bool next_ready = false;  // group-scaled form: early test of the next stage's barrier
  const uint32_t sStage_u32 = smem_u32(sStage);
  const int rA = 16 * rg + g;  // tile row of this lane's first fragment row
  // Dequantising form: lane t of k-half kh owns the 32-column chunk
  // c = 2t + kh of every stage (four 8-column blocks b; one 16-byte line of
  // each row at 4 bits), all inside quantization group t of the stage; its
  // scale / bias for each of its two rows and each projection are prefetched
  // into registers one stage ahead, across tile boundaries too.
  // Group-scaled form: warps of k-half kh take groups 2kh and 2kh + 1 of
  // every stage whole; the scales / biases arrive with the stage (producer).
  const int cs = 2 * t + kh;
  uint16_t scur[NPROJ][2], bcur[NPROJ][2], snext[NPROJ][2], bnext[NPROJ][2];
  auto load_sb = [&](int ti, int st) {
    const int4 tn = s_tiles[ti];
    const size_t row = static_cast<size_t>(tn.x * a.rows + tn.y + rA) * groups + static_cast<size_t>(st) * 4 + t;
#pragma unroll
    for (int p = 0; p < NPROJ; ++p) {
      snext[p][0] = __ldg(a.s[p] + row);
      snext[p][1] = __ldg(a.s[p] + row + 8 * groups);
      bnext[p][0] = __ldg(a.b[p] + row);
      bnext[p][1] = __ldg(a.b[p] + row + 8 * groups);
    }
  };
  // Group-scaled form, per-lane shared-memory offsets inside a stage.
  // ldmatrix: lane supplies row (lane & 7) of matrix (lane >> 3).  Codes of
  // group j (chunks 2j, 2j+1 of each row): matrix m = rows 8 (m & 1) ..,
  // chunk 2j + m / 2.  Activations of group j (box j): x4 load hw covers
  // k-steps 2hw (chunks 4hw, +1) and 2hw + 1 (chunks 4hw + 2, +3).
  const int lm = lane >> 3, lr = lane & 7;
  uint32_t offA[2] = {0, 0}, offB[2][2] = {{0, 0}, {0, 0}}, offSB = 0;
  if constexpr (G4) {
    const uint32_t a_row = static_cast<uint32_t>(16 * rg + lr + 8 * (lm & 1)) * 128u;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
      const int j = 2 * kh + gi;
      offA[gi] = a_row + ((static_cast<uint32_t>(2 * j + (lm >> 1)) ^ lr) << 4);
#pragma unroll
      for (int hw = 0; hw < 2; ++hw)
        offB[gi][hw] = S::kABytes + j * S::kBBox + lr * 128 + ((static_cast<uint32_t>(4 * hw + lm) ^ lr) << 4);
    }
    offSB = S::kSBOff + rA * 8 + kh * 4;  // bf16 pair (groups 2kh, 2kh + 1) of row rA
  } else {
    if (ntiles > 0) load_sb(0, 0);
  }
  for (int ti = 0; ti < ntiles && ok; ++ti) {
    const int4 tl = s_tiles[ti];
    float acc[NPROJ][NT][4];
#pragma unroll
    for (int p = 0; p < NPROJ; ++p)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[p][nt][i] = 0.f;
    for (int st = 0; st < nst; ++st) {
      if constexpr (!G4) {
#pragma unroll
        for (int p = 0; p < NPROJ; ++p) {
          scur[p][0] = snext[p][0]; scur[p][1] = snext[p][1];
          bcur[p][0] = bnext[p][0]; bcur[p][1] = bnext[p][1];
        }
        if (st + 1 < nst) load_sb(ti, st + 1);
        else if (ti + 1 < ntiles) load_sb(ti + 1, 0);
      }
      ok = __all_sync(0xffffffffu, next_ready || wait_or_abort(&bar_full[slot], ph, &s_abort, a.err));
      if (!ok) break;
      const unsigned char* base = sStage + slot * S::kStageBytes;
      const uint32_t sbase = sStage_u32 + slot * S::kStageBytes;
      const uint32_t bbase = sbase + S::kABytes;
      if constexpr (G4) {
        // ask now whether the next stage has landed: the barrier round trip
        // then overlaps this stage's work
        const int ns = slot + 1 == S::kStages ? 0 : slot + 1;
        next_ready = mbar_test_wait(&bar_full[ns], ns == 0 ? ph ^ 1 : ph);
        // scales / biases of rows rA, rA + 8: bf16 pairs, group 2kh low, 2kh + 1 high
        uint32_t sv[NPROJ][2], bv[NPROJ][2];
#pragma unroll
        for (int p = 0; p < NPROJ; ++p)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            sv[p][r] = *reinterpret_cast<const uint32_t*>(base + offSB + (2 * p) * kRows * 8 + r * 64);
            bv[p][r] = *reinterpret_cast<const uint32_t*>(base + offSB + (2 * p + 1) * kRows * 8 + r * 64);
          }
        // gate/up: group sums of slots 2t (c0, c2) and 2t + 1 (c1, c3) for
        // this k-half's groups 2kh, 2kh + 1
        float xlo[NT][2], xhi[NT][2];
        if constexpr (kGateUp) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float2 v0 = *reinterpret_cast<const float2*>(base + S::kXOff + (8 * nt + 2 * t) * 16 + kh * 8);
            const float2 v1 = *reinterpret_cast<const float2*>(base + S::kXOff + (8 * nt + 2 * t + 1) * 16 + kh * 8);
            xlo[nt][0] = v0.x; xlo[nt][1] = v0.y;
            xhi[nt][0] = v1.x; xhi[nt][1] = v1.y;
          }
        }
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
          uint32_t bf[NT][2][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            ldmatrix_x4(sbase + offB[gi][0] + nt * 1024, bf[nt][0]);
            ldmatrix_x4(sbase + offB[gi][1] + nt * 1024, bf[nt][1]);
          }
          // group sums of the activations, in units of 2^-24 (all rows alike):
          // gate/up reads them (gather_rows computed them), down forms them
          // with four more MMAs whose A is the constant 2^-24 / 2^-20
          float xs[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if constexpr (kGateUp) {
              xs[nt][0] = xs[nt][2] = xlo[nt][gi];
              xs[nt][1] = xs[nt][3] = xhi[nt][gi];
            } else {
              mma_z(xs[nt], kOne24, kOne24, kOne24, kOne24, bf[nt][0][0], bf[nt][0][1]);
              mma_acc(xs[nt], kOne20, kOne20, kOne20, kOne20, bf[nt][0][2], bf[nt][0][3]);
              mma_acc(xs[nt], kOne24, kOne24, kOne24, kOne24, bf[nt][1][0], bf[nt][1][1]);
              mma_acc(xs[nt], kOne20, kOne20, kOne20, kOne20, bf[nt][1][2], bf[nt][1][3]);
            }
          }
#pragma unroll
          for (int p = 0; p < NPROJ; ++p) {
            // words t (regs 0, 1: rows g, g+8) and 4 + t (regs 2, 3) of the group
            uint32_t w[4];
            ldmatrix_x4(sbase + offA[gi] + p * S::kABox, w);
            float grp[NT][4];
#pragma unroll
            for (int hw = 0; hw < 2; ++hw) {
              const uint32_t x0 = w[2 * hw], x1 = w[2 * hw + 1], y0 = x0 >> 8, y1 = x1 >> 8;
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                if (hw == 0)
                  mma_z(grp[nt], x0 & kCodeLo, x1 & kCodeLo, y0 & kCodeLo, y1 & kCodeLo, bf[nt][0][0], bf[nt][0][1]);
                else
                  mma_acc(grp[nt], x0 & kCodeLo, x1 & kCodeLo, y0 & kCodeLo, y1 & kCodeLo, bf[nt][1][0],
                          bf[nt][1][1]);
                mma_acc(grp[nt], x0 & kCodeHi, x1 & kCodeHi, y0 & kCodeHi, y1 & kCodeHi, bf[nt][hw][2],
                        bf[nt][hw][3]);
              }
            }
            const float s0 = gi ? bf16_hi(sv[p][0]) : bf16_lo(sv[p][0]);
            const float s1 = gi ? bf16_hi(sv[p][1]) : bf16_lo(sv[p][1]);
            const float b0 = gi ? bf16_hi(bv[p][0]) : bf16_lo(bv[p][0]);
            const float b1 = gi ? bf16_hi(bv[p][1]) : bf16_lo(bv[p][1]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[p][nt][0] = fmaf(s0, grp[nt][0], fmaf(b0, xs[nt][0], acc[p][nt][0]));
              acc[p][nt][1] = fmaf(s0, grp[nt][1], fmaf(b0, xs[nt][1], acc[p][nt][1]));
              acc[p][nt][2] = fmaf(s1, grp[nt][2], fmaf(b1, xs[nt][2], acc[p][nt][2]));
              acc[p][nt][3] = fmaf(s1, grp[nt][3], fmaf(b1, xs[nt][3], acc[p][nt][3]));
            }
          }
        }
      } else {
      GroupConst gc[NPROJ][2];
      bool all_sub = true;
#pragma unroll
      for (int p = 0; p < NPROJ; ++p)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          gc[p][r] = group_const<BITS>(scur[p][r], bcur[p][r]);
          all_sub = all_sub && gc[p][r].sub;
        }
      all_sub = __all_sync(0xffffffffu, all_sub);
      // this lane's packed words of the stage, per projection and row:
      // 4-bit: one 16-byte line (word b for block b); 8-bit: two lines
      // (words 2b, 2b+1 for block b), chunks 2(c%4), +1 of box c/4
      uint4 wl[NPROJ][2][BITS / 4];
#pragma unroll
      for (int p = 0; p < NPROJ; ++p)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = rA + 8 * r;
          if constexpr (BITS == 4) {
            wl[p][r][0] = *reinterpret_cast<const uint4*>(base + p * S::kABox + row * 128 + ((cs ^ (row & 7)) << 4));
          } else {
            const unsigned char* rowp = base + (p * S::kABoxes + (cs >> 2)) * S::kABox + row * 128;
            const int c0 = 2 * (cs & 3);
            wl[p][r][0] = *reinterpret_cast<const uint4*>(rowp + ((c0 ^ (row & 7)) << 4));
            wl[p][r][1] = *reinterpret_cast<const uint4*>(rowp + (((c0 + 1) ^ (row & 7)) << 4));
          }
        }
      auto run_blocks = [&](auto fast) {
        constexpr bool F = decltype(fast)::value;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          // B fragments (all n-tiles) for the block's two k-steps: segment
          // 16 kh + 4 b + p of the stage = box 2 kh + b/2, chunk 4 (b%2) + p
          uint32_t bf[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int n = lane & 7, mi = lane >> 3;
            const uint32_t addr = bbase + (2 * kh + (b >> 1)) * S::kBBox + (8 * nt + n) * 128 +
                                  ((((b & 1) * 4 + mi) ^ n) << 4);
            ldmatrix_x4(addr, bf[nt]);
          }
#pragma unroll
          for (int p = 0; p < NPROJ; ++p) {
            uint4 v[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              uint32_t w0, w1 = 0;
              if constexpr (BITS == 4) {
                const uint4& L4 = wl[p][r][0];
                w0 = b == 0 ? L4.x : b == 1 ? L4.y : b == 2 ? L4.z : L4.w;
              } else {
                const uint4& L8 = wl[p][r][b >> 1];
                w0 = (b & 1) ? L8.z : L8.x;
                w1 = (b & 1) ? L8.w : L8.y;
              }
              v[r] = dequant_pairs<BITS, F>(w0, w1, gc[p][r]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma16816(acc[p][nt], v[0].x, v[1].x, v[0].y, v[1].y, bf[nt][0], bf[nt][1]);
              mma16816(acc[p][nt], v[0].z, v[1].z, v[0].w, v[1].w, bf[nt][2], bf[nt][3]);
            }
          }
        }
      };
      if (all_sub) run_blocks(std::true_type{});
      else run_blocks(std::false_type{});
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_empty[slot]);
      if (++slot == S::kStages) { slot = 0; ph ^= 1; }
    }
    if (!ok) break;

    // ---- add the two k-halves: warp rg+8 hands its partials to warp rg
    float* red = sRed + (rg * 32 + lane) * (NPROJ * NT * 4);
    const uint32_t rph = ti & 1;
    if (kh == 1) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&bar_red_empty[rg], rph ^ 1, &s_abort, a.err));
      if (!ok) break;
#pragma unroll
      for (int p = 0; p < NPROJ; ++p)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          *reinterpret_cast<float4*>(red + (p * NT + nt) * 4) =
              make_float4(acc[p][nt][0], acc[p][nt][1], acc[p][nt][2], acc[p][nt][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_red_full[rg]);
      continue;
    }
    ok = __all_sync(0xffffffffu, wait_or_abort(&bar_red_full[rg], rph, &s_abort, a.err));
    if (!ok) break;
#pragma unroll
    for (int p = 0; p < NPROJ; ++p)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float4 o = *reinterpret_cast<const float4*>(red + (p * NT + nt) * 4);
        acc[p][nt][0] += o.x; acc[p][nt][1] += o.y; acc[p][nt][2] += o.z; acc[p][nt][3] += o.w;
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_red_empty[rg]);

    // ---- epilogue: lane holds rows (rA, rA+8) x slots (8nt + 2t, +1)
    bool range_ok = true;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int n = 8 * nt + 2 * t + (i & 1);
        if (n >= tl.w) continue;
        const int row = tl.y + rA + 8 * (i >> 1);
        const size_t o = static_cast<size_t>(tl.z + n) * a.out_stride;
        constexpr float kUnit = G4 ? kG4Scale : 1.0f;  // accumulator units (exact power of two)
        if constexpr (kGateUp) {
          const float gv = round_bf16(acc[0][nt][i] * kUnit), uv = round_bf16(acc[1][nt][i] * kUnit);
          const float h = a.act == 0 ? act_swiglu_mlx(gv, uv) : act_geglu_mlx(gv, uv);
          range_ok &= fabsf(h) < 65504.0f;
          if constexpr (G4)
            a.out[o + kperm_g4(row)] = __half_as_ushort(__float2half_rn((row & 1) ? h * 0.0625f : h));
          else
            a.out[o + kperm256(row)] = __half_as_ushort(__float2half_rn(h));
        } else {
#pragma unroll
          for (int p = 0; p < NPROJ; ++p)  // row blocks (DP: 128 rows apart)
            a.out[o + row + p * kRows] = f32_to_bf16_bits(acc[p][nt][i] * kUnit);
        }
      }
    }
    if (!range_ok) record_error(a.err, kDevFp16Range);
  }
}

// ---------------------------------------------------------------------------
// Group-scaled form, two CTAs per SM (qmma_q4_kernel, 8-slot tiles).  The
// kernel above runs 16 compute warps per SM, four per scheduler, each at the
// 96-register cap, and at decode sizes it is bound by how much MMA and
// shared-memory latency those warps hide, not by HBM (the same kernel with
// its weights resident in L2 is only ~10 % faster).  This form halves the
// tile (64 weight rows) and the per-warp state (one quantization group per
// stage) so that two CTAs fit on an SM: eight compute warps per scheduler.
//   warps 0-15   warp w: rows 16 (w % 4) .. +16 of the tile, quantization
//                group w / 4 (k-quarter kq) of every 256-column stage
//   warp 16      producer: TMA of the codes (64-row boxes) and activations,
//                cp.async of the stage's scales / biases
// The k-quarters are added in a fixed order (kq = 1, 2, 3 into kq = 0)
// through shared memory; warps kq = 0 run the epilogue.
constexpr int kQRows = 64;
template <int NPROJ>
struct QShape {
  static constexpr int kABox = kQRows * 128;                 // 8 KB: 64 rows x 128 B
  static constexpr int kABytes = NPROJ * kABox;
  static constexpr int kBBox = 8 * 128;                      // 64 fp16 columns x 8 slots
  static constexpr int kBBytes = 4 * kBBox;
  static constexpr int kTmaBytes = kABytes + kBBytes;
  static constexpr int kSBOff = kTmaBytes;                   // [proj][s, b][row][4 groups] bf16
  static constexpr int kSBBytes = NPROJ * 2 * kQRows * 8;
  static constexpr int kStageBytes = kTmaBytes + kSBBytes;   // 13 or 22 KB
  static constexpr int kRedSlice = 4 * 32 * NPROJ * 4;       // floats of one k-quarter's partials
  static constexpr int kRedBytes = 3 * kRedSlice * 4;
  static constexpr int kMisc = 4096;                         // barriers + tile list
  static constexpr int kBudget = 112 * 1024;                 // two CTAs per SM
  static constexpr int kFit = (kBudget - kRedBytes - kMisc - 1024) / kStageBytes;
  static constexpr int kStages = kFit > 8 ? 8 : kFit;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kRedBytes + kMisc;
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(kStageBytes % 1024 == 0, "stage alignment");
};

template <int NPROJ>
__global__ void __launch_bounds__(kThreads, 2)
    qmma_q4_kernel(const __grid_constant__ CUtensorMap tA0, const __grid_constant__ CUtensorMap tA1,
                   const __grid_constant__ CUtensorMap tB, TcGemmArgs a) {
  using S = QShape<NPROJ>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sStage = smem;
  float* sRed = reinterpret_cast<float*>(smem + S::kStages * S::kStageBytes);
  uint64_t* bar_full = reinterpret_cast<uint64_t*>(smem + S::kStages * S::kStageBytes + S::kRedBytes);
  uint64_t* bar_empty = bar_full + S::kStages;
  uint64_t* bar_red_full = bar_empty + S::kStages;   // [4] k-quarters 1-3 of row group rg written
  uint64_t* bar_red_empty = bar_red_full + 4;        // [4] consumed
  int4* s_tiles = reinterpret_cast<int4*>(bar_red_empty + 4);
  __shared__ int s_ntiles;
  __shared__ int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < S::kStages; ++i) {
      mbar_init(&bar_full[i], 33);  // the TMA thread + one cp.async arrival per producer lane
      mbar_init(&bar_empty[i], kComputeWarps);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar_red_full[i], 3);
      mbar_init(&bar_red_empty[i], 1);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  pdl_wait();  // active list / offsets (dispatch) and the activation rows (gather or gate/up)
  pdl_launch_dependents();
  const int nlisted = list_tiles(a.active, a.active_count, a.offsets, a.expert_begin, a.m_tiles, kQRows, 8, false,
                                 s_tiles, kMaxTiles, reinterpret_cast<int*>(sStage), a.err, a.slot_cap, a.cnt_lo,
                                 a.cnt_hi);
  if (threadIdx.x == 0) s_ntiles = nlisted;
  __syncthreads();
  const int ntiles = s_ntiles;
  const int nst = a.kdim / kStageCols;
  const int groups = a.kdim / 64;

  if (warp == kComputeWarps) {
    // ===================================================== producer
    int slot = 0;
    uint32_t ph = 0;
    int issued = 0;
    bool ok = true;
    for (int ti = 0; ti < ntiles && ok; ++ti) {
      const int4 tl = s_tiles[ti];
      const int arow = tl.x * a.rows + tl.y;
      const size_t sb_row0 = static_cast<size_t>(arow + lane) * groups;  // (row lane, group 0)
      for (int st = 0; st < nst; ++st, ++issued) {
        if (!(ok = __all_sync(0xffffffffu, wait_or_abort(&bar_empty[slot], ph ^ 1, &s_abort, a.err)))) break;
        unsigned char* base = sStage + slot * S::kStageBytes;
        if (lane == 0) {
          mbar_arrive_expect_tx(&bar_full[slot], S::kTmaBytes);
#pragma unroll
          for (int p = 0; p < NPROJ; ++p)
            tma_load_2d(base + p * S::kABox, p ? &tA1 : &tA0, st * 32, arow, &bar_full[slot]);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tma_load_2d(base + S::kABytes + j * S::kBBox, &tB, st * kStageCols + j * 64, tl.z, &bar_full[slot]);
        }
        // scale / bias runs: 8 bytes (4 groups of one row) each, NPROJ * 2 * 64 per stage
        const uint32_t dst = smem_u32(base + S::kSBOff) + lane * 8;
#pragma unroll
        for (int i = 0; i < 4 * NPROJ; ++i) {  // run (array pa = i / 2, row lane + 32 (i % 2))
          const int pa = i >> 1, r = 32 * (i & 1);
          const uint16_t* src = ((pa & 1) ? a.b[pa >> 1] : a.s[pa >> 1]) + sb_row0 +
                                static_cast<size_t>(r) * groups + 4 * st;
          cp_async_8(dst + (pa * kQRows + r) * 8, src);
        }
        cp_async_arrive_noinc(&bar_full[slot]);
        if (++slot == S::kStages) { slot = 0; ph ^= 1; }
      }
    }
    // drain: the copies of the last stages must land before the CTA may exit
    int never = 0;
    for (int k = (issued > S::kStages ? issued - S::kStages : 0); k < issued; ++k)
      wait_or_abort(&bar_full[k % S::kStages], (k / S::kStages) & 1, &never, nullptr);
    return;
  }

  // ======================================================= compute warps
  const int rg = warp & 3, kq = warp >> 2;
  const int g = lane >> 2, t = lane & 3, lm = lane >> 3, lr = lane & 7;
  const int rA = 16 * rg + g;
  const uint32_t sStage_u32 = smem_u32(sStage);
  // ldmatrix offsets inside a stage (see the k order of the group-scaled form)
  const uint32_t offA = static_cast<uint32_t>(16 * rg + lr + 8 * (lm & 1)) * 128u +
                        ((static_cast<uint32_t>(2 * kq + (lm >> 1)) ^ lr) << 4);
  const uint32_t offB0 = S::kABytes + kq * S::kBBox + lr * 128 + ((static_cast<uint32_t>(lm) ^ lr) << 4);
  const uint32_t offB1 = S::kABytes + kq * S::kBBox + lr * 128 + ((static_cast<uint32_t>(4 + lm) ^ lr) << 4);
  const int offSB = S::kSBOff + rA * 8 + kq * 2;  // bf16 of group kq, row rA
  int slot = 0;
  uint32_t ph = 0;
  bool ok = true;
  for (int ti = 0; ti < ntiles && ok; ++ti) {
    const int4 tl = s_tiles[ti];
    float acc[NPROJ][4];
#pragma unroll
    for (int p = 0; p < NPROJ; ++p)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[p][i] = 0.f;
    for (int st = 0; st < nst; ++st) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&bar_full[slot], ph, &s_abort, a.err));
      if (!ok) break;
      const unsigned char* base = sStage + slot * S::kStageBytes;
      const uint32_t sbase = sStage_u32 + slot * S::kStageBytes;
      uint32_t bf[2][4];
      ldmatrix_x4(sbase + offB0, bf[0]);
      ldmatrix_x4(sbase + offB1, bf[1]);
      float xs[4];  // group sums of the activations, units of 2^-24
      mma_z(xs, kOne24, kOne24, kOne24, kOne24, bf[0][0], bf[0][1]);
      mma_acc(xs, kOne20, kOne20, kOne20, kOne20, bf[0][2], bf[0][3]);
      mma_acc(xs, kOne24, kOne24, kOne24, kOne24, bf[1][0], bf[1][1]);
      mma_acc(xs, kOne20, kOne20, kOne20, kOne20, bf[1][2], bf[1][3]);
#pragma unroll
      for (int p = 0; p < NPROJ; ++p) {
        uint32_t w[4];
        ldmatrix_x4(sbase + offA + p * S::kABox, w);
        float grp[4];
#pragma unroll
        for (int hw = 0; hw < 2; ++hw) {
          const uint32_t x0 = w[2 * hw], x1 = w[2 * hw + 1], y0 = x0 >> 8, y1 = x1 >> 8;
          if (hw == 0)
            mma_z(grp, x0 & kCodeLo, x1 & kCodeLo, y0 & kCodeLo, y1 & kCodeLo, bf[0][0], bf[0][1]);
          else
            mma_acc(grp, x0 & kCodeLo, x1 & kCodeLo, y0 & kCodeLo, y1 & kCodeLo, bf[1][0], bf[1][1]);
          mma_acc(grp, x0 & kCodeHi, x1 & kCodeHi, y0 & kCodeHi, y1 & kCodeHi, bf[hw][2], bf[hw][3]);
        }
        const unsigned char* sbp = base + offSB + 2 * p * kQRows * 8;
        const float s0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sbp));
        const float s1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sbp + 64));
        const float b0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sbp + kQRows * 8));
        const float b1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(sbp + kQRows * 8 + 64));
        acc[p][0] = fmaf(s0, grp[0], fmaf(b0, xs[0], acc[p][0]));
        acc[p][1] = fmaf(s0, grp[1], fmaf(b0, xs[1], acc[p][1]));
        acc[p][2] = fmaf(s1, grp[2], fmaf(b1, xs[2], acc[p][2]));
        acc[p][3] = fmaf(s1, grp[3], fmaf(b1, xs[3], acc[p][3]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_empty[slot]);
      if (++slot == S::kStages) { slot = 0; ph ^= 1; }
    }
    if (!ok) break;

    // ---- add the k-quarters: warps kq = 1..3 hand their partials to kq = 0
    float* red = sRed + (rg * 32 + lane) * (NPROJ * 4);
    const uint32_t rph = ti & 1;
    if (kq != 0) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&bar_red_empty[rg], rph ^ 1, &s_abort, a.err));
      if (!ok) break;
#pragma unroll
      for (int p = 0; p < NPROJ; ++p)
        *reinterpret_cast<float4*>(red + (kq - 1) * S::kRedSlice + p * 4) =
            make_float4(acc[p][0], acc[p][1], acc[p][2], acc[p][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_red_full[rg]);
      continue;
    }
    ok = __all_sync(0xffffffffu, wait_or_abort(&bar_red_full[rg], rph, &s_abort, a.err));
    if (!ok) break;
#pragma unroll
    for (int q = 0; q < 3; ++q)
#pragma unroll
      for (int p = 0; p < NPROJ; ++p) {
        const float4 o = *reinterpret_cast<const float4*>(red + q * S::kRedSlice + p * 4);
        acc[p][0] += o.x; acc[p][1] += o.y; acc[p][2] += o.z; acc[p][3] += o.w;
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar_red_empty[rg]);

    // ---- epilogue: lane holds rows (rA, rA + 8) x slots (2t, 2t + 1)
    bool range_ok = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = 2 * t + (i & 1);
      if (n >= tl.w) continue;
      const int row = tl.y + rA + 8 * (i >> 1);
      const size_t o = static_cast<size_t>(tl.z + n) * a.out_stride;
      if constexpr (NPROJ == 2) {
        const float gv = round_bf16(acc[0][i] * kG4Scale), uv = round_bf16(acc[1][i] * kG4Scale);
        const float h = a.act == 0 ? act_swiglu_mlx(gv, uv) : act_geglu_mlx(gv, uv);
        range_ok &= fabsf(h) < 65504.0f;
        a.out[o + kperm_g4(row)] = __half_as_ushort(__float2half_rn((row & 1) ? h * 0.0625f : h));
      } else {
        a.out[o + row] = f32_to_bf16_bits(acc[0][i] * kG4Scale);
      }
    }
    if (!range_ok) record_error(a.err, kDevFp16Range);
  }
}

}  // namespace

// ------------------------------------------------------------------ host
template <int BITS, int NPROJ, int NT, bool G4, bool DP = false>
static cudaError_t launch_mma_t(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                                const TcGemmArgs& a, int tiles_upper, cudaStream_t st) {
  using S = MmaShape<BITS, NPROJ, NT, G4, DP>;
  auto kern = qmma_kernel<BITS, NPROJ, NT, G4, DP>;
  constexpr int threads = G4 ? kThreadsG4 : kThreads;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), S::kSmem);
  if (e != cudaSuccess) return e;
  int sms = 0, dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  int grid = tiles_upper < sms ? tiles_upper : sms;
  if (grid < 1) grid = 1;
  if ((tiles_upper + grid - 1) / grid > kMaxTiles) return cudaErrorNotSupported;
  return launch_pdl(kern, dim3(grid), dim3(threads), S::kSmem, st, tA0, tA1, tB, a);
}

template <int NPROJ>
static cudaError_t launch_q4_t(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                               const TcGemmArgs& a, int tiles_upper, cudaStream_t st) {
  using S = QShape<NPROJ>;
  auto kern = qmma_q4_kernel<NPROJ>;
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), S::kSmem);
  if (e != cudaSuccess) return e;
  int sms = 0, dev = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  int grid = tiles_upper < 2 * sms ? tiles_upper : 2 * sms;  // two CTAs per SM
  if (grid < 1) grid = 1;
  if ((tiles_upper + grid - 1) / grid > kMaxTiles) return cudaErrorNotSupported;
  return launch_pdl(kern, dim3(grid), dim3(kThreads), S::kSmem, st, tA0, tA1, tB, a);
}

cudaError_t launch_mma_q4(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                          const TcGemmArgs& a, int bits, int nproj, int tiles_upper, cudaStream_t st) {
  if (!mma_g4_supported(bits, 1, a)) return cudaErrorInvalidValue;
  if (nproj == 2) return launch_q4_t<2>(tA0, tA1, tB, a, tiles_upper, st);
  if (nproj == 1) return launch_q4_t<1>(tA0, tA1, tB, a, tiles_upper, st);
  return cudaErrorNotSupported;
}

size_t mma_smem_bytes(int bits, int nproj, int nt, bool g4) {
  if (g4 && bits == 4 && nt == 1) return nproj == 2 ? MmaShape<4, 2, 1, true>::kSmem : MmaShape<4, 1, 1, true>::kSmem;
  if (g4 && bits == 4 && nt == 2) return nproj == 2 ? MmaShape<4, 2, 2, true>::kSmem : MmaShape<4, 1, 2, true>::kSmem;
  if (g4) return 0;
#define SENMOE_MMA_SMEM(B, P, N) \
  if (bits == B && nproj == P && nt == N) return MmaShape<B, P, N, false>::kSmem;
  SENMOE_MMA_SMEM(4, 1, 1) SENMOE_MMA_SMEM(4, 1, 2) SENMOE_MMA_SMEM(4, 1, 4)
  SENMOE_MMA_SMEM(4, 2, 1) SENMOE_MMA_SMEM(4, 2, 2) SENMOE_MMA_SMEM(4, 2, 4)
  SENMOE_MMA_SMEM(8, 1, 1) SENMOE_MMA_SMEM(8, 1, 2) SENMOE_MMA_SMEM(8, 1, 4)
  SENMOE_MMA_SMEM(8, 2, 1) SENMOE_MMA_SMEM(8, 2, 2) SENMOE_MMA_SMEM(8, 2, 4)
#undef SENMOE_MMA_SMEM
  return 0;
}

bool mma_supported(int rows, int kdim, int bits) {
  return (bits == 4 || bits == 8) && rows > 0 && rows % kRows == 0 && kdim > 0 && kdim % kStageCols == 0;
}

bool mma_g4_supported(int bits, int nt, const TcGemmArgs& a) {
  auto aligned4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; };
  bool ok = bits == 4 && (nt == 1 || nt == 2);
  for (int p = 0; p < 2; ++p) ok = ok && aligned4(a.s[p]) && aligned4(a.b[p]);
  return ok;
}

bool mma_down_pair_supported(int bits, int nt, const TcGemmArgs& a) {
  return nt == 1 && mma_g4_supported(bits, nt, a) && a.rows % (2 * kRows) == 0 && a.m_tiles * 2 * kRows == a.rows;
}

cudaError_t launch_mma_down_pair(const CUtensorMap& tA, const CUtensorMap& tB, const TcGemmArgs& a, int bits, int nt,
                                 int tiles_upper, cudaStream_t st) {
  if (!mma_down_pair_supported(bits, nt, a)) return cudaErrorInvalidValue;
  return launch_mma_t<4, 2, 1, true, true>(tA, tA, tB, a, tiles_upper, st);
}

cudaError_t launch_mma_gemm(const CUtensorMap& tA0, const CUtensorMap& tA1, const CUtensorMap& tB,
                            const TcGemmArgs& a, int bits, int nproj, int nt, bool g4, int tiles_upper,
                            cudaStream_t st) {
  if (g4) {
    if (!mma_g4_supported(bits, nt, a)) return cudaErrorInvalidValue;
    if (nproj == 2 && !a.xsum) return cudaErrorInvalidValue;  // gate/up reads gather_rows' group sums
    if (nproj == 2) return nt == 1 ? launch_mma_t<4, 2, 1, true>(tA0, tA1, tB, a, tiles_upper, st)
                                   : launch_mma_t<4, 2, 2, true>(tA0, tA1, tB, a, tiles_upper, st);
    if (nproj == 1) return nt == 1 ? launch_mma_t<4, 1, 1, true>(tA0, tA1, tB, a, tiles_upper, st)
                                   : launch_mma_t<4, 1, 2, true>(tA0, tA1, tB, a, tiles_upper, st);
    return cudaErrorNotSupported;
  }
#define SENMOE_MMA_CASE(B, P, N) \
  if (bits == B && nproj == P && nt == N) return launch_mma_t<B, P, N, false>(tA0, tA1, tB, a, tiles_upper, st);
  SENMOE_MMA_CASE(4, 1, 1) SENMOE_MMA_CASE(4, 1, 2) SENMOE_MMA_CASE(4, 1, 4)
  SENMOE_MMA_CASE(4, 2, 1) SENMOE_MMA_CASE(4, 2, 2) SENMOE_MMA_CASE(4, 2, 4)
  SENMOE_MMA_CASE(8, 1, 1) SENMOE_MMA_CASE(8, 1, 2) SENMOE_MMA_CASE(8, 1, 4)
  SENMOE_MMA_CASE(8, 2, 1) SENMOE_MMA_CASE(8, 2, 2) SENMOE_MMA_CASE(8, 2, 4)
#undef SENMOE_MMA_CASE
  return cudaErrorNotSupported;
}

}  // namespace senmoe
