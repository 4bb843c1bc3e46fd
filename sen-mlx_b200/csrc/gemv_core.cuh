// gemv_core.cuh -- the dequant-dot arithmetic of one quantized row against
// one token row, shared by the grouped GEMV kernel and the single-token fused
// layer kernel (same code, so the same bits).  Lane l owns packed words l,
// l + 32, ... of the row; dequantisation follows MLX qmv's factorisation
// scale * sum(q x) + bias * sum(x) in fp32 (magic-number code extraction:
// bf16 128 + q for 4 bits, fp32 2^23 + q for 8 bits).
#pragma once

#include "common.cuh"

namespace senmoe {

// sum over one packed word's codes of q_code * x, with the magic offset
// (128 for 4-bit, none for 8-bit: the 8-bit path subtracts 2^23 exactly).
template <int BITS>
__device__ __forceinline__ float word_dot(uint32_t w, const float* xv);

template <>
__device__ __forceinline__ float word_dot<4>(uint32_t w, const float* xv) {
  // nibble k (k = 0..7) holds column 8*word + k.
  const uint32_t p0 = (w & 0x000F000Fu) | 0x43004300u;          // cols 0, 4
  const uint32_t p1 = ((w >> 4) & 0x000F000Fu) | 0x43004300u;   // cols 1, 5
  const uint32_t p2 = ((w >> 8) & 0x000F000Fu) | 0x43004300u;   // cols 2, 6
  const uint32_t p3 = ((w >> 12) & 0x000F000Fu) | 0x43004300u;  // cols 3, 7
  float a = bf16_lo(p0) * xv[0];
  a = fmaf(bf16_lo(p1), xv[1], a);
  a = fmaf(bf16_lo(p2), xv[2], a);
  a = fmaf(bf16_lo(p3), xv[3], a);
  a = fmaf(bf16_hi(p0), xv[4], a);
  a = fmaf(bf16_hi(p1), xv[5], a);
  a = fmaf(bf16_hi(p2), xv[6], a);
  a = fmaf(bf16_hi(p3), xv[7], a);
  return a;  // = sum (128 + q_k) x_k
}

template <>
__device__ __forceinline__ float word_dot<8>(uint32_t w, const float* xv) {
  // byte k holds column 4*word + k; 0x4B0000qq is 2^23 + q exactly.
  float a = (__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540)) - 8388608.0f) * xv[0];
  a = fmaf(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541)) - 8388608.0f, xv[1], a);
  a = fmaf(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542)) - 8388608.0f, xv[2], a);
  a = fmaf(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543)) - 8388608.0f, xv[3], a);
  return a;  // = sum q_k x_k
}

// Columns per packed word and the additive code offset of word_dot.
template <int BITS> struct Codes;
template <> struct Codes<4> { static constexpr int kPerWord = 8; static constexpr float kOffset = 128.0f; };
template <> struct Codes<8> { static constexpr int kPerWord = 4; static constexpr float kOffset = 0.0f; };

// Loads the lane's slice of one token row: for j < WPL, columns
// [cpw*(lane + 32 j), cpw*(lane + 32 j) + cpw) as fp32, and their sums.
template <int BITS, int WPL>
__device__ __forceinline__ void load_x_slice(const uint16_t* __restrict__ xrow, int lane, int words_per_row,
                                             float (&xv)[WPL][Codes<BITS>::kPerWord], float (&xs)[WPL]) {
  constexpr int CPW = Codes<BITS>::kPerWord;
#pragma unroll
  for (int j = 0; j < WPL; ++j) {
    const int col = CPW * (lane + 32 * j);
    float s = 0.f;
    if (lane + 32 * j >= words_per_row) {
#pragma unroll
      for (int k = 0; k < CPW; ++k) xv[j][k] = 0.f;
    } else if constexpr (CPW == 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xrow + col);
      xv[j][0] = bf16_lo(v.x); xv[j][1] = bf16_hi(v.x);
      xv[j][2] = bf16_lo(v.y); xv[j][3] = bf16_hi(v.y);
      xv[j][4] = bf16_lo(v.z); xv[j][5] = bf16_hi(v.z);
      xv[j][6] = bf16_lo(v.w); xv[j][7] = bf16_hi(v.w);
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(xrow + col);
      xv[j][0] = bf16_lo(v.x); xv[j][1] = bf16_hi(v.x);
      xv[j][2] = bf16_lo(v.y); xv[j][3] = bf16_hi(v.y);
    }
#pragma unroll
    for (int k = 0; k < CPW; ++k) s += xv[j][k];
    xs[j] = s;
  }
}

// One projection row against the lane's x slice; returns the lane's partial.
template <int BITS, int WPL>
__device__ __forceinline__ float row_partial(const uint32_t* __restrict__ wrow, const uint16_t* __restrict__ srow,
                                             const uint16_t* __restrict__ brow, int lane, int words_per_row,
                                             const float (&xv)[WPL][Codes<BITS>::kPerWord],
                                             const float (&xs)[WPL]) {
  constexpr int CPW = Codes<BITS>::kPerWord;
  constexpr int WPG = 64 / CPW;  // words per 64-column group
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < WPL; ++j) {
    const int word = lane + 32 * j;
    if (word >= words_per_row) break;
    const uint32_t w = wrow[word];
    const float sc = bf16_bits_to_f32(srow[word / WPG]);
    const float bi = bf16_bits_to_f32(brow[word / WPG]);
    const float qx = word_dot<BITS>(w, xv[j]);
    acc = fmaf(sc, qx, acc);
    acc = fmaf(bi - Codes<BITS>::kOffset * sc, xs[j], acc);
  }
  return acc;
}

}  // namespace senmoe
