// dequant.cuh -- affine 4-bit code -> fp16 weight conversions shared by the
// tensor-core expert kernels (tcgen05 and warp-level MMA).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

namespace senmoe {

// 8 consecutive 4-bit codes (one u32) -> 8 fp16 w = q * s + b, k-permuted.
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
  return make_uint4(o[0], o[1], o[2], o[3]);  // (0,4),(1,5),(2,6),(3,7)
}

// Same result through fp16 subnormals: (w << 6, << 2, >> 2, >> 6) & 0x03C003C0
// puts code k (and k + 4) in mantissa bits 6-9, i.e. the fp16 value q * 2^-18,
// and fma(q * 2^-18, s * 2^18, b) = q * s + b with one rounding.  s * 2^18 is
// exact in fp16 for 2^-32 < |s| < 0.2498; callers use dequant8_u4 otherwise.
__device__ __forceinline__ uint4 dequant8_u4_sub(uint32_t w, __half2 s18, __half2 b2) {
  const uint32_t m = 0x03C003C0u;
  const uint32_t v0 = (w << 6) & m, v1 = (w << 2) & m, v2 = (w >> 2) & m, v3 = (w >> 6) & m;
  __half2 r0 = __hfma2(*reinterpret_cast<const __half2*>(&v0), s18, b2);
  __half2 r1 = __hfma2(*reinterpret_cast<const __half2*>(&v1), s18, b2);
  __half2 r2 = __hfma2(*reinterpret_cast<const __half2*>(&v2), s18, b2);
  __half2 r3 = __hfma2(*reinterpret_cast<const __half2*>(&v3), s18, b2);
  return make_uint4(*reinterpret_cast<uint32_t*>(&r0), *reinterpret_cast<uint32_t*>(&r1),
                    *reinterpret_cast<uint32_t*>(&r2), *reinterpret_cast<uint32_t*>(&r3));
}

// Same result with the codes at mantissa bits 4-7 (q * 2^-20): (w << 4, w,
// w >> 4, w >> 8) & 0x00F000F0 -- one operation fewer per word (pair (1,5)
// needs no shift).  s * 2^20 is exact in fp16 for 2^-34 < |s| < 0.0624.
__device__ __forceinline__ uint4 dequant8_u4_sub20(uint32_t w, __half2 s20, __half2 b2) {
  const uint32_t m = 0x00F000F0u;
  const uint32_t v0 = (w << 4) & m, v1 = w & m, v2 = (w >> 4) & m, v3 = (w >> 8) & m;
  __half2 r0 = __hfma2(*reinterpret_cast<const __half2*>(&v0), s20, b2);
  __half2 r1 = __hfma2(*reinterpret_cast<const __half2*>(&v1), s20, b2);
  __half2 r2 = __hfma2(*reinterpret_cast<const __half2*>(&v2), s20, b2);
  __half2 r3 = __hfma2(*reinterpret_cast<const __half2*>(&v3), s20, b2);
  return make_uint4(*reinterpret_cast<uint32_t*>(&r0), *reinterpret_cast<uint32_t*>(&r1),
                    *reinterpret_cast<uint32_t*>(&r2), *reinterpret_cast<uint32_t*>(&r3));
}

}  // namespace senmoe
