// quant.cuh -- splitting an f32 activation into a sum of block-scaled E4M3
// terms (the operand format of kind::mxf8f6f4 with E8M0 scales).
//
// A block is 32 consecutive K elements held by the 32 lanes of one warp.  Term
// t is  code_t * 2^s_t  with s_t chosen so that the block's largest remaining
// magnitude fits E4M3 (<= 448); the residual after each term is exact in f32,
// so n terms carry about 4n significant bits: two terms reproduce a bf16 value
// exactly, three cover f32 inputs to ~2^-13.
#pragma once
#include <cuda_fp8.h>
#include <cstdint>

namespace mxmoe {

constexpr int kMaxTerms = 3;

// E8M0 exponent s (value 2^s) such that amax * 2^-s <= 448 (E4M3 max).
__device__ __forceinline__ int e4m3_block_exp(float amax) {
  const uint32_t bits = __float_as_uint(amax);
  const int ef = static_cast<int>((bits >> 23) & 0xFF);
  if (ef == 0) return -127;  // zero or subnormal block
  const uint32_t mant = bits & 0x7FFFFFu;
  const int s = (ef - 127) - (mant <= 0x600000u ? 8 : 7);  // 1.75 * 2^8 == 448
  return s < -127 ? -127 : (s > 127 ? 127 : s);
}

__device__ __forceinline__ float warp_max_abs(float v) {
  v = fabsf(v);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// Warp-collective: lane l holds element l of a 32-block.  Writes `terms`
// codes and the per-term E8M0 bytes (same in every lane).
__device__ __forceinline__ void split_e4m3_terms(float u, int terms, uint8_t (&code)[kMaxTerms],
                                                 uint8_t (&sbyte)[kMaxTerms]) {
  float r = u;
#pragma unroll
  for (int t = 0; t < kMaxTerms; ++t) {
    if (t < terms) {
      const int s = e4m3_block_exp(warp_max_abs(r));
      const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(ldexpf(r, -s), __NV_SATFINITE, __NV_E4M3);
      const float cv = __half2float(__half(__nv_cvt_fp8_to_halfraw(c, __NV_E4M3)));
      r = r - ldexpf(cv, s);
      code[t] = c;
      sbyte[t] = static_cast<uint8_t>(s + 127);
    }
  }
}

}  // namespace mxmoe

namespace mxmoe {

// Two f32 -> E4M3 codes in one instruction (lo lands in the low byte) and the
// exact decode of a code pair back to f32.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void dec_e4m3x2(uint32_t codes16, float& lo, float& hi) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(codes16)));
  lo = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
  hi = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 >> 16)));
}

// Thread-local variant: one thread owns a whole 32-element block `v` and
// writes `terms` x 32 codes (as 8 packed 32-bit words per term) plus the
// per-term E8M0 bytes.  Same arithmetic as split_e4m3_terms: the block
// exponent of every term keeps the block's largest residual within E4M3
// range, and each residual is exact in f32.
__device__ __forceinline__ void quantize_block32(float (&v)[32], int terms, uint32_t (&words)[kMaxTerms][8],
                                                 uint8_t (&sbyte)[kMaxTerms]) {
#pragma unroll
  for (int t = 0; t < kMaxTerms; ++t) {
    if (t < terms) {
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
      const int s = e4m3_block_exp(amax);
      // 2^-s and 2^s as normal floats when both exist; the extreme exponents
      // take the exact ldexpf path.
      const bool fast = (s > -126) && (s < 127);
      const float inv = fast ? __int_as_float((127 - s) << 23) : 0.0f;
      const float back = fast ? __int_as_float((127 + s) << 23) : 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          const int i = w * 4 + hp * 2;
          float a, b;
          if (fast) {
            a = v[i] * inv;
            b = v[i + 1] * inv;
          } else {
            a = ldexpf(v[i], -s);
            b = ldexpf(v[i + 1], -s);
          }
          const uint32_t c = cvt_e4m3x2(a, b);
          float da, db;
          dec_e4m3x2(c, da, db);
          if (fast) {
            v[i] = fmaf(-da, back, v[i]);
            v[i + 1] = fmaf(-db, back, v[i + 1]);
          } else {
            v[i] = v[i] - ldexpf(da, s);
            v[i + 1] = v[i + 1] - ldexpf(db, s);
          }
          word |= c << (16 * hp);
        }
        words[t][w] = word;
      }
      sbyte[t] = static_cast<uint8_t>(s + 127);
    }
  }
}

}  // namespace mxmoe
