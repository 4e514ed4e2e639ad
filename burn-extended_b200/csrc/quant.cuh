// quant.cuh -- splitting an f32 activation into a sum of block-scaled E4M3
// terms (the operand format of kind::mxf8f6f4 with E8M0 scales).
//
// A block is 32 consecutive K elements held by the 32 lanes of one warp.  Term
// t is  code_t * 2^s_t  with s_t chosen so that the block's largest remaining
// magnitude fits E4M3 (<= 448); the residual after each term is exact in f32,
// so n terms carry about 4n significant bits: two terms reproduce a bf16 value
// exactly, three cover f32 inputs to ~2^-13.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>

#include "layout.cuh"

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
      // 2^-s and 2^s as normal floats: a finite block has s <= 120, and a
      // block with s = -127 (amax below 2^-118) is written as zero codes
      const bool live = s > -127;
      const float inv = live ? __int_as_float((127 - s) << 23) : 0.0f;
      const float back = live ? __int_as_float((127 + s) << 23) : 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int hp = 0; hp < 2; ++hp) {
          const int i = w * 4 + hp * 2;
          const uint32_t c = cvt_e4m3x2(v[i] * inv, v[i + 1] * inv);
          float da, db;
          dec_e4m3x2(c, da, db);
          v[i] = fmaf(-da, back, v[i]);
          v[i + 1] = fmaf(-db, back, v[i + 1]);
          word |= c << (16 * hp);
        }
        words[t][w] = word;
      }
      sbyte[t] = static_cast<uint8_t>(s + 127);
    }
  }
}

}  // namespace mxmoe

namespace mxmoe {

// ---------------------------------------------------------------- E2M1 terms
// The FP4 decode operand: a sum of four block-scaled E2M1 terms (kind::mxf4).
// Term t of a 32-block is code_t * 2^s_t with s_t the smallest exponent that
// keeps the block's largest remaining magnitude within E2M1 range (<= 6); the
// residual after each term is exact in f32.  Each term removes two to three
// bits of the block's error, so four terms leave ~2^-9 of the block maximum.

// E8M0 exponent s (value 2^s) such that amax * 2^-s <= 6 (E2M1 max).
__device__ __forceinline__ int e2m1_block_exp(float amax) {
  const uint32_t bits = __float_as_uint(amax);
  const int ef = static_cast<int>((bits >> 23) & 0xFF);
  if (ef == 0) return -127;  // zero or subnormal block
  const uint32_t mant = bits & 0x7FFFFFu;
  const int s = (ef - 127) - (mant <= 0x400000u ? 2 : 1);  // 1.5 * 2^2 == 6
  return s < -127 ? -127 : (s > 127 ? 127 : s);
}

// Eight f32 -> eight E2M1 codes, element 2i in the low nibble of byte i.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float* a) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(a[0]), "f"(a[1]), "f"(a[2]), "f"(a[3]), "f"(a[4]), "f"(a[5]), "f"(a[6]), "f"(a[7]));
  return r;
}

// Exact value of one E2M1 code (sign bit 3, exponent bits 2..1, mantissa
// bit 0), built as f32 bits with integer operations.  The residual update
// decodes the codes it just packed this way rather than with the
// e2m1x2 -> f16x2 conversion, whose byte-register inputs did not survive
// being packed and unpacked within one function.
__device__ __forceinline__ float e2m1_value(uint32_t c) {
  const uint32_t e = (c >> 1) & 3u, m = c & 1u;
  uint32_t bits = e ? (((e + 126u) << 23) | (m << 22)) : (m ? 0x3F000000u : 0u);
  bits |= (c & 8u) << 28;
  return __uint_as_float(bits);
}

// Lane-pair cooperative: this lane holds 16 elements of a 32-block whose
// other half sits in lane ^ xor_mask.  Writes the four terms' codes (16
// nibbles = two words per term) and E8M0 bytes (equal in both lanes).  Every
// lane of the warp must call it (the block maximum is a shuffle).
__device__ __forceinline__ void quantize16_e2m1_terms(float (&v)[16], int xor_mask, uint32_t (&words)[kF4Terms][2],
                                                      uint8_t (&sbyte)[kF4Terms]) {
#pragma unroll
  for (int t = 0; t < kF4Terms; ++t) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, xor_mask));
    // A finite block never needs s > 126; s = -127 (amax below 2^-125) is
    // written as zero codes with the smallest scale, leaving the residual as is.
    const int s = e2m1_block_exp(amax);
    const bool live = s > -127;
    const float inv = live ? __int_as_float((127 - s) << 23) : 0.0f;
    const float back = live ? __int_as_float((127 + s) << 23) : 0.0f;
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      float sc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sc[i] = v[8 * w + i] * inv;
      const uint32_t c = cvt_e2m1x8(sc);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[8 * w + i] = fmaf(-e2m1_value(c >> (4 * i)), back, v[8 * w + i]);
      words[t][w] = c;
    }
    sbyte[t] = static_cast<uint8_t>(s + 127);
  }
}

}  // namespace mxmoe

namespace mxmoe {

// Lane-quad variant of quantize16_e2m1_terms: this lane holds 8 elements of
// a 32-block spread over lanes l, l ^ 1, l ^ 2, l ^ 3 (one code word per
// term).  Same arithmetic; every lane of the warp must call it.
__device__ __forceinline__ void quantize8_e2m1_terms(float (&v)[8], uint32_t (&words)[kF4Terms],
                                                     uint8_t (&sbyte)[kF4Terms]) {
#pragma unroll
  for (int t = 0; t < kF4Terms; ++t) {
    float m0 = fmaxf(fabsf(v[0]), fabsf(v[1])), m1 = fmaxf(fabsf(v[2]), fabsf(v[3]));
    float m2 = fmaxf(fabsf(v[4]), fabsf(v[5])), m3 = fmaxf(fabsf(v[6]), fabsf(v[7]));
    float amax = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
    const int s = e2m1_block_exp(amax);
    const bool live = s > -127;
    const float inv = live ? __int_as_float((127 - s) << 23) : 0.0f;
    const float back = live ? __int_as_float((127 + s) << 23) : 0.0f;
    float sc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) sc[i] = v[i] * inv;
    const uint32_t c = cvt_e2m1x8(sc);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = fmaf(-e2m1_value(c >> (4 * i)), back, v[i]);
    words[t] = c;
    sbyte[t] = static_cast<uint8_t>(s + 127);
  }
}

}  // namespace mxmoe
