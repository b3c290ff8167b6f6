// dequant.cuh -- packed-weight -> bf16 conversions shared by the standalone
// dequantize kernel and the GEMM's dequant warps, so both produce identical
// bits.
//
// Affine (MLX "affine" mode, loader/transformer_cache.py:1255): the bf16
// weight is RNE_bf16(scale * q + bias) computed exactly: q is rebuilt as an
// exact bf16 value with the magic-number technique of Kim et al., "Who Says
// Elephants Can't Run" (2022) -- the code is OR-ed into the mantissa of a
// float whose exponent makes the integer part exact, and the bias of that
// float is subtracted -- and the affine map is a single fma.rn.bf16x2, i.e.
// one rounding of the exact scale*q + bias.
//
// MXFP8 (OCP MX v1.0): E4M3 bytes widened exactly through cvt.rn.f16x2.e4m3x2,
// scaled by the E8M0 power of two in fp32 (exact) and rounded once to bf16.
// For data without NaN codes and with scales <= 134 (LTXQ_QW_MXFP8_FINITE)
// a shorter form gives the same bits: an E4M3 byte's sign and 7 low bits,
// moved to bf16 bit 15 and bits 10:4, are the bf16 encoding of its value
// times 2^-120 (normal codes keep exponent and mantissa, subnormal codes
// become bf16 subnormals); one bf16 multiply by 2^(s-7) then scales and
// rounds it once.
#pragma once

#include "common.cuh"

namespace ltxq {

__device__ __forceinline__ uint32_t fma_bf16x2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t sub_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bcast_bf16x2(uint32_t bits16) { return (bits16 & 0xFFFFu) * 0x00010001u; }

// int8: one packed word (elements k..k+3) -> two bf16x2 words (k,k+1), (k+2,k+3).
__device__ __forceinline__ void deq_affine8_word(uint32_t w, uint32_t s2, uint32_t b2, uint32_t& o01,
                                                 uint32_t& o23) {
  constexpr float kMagic = 8388608.0f;  // 2^23: float(0x4B0000xx) = 2^23 + xx exactly
  const float q0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650)) - kMagic;
  const float q1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651)) - kMagic;
  const float q2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7652)) - kMagic;
  const float q3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7653)) - kMagic;
  // q < 256 has <= 8 significant bits, so the low 16 bits of its fp32
  // pattern are zero and the upper half is its exact bf16: the pairs are
  // packed by a byte permute (integer pipe), not a conversion.
  o01 = fma_bf16x2(s2, __byte_perm(__float_as_uint(q0), __float_as_uint(q1), 0x7632), b2);
  o23 = fma_bf16x2(s2, __byte_perm(__float_as_uint(q2), __float_as_uint(q3), 0x7632), b2);
}

// int4: one packed word (elements k..k+7, nibble i = element k+i) -> four
// bf16x2 words (k,k+1) .. (k+6,k+7).
__device__ __forceinline__ void deq_affine4_word(uint32_t w, uint32_t s2, uint32_t b2, uint32_t (&o)[4]) {
  const uint32_t u = w >> 4;
  constexpr uint32_t kMagic = 0x43004300u;  // bf16x2 (128, 128): 0x43xx = 128 + xx for xx < 128
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // byte0 <- byte j of w (low nibble = element 2j), byte2 <- byte j of w>>4
    // (low nibble = element 2j+1)
    const uint32_t t = __byte_perm(w, u, static_cast<uint32_t>(j) | (static_cast<uint32_t>(4 + j) << 8));
    const uint32_t x = (t & 0x000F000Fu) | kMagic;
    o[j] = fma_bf16x2(s2, sub_bf16x2(x, kMagic), b2);
  }
}

__device__ __forceinline__ float e8m0_to_f32(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);  // 2^-127 (fp32 subnormal)
  if (s == 255u) return __uint_as_float(0x7FC00000u);  // NaN code
  return __uint_as_float(s << 23);
}

// mxfp8: one packed word (4 E4M3 bytes, elements k..k+3) and the group's
// fp32 scale -> two bf16x2 words.
__device__ __forceinline__ void deq_mxfp8_word(uint32_t w, float scale, uint32_t& o01, uint32_t& o23) {
  uint32_t h01, h23;
  const uint16_t lo = static_cast<uint16_t>(w & 0xFFFFu), hi = static_cast<uint16_t>(w >> 16);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h01) : "h"(lo));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h23) : "h"(hi));
  const __half2 a = *reinterpret_cast<const __half2*>(&h01);
  const __half2 b = *reinterpret_cast<const __half2*>(&h23);
  o01 = pack_bf16x2(__low2float(a) * scale, __high2float(a) * scale);
  o23 = pack_bf16x2(__low2float(b) * scale, __high2float(b) * scale);
}

// bf16x2 broadcast of 2^(s - 7), the multiplier of the short mxfp8 form
// (exact for E8M0 codes s <= 134)
__device__ __forceinline__ uint32_t e8m0_fast_scale2(uint32_t s) { return ((s + 120u) << 7) * 0x00010001u; }

// bytes (lo, hi) of w picked by a prmt selector whose high nibbles replicate
// each byte's sign -> bf16x2 of (E4M3 value * 2^-120)
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2_m120(uint32_t w, uint32_t sel) {
  uint32_t t;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(t) : "r"(w), "r"(sel));
  return (t << 4) & 0x87F087F0u;
}

// mxfp8 short form (LTXQ_QW_MXFP8_FINITE data): s2 = e8m0_fast_scale2(s)
__device__ __forceinline__ void deq_mxfp8_word_fast(uint32_t w, uint32_t s2, uint32_t& o01, uint32_t& o23) {
  o01 = fma_bf16x2(e4m3x2_to_bf16x2_m120(w, 0x9180u), s2, 0x80008000u);
  o23 = fma_bf16x2(e4m3x2_to_bf16x2_m120(w, 0xB3A2u), s2, 0x80008000u);
}

}  // namespace ltxq
