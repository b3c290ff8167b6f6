// mx_act.cuh -- MXFP8 activation terms (the input form of the block-scaled
// fp8 GEMM in mx.cu), shared by the standalone splitter and by the kernels
// that write their outputs directly in this form (the AdaLN pass, the head
// gate, the GEMM epilogue), so that every writer produces the same bits.
//
// Per group of 32 consecutive K of a row: E8M0 scale 2^e with the smallest
// e >= -127 for which max|v| * 2^-e <= 448, E4M3 codes RNE(v * 2^-e); the
// second term quantizes the exact residual v - decode(hi) the same way.
// Codes: [M, K] bytes per term.  Scales: atom (k-tile j = k / 128, row tile
// t = m / 128) at (j * row_tiles + t) * 512 holds the scale of row
// t*128 + 32*m1 + m0, group 4j + k1 at byte m0*16 + m1*4 + k1.
#pragma once

#include "common.cuh"

namespace ltxq {
namespace mx {

constexpr int kGroup = 32;   // K values per E8M0 scale
constexpr int kAtom = 512;   // scale-factor atom: 128 rows x 4 groups (one 128-K tile)

// ---------------------------------------------------------------- numerics

// E8M0 exponent of a group whose largest magnitude is amax: the smallest e
// with amax * 2^-e <= 448, and at least -127 (the smallest E8M0 value).
__device__ __forceinline__ int group_exp(float amax) {
  const uint32_t b = __float_as_uint(amax);
  const int ef = static_cast<int>(b >> 23);
  if (ef == 0) return -127;  // zero or an fp32 subnormal
  // amax = m 2^E, m in [1, 2): 256 m <= 448 exactly when m <= 1.75
  const int e = ef - 127 - 8 + ((b & 0x7FFFFFu) > 0x600000u ? 1 : 0);
  return e < -127 ? -127 : e;
}

// 2^e for e in [-127, 127]
__device__ __forceinline__ float exp2i(int e) {
  return e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23) : __uint_as_float(0x00400000u);
}

// four fp32 values -> four E4M3 codes (RNE, saturating at +-448), value 0 in the low byte
__device__ __forceinline__ uint32_t to_e4m3x4(float a0, float a1, float a2, float a3) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(a1), "f"(a0));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(a3), "f"(a2));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// the exact values of four E4M3 codes (code 0 = low byte)
__device__ __forceinline__ void e4m3x4_values(uint32_t c, float (&v)[4]) {
  uint32_t h0, h1;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h0) : "h"(static_cast<uint16_t>(c & 0xFFFFu)));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h1) : "h"(static_cast<uint16_t>(c >> 16)));
  v[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(h0 & 0xFFFFu)));
  v[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(h0 >> 16)));
  v[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(h1 & 0xFFFFu)));
  v[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(h1 >> 16)));
}

// Converts the 32 values of v (in place) to one MX term: codes c, E8M0 byte
// s; v becomes the residual v - decode(c) * 2^e when kResidual.
template <bool kResidual>
__device__ __forceinline__ void mx_term(float (&v)[32], uint32_t (&c)[8], uint32_t& s) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  const int e = group_exp(amax);
  const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e, e in [-127, 121]
  s = static_cast<uint32_t>(e + 127);
#pragma unroll
  for (int w = 0; w < 8; ++w)
    c[w] = to_e4m3x4(v[4 * w] * inv, v[4 * w + 1] * inv, v[4 * w + 2] * inv, v[4 * w + 3] * inv);
  if (kResidual) {
    const float sc = exp2i(e);
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      float d[4];
      e4m3x4_values(c[w], d);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * w + i] = __fsub_rn(v[4 * w + i], __fmul_rn(d[i], sc));  // exact
    }
  }
}


// Where a writer puts MX terms: codes [M, K] per term, scale atoms per term.
struct MxOut {
  uint8_t* hi;
  uint8_t* lo;
  uint8_t* sf_hi;
  uint8_t* sf_lo;
  int64_t K;       // row length (codes per row)
  int row_tiles;   // atoms per k-tile: ceil(M / 128) + 1
  int terms;       // 1 or 2
};

// Host side: an ltxq_mx_act is usable (1 or 2 terms, the pointers the term
// count needs, 16-byte aligned).
inline bool act_ok(const ltxq_mx_act* a) {
  if (!a || (a->terms != 1 && a->terms != 2) || !a->hi || !a->sf_hi) return false;
  if (a->terms == 2 && (!a->lo || !a->sf_lo)) return false;
  const uintptr_t bits = reinterpret_cast<uintptr_t>(a->hi) | reinterpret_cast<uintptr_t>(a->sf_hi) |
                         (a->terms == 2 ? reinterpret_cast<uintptr_t>(a->lo) | reinterpret_cast<uintptr_t>(a->sf_lo)
                                        : 0);
  return (bits & 15u) == 0;
}

// The writer's view of an ltxq_mx_act holding M rows of K values.
inline MxOut out_of(const ltxq_mx_act& a, int64_t M, int64_t K) {
  return MxOut{static_cast<uint8_t*>(a.hi), static_cast<uint8_t*>(a.lo), static_cast<uint8_t*>(a.sf_hi),
               static_cast<uint8_t*>(a.sf_lo), K, static_cast<int>((M + 127) / 128 + 1), a.terms};
}

// byte offset of the scale of (row m, group g) in the atom layout
__device__ __forceinline__ int64_t mx_scale_offset(int64_t m, int64_t g, int row_tiles) {
  const int mi = static_cast<int>(m & 127);
  return ((g >> 2) * row_tiles + (m >> 7)) * kAtom + (mi & 31) * 16 + (mi >> 5) * 4 + (g & 3);
}

// One group's term from eight values per lane of a quad: lanes q4..q4+3
// (q4 = lane & ~3, all four calling together, `mask` holding their bits) own
// the group's values in column order, eight each.  Returns this lane's two
// code words and the scale byte; v becomes the residual when kResidual.
template <bool kResidual>
__device__ __forceinline__ void mx_quad_term(float (&v)[8], uint32_t mask, uint32_t (&c)[2], uint32_t& s) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(mask, amax, 2));
  const int e = group_exp(amax);
  const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
  s = static_cast<uint32_t>(e + 127);
  c[0] = to_e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv);
  c[1] = to_e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv);
  if (kResidual) {
    const float sc = exp2i(e);
#pragma unroll
    for (int w = 0; w < 2; ++w) {
      float d[4];
      e4m3x4_values(c[w], d);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[4 * w + i] = __fsub_rn(v[4 * w + i], __fmul_rn(d[i], sc));  // exact
    }
  }
}

// Writes eight consecutive bf16 values u (row m, columns [c, c + 8), c % 8
// == 0) as MX terms.  The four lanes of this lane's quad must hold the rest
// of the 32-column group (columns c - 8 (lane & 3) ... in lane order) and
// call together with `mask` (their lane bits).  The same numerics as
// mx_split_kernel, so the same bits.
__device__ __forceinline__ void mx_write8(const uint32_t (&u)[4], int64_t m, int64_t c, const MxOut& o,
                                          uint32_t mask) {
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = lo_bf16(u[i]);
    v[2 * i + 1] = hi_bf16(u[i]);
  }
  uint32_t cw[2], s;
  const bool lead = (threadIdx.x & 3) == 0;
  const int64_t soff = mx_scale_offset(m, c >> 5, o.row_tiles);
  if (o.terms == 2) mx_quad_term<true>(v, mask, cw, s);
  else mx_quad_term<false>(v, mask, cw, s);
  *reinterpret_cast<uint2*>(o.hi + m * o.K + c) = make_uint2(cw[0], cw[1]);
  if (lead) o.sf_hi[soff] = static_cast<uint8_t>(s);
  if (o.terms == 2) {
    mx_quad_term<false>(v, mask, cw, s);
    *reinterpret_cast<uint2*>(o.lo + m * o.K + c) = make_uint2(cw[0], cw[1]);
    if (lead) o.sf_lo[soff] = static_cast<uint8_t>(s);
  }
}

}  // namespace mx
}  // namespace ltxq
