// gemm_epilogue.cuh -- pieces shared by the quantized GEMM kernels (qgemm.cu
// for the dequantizing path, mx.cu for the native block-scaled fp8 path):
// the launch parameters, the reference's GELU with its per-op bf16 rounding
// (exact table form), named barriers and the epilogue's row store with the
// gated residual fused.
#pragma once

#include "common.cuh"

namespace ltxq {
namespace gemm {

struct Params {
  int M, N, K, gs;
  int vec_groups;  // group parameters of a row are 16-byte aligned blocks (see GroupCursor)
  const void* scales;
  const uint16_t* biases;
  const uint16_t* bias;
  int epi;
  VecArg gate;
  const uint16_t* residual;
  uint16_t* out;
  unsigned int* err;
  // pair-kernel schedule: output tiles [0, dp_tiles) are computed whole; each
  // later tile is split into `splits` K ranges whose fp32 partials go to
  // `partial` ([tile - dp_tiles][split][256 tokens][256 features], tile-local)
  // and are summed by splitk_reduce_kernel
  int dp_tiles;
  int splits;
  float* partial;
};

// gelu_approx with the reference's per-op bf16 rounding (feed_forward.py:8-14;
// MLX evaluates each op of the expression on bf16 arrays, the constants
// 0.044715 and sqrt(2/pi) taking the bf16 values below).
__device__ __forceinline__ float gelu_ref(float x) {
  constexpr float c1 = 0.044677734375f;  // bf16(0.044715)
  constexpr float c2 = 0.796875f;        // bf16(sqrt(2/pi))
  const float x3 = rbf16(__fmul_rn(__fmul_rn(x, x), x));  // exact in fp32 for bf16 x
  float t = rbf16(__fmul_rn(c1, x3));
  t = rbf16(__fadd_rn(x, t));
  t = rbf16(__fmul_rn(c2, t));
  t = rbf16(tanhf(t));
  t = rbf16(__fadd_rn(1.0f, t));
  const float h = rbf16(__fmul_rn(0.5f, x));
  return rbf16(__fmul_rn(h, t));
}

// gelu_ref through a table.  Over all 65536 bf16 inputs gelu_ref(x) equals
// bf16(0.5 x) for |x| < 2^-9 (its 1 + tanh term rounds to 1), x for x >= 4
// (tanh rounds to 1), -0 for finite x <= -4 (1 + tanh rounds to 0) and NaN
// for -inf / NaN.  Between, the result is read from a table of gelu_ref
// values built by the kernel itself, so both forms give the same bits.
// Magnitudes [kGeluLo, kGeluLo + kGeluN) are tabulated, positive then negative.
constexpr uint32_t kGeluLo = 0x3B00u;  // 2^-9
constexpr uint32_t kGeluN = 0x4080u - kGeluLo;  // up to 4.0 (exclusive)
constexpr int kGeluTabBytes = static_cast<int>(2 * kGeluN * 2);

// b: bf16 bits (low 16), small: bf16 bits of bf16(0.5 b); returns the bf16
// bits of gelu_ref(b)
__device__ __forceinline__ uint32_t gelu_tab_sel(uint32_t b, uint32_t small, const uint16_t* tab) {
  const uint32_t mag = b & 0x7FFFu, neg = b >> 15;
  const uint32_t t = mag - kGeluLo;  // wraps for mag < kGeluLo
  const bool in_tab = t < kGeluN;
  const uint32_t tv = tab[in_tab ? t + neg * kGeluN : 0u];
  const uint32_t big = neg ? (mag >= 0x7F80u ? 0x7FC0u : 0x8000u) : b;
  return in_tab ? tv : (mag < kGeluLo ? small : big);
}

// gelu_ref on both halves of a bf16x2 word (one paired conversion for the
// small-input form)
__device__ __forceinline__ uint32_t gelu_tab_x2(uint32_t b2, const uint16_t* tab) {
  const uint32_t small2 = pack_bf16x2(__fmul_rn(0.5f, __uint_as_float(b2 << 16)),
                                      __fmul_rn(0.5f, __uint_as_float(b2 & 0xFFFF0000u)));
  return gelu_tab_sel(b2 & 0xFFFFu, small2 & 0xFFFFu, tab) | (gelu_tab_sel(b2 >> 16, small2 >> 16, tab) << 16);
}

// fills the table (n_threads threads, thread id tid); caller synchronizes
__device__ __forceinline__ void gelu_tab_fill(uint16_t* tab, int tid, int n_threads) {
  for (int i = tid; i < static_cast<int>(2 * kGeluN); i += n_threads) {
    const uint32_t neg = static_cast<uint32_t>(i) >= kGeluN;
    const uint32_t mag = kGeluLo + static_cast<uint32_t>(i) - (neg ? kGeluN : 0u);
    tab[i] = f32_to_bf16(gelu_ref(__uint_as_float(((neg << 15) | mag) << 16)));
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Row side of the smem-A epilogue: u = bf16x2 words of 8 consecutive
// features (bias / GELU already applied); gated residual, then a 16-byte store.
__device__ __forceinline__ void epi_row_store(const Params& p, uint32_t (&u)[4], int m, int nf, const float (&g8b)[8],
                                              bool gated, bool two_round, bool gate_bcast) {
  const int64_t off = static_cast<int64_t>(m) * p.N + nf;
  if (gated) {
    const uint4 rv = __ldg(reinterpret_cast<const uint4*>(p.residual + off));
    const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
    float g8[8];
    if (gate_bcast) {
#pragma unroll
      for (int k = 0; k < 8; ++k) g8[k] = g8b[k];
    } else {
      load_vec8(p.gate, vec_row(p.gate, m), nf, g8);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float p0 = __fmul_rn(lo_bf16(u[k]), g8[2 * k]);
      const float p1 = __fmul_rn(hi_bf16(u[k]), g8[2 * k + 1]);
      const float r0 = lo_bf16(rw[k]), r1 = hi_bf16(rw[k]);
      if (two_round) {
        const uint32_t pr = pack_bf16x2(p0, p1);
        u[k] = pack_bf16x2(__fadd_rn(r0, lo_bf16(pr)), __fadd_rn(r1, hi_bf16(pr)));
      } else {
        u[k] = pack_bf16x2(__fadd_rn(p0, r0), __fadd_rn(p1, r1));
      }
    }
  }
  *reinterpret_cast<uint4*>(p.out + off) = make_uint4(u[0], u[1], u[2], u[3]);
}

}  // namespace gemm
}  // namespace ltxq
