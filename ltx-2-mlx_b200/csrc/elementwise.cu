// elementwise.cu -- HBM-bound kernels of the block: AdaLN norm+modulate
// (fused_ops.py:237 adaln_norm_fused / transformer.py:21-37), the gated
// residual add (fused_ops.py:398 / transformer.py:40-50, 387) and the
// per-head attention output gate (attention.py:559-601).
//
// Rounding points follow the reference composition: rms_norm/layer_norm
// output rounded to bf16; fp32 AdaLN vectors give fp32 product and sum (no
// FMA contraction) and one bf16 rounding; bf16 vectors round after every op.
// Row statistics are accumulated in fp64 so that they are independent of the
// reduction order.
#include "common.cuh"
#include "mx_act.cuh"

namespace ltxq {

__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// modulate one element: normed (bf16-exact for bf16 output) * (1+s) + t
template <bool kVecBf16>
__device__ __forceinline__ float modulate1(float n, float s, float t) {
  if (kVecBf16) {
    const float one_p = rbf16(__fadd_rn(1.0f, s));
    return __fadd_rn(rbf16(__fmul_rn(n, one_p)), t);
  }
  return __fadd_rn(__fmul_rn(n, __fadd_rn(1.0f, s)), t);
}

// One CTA per row; each thread owns up to 16 consecutive channels (two
// 16-byte chunks of bf16).  kXF32: x/out are fp32 (the reference's fp32
// fallback keeps fp32 output without rounding).
template <bool kXF32, bool kVecBf16>
__global__ void __launch_bounds__(512) adaln_modulate_kernel(const void* __restrict__ x, int64_t C, int norm,
                                                              float eps, VecArg scale, VecArg shift,
                                                              void* __restrict__ out) {
  __shared__ double red[32];
  const double inv_c = 1.0 / static_cast<double>(C);
  const int64_t row = blockIdx.x;
  const int64_t c0 = static_cast<int64_t>(threadIdx.x) * 16;
  float v[16];
  int nvalid = 0;
  if (c0 < C) nvalid = (C - c0 >= 16) ? 16 : static_cast<int>(C - c0);  // 8 or 16 (C % 8 == 0)
  if (kXF32) {
    const float* xr = static_cast<const float*>(x) + row * C;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h * 8 < nvalid) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr + c0 + h * 8));
        const float4 b = __ldg(reinterpret_cast<const float4*>(xr + c0 + h * 8 + 4));
        v[h * 8 + 0] = a.x; v[h * 8 + 1] = a.y; v[h * 8 + 2] = a.z; v[h * 8 + 3] = a.w;
        v[h * 8 + 4] = b.x; v[h * 8 + 5] = b.y; v[h * 8 + 6] = b.z; v[h * 8 + 7] = b.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[h * 8 + i] = 0.f;
      }
    }
  } else {
    const uint16_t* xr = static_cast<const uint16_t*>(x) + row * C;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h * 8 < nvalid) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(xr + c0 + h * 8));
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[h * 8 + 2 * i] = lo_bf16(w[i]);
          v[h * 8 + 2 * i + 1] = hi_bf16(w[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[h * 8 + i] = 0.f;
      }
    }
  }

  float mu_f = 0.f, inv = 1.f;
  if (norm == LTXQ_NORM_RMS) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 16; ++i) ss += static_cast<double>(v[i]) * static_cast<double>(v[i]);
    const double tot = block_sum(ss, red);
    const float ms = static_cast<float>(tot * inv_c);
    inv = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(ms, eps))));
  } else if (norm == LTXQ_NORM_LAYER) {
    double s1 = 0.0;
#pragma unroll
    for (int i = 0; i < 16; ++i) s1 += static_cast<double>(v[i]);
    const double mu = block_sum(s1, red) * inv_c;
    double s2 = 0.0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < nvalid) {
        const double d = static_cast<double>(v[i]) - mu;
        s2 += d * d;
      }
    }
    const float var = static_cast<float>(block_sum(s2, red) * inv_c);
    inv = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(var, eps))));
    mu_f = static_cast<float>(mu);
  }
  if (nvalid == 0) return;

  const char* sc = vec_row(scale, row);
  const char* sh = vec_row(shift, row);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (h * 8 >= nvalid) break;
    float s[8], t[8], o[8];
    load_vec8(scale, sc, c0 + h * 8, s);
    load_vec8(shift, sh, c0 + h * 8, t);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float n = v[h * 8 + i];
      if (norm == LTXQ_NORM_RMS) n = __fmul_rn(n, inv);
      else if (norm == LTXQ_NORM_LAYER) n = __fmul_rn(__fsub_rn(n, mu_f), inv);
      if (!kXF32) n = rbf16(n);
      o[i] = modulate1<kVecBf16>(n, s[i], t[i]);
    }
    if (kXF32) {
      float* orow = static_cast<float*>(out) + row * C + c0 + h * 8;
      reinterpret_cast<float4*>(orow)[0] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(orow)[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
      uint4 pk;
      pk.x = pack_bf16x2(o[0], o[1]);
      pk.y = pack_bf16x2(o[2], o[3]);
      pk.z = pack_bf16x2(o[4], o[5]);
      pk.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + row * C + c0 + h * 8) = pk;
    }
  }
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row tiles for bf16 rows of C <= 256 * 8 * kCPT channels: a CTA of 256
// threads takes kR consecutive rows; thread t owns the 8-channel chunks
// t + 256 j (j < kCPT) of every row, so all kR * kCPT 16-byte loads of a
// thread are in flight at once, and the scale / shift entries of a chunk are
// loaded once for the kR rows when the rows share their vectors.  RMS
// statistics: an fp32 sum of squares per thread and row (the reference's
// fp32 mean, up to its last ulp), added across threads in fp64 in a fixed
// order; LayerNorm sums and centred squares in fp64.  One thread per row
// forms 1/sqrt.  kMx: the result is written as MX terms (C % 128 == 0: the
// four lanes of a quad hold one 32-channel group of one row) and, when
// out != NULL, also as bf16 rows.
constexpr int kTileThreads = 256;

template <int kR, int kCPT, int kNorm, bool kVecBf16, bool kMx>
__global__ void __launch_bounds__(kTileThreads, kNorm == LTXQ_NORM_LAYER ? 2 : 3)
    adaln_tile_kernel(const uint16_t* __restrict__ x, int64_t rows, int C, float eps, VecArg scale, VecArg shift,
                      uint16_t* __restrict__ out, const mx::MxOut mo) {
  constexpr int kWarps = kTileThreads / 32;
  __shared__ double red[kWarps][kR];
  __shared__ float inv_s[kR], mu_s[kR];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kR;
  const int nch = C >> 3;
  uint4 v[kR][kCPT];
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int j = 0; j < kCPT; ++j) {
      const int c = threadIdx.x + kTileThreads * j;
      v[r][j] = (r0 + r < rows && c < nch) ? __ldg(reinterpret_cast<const uint4*>(x + (r0 + r) * C) + c)
                                          : make_uint4(0, 0, 0, 0);
    }
  const double inv_c = __drcp_rn(static_cast<double>(C));
  if constexpr (kNorm == LTXQ_NORM_RMS) {
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      float q = 0.f;
#pragma unroll
      for (int j = 0; j < kCPT; ++j) {
        const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          q = __fmaf_rn(hi_bf16(w[i]), hi_bf16(w[i]), __fmaf_rn(lo_bf16(w[i]), lo_bf16(w[i]), q));
      }
      const double d = warp_sum(static_cast<double>(q));
      if (lane == 0) red[warp][r] = d;
    }
    __syncthreads();
    if (threadIdx.x < kR) {
      double t = 0.0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += red[w][threadIdx.x];
      const float ms = static_cast<float>(t * inv_c);
      inv_s[threadIdx.x] = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(ms, eps))));
      mu_s[threadIdx.x] = 0.f;
    }
    __syncthreads();
  } else if constexpr (kNorm == LTXQ_NORM_LAYER) {
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      double s1 = 0.0;
#pragma unroll
      for (int j = 0; j < kCPT; ++j) {
        const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) s1 += static_cast<double>(lo_bf16(w[i])) + static_cast<double>(hi_bf16(w[i]));
      }
      s1 = warp_sum(s1);
      if (lane == 0) red[warp][r] = s1;
    }
    __syncthreads();
    double mu[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      double t = 0.0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += red[w][r];
      mu[r] = t * inv_c;
    }
    __syncthreads();  // red is reused for the centred squares
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      double d2 = 0.0;
#pragma unroll
      for (int j = 0; j < kCPT; ++j) {
        if (threadIdx.x + kTileThreads * j < nch) {
          const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const double a = lo_bf16(w[i]) - mu[r], b = hi_bf16(w[i]) - mu[r];
            d2 += a * a + b * b;
          }
        }
      }
      d2 = warp_sum(d2);
      if (lane == 0) red[warp][r] = d2;
    }
    __syncthreads();
    if (threadIdx.x < kR) {
      double t = 0.0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += red[w][threadIdx.x];
      const float var = static_cast<float>(t * inv_c);
      inv_s[threadIdx.x] = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(var, eps))));
      mu_s[threadIdx.x] = static_cast<float>(mu[threadIdx.x]);
    }
    __syncthreads();
  }
  // the kR rows read the same vector entries (broadcast, or one vector per
  // group of rows that the tile does not straddle)
  const bool shared_vec = (scale.rows_per_vec == 0 || (scale.rows_per_vec % kR) == 0) &&
                          (shift.rows_per_vec == 0 || (shift.rows_per_vec % kR) == 0);
#pragma unroll
  for (int j = 0; j < kCPT; ++j) {
    const int c = threadIdx.x + kTileThreads * j;
    if (c >= nch) break;
    float s8[8], t8[8];
    if (shared_vec) {
      load_vec8(scale, vec_row(scale, r0), static_cast<int64_t>(c) * 8, s8);
      load_vec8(shift, vec_row(shift, r0), static_cast<int64_t>(c) * 8, t8);
    }
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int64_t row = r0 + r;
      if (row >= rows) break;
      if (!shared_vec) {
        load_vec8(scale, vec_row(scale, row), static_cast<int64_t>(c) * 8, s8);
        load_vec8(shift, vec_row(shift, row), static_cast<int64_t>(c) * 8, t8);
      }
      const float inv = kNorm == LTXQ_NORM_NONE ? 1.f : inv_s[r];
      const float mu_f = kNorm == LTXQ_NORM_LAYER ? mu_s[r] : 0.f;
      const uint32_t w[4] = {v[r][j].x, v[r][j].y, v[r][j].z, v[r][j].w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float e[2] = {lo_bf16(w[i]), hi_bf16(w[i])};
        if (kNorm != LTXQ_NORM_NONE) {
          // the norm's bf16 rounding, two values per conversion
          const uint32_t nw = kNorm == LTXQ_NORM_RMS
                                  ? pack_bf16x2(__fmul_rn(e[0], inv), __fmul_rn(e[1], inv))
                                  : pack_bf16x2(__fmul_rn(__fsub_rn(e[0], mu_f), inv),
                                                __fmul_rn(__fsub_rn(e[1], mu_f), inv));
          e[0] = lo_bf16(nw);
          e[1] = hi_bf16(nw);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) e[h] = modulate1<kVecBf16>(e[h], s8[2 * i + h], t8[2 * i + h]);
        o[i] = pack_bf16x2(e[0], e[1]);
      }
      if (kMx) mx::mx_write8(o, row, static_cast<int64_t>(c) * 8, mo, 0xFu << (lane & ~3));
      if (out != nullptr) reinterpret_cast<uint4*>(out + row * C)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// out = residual + gate * branch over bf16 [rows, C]; 8 channels per thread.
template <bool kVecBf16, bool kTwoRound>
__global__ void gated_add_kernel(const uint16_t* __restrict__ res, const uint16_t* __restrict__ br, VecArg gate,
                                 int64_t rows, int64_t C, uint16_t* __restrict__ out) {
  const int64_t chunks_per_row = C >> 3;
  const int64_t total = rows * chunks_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / chunks_per_row;
    const int64_t c = (i - row * chunks_per_row) << 3;
    const uint4 r4 = __ldg(reinterpret_cast<const uint4*>(res + row * C + c));
    const uint4 b4 = __ldg(reinterpret_cast<const uint4*>(br + row * C + c));
    float g[8];
    load_vec8(gate, vec_row(gate, row), c, g);
    const uint32_t rw[4] = {r4.x, r4.y, r4.z, r4.w};
    const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float o2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float r = h ? hi_bf16(rw[k]) : lo_bf16(rw[k]);
        const float b = h ? hi_bf16(bw[k]) : lo_bf16(bw[k]);
        const float p = __fmul_rn(b, g[2 * k + h]);
        o2[h] = (kVecBf16 || kTwoRound) ? __fadd_rn(r, rbf16(p)) : __fadd_rn(p, r);
      }
      ow[k] = pack_bf16x2(o2[0], o2[1]);
    }
    *reinterpret_cast<uint4*>(out + row * C + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
  }
}

// out[m, h, :] = o[m, h, :] * bf16(2 * bf16(sigmoid(logit[m, h]))); one
// thread per 8 channels.  Row m's logits start at logits + m * lstride (a
// column slice of a fused projection output needs no copy).
// kMx: as adaln_tile_kernel's (width % 128 == 0: the grid stride and the row
// width are multiples of 4 chunks, so a quad stays one 32-channel group).
template <bool kMx>
__global__ void head_gate_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ logits, int64_t lstride,
                                 int64_t rows, int64_t heads, int64_t head_dim, uint16_t* __restrict__ out,
                                 const mx::MxOut mo) {
  const int64_t width = heads * head_dim;
  const int64_t total = rows * (width >> 3);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / (width >> 3);
    const int64_t c = (i - row * (width >> 3)) << 3;
    const int64_t h = c / head_dim;
    const double lg = static_cast<double>(bf16_to_f32(__ldg(logits + row * lstride + h)));
    const float sig = rbf16(static_cast<float>(1.0 / (1.0 + exp(-lg))));
    const float g = rbf16(__fmul_rn(2.0f, sig));
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(o + row * width + c));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
    uint32_t r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) r[k] = pack_bf16x2(__fmul_rn(lo_bf16(w[k]), g), __fmul_rn(hi_bf16(w[k]), g));
    if (kMx) mx::mx_write8(r, row, c, mo, 0xFu << (threadIdx.x & 28));
    if (out != nullptr) *reinterpret_cast<uint4*>(out + row * width + c) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static ltxq_status check_vec(const ltxq_vec& v, int64_t C, const char* name) {
  if (!v.ptr) return fail(LTXQ_ERR_INVALID, std::string(name) + " pointer is NULL");
  if (v.dtype != LTXQ_BF16 && v.dtype != LTXQ_F32)
    return fail(LTXQ_ERR_UNSUPPORTED, std::string(name) + " dtype must be bf16 or f32");
  if (!aligned16(v.ptr)) return fail(LTXQ_ERR_UNSUPPORTED, std::string(name) + " must be 16-byte aligned");
  if (v.rows_per_vec < 0) return fail(LTXQ_ERR_INVALID, std::string(name) + " rows_per_vec < 0");
  if (v.rows_per_vec > 0) {
    if (v.row_stride < C) return fail(LTXQ_ERR_INVALID, std::string(name) + " row_stride < C");
    const int64_t es = v.dtype == LTXQ_F32 ? 4 : 2;
    if ((v.row_stride * es) % 16 != 0)
      return fail(LTXQ_ERR_UNSUPPORTED, std::string(name) + " row stride must be a multiple of 16 bytes");
  }
  return LTXQ_OK;
}

ltxq_status launch_adaln_modulate(const void* x, int x_dtype, int64_t rows, int64_t C, const ltxq_prologue& pro,
                                  void* out, cudaStream_t stream, const ltxq_mx_act* out_mx) {
  if (!x || (!out && !out_mx)) return fail(LTXQ_ERR_INVALID, "adaln_modulate: x/out is NULL");
  if (out_mx) {
    if (!mx::act_ok(out_mx)) return fail(LTXQ_ERR_INVALID, "adaln_modulate: out_mx terms / pointers invalid");
    if (x_dtype != LTXQ_BF16 || C % 128 != 0 || C > 4096)
      return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: MX output needs bf16 x, C % 128 == 0 and C <= 4096");
  }
  if (rows < 0 || C <= 0) return fail(LTXQ_ERR_INVALID, "adaln_modulate: bad shape");
  if (C % 8 != 0 || C > 8192)
    return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: C must be a multiple of 8 and <= 8192");
  if (x_dtype != LTXQ_BF16 && x_dtype != LTXQ_F32) return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: x dtype");
  if (pro.norm != LTXQ_NORM_NONE && pro.norm != LTXQ_NORM_RMS && pro.norm != LTXQ_NORM_LAYER)
    return fail(LTXQ_ERR_INVALID, "adaln_modulate: unknown norm kind");
  if (!(pro.eps >= 0.f)) return fail(LTXQ_ERR_INVALID, "adaln_modulate: eps must be >= 0");
  if (ltxq_status st = check_vec(pro.scale, C, "scale")) return st;
  if (ltxq_status st = check_vec(pro.shift, C, "shift")) return st;
  if (pro.scale.dtype != pro.shift.dtype)
    return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: scale and shift must share a dtype");
  if (!aligned16(x) || !aligned16(out)) return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: x/out not 16B aligned");
  const mx::MxOut mo = out_mx ? mx::out_of(*out_mx, rows, C) : mx::MxOut{};
  if (rows == 0) return LTXQ_OK;
  if (rows > 0x7FFFFFFF) return fail(LTXQ_ERR_UNSUPPORTED, "adaln_modulate: too many rows");
  const VecArg s = to_vec(pro.scale), t = to_vec(pro.shift);
  const bool vb = pro.scale.dtype == LTXQ_BF16;
  if (x_dtype == LTXQ_BF16 && C <= 4096) {
    auto* xb = static_cast<const uint16_t*>(x);
    auto* ob = static_cast<uint16_t*>(out);
    const int ci = static_cast<int>(C);
#define LTXQ_TILE_N(R, CPT, NORM)                                                                          \
  do {                                                                                                      \
    const unsigned blocks = static_cast<unsigned>((rows + (R) - 1) / (R));                                  \
    if (out_mx) {                                                                                           \
      if (vb) adaln_tile_kernel<R, CPT, NORM, true, true><<<blocks, kTileThreads, 0, stream>>>(xb, rows, ci, pro.eps, s, t, ob, mo); \
      else adaln_tile_kernel<R, CPT, NORM, false, true><<<blocks, kTileThreads, 0, stream>>>(xb, rows, ci, pro.eps, s, t, ob, mo);  \
    } else {                                                                                                \
      if (vb) adaln_tile_kernel<R, CPT, NORM, true, false><<<blocks, kTileThreads, 0, stream>>>(xb, rows, ci, pro.eps, s, t, ob, mo); \
      else adaln_tile_kernel<R, CPT, NORM, false, false><<<blocks, kTileThreads, 0, stream>>>(xb, rows, ci, pro.eps, s, t, ob, mo);  \
    }                                                                                                       \
  } while (0)
#define LTXQ_TILE(R, CPT)                                                       \
  do {                                                                          \
    if (pro.norm == LTXQ_NORM_RMS) LTXQ_TILE_N(R, CPT, LTXQ_NORM_RMS);          \
    else if (pro.norm == LTXQ_NORM_LAYER) LTXQ_TILE_N(R, CPT, LTXQ_NORM_LAYER); \
    else LTXQ_TILE_N(R, CPT, LTXQ_NORM_NONE);                                   \
  } while (0)
    if (C <= 2048) LTXQ_TILE(8, 1);
    else LTXQ_TILE(4, 2);
#undef LTXQ_TILE
#undef LTXQ_TILE_N
    return launch_check("adaln_modulate launch");
  }
  int threads = static_cast<int>((C + 15) / 16);
  threads = ((threads + 31) / 32) * 32;
  const dim3 grid(static_cast<unsigned>(rows));
  if (x_dtype == LTXQ_F32) {
    if (vb) adaln_modulate_kernel<true, true><<<grid, threads, 0, stream>>>(x, C, pro.norm, pro.eps, s, t, out);
    else adaln_modulate_kernel<true, false><<<grid, threads, 0, stream>>>(x, C, pro.norm, pro.eps, s, t, out);
  } else {
    if (vb) adaln_modulate_kernel<false, true><<<grid, threads, 0, stream>>>(x, C, pro.norm, pro.eps, s, t, out);
    else adaln_modulate_kernel<false, false><<<grid, threads, 0, stream>>>(x, C, pro.norm, pro.eps, s, t, out);
  }
  return launch_check("adaln_modulate launch");
}

ltxq_status launch_gated_add(const void* residual, const void* branch, const ltxq_vec& gate, int64_t rows,
                             int64_t C, int mode, void* out, cudaStream_t stream) {
  if (!residual || !branch || !out) return fail(LTXQ_ERR_INVALID, "gated_add: NULL tensor");
  if (rows < 0 || C <= 0) return fail(LTXQ_ERR_INVALID, "gated_add: bad shape");
  if (C % 8 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "gated_add: C must be a multiple of 8");
  if (mode != LTXQ_GATED_ADD && mode != LTXQ_GATE_THEN_ADD) return fail(LTXQ_ERR_INVALID, "gated_add: bad mode");
  if (ltxq_status st = check_vec(gate, C, "gate")) return st;
  if (!aligned16(residual) || !aligned16(branch) || !aligned16(out))
    return fail(LTXQ_ERR_UNSUPPORTED, "gated_add: tensors must be 16-byte aligned");
  if (rows == 0) return LTXQ_OK;
  const int64_t work = rows * (C / 8);
  const int threads = 256;
  const int64_t want = (work + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(want < num_sms() * 16 ? want : num_sms() * 16);
  const VecArg g = to_vec(gate);
  auto* r = static_cast<const uint16_t*>(residual);
  auto* b = static_cast<const uint16_t*>(branch);
  auto* o = static_cast<uint16_t*>(out);
  const bool vb = gate.dtype == LTXQ_BF16;
  if (vb) gated_add_kernel<true, true><<<blocks, threads, 0, stream>>>(r, b, g, rows, C, o);
  else if (mode == LTXQ_GATE_THEN_ADD) gated_add_kernel<false, true><<<blocks, threads, 0, stream>>>(r, b, g, rows, C, o);
  else gated_add_kernel<false, false><<<blocks, threads, 0, stream>>>(r, b, g, rows, C, o);
  return launch_check("gated_add launch");
}

}  // namespace ltxq

extern "C" {

ltxq_status ltxq_adaln_modulate(const void* x, int32_t x_dtype, int64_t rows, int64_t C, const ltxq_prologue* pro,
                                void* out, void* stream) {
  if (!pro) return ltxq::fail(LTXQ_ERR_INVALID, "adaln_modulate: prologue is NULL");
  if (!out) return ltxq::fail(LTXQ_ERR_INVALID, "adaln_modulate: x/out is NULL");
  return ltxq::launch_adaln_modulate(x, x_dtype, rows, C, *pro, out, static_cast<cudaStream_t>(stream), nullptr);
}

ltxq_status ltxq_adaln_modulate_mx(const void* x, int64_t rows, int64_t C, const ltxq_prologue* pro, void* out,
                                   const ltxq_mx_act* out_mx, void* stream) {
  if (!pro) return ltxq::fail(LTXQ_ERR_INVALID, "adaln_modulate_mx: prologue is NULL");
  if (!out_mx) return ltxq::fail(LTXQ_ERR_INVALID, "adaln_modulate_mx: out_mx is NULL");
  return ltxq::launch_adaln_modulate(x, LTXQ_BF16, rows, C, *pro, out, static_cast<cudaStream_t>(stream), out_mx);
}

ltxq_status ltxq_gated_add(const void* residual, const void* branch, const ltxq_vec* gate, int64_t rows, int64_t C,
                           int32_t mode, void* out, void* stream) {
  if (!gate) return ltxq::fail(LTXQ_ERR_INVALID, "gated_add: gate is NULL");
  return ltxq::launch_gated_add(residual, branch, *gate, rows, C, mode, out, static_cast<cudaStream_t>(stream));
}

static ltxq_status head_gate(const void* o, const void* logits, int64_t lstride, int64_t rows, int64_t heads,
                             int64_t head_dim, void* out, const ltxq_mx_act* out_mx, cudaStream_t stream) {
  using namespace ltxq;
  if (!o || !logits || (!out && !out_mx)) return fail(LTXQ_ERR_INVALID, "head_gate: NULL tensor");
  if (rows < 0 || heads <= 0 || head_dim <= 0) return fail(LTXQ_ERR_INVALID, "head_gate: bad shape");
  if (lstride == 0) lstride = heads;
  if (lstride < heads) return fail(LTXQ_ERR_INVALID, "head_gate: logits row stride < heads");
  if (head_dim % 8 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "head_gate: head_dim must be a multiple of 8");
  if ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "head_gate: o/out must be 16-byte aligned");
  if (out_mx) {
    if (!mx::act_ok(out_mx)) return fail(LTXQ_ERR_INVALID, "head_gate: out_mx terms / pointers invalid");
    if ((heads * head_dim) % 128 != 0)
      return fail(LTXQ_ERR_UNSUPPORTED, "head_gate: MX output needs heads * head_dim % 128 == 0");
  }
  if (rows == 0) return LTXQ_OK;
  const int64_t work = rows * heads * head_dim / 8;
  const int threads = 256;
  const int64_t want = (work + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(want < num_sms() * 16 ? want : num_sms() * 16);
  auto* oi = static_cast<const uint16_t*>(o);
  auto* li = static_cast<const uint16_t*>(logits);
  auto* oo = static_cast<uint16_t*>(out);
  if (out_mx)
    head_gate_kernel<true><<<blocks, threads, 0, stream>>>(oi, li, lstride, rows, heads, head_dim, oo,
                                                           mx::out_of(*out_mx, rows, heads * head_dim));
  else
    head_gate_kernel<false><<<blocks, threads, 0, stream>>>(oi, li, lstride, rows, heads, head_dim, oo,
                                                            mx::MxOut{});
  return launch_check("head_gate launch");
}

ltxq_status ltxq_head_gate(const void* o, const void* logits, int64_t rows, int64_t heads, int64_t head_dim,
                           void* out, void* stream) {
  if (!out) return ltxq::fail(LTXQ_ERR_INVALID, "head_gate: NULL tensor");
  return head_gate(o, logits, 0, rows, heads, head_dim, out, nullptr, static_cast<cudaStream_t>(stream));
}

ltxq_status ltxq_head_gate_mx(const void* o, const void* logits, int64_t rows, int64_t heads, int64_t head_dim,
                              void* out, const ltxq_mx_act* out_mx, void* stream) {
  if (!out_mx) return ltxq::fail(LTXQ_ERR_INVALID, "head_gate_mx: out_mx is NULL");
  return head_gate(o, logits, 0, rows, heads, head_dim, out, out_mx, static_cast<cudaStream_t>(stream));
}

ltxq_status ltxq_head_gate_ex(const void* o, const void* logits, int64_t logits_stride, int64_t rows, int64_t heads,
                              int64_t head_dim, void* out, const ltxq_mx_act* out_mx, void* stream) {
  if (logits_stride <= 0) return ltxq::fail(LTXQ_ERR_INVALID, "head_gate_ex: logits_stride must be positive");
  return head_gate(o, logits, logits_stride, rows, heads, head_dim, out, out_mx, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace ltxq {

// ---------------------------------------------------------------------------
// QK RMSNorm (weighted, attention.py:320-329) followed by the split rotary
// embedding (rope.py:53-90): y = bf16(x * rsqrt(mean(x^2) + eps) * w), then
// per head, with h1/h2 the two halves of the head vector,
//   out = bf16([h1 * cos - h2 * sin, h1 * sin + h2 * cos])      (fp32 math).
// One warp per row.  For head_dim D each head is D/16 lanes wide: lane l
// owns the 8-element chunk (l % (D/16)) of both halves of heads
// l / (D/16) + (512 / D) * i, so the rotation pairs stay in registers.  x may
// be a column slice of a wider row (row_stride elements); out is contiguous.
template <int kD, int kHeadsPerLane>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const uint16_t* __restrict__ x, int64_t rows,
                                                           int64_t row_stride, int heads, const float* __restrict__ w,
                                                           float eps, const float* __restrict__ cosv,
                                                           const float* __restrict__ sinv, int64_t pe_tokens,
                                                           uint16_t* __restrict__ out) {
  constexpr int kLanesPerHead = kD / 16;
  constexpr int kHeadStep = 32 / kLanesPerHead;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int c = lane % kLanesPerHead;  // chunk within each half
  const int h0 = lane / kLanesPerHead;
  const uint16_t* xr = x + row * row_stride;
  uint4 lo[kHeadsPerLane], hi[kHeadsPerLane];
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < kHeadsPerLane; ++i) {
    const int h = h0 + kHeadStep * i;
    if (h < heads) {
      lo[i] = __ldg(reinterpret_cast<const uint4*>(xr + h * kD + 8 * c));
      hi[i] = __ldg(reinterpret_cast<const uint4*>(xr + h * kD + kD / 2 + 8 * c));
    } else {
      lo[i] = make_uint4(0, 0, 0, 0);
      hi[i] = make_uint4(0, 0, 0, 0);
    }
    const uint32_t a[8] = {lo[i].x, lo[i].y, lo[i].z, lo[i].w, hi[i].x, hi[i].y, hi[i].z, hi[i].w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const double e0 = lo_bf16(a[k]), e1 = hi_bf16(a[k]);
      ss += e0 * e0 + e1 * e1;
    }
  }
  ss = warp_sum(ss);
  const float ms = static_cast<float>(ss / static_cast<double>(heads * kD));
  const float inv = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(ms, eps))));
  const int64_t b = cosv != nullptr ? row / pe_tokens : 0;
  const int64_t t = cosv != nullptr ? row - b * pe_tokens : 0;
  uint16_t* orow = out + row * static_cast<int64_t>(heads) * kD;
#pragma unroll
  for (int i = 0; i < kHeadsPerLane; ++i) {
    const int h = h0 + kHeadStep * i;
    if (h >= heads) break;
    const uint32_t al[4] = {lo[i].x, lo[i].y, lo[i].z, lo[i].w};
    const uint32_t ah[4] = {hi[i].x, hi[i].y, hi[i].z, hi[i].w};
    float y1[8], y2[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      y1[2 * k] = lo_bf16(al[k]);
      y1[2 * k + 1] = hi_bf16(al[k]);
      y2[2 * k] = lo_bf16(ah[k]);
      y2[2 * k + 1] = hi_bf16(ah[k]);
    }
    const float* w1 = w + h * kD + 8 * c;
    const float* w2 = w1 + kD / 2;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      y1[k] = rbf16(__fmul_rn(__fmul_rn(y1[k], inv), __ldg(w1 + k)));
      y2[k] = rbf16(__fmul_rn(__fmul_rn(y2[k], inv), __ldg(w2 + k)));
    }
    if (cosv != nullptr) {
      const int64_t off = ((b * heads + h) * pe_tokens + t) * (kD / 2) + 8 * c;
      float cs[8], sn[8];
      const float4 c0 = __ldg(reinterpret_cast<const float4*>(cosv + off));
      const float4 c1 = __ldg(reinterpret_cast<const float4*>(cosv + off + 4));
      const float4 s0 = __ldg(reinterpret_cast<const float4*>(sinv + off));
      const float4 s1 = __ldg(reinterpret_cast<const float4*>(sinv + off + 4));
      cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
      sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float a1 = y1[k], a2 = y2[k];
        y1[k] = __fsub_rn(__fmul_rn(a1, cs[k]), __fmul_rn(a2, sn[k]));
        y2[k] = __fadd_rn(__fmul_rn(a1, sn[k]), __fmul_rn(a2, cs[k]));
      }
    }
    uint4 o1, o2;
    o1.x = pack_bf16x2(y1[0], y1[1]); o1.y = pack_bf16x2(y1[2], y1[3]);
    o1.z = pack_bf16x2(y1[4], y1[5]); o1.w = pack_bf16x2(y1[6], y1[7]);
    o2.x = pack_bf16x2(y2[0], y2[1]); o2.y = pack_bf16x2(y2[2], y2[3]);
    o2.z = pack_bf16x2(y2[4], y2[5]); o2.w = pack_bf16x2(y2[6], y2[7]);
    *reinterpret_cast<uint4*>(orow + h * kD + 8 * c) = o1;
    *reinterpret_cast<uint4*>(orow + h * kD + kD / 2 + 8 * c) = o2;
  }
}

// Tile form: a unit is (head h, 8-wide chunk c): the chunk c of both halves
// of head h (the rotation pairs element i of the first half with element i of
// the second).  A row has U = heads * D / 16 units (a multiple of 32); a CTA
// of 256 threads covers 256 / U rows per pass and kR passes, so every thread
// issues all its 16-byte row and table loads at once.  kPair: a second
// operand (K next to Q) on the same rows, rotated by the same tables, which
// are then read once for both.  Row statistics: an fp32 sum of squares per
// thread, added across the row's threads in fp64 in a fixed order.
constexpr int kRopeThreads = 256;

template <int kD, int kR, bool kPair>
__global__ void __launch_bounds__(kRopeThreads, 2)
    qk_rope_tile_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ x2, int64_t rows,
                        int64_t stride, int64_t stride2, int heads, const float* __restrict__ w,
                        const float* __restrict__ w2, float eps, const float* __restrict__ cosv,
                        const float* __restrict__ sinv, int64_t pe_tokens, uint16_t* __restrict__ out,
                        uint16_t* __restrict__ out2) {
  constexpr int kCh = kD / 16;  // chunks per half head
  constexpr int kOps = kPair ? 2 : 1;
  __shared__ double red[kR][kOps][kRopeThreads / 32];
  __shared__ float inv_s[kR][kOps][kRopeThreads / 32];  // per row of the pass (at most 8 rows)
  const int U = heads * kCh;
  const int rpp = kRopeThreads / U;  // rows per pass
  const int tid = threadIdx.x;
  const int rr = tid / U, u = tid - rr * U;  // row within the pass, unit
  const bool active = rr < rpp;
  const int h = u / kCh, c = u - h * kCh;
  const int col_lo = h * kD + 8 * c, col_hi = col_lo + kD / 2;
  const int lane = tid & 31, warp = tid >> 5;
  const int wpr = U / 32;  // warps per row
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * rpp * kR;
  const uint16_t* xs[2] = {x, x2};
  const int64_t strides[2] = {stride, stride2};
  uint4 lo[kR][kOps], hi[kR][kOps];
  float4 cs[kR][2], sn[kR][2];
#pragma unroll
  for (int p = 0; p < kR; ++p) {
    const int64_t row = row0 + p * rpp + rr;
    const bool live = active && row < rows;
#pragma unroll
    for (int o = 0; o < kOps; ++o) {
      const uint16_t* xr = xs[o] + (live ? row : 0) * strides[o];
      lo[p][o] = live ? __ldg(reinterpret_cast<const uint4*>(xr + col_lo)) : make_uint4(0, 0, 0, 0);
      hi[p][o] = live ? __ldg(reinterpret_cast<const uint4*>(xr + col_hi)) : make_uint4(0, 0, 0, 0);
    }
    if (cosv != nullptr && live) {
      const int64_t b = row / pe_tokens, tt = row - b * pe_tokens;
      const int64_t off = ((b * heads + h) * pe_tokens + tt) * (kD / 2) + 8 * c;
      cs[p][0] = __ldg(reinterpret_cast<const float4*>(cosv + off));
      cs[p][1] = __ldg(reinterpret_cast<const float4*>(cosv + off + 4));
      sn[p][0] = __ldg(reinterpret_cast<const float4*>(sinv + off));
      sn[p][1] = __ldg(reinterpret_cast<const float4*>(sinv + off + 4));
    }
  }
  // per-row sums of squares: fp32 per thread, fp64 across the row's warps
#pragma unroll
  for (int p = 0; p < kR; ++p)
#pragma unroll
    for (int o = 0; o < kOps; ++o) {
      const uint32_t a[8] = {lo[p][o].x, lo[p][o].y, lo[p][o].z, lo[p][o].w,
                             hi[p][o].x, hi[p][o].y, hi[p][o].z, hi[p][o].w};
      float q = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        q = __fmaf_rn(hi_bf16(a[k]), hi_bf16(a[k]), __fmaf_rn(lo_bf16(a[k]), lo_bf16(a[k]), q));
      const double d = warp_sum(static_cast<double>(q));
      if (lane == 0) red[p][o][warp] = d;
    }
  __syncthreads();
  if (active && u % 32 == 0 && u / 32 == 0) {  // the first warp of each row of the pass
#pragma unroll
    for (int p = 0; p < kR; ++p)
#pragma unroll
      for (int o = 0; o < kOps; ++o)
        if (lane == 0) {
          double t = 0.0;
          for (int i = 0; i < wpr; ++i) t += red[p][o][rr * wpr + i];
          const float ms = static_cast<float>(t / static_cast<double>(heads * kD));
          inv_s[p][o][rr] = static_cast<float>(rsqrt(static_cast<double>(__fadd_rn(ms, eps))));
        }
  }
  __syncthreads();
  if (!active) return;
  const float* ws[2] = {w, w2};
  uint16_t* outs[2] = {out, out2};
#pragma unroll
  for (int o = 0; o < kOps; ++o) {
    float w1[8], w2v[8];
    {
      const float4 a0 = __ldg(reinterpret_cast<const float4*>(ws[o] + col_lo));
      const float4 a1 = __ldg(reinterpret_cast<const float4*>(ws[o] + col_lo + 4));
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(ws[o] + col_hi));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(ws[o] + col_hi + 4));
      w1[0] = a0.x; w1[1] = a0.y; w1[2] = a0.z; w1[3] = a0.w; w1[4] = a1.x; w1[5] = a1.y; w1[6] = a1.z; w1[7] = a1.w;
      w2v[0] = b0.x; w2v[1] = b0.y; w2v[2] = b0.z; w2v[3] = b0.w; w2v[4] = b1.x; w2v[5] = b1.y; w2v[6] = b1.z;
      w2v[7] = b1.w;
    }
#pragma unroll
    for (int p = 0; p < kR; ++p) {
      const int64_t row = row0 + p * rpp + rr;
      if (row >= rows) break;
      const float inv = inv_s[p][o][rr];
      const uint32_t al[4] = {lo[p][o].x, lo[p][o].y, lo[p][o].z, lo[p][o].w};
      const uint32_t ah[4] = {hi[p][o].x, hi[p][o].y, hi[p][o].z, hi[p][o].w};
      float y1[8], y2[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        y1[2 * k] = lo_bf16(al[k]);
        y1[2 * k + 1] = hi_bf16(al[k]);
        y2[2 * k] = lo_bf16(ah[k]);
        y2[2 * k + 1] = hi_bf16(ah[k]);
      }
#pragma unroll
      for (int k = 0; k < 8; k += 2) {
        // y = bf16(x * inv * w), two values per conversion
        const uint32_t r1 = pack_bf16x2(__fmul_rn(__fmul_rn(y1[k], inv), w1[k]),
                                        __fmul_rn(__fmul_rn(y1[k + 1], inv), w1[k + 1]));
        const uint32_t r2 = pack_bf16x2(__fmul_rn(__fmul_rn(y2[k], inv), w2v[k]),
                                        __fmul_rn(__fmul_rn(y2[k + 1], inv), w2v[k + 1]));
        y1[k] = lo_bf16(r1);
        y1[k + 1] = hi_bf16(r1);
        y2[k] = lo_bf16(r2);
        y2[k + 1] = hi_bf16(r2);
      }
      if (cosv != nullptr) {
        const float cv[8] = {cs[p][0].x, cs[p][0].y, cs[p][0].z, cs[p][0].w, cs[p][1].x, cs[p][1].y, cs[p][1].z,
                             cs[p][1].w};
        const float sv[8] = {sn[p][0].x, sn[p][0].y, sn[p][0].z, sn[p][0].w, sn[p][1].x, sn[p][1].y, sn[p][1].z,
                             sn[p][1].w};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float a1 = y1[k], a2 = y2[k];
          y1[k] = __fsub_rn(__fmul_rn(a1, cv[k]), __fmul_rn(a2, sv[k]));
          y2[k] = __fadd_rn(__fmul_rn(a1, sv[k]), __fmul_rn(a2, cv[k]));
        }
      }
      uint16_t* orow = outs[o] + row * static_cast<int64_t>(heads) * kD;
      uint4 o1, o2;
      o1.x = pack_bf16x2(y1[0], y1[1]); o1.y = pack_bf16x2(y1[2], y1[3]);
      o1.z = pack_bf16x2(y1[4], y1[5]); o1.w = pack_bf16x2(y1[6], y1[7]);
      o2.x = pack_bf16x2(y2[0], y2[1]); o2.y = pack_bf16x2(y2[2], y2[3]);
      o2.z = pack_bf16x2(y2[4], y2[5]); o2.w = pack_bf16x2(y2[6], y2[7]);
      *reinterpret_cast<uint4*>(orow + col_lo) = o1;
      *reinterpret_cast<uint4*>(orow + col_hi) = o2;
    }
  }
}

constexpr int kRopeRows = 2;  // passes per CTA

template <bool kPair>
static ltxq_status launch_rope_tile(const uint16_t* x, const uint16_t* x2, int64_t rows, int64_t stride,
                                   int64_t stride2, int heads, int D, const float* w, const float* w2, float eps,
                                   const float* cosv, const float* sinv, int64_t pe_tokens, uint16_t* out,
                                   uint16_t* out2, cudaStream_t s) {
  const int U = heads * (D / 16);
  const int64_t per_cta = static_cast<int64_t>(kRopeThreads / U) * kRopeRows;
  const unsigned blocks = static_cast<unsigned>((rows + per_cta - 1) / per_cta);
  if (D == 128)
    qk_rope_tile_kernel<128, kRopeRows, kPair><<<blocks, kRopeThreads, 0, s>>>(
        x, x2, rows, stride, stride2, heads, w, w2, eps, cosv, sinv, pe_tokens, out, out2);
  else
    qk_rope_tile_kernel<64, kRopeRows, kPair><<<blocks, kRopeThreads, 0, s>>>(
        x, x2, rows, stride, stride2, heads, w, w2, eps, cosv, sinv, pe_tokens, out, out2);
  return launch_check("qk_norm_rope launch");
}

}  // namespace ltxq

extern "C" ltxq_status ltxq_qk_norm_rope(const void* x, int64_t rows, int64_t row_stride, int64_t heads,
                                         int64_t head_dim, const float* weight, float eps, const float* cos_table,
                                         const float* sin_table, int64_t pe_tokens, void* out, void* stream) {
  using namespace ltxq;
  if (!x || !out || !weight) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: NULL tensor");
  if (rows < 0 || heads <= 0 || row_stride < heads * head_dim) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: bad shape");
  if (head_dim != 64 && head_dim != 128) return fail(LTXQ_ERR_UNSUPPORTED, "qk_norm_rope: head_dim must be 64 or 128");
  if (heads > 32) return fail(LTXQ_ERR_UNSUPPORTED, "qk_norm_rope: at most 32 heads");
  if ((cos_table == nullptr) != (sin_table == nullptr)) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: cos/sin pairing");
  if (cos_table && pe_tokens <= 0) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: pe_tokens must be > 0");
  if (cos_table && rows % pe_tokens != 0) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: rows must be a multiple of pe_tokens");
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(cos_table) |
        reinterpret_cast<uintptr_t>(sin_table)) & 15u) || (row_stride % 8) != 0)
    return fail(LTXQ_ERR_UNSUPPORTED, "qk_norm_rope: tensors must be 16-byte aligned (row stride a multiple of 8)");
  if (!(eps >= 0.f)) return fail(LTXQ_ERR_INVALID, "qk_norm_rope: eps must be >= 0");
  if (rows == 0) return LTXQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* xi = static_cast<const uint16_t*>(x);
  auto* o = static_cast<uint16_t*>(out);
  const int h = static_cast<int>(heads);
  if ((heads * (head_dim / 16)) % 32 == 0 && !(reinterpret_cast<uintptr_t>(weight) & 15u))
    return launch_rope_tile<false>(xi, nullptr, rows, row_stride, 0, h, static_cast<int>(head_dim), weight, nullptr,
                                   eps, cos_table, sin_table, pe_tokens, o, nullptr, s);
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  // heads per lane: heads / (32 / (D/16)), <= 32 heads
  if (head_dim == 128)
    qk_norm_rope_kernel<128, 8><<<blocks, 256, 0, s>>>(xi, rows, row_stride, h, weight, eps, cos_table, sin_table, pe_tokens, o);
  else
    qk_norm_rope_kernel<64, 4><<<blocks, 256, 0, s>>>(xi, rows, row_stride, h, weight, eps, cos_table, sin_table, pe_tokens, o);
  return launch_check("qk_norm_rope launch");
}

extern "C" ltxq_status ltxq_qk_norm_rope_pair(const void* q, const void* k, int64_t rows, int64_t q_stride,
                                              int64_t k_stride, int64_t heads, int64_t head_dim, const float* q_weight,
                                              const float* k_weight, float eps, const float* cos_table,
                                              const float* sin_table, int64_t pe_tokens, void* q_out, void* k_out,
                                              void* stream) {
  using namespace ltxq;
  if (!q || !k || !q_out || !k_out || !q_weight || !k_weight)
    return fail(LTXQ_ERR_INVALID, "qk_norm_rope_pair: NULL tensor");
  if (rows < 0 || heads <= 0 || q_stride < heads * head_dim || k_stride < heads * head_dim)
    return fail(LTXQ_ERR_INVALID, "qk_norm_rope_pair: bad shape");
  if (head_dim != 64 && head_dim != 128)
    return fail(LTXQ_ERR_UNSUPPORTED, "qk_norm_rope_pair: head_dim must be 64 or 128");
  if ((heads * (head_dim / 16)) % 32 != 0 || heads * (head_dim / 16) > kRopeThreads)
    return fail(LTXQ_ERR_UNSUPPORTED, "qk_norm_rope_pair: heads * head_dim / 16 must be a multiple of 32, <= 256");
  if ((cos_table == nullptr) != (sin_table == nullptr))
    return fail(LTXQ_ERR_INVALID, "qk_norm_rope_pair: cos/sin pairing");
  if (cos_table && (pe_tokens <= 0 || rows % pe_tokens != 0))
    return fail(LTXQ_ERR_INVALID, "qk_norm_rope_pair: rows must be a multiple of pe_tokens > 0");
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(q_out) |
        reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(cos_table) |
        reinterpret_cast<uintptr_t>(sin_table) | reinterpret_cast<uintptr_t>(q_weight) |
        reinterpret_cast<uintptr_t>(k_weight)) & 15u) ||
      (q_stride % 8) != 0 || (k_stride % 8) != 0)
    return fail(LTXQ_ERR_UNSUPPORTED,
                "qk_norm_rope_pair: tensors must be 16-byte aligned (row strides multiples of 8)");
  if (!(eps >= 0.f)) return fail(LTXQ_ERR_INVALID, "qk_norm_rope_pair: eps must be >= 0");
  if (rows == 0) return LTXQ_OK;
  return launch_rope_tile<true>(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k), rows, q_stride,
                                k_stride, static_cast<int>(heads), static_cast<int>(head_dim), q_weight, k_weight,
                                eps, cos_table, sin_table, pe_tokens, static_cast<uint16_t*>(q_out),
                                static_cast<uint16_t*>(k_out), static_cast<cudaStream_t>(stream));
}
