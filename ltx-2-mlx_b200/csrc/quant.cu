// quant.cu -- on-device builders/readers of the reference's quantized-weight
// cache entries (loader/transformer_cache.py:1238-1267 writes the outputs of
// mx.quantize; :1436-1462 / :177-193 read them back).
//
// ltxq_quantize restates MLX's affine quantizer (fp32 group min/max, the
// larger-magnitude edge snapped so that zero is an exact code, RNE rounding,
// clip, scales/biases cast to bf16) and the OCP MX v1.0 MXFP8 quantizer
// (E8M0 shared exponent floor(log2(amax)) - 8, E4M3 RNE with saturation).
// ltxq_dequantize produces the bf16 weight the GEMM consumes, bit for bit
// (the same device functions as the GEMM's dequant warps).
#include <mutex>

#include "common.cuh"
#include "dequant.cuh"

namespace ltxq {

// Quantize along the contiguous dimension of a [R, L] bf16 matrix; one
// thread per group.
template <int kBits>
__global__ void affine_quantize_kernel(const uint16_t* __restrict__ w, int64_t R, int64_t L, int gs,
                                       uint32_t* __restrict__ wq, uint16_t* __restrict__ scales,
                                       uint16_t* __restrict__ biases) {
  const int64_t groups_per_row = L / gs;
  const int64_t total = R * groups_per_row;
  constexpr int kPer = 32 / kBits;
  const float n_bins = static_cast<float>((1 << kBits) - 1);
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < total;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = gi / groups_per_row;
    const int64_t g = gi - row * groups_per_row;
    const uint16_t* src = w + row * L + g * gs;
    float wmax = -INFINITY, wmin = INFINITY;
    for (int i = 0; i < gs; ++i) {
      const float v = bf16_to_f32(src[i]);
      wmax = fmaxf(wmax, v);
      wmin = fminf(wmin, v);
    }
    const bool mask = fabsf(wmin) > fabsf(wmax);
    float scale = fmaxf(__fdiv_rn(__fsub_rn(wmax, wmin), n_bins), 1e-7f);
    scale = mask ? scale : -scale;
    const float edge = mask ? wmin : wmax;
    const float q0 = rintf(__fdiv_rn(edge, scale));
    if (q0 != 0.f) scale = __fdiv_rn(edge, q0);
    const float bias = (q0 == 0.f) ? 0.f : edge;
    scales[row * groups_per_row + g] = f32_to_bf16(scale);
    biases[row * groups_per_row + g] = f32_to_bf16(bias);
    uint32_t* dst = wq + (row * L + g * gs) / kPer;
    for (int i = 0; i < gs; i += kPer) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const float v = bf16_to_f32(src[i + j]);
        float q = rintf(__fdiv_rn(__fsub_rn(v, bias), scale));
        q = fminf(fmaxf(q, 0.f), n_bins);
        word |= static_cast<uint32_t>(q) << (j * kBits);
      }
      dst[i / kPer] = word;
    }
  }
}

__global__ void mxfp8_quantize_kernel(const uint16_t* __restrict__ w, int64_t R, int64_t L, int gs,
                                      uint32_t* __restrict__ wq, uint8_t* __restrict__ scales) {
  const int64_t groups_per_row = L / gs;
  const int64_t total = R * groups_per_row;
  for (int64_t gi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gi < total;
       gi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = gi / groups_per_row;
    const int64_t g = gi - row * groups_per_row;
    const uint16_t* src = w + row * L + g * gs;
    float amax = 0.f;
    for (int i = 0; i < gs; ++i) amax = fmaxf(amax, fabsf(bf16_to_f32(src[i])));
    int e = (amax > 0.f) ? ilogbf(amax) - 8 : -127;  // E4M3 emax = 8
    e = max(-127, min(127, e));
    scales[row * groups_per_row + g] = static_cast<uint8_t>(e + 127);
    // 2^-e as an exact normal fp32 value: bf16 inputs bound e to [-127, 119]
    const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
    uint32_t* dst = wq + (row * L + g * gs) / 4;
    for (int i = 0; i < gs; i += 4) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = bf16_to_f32(src[i + j]) * inv;
      uint16_t p01, p23;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p01) : "f"(v[1]), "f"(v[0]));
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(p23) : "f"(v[3]), "f"(v[2]));
      dst[i / 4] = static_cast<uint32_t>(p01) | (static_cast<uint32_t>(p23) << 16);
    }
  }
}

// One thread per packed word of a [R, L] packed matrix (L = packed-dim
// length in elements) -> bf16 [R, L].
template <int kKind>  // 0 affine8, 1 affine4, 2 mxfp8, 3 mxfp8 flagged LTXQ_QW_MXFP8_FINITE
__global__ void dequantize_kernel(const uint32_t* __restrict__ wq, const void* __restrict__ scales,
                                  const uint16_t* __restrict__ biases, int64_t R, int64_t L, int gs,
                                  uint16_t* __restrict__ out) {
  constexpr int kPer = kKind == 1 ? 8 : 4;
  const int64_t words_per_row = L / kPer;
  const int64_t total = R * words_per_row;
  const int64_t groups_per_row = L / gs;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / words_per_row;
    const int64_t k0 = (i - row * words_per_row) * kPer;
    const int64_t g = row * groups_per_row + k0 / gs;
    const uint32_t w = __ldg(wq + i);
    if (kKind == 2) {
      const float sc = e8m0_to_f32(static_cast<const uint8_t*>(scales)[g]);
      uint32_t o01, o23;
      deq_mxfp8_word(w, sc, o01, o23);
      *reinterpret_cast<uint2*>(out + row * L + k0) = make_uint2(o01, o23);
    } else if (kKind == 3) {
      uint32_t o01, o23;
      deq_mxfp8_word_fast(w, e8m0_fast_scale2(static_cast<const uint8_t*>(scales)[g]), o01, o23);
      *reinterpret_cast<uint2*>(out + row * L + k0) = make_uint2(o01, o23);
    } else {
      const uint32_t s2 = bcast_bf16x2(static_cast<const uint16_t*>(scales)[g]);
      const uint32_t b2 = bcast_bf16x2(biases[g]);
      if (kKind == 0) {
        uint32_t o01, o23;
        deq_affine8_word(w, s2, b2, o01, o23);
        *reinterpret_cast<uint2*>(out + row * L + k0) = make_uint2(o01, o23);
      } else {
        uint32_t o[4];
        deq_affine4_word(w, s2, b2, o);
        *reinterpret_cast<uint4*>(out + row * L + k0) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
}

// Validates a qweight descriptor; returns the packed matrix geometry
// (R rows, L elements along the packed dimension).
ltxq_status check_qweight(const ltxq_qweight& w, bool need_data, int64_t* R, int64_t* L) {
  if (w.n_out <= 0 || w.k_in <= 0) return fail(LTXQ_ERR_INVALID, "qweight: n_out/k_in must be positive");
  if (w.layout != LTXQ_LAYOUT_STD && w.layout != LTXQ_LAYOUT_PRETRANSPOSED)
    return fail(LTXQ_ERR_INVALID, "qweight: unknown layout");
  if (w.mode == LTXQ_AFFINE) {
    if (w.bits != 4 && w.bits != 8) return fail(LTXQ_ERR_UNSUPPORTED, "qweight: affine bits must be 4 or 8");
    if (w.group_size != 32 && w.group_size != 64 && w.group_size != 128)
      return fail(LTXQ_ERR_UNSUPPORTED, "qweight: affine group_size must be 32, 64 or 128");
  } else if (w.mode == LTXQ_MXFP8) {
    if (w.bits != 8 || w.group_size != 32) return fail(LTXQ_ERR_UNSUPPORTED, "qweight: mxfp8 needs bits 8, gs 32");
  } else {
    return fail(LTXQ_ERR_UNSUPPORTED, "qweight: mode must be affine or mxfp8");
  }
  const bool pt = w.layout == LTXQ_LAYOUT_PRETRANSPOSED;
  *R = pt ? w.k_in : w.n_out;
  *L = pt ? w.n_out : w.k_in;
  if (*L % w.group_size != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qweight: packed dimension not a multiple of group_size");
  if (need_data) {
    if (!w.weight || !w.scales) return fail(LTXQ_ERR_INVALID, "qweight: weight/scales NULL");
    if (w.mode == LTXQ_AFFINE && !w.biases) return fail(LTXQ_ERR_INVALID, "qweight: affine biases NULL");
  }
  return LTXQ_OK;
}

// LTXQ_QW_MXFP8_FINITE check: sets *bad if any E4M3 byte is a NaN code or
// any E8M0 scale exceeds 134.  `vec`: codes are 16-byte aligned (16-byte
// loads for all but the tail).
__global__ void mxfp8_scan_kernel(const uint8_t* __restrict__ codes, int64_t n_codes, bool vec,
                                  const uint8_t* __restrict__ scales, int64_t n_scales, unsigned int* bad) {
  bool b = false;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t n16 = vec ? n_codes / 16 : 0;
  for (int64_t i = t0; i < n16; i += stride) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(codes) + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) b |= (((w[j] & 0x7F7F7F7Fu) + 0x01010101u) & 0x80808080u) != 0u;
  }
  for (int64_t i = n16 * 16 + t0; i < n_codes; i += stride) b |= (codes[i] & 0x7Fu) == 0x7Fu;
  for (int64_t i = t0; i < n_scales; i += stride) b |= scales[i] > 134u;
  if (__syncthreads_or(b) && threadIdx.x == 0) atomicOr(bad, 1u);
}

__device__ unsigned int g_scan_word = 0;
static std::mutex g_scan_mutex;

static unsigned grid_for(int64_t work, int threads) {
  const int64_t want = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 32;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace ltxq

extern "C" {

ltxq_status ltxq_quantize(const void* w_bf16, const ltxq_qweight* w, void* stream) {
  using namespace ltxq;
  if (!w_bf16 || !w) return fail(LTXQ_ERR_INVALID, "quantize: NULL argument");
  int64_t R, L;
  if (ltxq_status st = check_qweight(*w, true, &R, &L)) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256;
  const unsigned blocks = grid_for(R * (L / w->group_size), threads);
  auto* src = static_cast<const uint16_t*>(w_bf16);
  auto* wq = static_cast<uint32_t*>(const_cast<void*>(w->weight));
  if (w->mode == LTXQ_AFFINE) {
    auto* sc = static_cast<uint16_t*>(const_cast<void*>(w->scales));
    auto* bi = static_cast<uint16_t*>(const_cast<void*>(w->biases));
    if (w->bits == 8) affine_quantize_kernel<8><<<blocks, threads, 0, s>>>(src, R, L, w->group_size, wq, sc, bi);
    else affine_quantize_kernel<4><<<blocks, threads, 0, s>>>(src, R, L, w->group_size, wq, sc, bi);
  } else {
    auto* sc = static_cast<uint8_t*>(const_cast<void*>(w->scales));
    mxfp8_quantize_kernel<<<blocks, threads, 0, s>>>(src, R, L, w->group_size, wq, sc);
  }
  return launch_check("quantize launch");
}

ltxq_status ltxq_dequantize(const ltxq_qweight* w, void* out_bf16, void* stream) {
  using namespace ltxq;
  if (!w || !out_bf16) return fail(LTXQ_ERR_INVALID, "dequantize: NULL argument");
  int64_t R, L;
  if (ltxq_status st = check_qweight(*w, true, &R, &L)) return st;
  if (reinterpret_cast<uintptr_t>(out_bf16) & 15u) return fail(LTXQ_ERR_UNSUPPORTED, "dequantize: out not 16B aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256;
  auto* wq = static_cast<const uint32_t*>(w->weight);
  auto* bi = static_cast<const uint16_t*>(w->biases);
  auto* o = static_cast<uint16_t*>(out_bf16);
  if (w->mode == LTXQ_MXFP8 && (w->flags & LTXQ_QW_MXFP8_FINITE)) {
    dequantize_kernel<3><<<grid_for(R * L / 4, threads), threads, 0, s>>>(wq, w->scales, bi, R, L, w->group_size, o);
  } else if (w->mode == LTXQ_MXFP8) {
    dequantize_kernel<2><<<grid_for(R * L / 4, threads), threads, 0, s>>>(wq, w->scales, bi, R, L, w->group_size, o);
  } else if (w->bits == 8) {
    dequantize_kernel<0><<<grid_for(R * L / 4, threads), threads, 0, s>>>(wq, w->scales, bi, R, L, w->group_size, o);
  } else {
    dequantize_kernel<1><<<grid_for(R * L / 8, threads), threads, 0, s>>>(wq, w->scales, bi, R, L, w->group_size, o);
  }
  return launch_check("dequantize launch");
}

ltxq_status ltxq_qweight_scan(const ltxq_qweight* w, uint32_t* flags_out, void* stream) {
  using namespace ltxq;
  if (!w || !flags_out) return fail(LTXQ_ERR_INVALID, "qweight_scan: NULL argument");
  int64_t R, L;
  if (ltxq_status st = check_qweight(*w, true, &R, &L)) return st;
  *flags_out = 0;
  if (w->mode != LTXQ_MXFP8) return LTXQ_OK;
  std::lock_guard<std::mutex> lock(g_scan_mutex);  // one scan word per device
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* word = nullptr;
  if (ltxq_status st = cuda_check(cudaGetSymbolAddress(&word, g_scan_word), "scan word")) return st;
  if (ltxq_status st = cuda_check(cudaMemsetAsync(word, 0, sizeof(unsigned int), s), "scan reset")) return st;
  const int64_t n_codes = R * L, n_scales = R * (L / w->group_size);
  const bool al = (reinterpret_cast<uintptr_t>(w->weight) & 15u) == 0;
  mxfp8_scan_kernel<<<grid_for(al ? n_codes / 16 + 1 : n_codes, 256), 256, 0, s>>>(
      static_cast<const uint8_t*>(w->weight), n_codes, al, static_cast<const uint8_t*>(w->scales), n_scales,
      static_cast<unsigned int*>(word));
  if (ltxq_status st = launch_check("qweight scan launch")) return st;
  unsigned int bad = 0;
  if (ltxq_status st = cuda_check(cudaMemcpyAsync(&bad, word, sizeof(bad), cudaMemcpyDeviceToHost, s), "scan read"))
    return st;
  if (ltxq_status st = cuda_check(cudaStreamSynchronize(s), "scan sync")) return st;
  *flags_out = bad ? 0u : static_cast<uint32_t>(LTXQ_QW_MXFP8_FINITE);
  return LTXQ_OK;
}

}  // extern "C"
