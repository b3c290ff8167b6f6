// qgemm.cu -- quantized linear layers of the DiT block on sm_100a tensor
// cores (tcgen05), with the block's epilogues fused.
//
// Reference semantics (LTX_2_MLX/loader/transformer_cache.py:177-193 and
// MLX nn.QuantizedLinear): y = bf16(x . dequant(W)^T), then bf16(y + bias),
// then the block's consumer: GELU-tanh (feed_forward.py:101-102), the gated
// residual add (transformer.py:40-50, 469, 650) or the text cross-attention
// gate-then-add (transformer.py:387, 484).
//
// Kernel design (one CTA computes 128 output features x BN tokens):
//   * operands are swapped: the dequantized weight tile (128 features x 64 K)
//     is the MMA "A" operand and lives in tensor memory; the activation tile
//     (BN tokens x 64 K, bf16) is the "B" operand, staged in shared memory by
//     TMA with the 128-byte swizzle.  The weight never round-trips through
//     shared memory as bf16: packed bytes arrive by TMA, 4 dequant warps
//     convert them in registers (dequant.cuh) and write them to TMEM with
//     tcgen05.st, one TMEM lane per output feature.
//   * warp 4 issues TMA loads (activations and packed weights, multi-stage
//     mbarrier ring), warp 5 owns the TMEM allocation and issues
//     tcgen05.mma kind::f16 (M=128, N=BN, K=16) with fp32 accumulators in
//     TMEM, and tcgen05.commit releases stages back to the producers.
//   * the epilogue (the dequant warps, after the main loop) reads the
//     accumulator with tcgen05.ld (thread = feature, registers = tokens),
//     applies bias/GELU with the reference's rounding points, transposes
//     through shared memory and writes 16-byte coalesced rows, fusing the
//     gated residual with 16-byte residual loads.
//   * every mbarrier wait is bounded (common.cuh mbar_wait); an expired wait
//     raises the device error word and the CTA unwinds, releasing TMEM.
#include "common.cuh"
#include "dequant.cuh"

namespace ltxq {

ltxq_status check_qweight(const ltxq_qweight& w, bool need_data, int64_t* R, int64_t* L);
ltxq_status launch_adaln_modulate(const void* x, int x_dtype, int64_t rows, int64_t C, const ltxq_prologue& pro,
                                  void* out, cudaStream_t stream);

namespace gemm {

constexpr int BM = 128;  // output features per CTA (MMA M, TMEM lanes)
constexpr int BK = 64;   // K per pipeline stage
constexpr int kTmaWarp = 4, kMmaWarp = 5, kThreads = 192;
constexpr int kAStages = 4;  // TMEM A-operand ring
constexpr int kStagePitch = 136;  // epilogue staging row pitch in bf16 (128 + 8 pad)

enum QKind { kAffine8 = 0, kAffine4 = 1, kMxfp8 = 2 };

template <int QK>
struct QTraits {
  static constexpr int kWBytes = QK == kAffine4 ? 32 : 64;  // packed bytes per row per stage
  static constexpr CUtensorMapSwizzle kSwizzle =
      QK == kAffine4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
};

template <int QK, int BN>
struct Cfg {
  static constexpr int kXStage = BN * BK * 2;
  static constexpr int kWStage = BM * QTraits<QK>::kWBytes;
  static constexpr int kBudget = 200 * 1024;
  static constexpr int kStagesRaw = kBudget / (kXStage + kWStage);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kBarOff = kStages * (kXStage + kWStage);
  static constexpr int kSmem = 1024 + kBarOff + 256;
  static constexpr uint32_t kTmemCols = (BN + kAStages * 32) <= 256 ? 256 : 512;
  static constexpr uint32_t kACol = BN;  // A-operand stages follow the accumulator
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(BN + kAStages * 32 <= 512, "TMEM budget");
};

struct Params {
  int M, N, K, gs;
  const void* scales;
  const uint16_t* biases;
  const uint16_t* bias;
  int epi;
  VecArg gate;
  const uint16_t* residual;
  uint16_t* out;
  unsigned int* err;
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

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <int QK, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const Params p) {
  using C = Cfg<QK, BN>;
  constexpr int S = C::kStages;
  constexpr int WB = QTraits<QK>::kWBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint8_t* ws = smem + S * C::kXStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + S;
  uint64_t* w_full = bars + 2 * S;
  uint64_t* w_empty = bars + 3 * S;
  uint64_t* a_full = bars + 4 * S;
  uint64_t* a_empty = bars + 4 * S + kAStages;
  uint64_t* acc_full = bars + 4 * S + 2 * kAStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BM;
  const int m0 = blockIdx.y * BN;
  const int num_kb = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 1);
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 4);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&x_empty[s], ph ^ 1, abort_flag, p.err)) break;
        mbar_arrive_expect_tx(&x_full[s], C::kXStage);
        tma_load_2d(xs + s * C::kXStage, &tmap_x, &x_full[s], kb * BK, m0);
        if (!mbar_wait(&w_empty[s], ph ^ 1, abort_flag, p.err)) {
          issued = kb + 1;
          break;
        }
        mbar_arrive_expect_tx(&w_full[s], C::kWStage);
        tma_load_2d(ws + s * C::kWStage, &tmap_w, &w_full[s], kb * WB, n0);
        issued = kb + 1;
      }
      if (*abort_flag) {
        // let the copies already issued land before the CTA's smem is released
        int dummy_abort = 0;
        for (int kb = issued - 1; kb >= 0 && kb >= issued - S; --kb) {
          const int s = kb % S;
          const uint32_t ph = (kb / S) & 1;
          mbar_wait(&x_full[s], ph, reinterpret_cast<volatile int*>(&dummy_abort), p.err);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        const int as = kb % kAStages;
        const uint32_t aph = (kb / kAStages) & 1;
        if (!mbar_wait(&x_full[s], ph, abort_flag, p.err)) break;
        if (!mbar_wait(&a_full[as], aph, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t xaddr = smem_u32(xs + s * C::kXStage);
#pragma unroll
        for (int j = 0; j < BK / 16; ++j) {
          const uint64_t bdesc = smem_desc_sw128(xaddr + j * 32);
          mma_bf16_ts(tmem, tmem + C::kACol + as * 32 + j * 8, bdesc, idesc, (kb | j) != 0 ? 1u : 0u);
        }
        mma_commit(&x_empty[s]);
        mma_commit(&a_empty[as]);
      }
      mma_commit(acc_full);  // also drains in-flight MMAs on the abort path
      if (*abort_flag) {
        int dummy_abort = 0;
        mbar_wait(acc_full, 0, reinterpret_cast<volatile int*>(&dummy_abort), p.err);
      }
    }
  } else {
    // ------------------------------------------------ dequant warps 0..3
    const int r = warp * 32 + lane;  // feature row within the tile == TMEM lane
    const int n = n0 + r;
    const bool row_ok = n < p.N;
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    for (int kb = 0; kb < num_kb; ++kb) {
      const int s = kb % S;
      const uint32_t ph = (kb / S) & 1;
      const int as = kb % kAStages;
      const uint32_t aph = (kb / kAStages) & 1;
      // group parameters of this row for the two 32-wide halves of the stage
      uint32_t s2[2] = {0u, 0u}, b2[2] = {0u, 0u};
      float fs[2] = {0.f, 0.f};
      if (row_ok) {
        if (QK == kMxfp8) {
          const uint8_t* sc = static_cast<const uint8_t*>(p.scales) + static_cast<int64_t>(n) * (p.K / 32) + kb * 2;
          fs[0] = e8m0_to_f32(__ldg(sc));
          fs[1] = e8m0_to_f32(__ldg(sc + 1));
        } else {
          const int gpr = p.K / p.gs;
          const uint16_t* sc = static_cast<const uint16_t*>(p.scales) + static_cast<int64_t>(n) * gpr;
          const uint16_t* bi = p.biases + static_cast<int64_t>(n) * gpr;
          const int g0 = (kb * BK) / p.gs, g1 = (kb * BK + 32) / p.gs;
          s2[0] = bcast_bf16x2(__ldg(sc + g0));
          b2[0] = bcast_bf16x2(__ldg(bi + g0));
          s2[1] = bcast_bf16x2(__ldg(sc + g1));
          b2[1] = bcast_bf16x2(__ldg(bi + g1));
        }
      }
      if (!mbar_wait(&w_full[s], ph, abort_flag, p.err)) break;
      if (!mbar_wait(&a_empty[as], aph ^ 1, abort_flag, p.err)) break;
      const uint8_t* wrow = ws + s * C::kWStage + r * WB;
      uint32_t o[32];
      if (QK == kAffine4) {
        // 32-byte rows, 32B swizzle: 16-byte chunk c sits at c ^ ((r >> 2) & 1)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ ((r >> 2) & 1)) << 4));
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t q4[4];
            deq_affine4_word(wv[i], s2[c], b2[c], q4);
#pragma unroll
            for (int t = 0; t < 4; ++t) o[c * 16 + i * 4 + t] = q4[t];
          }
        }
      } else {
        // 64-byte rows, 64B swizzle: 16-byte chunk c sits at c ^ ((r >> 1) & 3)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ ((r >> 1) & 3)) << 4));
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (QK == kMxfp8) deq_mxfp8_word(wv[i], fs[c >> 1], o[c * 8 + i * 2], o[c * 8 + i * 2 + 1]);
            else deq_affine8_word(wv[i], s2[c >> 1], b2[c >> 1], o[c * 8 + i * 2], o[c * 8 + i * 2 + 1]);
          }
        }
      }
      tmem_st_32x32b_x32(tmem + t_lane + C::kACol + as * 32, o);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        mbar_arrive(&w_empty[s]);
      }
    }

    // ------------------------------------------------ epilogue
    if (!*abort_flag && mbar_wait(acc_full, 0, abort_flag, p.err)) {
      tc_fence_after();
      uint16_t* stg = reinterpret_cast<uint16_t*>(xs);  // all stages are drained by now
      const float bias_n = (p.bias != nullptr && row_ok) ? bf16_to_f32(__ldg(p.bias + n)) : 0.f;
      const bool gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
      const bool two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + t_lane + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float a = rbf16(__uint_as_float(v[j]));
          if (p.bias != nullptr) a = rbf16(__fadd_rn(a, bias_n));
          if (p.epi == LTXQ_EPI_GELU) a = gelu_ref(a);
          stg[j * kStagePitch + r] = f32_to_bf16(a);
        }
        named_bar_sync(1, 128);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = i * 128 + static_cast<int>(threadIdx.x);
          const int j = q >> 4, f = (q & 15) * 8;
          const int m = m0 + c * 32 + j, nf = n0 + f;
          if (m < p.M && nf < p.N) {
            uint4 bw = *reinterpret_cast<const uint4*>(stg + j * kStagePitch + f);
            const int64_t off = static_cast<int64_t>(m) * p.N + nf;
            if (gated) {
              const uint4 rv = __ldg(reinterpret_cast<const uint4*>(p.residual + off));
              float g[8];
              load_vec8(p.gate, vec_row(p.gate, m), nf, g);
              const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
              uint32_t bwv[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float p0 = __fmul_rn(lo_bf16(bwv[k]), g[2 * k]);
                const float p1 = __fmul_rn(hi_bf16(bwv[k]), g[2 * k + 1]);
                const float r0 = lo_bf16(rw[k]), r1 = hi_bf16(rw[k]);
                bwv[k] = two_round ? pack_bf16x2(__fadd_rn(r0, rbf16(p0)), __fadd_rn(r1, rbf16(p1)))
                                   : pack_bf16x2(__fadd_rn(p0, r0), __fadd_rn(p1, r1));
              }
              bw = make_uint4(bwv[0], bwv[1], bwv[2], bwv[3]);
            }
            *reinterpret_cast<uint4*>(p.out + off) = bw;
          }
        }
        named_bar_sync(1, 128);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <int QK, int BN>
static ltxq_status launch_cfg(const CUtensorMap& tx, const CUtensorMap& tw, const Params& p, cudaStream_t stream) {
  using C = Cfg<QK, BN>;
  auto kern = qgemm_kernel<QK, BN>;
  ltxq_status st =
      cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem), "smem attribute");
  if (st) return st;
  const dim3 grid((p.N + BM - 1) / BM, (p.M + BN - 1) / BN);
  kern<<<grid, kThreads, C::kSmem, stream>>>(tx, tw, p);
  return cuda_check(cudaGetLastError(), "qgemm launch");
}

template <int QK>
static ltxq_status launch_qk(int bn, const CUtensorMap& tx, const CUtensorMap& tw, const Params& p,
                             cudaStream_t stream) {
  if (bn == 64) return launch_cfg<QK, 64>(tx, tw, p, stream);
  if (bn == 128) return launch_cfg<QK, 128>(tx, tw, p, stream);
  return launch_cfg<QK, 256>(tx, tw, p, stream);
}

}  // namespace gemm

static ltxq_status check_epilogue(const ltxq_epilogue* epi, int64_t M, int64_t N) {
  if (!epi) return LTXQ_OK;
  switch (epi->kind) {
    case LTXQ_EPI_NONE:
    case LTXQ_EPI_GELU:
      return LTXQ_OK;
    case LTXQ_EPI_GATED_RESIDUAL:
    case LTXQ_EPI_GATE_THEN_ADD: {
      if (!epi->residual) return fail(LTXQ_ERR_INVALID, "epilogue: residual is NULL");
      if (reinterpret_cast<uintptr_t>(epi->residual) & 15u)
        return fail(LTXQ_ERR_UNSUPPORTED, "epilogue: residual must be 16-byte aligned");
      const ltxq_vec& g = epi->gate;
      if (!g.ptr) return fail(LTXQ_ERR_INVALID, "epilogue: gate is NULL");
      if (g.dtype != LTXQ_BF16 && g.dtype != LTXQ_F32) return fail(LTXQ_ERR_UNSUPPORTED, "epilogue: gate dtype");
      if (reinterpret_cast<uintptr_t>(g.ptr) & 15u) return fail(LTXQ_ERR_UNSUPPORTED, "epilogue: gate not 16B aligned");
      if (g.rows_per_vec < 0) return fail(LTXQ_ERR_INVALID, "epilogue: gate rows_per_vec < 0");
      if (g.rows_per_vec > 0 && (g.row_stride < N || (g.row_stride * (g.dtype == LTXQ_F32 ? 4 : 2)) % 16 != 0))
        return fail(LTXQ_ERR_UNSUPPORTED, "epilogue: gate row stride");
      (void)M;
      return LTXQ_OK;
    }
    default:
      return fail(LTXQ_ERR_INVALID, "epilogue: unknown kind");
  }
}

ltxq_status launch_qlinear(const void* x, int64_t M, const ltxq_qweight& w, const ltxq_epilogue* epi, void* out,
                           cudaStream_t stream) {
  int64_t R, L;
  if (ltxq_status st = check_qweight(w, true, &R, &L)) return st;
  if (!x || !out) return fail(LTXQ_ERR_INVALID, "qlinear: x/out is NULL");
  if (M < 0) return fail(LTXQ_ERR_INVALID, "qlinear: M < 0");
  if (w.layout != LTXQ_LAYOUT_STD)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: pretransposed weights are not supported by the GEMM yet");
  const int64_t N = w.n_out, K = w.k_in;
  if (K % gemm::BK != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: K must be a multiple of 64");
  if (N % 8 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: N must be a multiple of 8");
  if (M > 0x7FFFFFFF / 2 || N > 0x7FFFFFFF / 2 || K > 0x7FFFFFFF / 2)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: dimension too large");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: x/out must be 16-byte aligned");
  if (w.bias && (reinterpret_cast<uintptr_t>(w.bias) & 1u)) return fail(LTXQ_ERR_INVALID, "qlinear: bias misaligned");
  if (ltxq_status st = check_epilogue(epi, M, N)) return st;
  if (M == 0) return LTXQ_OK;

  const int qk = w.mode == LTXQ_MXFP8 ? gemm::kMxfp8 : (w.bits == 8 ? gemm::kAffine8 : gemm::kAffine4);
  const int bn = M <= 64 ? 64 : (M <= 128 ? 128 : 256);
  CUtensorMap tx, tw;
  if (ltxq_status st = encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, K * 2, gemm::BK, bn,
                                      CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  const int wbytes_row = static_cast<int>(K * w.bits / 8);
  const uint32_t wbox = qk == gemm::kAffine4 ? 32 : 64;
  const CUtensorMapSwizzle wsw = qk == gemm::kAffine4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (ltxq_status st =
          encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.weight, wbytes_row, N, wbytes_row, wbox, gemm::BM, wsw))
    return st;

  gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.gs = w.group_size;
  p.scales = w.scales;
  p.biases = static_cast<const uint16_t*>(w.biases);
  p.bias = static_cast<const uint16_t*>(w.bias);
  p.epi = epi ? epi->kind : LTXQ_EPI_NONE;
  if (epi && (p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD)) {
    p.gate = to_vec(epi->gate);
    p.residual = static_cast<const uint16_t*>(epi->residual);
  } else {
    p.gate = VecArg{nullptr, LTXQ_F32, 0, 0};
    p.residual = nullptr;
  }
  p.out = static_cast<uint16_t*>(out);
  p.err = dev_error_word();
  if (!p.err) return fail(LTXQ_ERR_CUDA, "qlinear: device error word unavailable");
  switch (qk) {
    case gemm::kAffine8: return gemm::launch_qk<gemm::kAffine8>(bn, tx, tw, p, stream);
    case gemm::kAffine4: return gemm::launch_qk<gemm::kAffine4>(bn, tx, tw, p, stream);
    default: return gemm::launch_qk<gemm::kMxfp8>(bn, tx, tw, p, stream);
  }
}

static size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace ltxq

extern "C" {

size_t ltxq_qlinear_workspace_size(int64_t M, const ltxq_qweight* w) {
  (void)M;
  (void)w;
  return 0;
}

size_t ltxq_adaln_qlinear_workspace_size(int64_t M, const ltxq_qweight* w) {
  if (!w || M <= 0) return 0;
  return ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w->k_in) * 2);
}

size_t ltxq_feed_forward_workspace_size(int64_t M, const ltxq_qweight* w_in, const ltxq_qweight* w_out) {
  if (!w_in || !w_out || M <= 0) return 0;
  return ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->k_in) * 2) +
         ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->n_out) * 2);
}

ltxq_status ltxq_qlinear(const void* x, int64_t M, const ltxq_qweight* w, const ltxq_epilogue* epi, void* out,
                         void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  if (!w) return ltxq::fail(LTXQ_ERR_INVALID, "qlinear: weight is NULL");
  return ltxq::launch_qlinear(x, M, *w, epi, out, static_cast<cudaStream_t>(stream));
}

ltxq_status ltxq_adaln_qlinear(const void* x, int64_t M, const ltxq_prologue* pro, const ltxq_qweight* w,
                               const ltxq_epilogue* epi, void* out, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (!w || !pro) return ltxq::fail(LTXQ_ERR_INVALID, "adaln_qlinear: NULL argument");
  const size_t need = ltxq_adaln_qlinear_workspace_size(M, w);
  if (workspace_bytes < need || (need && !workspace))
    return ltxq::fail(LTXQ_ERR_INVALID, "adaln_qlinear: workspace too small");
  if (M == 0) return LTXQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w->k_in, *pro, workspace, s)) return st;
  return ltxq::launch_qlinear(workspace, M, *w, epi, out, s);
}

ltxq_status ltxq_feed_forward(const void* x, int64_t M, const ltxq_prologue* pro, const ltxq_qweight* w_in,
                              const ltxq_qweight* w_out, const ltxq_epilogue* epi, void* out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!w_in || !w_out) return ltxq::fail(LTXQ_ERR_INVALID, "feed_forward: NULL weight");
  if (w_out->k_in != w_in->n_out) return ltxq::fail(LTXQ_ERR_INVALID, "feed_forward: inner dimensions differ");
  const size_t need = ltxq_feed_forward_workspace_size(M, w_in, w_out);
  if (workspace_bytes < need || (need && !workspace))
    return ltxq::fail(LTXQ_ERR_INVALID, "feed_forward: workspace too small");
  if (M == 0) return LTXQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const void* a = x;
  if (pro) {
    if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w_in->k_in, *pro, ws, s)) return st;
    a = ws;
  }
  void* hidden = ws + ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->k_in) * 2);
  ltxq_epilogue gelu{};
  gelu.kind = LTXQ_EPI_GELU;
  if (ltxq_status st = ltxq::launch_qlinear(a, M, *w_in, &gelu, hidden, s)) return st;
  return ltxq::launch_qlinear(hidden, M, *w_out, epi, out, s);
}

}  // extern "C"
