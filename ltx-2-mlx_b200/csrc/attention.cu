// attention.cu -- scaled-dot-product attention forward without a mask, the
// block's attention core: O = softmax(Q K^T * scale) V per (batch, head),
// what mx.fast.scaled_dot_product_attention computes for the reference
// (model/transformer/attention.py:170-302, its steel_attention Metal kernel
// kernels/steel_attention.py:251-280), for head_dim 128 (video) and 64
// (audio / audio-video cross attention).
//
// One CTA takes two 128-query tiles (A, B) of one (batch, head) and streams
// the keys in 128-row stages:
//   warp 8  (TMA)     Q_A, Q_B once; then K_j, V_j into a ring of stages,
//                     3D tensor maps (columns, rows, batch) so that rows
//                     past the batch's end read as zeros, never the next
//                     batch's rows;
//   warp 9  (MMA)     S_t = Q_t K_j^T into TMEM (tcgen05.mma kind::f16, both
//                     operands from 128B-swizzled shared memory), then
//                     O_t += P_t V_j with P_t read from TMEM and V_j as an
//                     MN-major operand;
//   warps 0-3 / 4-7   the softmax of tile A / B: thread = query row = TMEM
//                     lane.  Per stage: the row maximum of S (masked past the
//                     last key), exp2 of the scaled scores against the
//                     running maximum, the running sum in fp32, and P in bf16
//                     written over the S columns it came from (P of key pair
//                     (2c, 2c+1) in column c, read only after S columns 0..2c+1
//                     were).  The running maximum is raised only when a
//                     row's maximum grows by more than 2^8 (then O is rescaled
//                     in TMEM, after the previous P V product completed), so
//                     P stays below 256 and most stages touch O not at all.
//                     A full stage after the first takes one pass over S,
//                     with P held in registers until the maximum is known
//                     to stay.
//   epilogue          O / sum, rounded to bf16, one row per thread.
// S_t(j) overwrites P_t(j-1), so it is issued once PV_t(j-1) completed.
// Measured and not kept: 64-key stages with S double-buffered per tile (S of
// the next stage computed during the softmax of this one) ran 20 % slower,
// the per-stage hand-offs doubling; a quarter of the exponentials on the
// FMA pipe (polynomial) ran 6 % slower: the softmax is issue-bound, not
// bound by the MUFU.
// TMEM: S_A [0, 128), S_B [128, 256), O_A [256, 256 + D), O_B [256 + D, ...).
// Every mbarrier wait is bounded; an expired wait raises the device error
// word and the CTA unwinds.
#include "common.cuh"

namespace ltxq {
namespace fmha {

constexpr int BQ = 128;   // queries per tile (MMA M, TMEM lanes)
constexpr int BKV = 128;  // keys per stage (MMA N of S = Q K^T, MMA K of P V)
constexpr int kTmaWarp = 8, kMmaWarp = 9, kThreads = 320;
constexpr float kRescaleLog2 = 8.f;  // the running maximum lags a row's maximum by at most this (log2 units)

template <int D>
struct Plan {
  static constexpr int kRegion = BQ * 64 * 2;  // 128 rows x 64 bf16, 128-byte swizzle
  static constexpr int kRegions = D / 64;
  static constexpr int kTile = kRegion * kRegions;
  static constexpr int kStages = D == 128 ? 2 : 4;
  static constexpr int kKOff = 2 * kTile;  // Q_A, Q_B first
  static constexpr int kVOff = kKOff + kStages * kTile;
  static constexpr int kBarOff = kVOff + kStages * kTile;
  static constexpr int kSmem = 1024 + kBarOff + 256;
  static constexpr uint32_t kOCol = 256;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

struct Bars {
  uint64_t *q_full, *k_full, *v_full, *kv_empty, *s_full, *p_full, *o_done;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, int Tq, int Tk, float scale_log2,
                    uint16_t* __restrict__ out, int64_t out_stride, unsigned int* err) {
  using P = Plan<D>;
  constexpr int S = P::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* b = reinterpret_cast<uint64_t*>(smem + P::kBarOff);
  Bars bb;
  bb.q_full = b;
  bb.k_full = b + 1;
  bb.v_full = b + 1 + S;
  bb.kv_empty = b + 1 + 2 * S;
  bb.s_full = b + 1 + 3 * S;
  bb.p_full = b + 3 + 3 * S;
  bb.o_done = b + 5 + 3 * S;
  bb.tmem_slot = reinterpret_cast<uint32_t*>(b + 7 + 3 * S);
  bb.abort_flag = reinterpret_cast<volatile int*>(bb.tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 2 * BQ;
  const int head = blockIdx.y, batch = blockIdx.z;
  const int n_kv = (Tk + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(bb.q_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(&bb.k_full[s], 1);
      mbar_init(&bb.v_full[s], 1);
      mbar_init(&bb.kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bb.s_full[t], 1);
      mbar_init(&bb.p_full[t], 4);  // one arrive per softmax warp of the tile
      mbar_init(&bb.o_done[t], 1);
    }
    *bb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(bb.tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bb.tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      const int col0 = head * D;
      mbar_arrive_expect_tx(bb.q_full, 2 * P::kTile);
      for (int t = 0; t < 2; ++t)
        for (int r = 0; r < P::kRegions; ++r)
          tma_load_3d(smem + t * P::kTile + r * P::kRegion, &tq, bb.q_full, col0 + 64 * r, q0 + t * BQ, batch);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % S;
        if (!mbar_wait(&bb.kv_empty[s], ((j / S) & 1) ^ 1, bb.abort_flag, err)) break;
        mbar_arrive_expect_tx(&bb.k_full[s], P::kTile);
        for (int r = 0; r < P::kRegions; ++r)
          tma_load_3d(smem + P::kKOff + s * P::kTile + r * P::kRegion, &tk, &bb.k_full[s], col0 + 64 * r, j * BKV,
                      batch);
        mbar_arrive_expect_tx(&bb.v_full[s], P::kTile);
        for (int r = 0; r < P::kRegions; ++r)
          tma_load_3d(smem + P::kVOff + s * P::kTile + r * P::kRegion, &tv, &bb.v_full[s], col0 + 64 * r, j * BKV,
                      batch);
        issued = j + 1;
      }
      if (*bb.abort_flag) {
        // let the copies already issued land before the CTA's shared memory is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
      (void)issued;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16_f32(BQ, BKV);
      const uint32_t idesc_o = idesc_bf16_f32(BQ, D) | (1u << 16);  // B (V) MN-major
      bool ok = mbar_wait(bb.q_full, 0, bb.abort_flag, err);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j % S;
        const uint32_t ph = (j / S) & 1;
        if (!mbar_wait(&bb.k_full[s], ph, bb.abort_flag, err)) break;
        const uint32_t kbase = smem_u32(smem + P::kKOff + s * P::kTile);
        for (int t = 0; t < 2 && ok; ++t) {
          // S_t's columns hold P_t of the previous stage until that P V product completes
          if (j > 0 && !mbar_wait(&bb.o_done[t], (j - 1) & 1, bb.abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t qbase = smem_u32(smem + t * P::kTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * P::kRegion + (kk & 3) * 32;
            mma_bf16_ss(tmem + 128u * t, smem_desc_sw128(qbase + off), smem_desc_sw128(kbase + off), idesc_s,
                        kk != 0 ? 1u : 0u);
          }
          mma_commit(&bb.s_full[t]);
        }
        if (!ok || !mbar_wait(&bb.v_full[s], ph, bb.abort_flag, err)) break;
        const uint32_t vbase = smem_u32(smem + P::kVOff + s * P::kTile);
        for (int t = 0; t < 2 && ok; ++t) {
          if (!mbar_wait(&bb.p_full[t], j & 1, bb.abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            mma_bf16_ts(tmem + P::kOCol + D * t, tmem + 128u * t + kk * 8,
                        smem_desc_sw128_mn(vbase + kk * 2048, P::kRegion, 1024), idesc_o, (j | kk) != 0 ? 1u : 0u);
          mma_commit(&bb.o_done[t]);
        }
        mma_commit(&bb.kv_empty[s]);
      }
      if (*bb.abort_flag) {
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------ softmax of tile t
    const int t = warp >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t s_col = tmem + t_lane + 128u * t;
    const uint32_t o_col = tmem + t_lane + P::kOCol + D * t;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool got = mbar_wait(&bb.s_full[t], j & 1, bb.abort_flag, err);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int n_valid = min(BKV, Tk - j * BKV);
      // Fast path (a full stage after the first): one pass over S, exps
      // against the running maximum, P kept in registers and stored only if
      // no row's maximum grew past the threshold.
      bool redo = true;
      float ls = 0.f;

      if (j > 0 && n_valid == BKV) {
        uint32_t pw[BKV / 2];
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < BKV / 32; c += 2) {
          uint32_t v[2][32];  // two loads in flight per wait
          tmem_ld_32x32b_x32(s_col + c * 32, v[0]);
          tmem_ld_32x32b_x32(s_col + c * 32 + 32, v[1]);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float s0 = __uint_as_float(v[h][2 * i]), s1 = __uint_as_float(v[h][2 * i + 1]);
              mt = fmaxf(mt, fmaxf(s0, s1));
              const float p0 = ex2(__fmaf_rn(s0, scale_log2, -m_run));
              const float p1 = ex2(__fmaf_rn(s1, scale_log2, -m_run));
              ls += p0 + p1;
              pw[(c + h) * 16 + i] = pack_bf16x2(p0, p1);
            }
        }
        redo = __any_sync(0xffffffffu, mt * scale_log2 > m_run + kRescaleLog2);
        if (!redo) {
#pragma unroll
          for (int c = 0; c < BKV / 32; ++c) tmem_st_32x32b_x16(s_col + c * 16, pw + c * 16);
        }
      }
      if (redo) {
        ls = 0.f;
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(s_col + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i < n_valid) mt = fmaxf(mt, __uint_as_float(v[i]));
        }
        mt *= scale_log2;
        if (j == 0) {
          m_run = mt;
        } else {
          const bool grow = mt > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, grow)) {
            // O holds the products up to stage j-1: rescale it once they are complete
            const bool done = mbar_wait(&bb.o_done[t], (j - 1) & 1, bb.abort_flag, err);
            if (!__all_sync(0xffffffffu, done)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const float f = grow ? ex2(m_run - mt) : 1.f;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t v[32];
              tmem_ld_32x32b_x32(o_col + c * 32, v);
              tmem_wait_ld();
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(__uint_as_float(v[h * 16 + i]) * f);
                tmem_st_32x32b_x16(o_col + c * 32 + h * 16, w);
              }
            }
            if (grow) {
              l_run *= f;
              m_run = mt;
            }
          }
        }
#pragma unroll
        for (int c = 0; c < BKV / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(s_col + c * 32, v);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int k0 = c * 32 + 2 * i;
            const float p0 = k0 < n_valid ? ex2(__fmaf_rn(__uint_as_float(v[2 * i]), scale_log2, -m_run)) : 0.f;
            const float p1 =
                k0 + 1 < n_valid ? ex2(__fmaf_rn(__uint_as_float(v[2 * i + 1]), scale_log2, -m_run)) : 0.f;
            ls += p0 + p1;
            w[i] = pack_bf16x2(p0, p1);
          }
          tmem_st_32x32b_x16(s_col + c * 16, w);
        }
      }
      l_run += ls;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bb.p_full[t]);
    }
    if (ok && n_kv > 0) {
      const bool done = mbar_wait(&bb.o_done[t], (n_kv - 1) & 1, bb.abort_flag, err);
      if (__all_sync(0xffffffffu, done)) {
        tc_fence_after();
        const float inv = 1.f / l_run;
        const int qrow = q0 + t * BQ + row;
        uint16_t* orow = out + (static_cast<int64_t>(batch) * Tq + qrow) * out_stride + head * D;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(o_col + c * 32, v);
          tmem_wait_ld();
          if (qrow < Tq) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 o4;
              o4.x = pack_bf16x2(__uint_as_float(v[8 * g + 0]) * inv, __uint_as_float(v[8 * g + 1]) * inv);
              o4.y = pack_bf16x2(__uint_as_float(v[8 * g + 2]) * inv, __uint_as_float(v[8 * g + 3]) * inv);
              o4.z = pack_bf16x2(__uint_as_float(v[8 * g + 4]) * inv, __uint_as_float(v[8 * g + 5]) * inv);
              o4.w = pack_bf16x2(__uint_as_float(v[8 * g + 6]) * inv, __uint_as_float(v[8 * g + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c * 32 + 8 * g) = o4;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
static ltxq_status launch(const void* q, const void* k, const void* v, int64_t B, int64_t Tq, int64_t Tk,
                          int64_t heads, int64_t qs, int64_t ks, int64_t vs, float scale, void* out,
                          cudaStream_t stream) {
  using P = Plan<D>;
  CUtensorMap mq, mk, mv;
  const uint32_t box[3] = {64, BQ, 1};
  const uint64_t w = static_cast<uint64_t>(heads * D);
  {
    const uint64_t dims[3] = {w, static_cast<uint64_t>(Tq), static_cast<uint64_t>(B)};
    const uint64_t str[2] = {static_cast<uint64_t>(qs) * 2, static_cast<uint64_t>(qs * Tq) * 2};
    if (ltxq_status st = encode_tmap_3d(&mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, dims, str, box,
                                        CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  {
    const uint64_t dims[3] = {w, static_cast<uint64_t>(Tk), static_cast<uint64_t>(B)};
    const uint64_t sk[2] = {static_cast<uint64_t>(ks) * 2, static_cast<uint64_t>(ks * Tk) * 2};
    const uint64_t sv[2] = {static_cast<uint64_t>(vs) * 2, static_cast<uint64_t>(vs * Tk) * 2};
    if (ltxq_status st = encode_tmap_3d(&mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, dims, sk, box,
                                        CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
    if (ltxq_status st = encode_tmap_3d(&mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, v, dims, sv, box,
                                        CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
  }
  unsigned int* err = dev_error_word();
  if (!err) return fail(LTXQ_ERR_CUDA, "attention: device error word unavailable");
  static const bool attr_ok = cudaFuncSetAttribute(fmha_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   P::kSmem) == cudaSuccess;
  if (!attr_ok) return fail(LTXQ_ERR_CUDA, "attention: shared-memory attribute");
  const dim3 grid(static_cast<unsigned>((Tq + 2 * BQ - 1) / (2 * BQ)), static_cast<unsigned>(heads),
                  static_cast<unsigned>(B));
  const float scale_log2 = scale * 1.4426950408889634f;
  fmha_fwd_kernel<D><<<grid, kThreads, P::kSmem, stream>>>(mq, mk, mv, static_cast<int>(Tq), static_cast<int>(Tk),
                                                            scale_log2, static_cast<uint16_t*>(out), heads * D, err);
  return launch_check("attention launch");
}

}  // namespace fmha
}  // namespace ltxq

extern "C" ltxq_status ltxq_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t q_rows,
                                      int64_t kv_rows, int64_t heads, int64_t head_dim, int64_t q_stride,
                                      int64_t k_stride, int64_t v_stride, float scale, void* out, void* stream) {
  using namespace ltxq;
  if (!q || !k || !v || !out) return fail(LTXQ_ERR_INVALID, "attention: NULL tensor");
  if (batch < 0 || q_rows < 0 || heads <= 0) return fail(LTXQ_ERR_INVALID, "attention: bad shape");
  if (head_dim != 64 && head_dim != 128) return fail(LTXQ_ERR_UNSUPPORTED, "attention: head_dim must be 64 or 128");
  if (kv_rows <= 0) return fail(LTXQ_ERR_INVALID, "attention: kv_rows must be >= 1");
  const int64_t w = heads * head_dim;
  if (q_stride < w || k_stride < w || v_stride < w) return fail(LTXQ_ERR_INVALID, "attention: row stride < heads*head_dim");
  if ((q_stride | k_stride | v_stride) % 8 != 0)
    return fail(LTXQ_ERR_UNSUPPORTED, "attention: row strides must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
       reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "attention: tensors must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(LTXQ_ERR_INVALID, "attention: scale must be > 0");
  if (q_rows > 0x3FFFFFFF || kv_rows > 0x3FFFFFFF || batch > 65535 || heads > 65535)
    return fail(LTXQ_ERR_UNSUPPORTED, "attention: dimension too large");
  if (batch == 0 || q_rows == 0) return LTXQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    return fmha::launch<128>(q, k, v, batch, q_rows, kv_rows, heads, q_stride, k_stride, v_stride, scale, out, s);
  return fmha::launch<64>(q, k, v, batch, q_rows, kv_rows, heads, q_stride, k_stride, v_stride, scale, out, s);
}
