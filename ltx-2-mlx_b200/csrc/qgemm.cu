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
#include "gemm_epilogue.cuh"

namespace ltxq {

ltxq_status check_qweight(const ltxq_qweight& w, bool need_data, int64_t* R, int64_t* L);
ltxq_status launch_adaln_modulate(const void* x, int x_dtype, int64_t rows, int64_t C, const ltxq_prologue& pro,
                                  void* out, cudaStream_t stream, const ltxq_mx_act* out_mx);
ltxq_status launch_mx_split(const void* x, int64_t M, int64_t K, int terms, void* hi, void* lo, void* sf_hi,
                            void* sf_lo, cudaStream_t stream);
ltxq_mx_act mx_workspace_act(int64_t M, int64_t K, int terms, void* workspace);
namespace gemm {
struct Params;
}
size_t mx_workspace_bytes(int64_t M, const ltxq_qweight& w);
ltxq_status launch_qlinear_mx(const void* x, int64_t M, const ltxq_qweight& w, const gemm::Params& p, void* workspace,
                              cudaStream_t stream);

namespace gemm {

constexpr int BM = 128;  // output features per CTA (MMA M, TMEM lanes)
constexpr int BK = 64;   // K per pipeline stage
constexpr int kDeqWarps = 8;  // two per TMEM lane quarter; each converts one 32-wide half of a stage
constexpr int kTmaWarp = 8, kMmaWarp = 9, kThreads = 320;
constexpr int kStagePitch = 136;  // epilogue staging row pitch in bf16 (128 + 8 pad)
constexpr int kPrefetch = 2;      // scale/bias register prefetch distance (stages); also the dequant loop's unroll

// kMxfp8F: mxfp8 data flagged LTXQ_QW_MXFP8_FINITE (short conversion)
enum QKind { kAffine8 = 0, kAffine4 = 1, kMxfp8 = 2, kMxfp8F = 3 };
constexpr bool is_mx(int qk) { return qk == kMxfp8 || qk == kMxfp8F; }

template <int QK>
struct QTraits {
  static constexpr int kWBytes = QK == kAffine4 ? 32 : 64;  // packed bytes per row per stage
};

// output tiles of the pair kernel, how many stay whole, K splits of the rest
struct Sched {
  int tiles, dp, splits;
};

// 16-byte blocks of a row's group parameters (8 bf16 scales / biases for
// affine, 16 E8M0 bytes for mxfp8) held in registers, with the next block
// prefetched one block ahead: one vector load per 4..16 stages instead of two
// scattered 2-byte loads per stage.
template <int QK>
struct GroupCursor {
  static constexpr int kPerBlk = is_mx(QK) ? 16 : 8;
  const uint4* sb;
  const uint4* bb;
  int nblk, cur;
  uint4 cs, cb, ns, nb;
  // g0: the first group get() will be asked for
  __device__ __forceinline__ void init(const Params& p, int64_t srow, bool ok, int g0) {
    const int gpr = is_mx(QK) ? p.K / 32 : p.K / p.gs;
    nblk = ok ? gpr / kPerBlk : 0;
    sb = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.scales) + srow * (is_mx(QK) ? 1 : 2));
    bb = is_mx(QK) ? nullptr : reinterpret_cast<const uint4*>(p.biases + srow);
    cur = g0 / kPerBlk;
    const uint4 z = make_uint4(0, 0, 0, 0);
    cs = cur < nblk ? __ldg(sb + cur) : z;
    cb = (!is_mx(QK) && cur < nblk) ? __ldg(bb + cur) : z;
    ns = cur + 1 < nblk ? __ldg(sb + cur + 1) : z;
    nb = (!is_mx(QK) && cur + 1 < nblk) ? __ldg(bb + cur + 1) : z;
  }
  // parameters of group g (monotone, advancing by at most one block per call)
  __device__ __forceinline__ void get(int g, uint32_t& s, uint32_t& b) {
    const int blk = g / kPerBlk;
    if (blk != cur && nblk > 0) {
      cs = ns;
      cb = nb;
      cur = blk;
      if (blk + 1 < nblk) {
        ns = __ldg(sb + blk + 1);
        if (!is_mx(QK)) nb = __ldg(bb + blk + 1);
      }
    }
    const int e = g - blk * kPerBlk;
    if (is_mx(QK)) {
      const int wi = e >> 2;
      const uint32_t w = wi == 0 ? cs.x : wi == 1 ? cs.y : wi == 2 ? cs.z : cs.w;
      s = (w >> (8 * (e & 3))) & 0xFFu;
      b = 0u;
    } else {
      const int wi = e >> 1;
      const uint32_t ws_ = wi == 0 ? cs.x : wi == 1 ? cs.y : wi == 2 ? cs.z : cs.w;
      const uint32_t wb_ = wi == 0 ? cb.x : wi == 1 ? cb.y : wi == 2 ? cb.z : cb.w;
      const int sh = 16 * (e & 1);
      s = bcast_bf16x2(ws_ >> sh);
      b = bcast_bf16x2(wb_ >> sh);
    }
  }
};

// Group parameters of (row n, K-half starting at element k) as the packed
// form the converters take: affine -> bf16x2 broadcast scale / bias;
// mxfp8 -> E8M0 byte in `s`.
template <int QK>
__device__ __forceinline__ void load_group(const Params& p, int64_t row_off_scales, int k, bool ok, uint32_t& s,
                                           uint32_t& b) {
  if (!ok) {
    s = 0u;
    b = 0u;
    return;
  }
  if (is_mx(QK)) {
    s = __ldg(static_cast<const uint8_t*>(p.scales) + row_off_scales + (k >> 5));
    b = 0u;
  } else {
    const int g = k / p.gs;
    s = bcast_bf16x2(__ldg(static_cast<const uint16_t*>(p.scales) + row_off_scales + g));
    b = bcast_bf16x2(__ldg(p.biases + row_off_scales + g));
  }
}

// ---------------------------------------------------------------------------
// Shared-memory / barrier plan of one CTA.  BNC = tokens whose activation
// rows this CTA stages (the MMA's N in single-CTA mode; half of it in pair
// mode).  BN = MMA N = accumulator columns.
template <int QK, int BN, int BNC>
struct Plan {
  static constexpr int kXStage = BNC * BK * 2;
  static constexpr int kWStage = BM * QTraits<QK>::kWBytes;
  static constexpr int kStagingBytes = 2 * 32 * kStagePitch * 2;  // two epilogue staging tiles
  static constexpr int kBudget = 200 * 1024;
  static constexpr int kStagesRaw = kBudget / (kXStage + kWStage);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kBarOff = kStages * (kXStage + kWStage);
  static constexpr int kSmem = 1024 + kBarOff + 512;
  // TMEM: fp32 accumulator (BN columns) followed by the bf16 A-operand ring
  // (32 columns per 64-wide K stage).
  static constexpr uint32_t kTmemCols = BN >= 256 ? 512 : 256;
  static constexpr int kAStages =
      (static_cast<int>(kTmemCols) - BN) / 32 > 8 ? 8 : (static_cast<int>(kTmemCols) - BN) / 32;
  static constexpr uint32_t kACol = BN;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kAStages >= 2, "TMEM A ring needs two stages");
  static_assert(kStagingBytes <= kStages * kXStage, "epilogue staging reuses the drained activation stages");
};

struct Bars {
  uint64_t *x_full, *x_empty, *w_full, *w_empty, *a_full, *a_empty, *acc_full, *acc_empty;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
};

template <int S, int AS>
__device__ __forceinline__ Bars carve_bars(uint8_t* base) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  Bars r;
  r.x_full = b;
  r.x_empty = b + S;
  r.w_full = b + 2 * S;
  r.w_empty = b + 3 * S;
  r.a_full = b + 4 * S;
  r.a_empty = b + 4 * S + AS;
  r.acc_full = b + 4 * S + 2 * AS;
  r.acc_empty = b + 4 * S + 2 * AS + 1;
  r.tmem_slot = reinterpret_cast<uint32_t*>(r.acc_empty + 1);
  r.abort_flag = reinterpret_cast<volatile int*>(r.tmem_slot + 1);
  return r;
}

// Dequant warps (warp 0..7): convert this CTA's 128 packed weight rows stage
// by stage into the TMEM A ring.  `a_full_remote` != 0 means the A-full
// barriers live in the pair leader (cluster address of a_full[0]).  The
// num_kb stages cover K stages [kb_first, kb_first + num_kb); kb_base is the
// position of the first one in the smem / TMEM rings.
template <int QK, int S, int AS, uint32_t kACol>
__device__ __forceinline__ void dequant_loop(const Params& p, const Bars& bb, uint8_t* ws, uint32_t tmem, int warp,
                                             int lane, int n0, int num_kb, uint32_t a_full_remote, int kb_base,
                                             int kb_first) {
  constexpr int WB = QTraits<QK>::kWBytes;
  constexpr int kWStage = BM * WB;
  const int q = warp & 3;      // TMEM lane quarter
  const int half = warp >> 2;  // which 32-wide half of every K stage
  const int r = q * 32 + lane; // feature row within the tile == TMEM lane
  const int n = n0 + r;
  const bool row_ok = n < p.N;
  const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
  const int64_t srow = static_cast<int64_t>(n) * (is_mx(QK) ? p.K / 32 : p.K / p.gs);
  // group parameters of stage kb live in qs/qb[kb % kPrefetch]; the K loop
  // is unrolled by kPrefetch so every register is read kPrefetch stages
  // after its load was issued (no register moves that would wait on it)
  const bool vec = p.vec_groups != 0;
  const int k_first = kb_first * BK + half * 32;
  GroupCursor<QK> gc;
  if (vec) gc.init(p, srow, row_ok, is_mx(QK) ? (k_first >> 5) : k_first / p.gs);
  uint32_t qs[kPrefetch], qb[kPrefetch];
#pragma unroll
  for (int i = 0; i < kPrefetch; ++i)
    load_group<QK>(p, srow, k_first + i * BK, !vec && row_ok && i < num_kb, qs[i], qb[i]);
  auto publish = [&](int as_done) {
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (a_full_remote) mbar_arrive_cluster(a_full_remote + 8u * static_cast<uint32_t>(as_done));
      else mbar_arrive(&bb.a_full[as_done]);
    }
  };
  // the TMEM store of stage kb is completed (wait::st) and published
  // (a_full) only after stage kb+1 has been converted, hiding its latency
  int pend_as = -1;
  bool ok = true;
  for (int kb0 = 0; kb0 < num_kb && ok; kb0 += kPrefetch) {
#pragma unroll
    for (int i = 0; i < kPrefetch; ++i) {
      const int kb = kb0 + i;
      if (kb >= num_kb) break;
      const int g = kb_base + kb;  // position in the smem / TMEM rings
      const int s = g % S;
      const uint32_t ph = (g / S) & 1;
      const int as = g % AS;
      const uint32_t aph = (g / AS) & 1;
      uint32_t s_cur = qs[i], b_cur = qb[i];
      if (vec) {
        const int k = k_first + kb * BK;
        gc.get(is_mx(QK) ? (k >> 5) : k / p.gs, s_cur, b_cur);
        if (!row_ok) {
          s_cur = 0u;
          b_cur = 0u;
        }
      }
      if (!mbar_wait(&bb.w_full[s], ph, bb.abort_flag, p.err)) {
        ok = false;
        break;
      }
      const uint8_t* wrow = ws + s * kWStage + r * WB;
      uint32_t o[16];
      if (QK == kAffine4) {
        // 32-byte rows, 32B swizzle: 16-byte chunk c sits at c ^ ((r >> 2) & 1);
        // this warp's half is chunk `half`
        const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((half ^ ((r >> 2) & 1)) << 4));
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          uint32_t q4[4];
          deq_affine4_word(wv[w4], s_cur, b_cur, q4);
#pragma unroll
          for (int t = 0; t < 4; ++t) o[w4 * 4 + t] = q4[t];
        }
      } else {
        // 64-byte rows, 64B swizzle: 16-byte chunk c sits at c ^ ((r >> 1) & 3);
        // this warp's half is chunks 2*half, 2*half+1
        const float fsc = QK == kMxfp8 ? e8m0_to_f32(s_cur) : 0.f;
        const uint32_t s2 = QK == kMxfp8F ? e8m0_fast_scale2(s_cur) : 0u;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = half * 2 + cc;
          const uint4 v = *reinterpret_cast<const uint4*>(wrow + ((c ^ ((r >> 1) & 3)) << 4));
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            if (QK == kMxfp8) deq_mxfp8_word(wv[w4], fsc, o[cc * 8 + w4 * 2], o[cc * 8 + w4 * 2 + 1]);
            else if (QK == kMxfp8F) deq_mxfp8_word_fast(wv[w4], s2, o[cc * 8 + w4 * 2], o[cc * 8 + w4 * 2 + 1]);
            else deq_affine8_word(wv[w4], s_cur, b_cur, o[cc * 8 + w4 * 2], o[cc * 8 + w4 * 2 + 1]);
          }
        }
      }
      if (!row_ok) {
#pragma unroll
        for (int t = 0; t < 16; ++t) o[t] = 0u;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bb.w_empty[s]);  // packed bytes consumed
      if (pend_as >= 0) publish(pend_as);
      pend_as = -1;
      if (!mbar_wait(&bb.a_empty[as], aph ^ 1, bb.abort_flag, p.err)) {
        ok = false;
        break;
      }
      tmem_st_32x32b_x16(tmem + t_lane + kACol + as * 32 + half * 16, o);
      pend_as = as;
      // issued late so that no arrive (release) of this stage waits for it
      if (!vec)
        load_group<QK>(p, srow, k_first + (kb + kPrefetch) * BK, row_ok && kb + kPrefetch < num_kb, qs[i], qb[i]);
    }
  }
  if (pend_as >= 0) publish(pend_as);
}

// Epilogue (warps 0..7): drain this CTA's 128 x BN accumulator, apply the
// reference's bias / GELU rounding points, transpose through shared memory
// (warps of `half` h take 32-token chunks c = h, h+2, ...) and write 16-byte
// coalesced rows with the gated residual fused in.
template <int BN>
__device__ __forceinline__ void epilogue(const Params& p, uint8_t* staging, uint32_t tmem, int warp, int lane, int n0,
                                         int m0) {
  const int q = warp & 3;
  const int half = warp >> 2;
  const int r = q * 32 + lane;
  const int n = n0 + r;
  const bool row_ok = n < p.N;
  const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
  uint16_t* stg = reinterpret_cast<uint16_t*>(staging) + half * 32 * kStagePitch;
  const int tid = q * 32 + lane;  // 0..127 within the group
  const float bias_n = (p.bias != nullptr && row_ok) ? bf16_to_f32(__ldg(p.bias + n)) : 0.f;
  const bool gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
  const bool two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
  for (int c = half; c < BN / 32; c += 2) {
    if (m0 + c * 32 >= p.M) break;  // uniform across the group
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
    named_bar_sync(1 + half, 128);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qq = i * 128 + tid;
      const int j = qq >> 4, f = (qq & 15) * 8;
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
    named_bar_sync(1 + half, 128);
  }
}

// ---------------------------------------------------------------------------
// Single-CTA kernel: 128 features x BN tokens per CTA (used for small token
// counts, BN in {64, 128}).
template <int QK, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                 const Params p) {
  using P = Plan<QK, BN, BN>;
  constexpr int S = P::kStages;
  constexpr int AS = P::kAStages;
  constexpr int WB = QTraits<QK>::kWBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint8_t* ws = smem + S * P::kXStage;
  const Bars bb = carve_bars<S, AS>(smem + P::kBarOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BM;
  const int m0 = blockIdx.y * BN;
  const int num_kb = p.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bb.x_full[s], 1);
      mbar_init(&bb.x_empty[s], 1);
      mbar_init(&bb.w_full[s], 1);
      mbar_init(&bb.w_empty[s], kDeqWarps);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&bb.a_full[s], kDeqWarps);
      mbar_init(&bb.a_empty[s], 1);
    }
    mbar_init(bb.acc_full, 1);
    *bb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(bb.tmem_slot, P::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bb.tmem_slot;

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&bb.w_empty[s], ph ^ 1, bb.abort_flag, p.err)) break;
        mbar_arrive_expect_tx(&bb.w_full[s], P::kWStage);
        tma_load_2d(ws + s * P::kWStage, &tmap_w, &bb.w_full[s], kb * WB, n0);
        if (!mbar_wait(&bb.x_empty[s], ph ^ 1, bb.abort_flag, p.err)) {
          issued = kb;  // the weight copy of stage kb is in flight
          break;
        }
        mbar_arrive_expect_tx(&bb.x_full[s], P::kXStage);
        tma_load_2d(xs + s * P::kXStage, &tmap_x, &bb.x_full[s], kb * BK, m0);
        issued = kb + 1;
      }
      if (*bb.abort_flag) {
        // let the copies already issued land before the CTA's smem is released
        int dummy_abort = 0;
        for (int kb = issued - 1; kb >= 0 && kb >= issued - S; --kb) {
          const int s = kb % S;
          const uint32_t ph = (kb / S) & 1;
          mbar_wait(&bb.x_full[s], ph, reinterpret_cast<volatile int*>(&dummy_abort), p.err);
          mbar_wait(&bb.w_full[s], ph, reinterpret_cast<volatile int*>(&dummy_abort), p.err);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(BM, BN);
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        const int as = kb % AS;
        const uint32_t aph = (kb / AS) & 1;
        if (!mbar_wait(&bb.a_full[as], aph, bb.abort_flag, p.err)) break;
        if (!mbar_wait(&bb.x_full[s], ph, bb.abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t xaddr = smem_u32(xs + s * P::kXStage);
#pragma unroll
        for (int j = 0; j < BK / 16; ++j) {
          const uint64_t bdesc = smem_desc_sw128(xaddr + j * 32);
          mma_bf16_ts(tmem, tmem + P::kACol + as * 32 + j * 8, bdesc, idesc, (kb | j) != 0 ? 1u : 0u);
        }
        mma_commit(&bb.x_empty[s]);
        mma_commit(&bb.a_empty[as]);
      }
      mma_commit(bb.acc_full);  // also drains in-flight MMAs on the abort path
      if (*bb.abort_flag) {
        int dummy_abort = 0;
        mbar_wait(bb.acc_full, 0, reinterpret_cast<volatile int*>(&dummy_abort), p.err);
      }
    }
  } else {
    dequant_loop<QK, S, AS, P::kACol>(p, bb, ws, tmem, warp, lane, n0, num_kb, 0u, 0, 0);
    if (!*bb.abort_flag && mbar_wait(bb.acc_full, 0, bb.abort_flag, p.err)) {
      tc_fence_after();
      epilogue<BN>(p, xs, tmem, warp, lane, n0, m0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, P::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Persistent CTA-pair kernel (cluster of 2, tcgen05 cta_group::2).  Each
// cluster walks the output tiles (256 features x 256 tokens) in a static
// round robin.  Per tile, CTA r of the pair dequantizes feature rows
// [n0 + 128 r, +128) into its own TMEM and stages activation rows
// [m0 + 128 r, +128) in its own smem, so each SM streams half of the
// activation tile; the leader (rank 0) issues one M=256 x N=256 MMA per K
// step and collects both CTAs' readiness on its barriers; tcgen05.commit
// multicasts stage releases and accumulator readiness to both CTAs.
//
// Four epilogue warps per CTA drain the 128 x 256 fp32 accumulator into a
// bf16 copy in spare TMEM columns (the reference's first rounding point;
// TMEM -> registers -> TMEM, each thread its own lane), hand the accumulator
// back to the MMA through the leader's acc_empty barrier, and only then apply
// bias / GELU / gated residual from the copy, through a 2 KB per-warp
// transpose tile, with 16-byte row stores -- overlapped with the next tile's
// main loop.  With no shared-memory staging tile, the operand ring gets the
// shared memory (8 stages of 24 KB, 10 of 20 KB).  The smem and TMEM rings
// continue across tiles.
//
// TMEM columns: [0, 256) fp32 accumulator (lane = feature, column = token);
// [256, 384) the A ring (4 stages x 32 columns of bf16 pairs); [384, 512) the
// bf16 accumulator copy (column c = tokens 2c, 2c + 1).
constexpr int kEpiWarp0 = 10, kPairThreads = 448;  // warps 10..13: epilogue

template <int QK>
struct PairPlan {
  static constexpr int BN = 256;
  static constexpr int kXStage = (BN / 2) * BK * 2;  // this CTA's half of the activation tile
  static constexpr int kWStage = BM * QTraits<QK>::kWBytes;
  static constexpr int kStgBytes = 4 * 32 * 32 * 2;  // per-warp 32 x 32 bf16 transpose tiles
  static constexpr int kFixed = 1024 + kStgBytes + 512 + kGeluTabBytes;
  static constexpr int kStagesRaw = (227 * 1024 - kFixed) / (kXStage + kWStage);
  static constexpr int kStages = kStagesRaw > 10 ? 10 : kStagesRaw;
  static constexpr int kStgOff = kStages * (kXStage + kWStage);
  static constexpr int kBarOff = kStgOff + kStgBytes;
  static constexpr int kTabOff = kBarOff + 512;  // GELU table (epilogue)
  static constexpr int kSmem = 1024 + kTabOff + kGeluTabBytes;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kAStages = 4;
  static constexpr uint32_t kACol = BN;
  static constexpr uint32_t kCopyCol = BN + kAStages * 32;
  static_assert(kCopyCol + BN / 2 <= kTmemCols, "TMEM columns");
  static_assert(kStages >= 4, "pipeline depth");
  static_assert(4 * kStages * 8 + 2 * kAStages * 8 + 24 <= 512, "barrier block");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

// Epilogue state of one thread for a fixed chunk of 8 features [nf, nf + 8):
// the linear bias and a broadcast gate are loaded once.  store() takes the
// bf16-rounded accumulators of one token (the reference's first rounding
// point) and applies bias / GELU / gated residual with the reference's
// rounding points, then writes 16 bytes.
struct Epi8 {
  float bias8[8];
  float g8[8];
  bool gated, two_round, gate_bcast;
  __device__ __forceinline__ void init(const Params& p, int nf) {
    gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
    two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
    gate_bcast = p.gate.rows_per_vec == 0;
    if (p.bias != nullptr) {
      const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + nf));
      const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        bias8[2 * k] = lo_bf16(bw[k]);
        bias8[2 * k + 1] = hi_bf16(bw[k]);
      }
    }
    if (gated && gate_bcast) load_vec8(p.gate, vec_row(p.gate, 0), nf, g8);
  }
  // conversions to bf16 are paired (cvt.rn.bf16x2.f32), never one value at a time
  __device__ __forceinline__ void store(const Params& p, const float (&a)[8], int m, int nf, const uint16_t* gtab) {
    uint32_t u[4];
    if (p.bias != nullptr) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        u[k] = pack_bf16x2(__fadd_rn(a[2 * k], bias8[2 * k]), __fadd_rn(a[2 * k + 1], bias8[2 * k + 1]));
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) u[k] = pack_bf16x2(a[2 * k], a[2 * k + 1]);  // exact: a is bf16-valued
    }
    if (p.epi == LTXQ_EPI_GELU) {
      if (gtab != nullptr) {
#pragma unroll
        for (int k = 0; k < 4; ++k) u[k] = gelu_tab_x2(u[k], gtab);
      } else {  // no table: the same function evaluated directly
#pragma unroll
        for (int k = 0; k < 4; ++k)
          u[k] = pack_bf16x2(gelu_ref(lo_bf16(u[k])), gelu_ref(hi_bf16(u[k])));
      }
    }
    const int64_t off = static_cast<int64_t>(m) * p.N + nf;
    if (gated) {
      const uint4 rv = __ldg(reinterpret_cast<const uint4*>(p.residual + off));
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
      if (!gate_bcast) load_vec8(p.gate, vec_row(p.gate, m), nf, g8);
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
};

// Split tiles: out[m, nf..nf+8) from the fp32 partial sums of a split
// tile's K ranges, added in split order (deterministic), rounded to bf16,
// then the same epilogue as whole tiles.  One thread per (split tile,
// token row, 8 features).
constexpr int kPairTile = 256;  // features and tokens per pair-kernel tile
constexpr int kGroupM = 16;     // token tiles that walk a feature tile together

// Pair-kernel tile t -> (feature tile nt, token tile mt).  Groups of kGroupM
// token tiles walk the feature tiles together, so the clusters that run at
// the same time share a few weight tiles (read from HBM about once per group
// while they sit in L2) and a group's activation rows stay L2-resident.
__device__ __forceinline__ void pair_tile_coords(int t, int n_pt, int m_tiles, int& nt, int& mt) {
  const int span = kGroupM * n_pt;
  const int grp = t / span;
  const int rem_m = m_tiles - grp * kGroupM;
  const int gm = rem_m < kGroupM ? rem_m : kGroupM;
  const int w = t - grp * span;
  nt = w / gm;
  mt = grp * kGroupM + w % gm;
}
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const Params p) {
  // GELU is evaluated directly here (a handful of elements per thread: a
  // per-block table would cost more to build than it saves)
  const int n_pt = (p.N + kPairTile - 1) / kPairTile;
  const int tiles = n_pt * ((p.M + kPairTile - 1) / kPairTile);
  const int64_t items = static_cast<int64_t>(tiles - p.dp_tiles) * kPairTile * (kPairTile / 8);
  constexpr size_t kTileElems = static_cast<size_t>(kPairTile) * kPairTile;
  constexpr int kBatch = 4;  // splits whose partials are loaded before they are added (loads in flight)
  for (int64_t it = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; it < items;
       it += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ti = static_cast<int>(it / (kPairTile * (kPairTile / 8)));
    const int rem = static_cast<int>(it - static_cast<int64_t>(ti) * (kPairTile * (kPairTile / 8)));
    const int j = rem / (kPairTile / 8), f = (rem % (kPairTile / 8)) * 8;
    int nt, mt;
    pair_tile_coords(p.dp_tiles + ti, n_pt, (p.M + kPairTile - 1) / kPairTile, nt, mt);
    const int m = mt * kPairTile + j;
    const int nf = nt * kPairTile + f;
    if (m >= p.M || nf >= p.N) continue;
    const float* src = p.partial + static_cast<size_t>(ti) * p.splits * kTileElems + j * kPairTile + f;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp0 = 0; sp0 < p.splits; sp0 += kBatch) {
      float4 lo[kBatch], hi[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (sp0 + b < p.splits) {
          lo[b] = __ldcg(reinterpret_cast<const float4*>(src + (sp0 + b) * kTileElems));
          hi[b] = __ldcg(reinterpret_cast<const float4*>(src + (sp0 + b) * kTileElems + 4));
        }
      }
      // added in split order; split 0 starts the sum (0 + x = x exactly, -0 aside: the
      // first partial is taken as is)
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (sp0 + b >= p.splits) break;
        if (sp0 + b == 0) {
          a[0] = lo[b].x; a[1] = lo[b].y; a[2] = lo[b].z; a[3] = lo[b].w;
          a[4] = hi[b].x; a[5] = hi[b].y; a[6] = hi[b].z; a[7] = hi[b].w;
        } else {
          a[0] = __fadd_rn(a[0], lo[b].x); a[1] = __fadd_rn(a[1], lo[b].y);
          a[2] = __fadd_rn(a[2], lo[b].z); a[3] = __fadd_rn(a[3], lo[b].w);
          a[4] = __fadd_rn(a[4], hi[b].x); a[5] = __fadd_rn(a[5], hi[b].y);
          a[6] = __fadd_rn(a[6], hi[b].z); a[7] = __fadd_rn(a[7], hi[b].w);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      const uint32_t r = pack_bf16x2(a[k], a[k + 1]);  // the first rounding point, bf16(acc)
      a[k] = lo_bf16(r);
      a[k + 1] = hi_bf16(r);
    }
    Epi8 e;
    e.init(p, nf);
    e.store(p, a, m, nf, nullptr);
  }
}

template <int QK>
__global__ void __launch_bounds__(kPairThreads, 1)
    qgemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                      const Params p) {
  using P = PairPlan<QK>;
  constexpr int BN = P::BN;
  constexpr int S = P::kStages;
  constexpr int AS = P::kAStages;
  constexpr int WB = QTraits<QK>::kWBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint8_t* ws = smem + S * P::kXStage;
  uint16_t* gtab = reinterpret_cast<uint16_t*>(smem + P::kTabOff);
  const Bars bb = carve_bars<S, AS>(smem + P::kBarOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_kb = p.K / BK;
  const int n_pt = (p.N + 2 * BM - 1) / (2 * BM);
  const int m_tiles = (p.M + BN - 1) / BN;
  const int tiles = n_pt * m_tiles;
  // work unit u < dp: whole tile u; u >= dp: K range sp of tile
  // dp + (u - dp) / splits.  Every role walks the same units in the same order.
  const int dp = p.dp_tiles;
  const int splits = p.splits;
  const int units = dp + (tiles - dp) * splits;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int n_clusters = static_cast<int>(gridDim.x >> 1);
  auto unit = [&](int u, int& n0, int& m0, int& sp, int& kb_lo, int& kb_hi) {
    int tile;
    if (u < dp) {
      tile = u;
      sp = -1;
      kb_lo = 0;
      kb_hi = num_kb;
    } else {
      tile = dp + (u - dp) / splits;
      sp = (u - dp) - (tile - dp) * splits;
      kb_lo = sp * num_kb / splits;
      kb_hi = (sp + 1) * num_kb / splits;
    }
    int nt, mt;
    pair_tile_coords(tile, n_pt, m_tiles, nt, mt);
    n0 = nt * (2 * BM) + static_cast<int>(rank) * BM;
    m0 = mt * BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bb.x_full[s], 1);
      mbar_init(&bb.x_empty[s], 1);
      mbar_init(&bb.w_full[s], 1);
      mbar_init(&bb.w_empty[s], kDeqWarps);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&bb.a_full[s], 2 * kDeqWarps);  // both CTAs' dequant warps (the leader's copy is used)
      mbar_init(&bb.a_empty[s], 1);
    }
    mbar_init(bb.acc_full, 1);
    mbar_init(bb.acc_empty, 2);  // both CTAs' epilogue groups (the leader's copy is used)
    *bb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(bb.tmem_slot, P::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialized, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *bb.tmem_slot;
  const uint32_t leader_x_full = mapa_shared(smem_u32(bb.x_full), 0);
  const uint32_t leader_a_full = mapa_shared(smem_u32(bb.a_full), 0);
  const uint32_t leader_acc_empty = mapa_shared(smem_u32(bb.acc_empty), 0);

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      bool ok = true;
      int g0 = 0;
      for (int u = cluster_id; u < units && ok; u += n_clusters) {
        int n0, m0, sp, kb_lo, kb_hi;
        unit(u, n0, m0, sp, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          const int g = g0 + (kb - kb_lo);
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&bb.w_empty[s], ph ^ 1, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bb.w_full[s], P::kWStage);
          tma_load_2d(ws + s * P::kWStage, &tmap_w, &bb.w_full[s], kb * WB, n0);
          if (!mbar_wait(&bb.x_empty[s], ph ^ 1, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          // the leader expects both halves; each CTA's copy completes on the leader's barrier
          if (leader) mbar_arrive_expect_tx(&bb.x_full[s], 2 * P::kXStage);
          tma_load_2d_pair(xs + s * P::kXStage, &tmap_x, leader_x_full + 8u * s, kb * BK,
                           m0 + static_cast<int>(rank) * (BN / 2));
        }
        g0 += kb_hi - kb_lo;
      }
      if (*bb.abort_flag) {
        // give copies already in flight time to land before smem is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(2 * BM, BN);
      bool ok = true;
      int it = 0, g0 = 0;
      for (int u = cluster_id; u < units && ok; u += n_clusters, ++it) {
        int n0, m0, sp, kb_lo, kb_hi;
        unit(u, n0, m0, sp, kb_lo, kb_hi);
        // both epilogue groups must have drained the previous unit's accumulator
        if (!mbar_wait(bb.acc_empty, (it & 1) ^ 1, bb.abort_flag, p.err)) break;
        tc_fence_after();
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          const int g = g0 + (kb - kb_lo);
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          const int as = g % AS;
          const uint32_t aph = (g / AS) & 1;
          if (!mbar_wait(&bb.a_full[as], aph, bb.abort_flag, p.err) ||
              !mbar_wait(&bb.x_full[s], ph, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(xs + s * P::kXStage);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            const uint64_t bdesc = smem_desc_sw128(xaddr + j * 32);
            mma_bf16_ts_pair(tmem, tmem + P::kACol + as * 32 + j * 8, bdesc, idesc,
                             (kb != kb_lo || j != 0) ? 1u : 0u);
          }
          mma_commit_pair(&bb.x_empty[s], 0x3);
          mma_commit_pair(&bb.a_empty[as], 0x3);
        }
        mma_commit_pair(bb.acc_full, 0x3);  // accumulator of this unit ready in both CTAs
        g0 += kb_hi - kb_lo;
      }
      if (*bb.abort_flag) {
        // give MMAs already issued time to complete before TMEM is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp < kDeqWarps) {
    int g0 = 0;
    for (int u = cluster_id; u < units && !*bb.abort_flag; u += n_clusters) {
      int n0, m0, sp, kb_lo, kb_hi;
      unit(u, n0, m0, sp, kb_lo, kb_hi);
      dequant_loop<QK, S, AS, P::kACol>(p, bb, ws, tmem, warp, lane, n0, kb_hi - kb_lo, leader_a_full, g0, kb_lo);
      g0 += kb_hi - kb_lo;
    }
  } else {
    // ------------------------------------------------ epilogue warps 10..13
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int r = q * 32 + lane;
    const int tid = (warp - kEpiWarp0) * 32 + lane;  // 0..127
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    uint16_t* stw = reinterpret_cast<uint16_t*>(smem + P::kStgOff) + q * (32 * 32);
    const bool gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
    const bool two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
    const bool gate_bcast = p.gate.rows_per_vec == 0;
    if (p.epi == LTXQ_EPI_GELU) {
      gelu_tab_fill(gtab, tid, 128);  // while the first tile's main loop runs
      named_bar_sync(1, 128);
    }
    for (int u = cluster_id, it = 0; u < units; u += n_clusters, ++it) {
      int n0, m0, sp, kb_lo, kb_hi;
      unit(u, n0, m0, sp, kb_lo, kb_hi);
      if (!mbar_wait(bb.acc_full, it & 1, bb.abort_flag, p.err)) break;
      tc_fence_after();
      if (sp >= 0) {
        // fp32 partial of split sp of this tile: TMEM lane r = feature n0 + r,
        // column = token; tile-local [token][feature] layout
        const int tile_i = (u - dp) / splits;
        float* dst = p.partial + (static_cast<size_t>(tile_i) * splits + sp) * (kPairTile * kPairTile) +
                     static_cast<int>(rank) * BM + r;
        const int n = n0 + r;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          if (m0 + c * 32 >= p.M) break;  // uniform
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + t_lane + c * 32, v);
          tmem_wait_ld();
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = m0 + c * 32 + j;
              if (m < p.M) dst[(c * 32 + j) * kPairTile] = __uint_as_float(v[j]);
            }
          }
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (tid == 0) mbar_arrive_cluster(leader_acc_empty);
        continue;
      }
      // drain: fp32 accumulator columns of TMEM lane r -> bf16(acc) pairs in
      // the copy columns of the same lane (the MMA waits on this drain only);
      // chunks past the last token row are neither read nor written
      const int chunks = min(BN / 32, (p.M - m0 + 31) / 32);
#pragma unroll 1
      for (int c = 0; c < chunks; c += 2) {
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(tmem + t_lane + c * 32, v[0]);
        tmem_ld_32x32b_x32(tmem + t_lane + (c + 1) * 32, v[1]);
        tmem_wait_ld();
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t h[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) h[j] = pack_bf16x2(__uint_as_float(v[h2][2 * j]), __uint_as_float(v[h2][2 * j + 1]));
          tmem_st_32x32b_x16(tmem + t_lane + P::kCopyCol + (c + h2) * 16, h);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      named_bar_sync(1, 128);
      if (tid == 0) mbar_arrive_cluster(leader_acc_empty);  // TMEM accumulator may be overwritten
      // epilogue from the copy: thread = feature r, registers = tokens; bias
      // and GELU in registers, a 32 x 32 transpose per warp, then 8 features
      // of one token row per lane quad and 16-byte stores
      const int n = n0 + r;
      const float bias_n = (p.bias != nullptr && n < p.N) ? bf16_to_f32(__ldg(p.bias + n)) : 0.f;
      const int nf = n0 + q * 32 + (lane & 3) * 8;
      float g8b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (gated && gate_bcast && nf < p.N) load_vec8(p.gate, vec_row(p.gate, 0), nf, g8b);
#pragma unroll 1
      for (int c = 0; c < chunks; c += 2) {
        uint32_t w2[2][16];
        tmem_ld_32x32b_x16(tmem + t_lane + P::kCopyCol + c * 16, w2[0]);
        tmem_ld_32x32b_x16(tmem + t_lane + P::kCopyCol + (c + 1) * 16, w2[1]);
        tmem_wait_ld();
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int m_c = m0 + (c + h2) * 32;
          if (m_c >= p.M) break;  // uniform
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            uint32_t w = w2[h2][j];
            if (p.bias != nullptr) w = pack_bf16x2(__fadd_rn(lo_bf16(w), bias_n), __fadd_rn(hi_bf16(w), bias_n));
            if (p.epi == LTXQ_EPI_GELU) w = gelu_tab_x2(w, gtab);
            stw[(2 * j) * 32 + lane] = static_cast<uint16_t>(w & 0xFFFFu);
            stw[(2 * j + 1) * 32 + lane] = static_cast<uint16_t>(w >> 16);
          }
          __syncwarp();
#pragma unroll
          for (int pass = 0; pass < 4; ++pass) {
            const int jr = (lane >> 2) + 8 * pass;
            const uint4 a = *reinterpret_cast<const uint4*>(stw + jr * 32 + (lane & 3) * 8);
            if (m_c + jr < p.M && nf < p.N) {
              uint32_t uw[4] = {a.x, a.y, a.z, a.w};
              epi_row_store(p, uw, m_c + jr, nf, g8b, gated, two_round, gate_bcast);
            }
          }
          __syncwarp();  // transpose tile consumed
        }
      }
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal or read it
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, P::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Pretransposed mxfp8 weights (the cache's `mxfp8-blocks-pretranspose` mode,
// loader/transformer_cache.py:177-193, 1240-1244): the packed array is W^T,
// [K rows][N bytes] of E4M3 codes with E8M0 scales [K, N/32] (groups along N).
// Persistent CTA-pair kernel as qgemm_pair_kernel, but the A operand is built
// in shared memory: TMA brings a [64 K][128 N] byte tile per stage, the
// dequant warps write it as an MN-major 128B-swizzled bf16 tile, and the MMA
// reads A through an MN-major descriptor (`tcgen05.mma ... [d], a_desc,
// b_desc` with the A-transpose bit).  With A out of TMEM, all 512 columns hold
// two 256-column accumulators: the epilogue of tile i reads accumulator i & 1
// straight from TMEM while the MMAs of tile i + 1 fill the other one.
// (For the standard layout this form measured slower than qgemm_pair_kernel:
// it adds 32 KB of shared-memory traffic per stage per SM.)
//
// Epilogue (warps 10-13, warp w owns TMEM lanes 32w..32w+31 = features): per
// 32-token chunk, bf16(acc), bias and GELU are applied in registers (thread =
// feature, registers = tokens), the 32 x 32 block is transposed through a
// 2 KB per-warp shared tile, and rows of 32 features are written with 16-byte
// stores (the gated residual fused in on that side).
template <int QK>
struct PairPlanPT {
  static constexpr int BN = 256;
  static constexpr int kXStage = (BN / 2) * BK * 2;  // this CTA's half of the activation tile
  static constexpr int kWStage = BK * BM;  // [64 K][128 N] E4M3 bytes
  static constexpr int kAStage = BM * BK * 2;        // bf16 A tile, 128B-swizzled K-major
  static constexpr int kAStages = 4;
  static constexpr int kStgBytes = 4 * 32 * 32 * 2;  // per-warp 32 x 32 transpose tiles
  static constexpr int kFixed = 1024 + kAStages * kAStage + kStgBytes + 512 + kGeluTabBytes;
  static constexpr int kStagesRaw = (227 * 1024 - kFixed) / (kXStage + kWStage);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kAOff = kStages * kXStage;            // 1024-aligned (16 KB stages)
  static constexpr int kWOff = kAOff + kAStages * kAStage;
  static constexpr int kStgOff = kWOff + kStages * kWStage;
  static constexpr int kBarOff = kStgOff + kStgBytes;
  static constexpr int kTabOff = kBarOff + 512;
  static constexpr int kSmem = 1024 + kTabOff + kGeluTabBytes;
  static constexpr uint32_t kTmemCols = 512;  // two accumulators
  static_assert(kStages >= 4, "pipeline depth");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static_assert(kXStage % 1024 == 0 && kAStage % 1024 == 0, "128B-swizzle atoms need 1024-byte alignment");
};

template <int S, int AS>
__device__ __forceinline__ Bars carve_bars_pt(uint8_t* base, uint64_t*& acc_full2, uint64_t*& acc_empty2) {
  uint64_t* b = reinterpret_cast<uint64_t*>(base);
  Bars r;
  r.x_full = b;
  r.x_empty = b + S;
  r.w_full = b + 2 * S;
  r.w_empty = b + 3 * S;
  r.a_full = b + 4 * S;
  r.a_empty = b + 4 * S + AS;
  acc_full2 = b + 4 * S + 2 * AS;       // [2]
  acc_empty2 = b + 4 * S + 2 * AS + 2;  // [2]
  r.acc_full = acc_full2;
  r.acc_empty = acc_empty2;
  r.tmem_slot = reinterpret_cast<uint32_t*>(b + 4 * S + 2 * AS + 4);
  r.abort_flag = reinterpret_cast<volatile int*>(r.tmem_slot + 1);
  return r;
}


// Dequant warps of the pretransposed form.  Thread t (0..255) converts K row
// t >> 2 of the stage for feature group t & 3 (32 features = one E8M0
// scale): 32 bytes of the [64 K][128 N] packed tile -> four 16-byte chunks of
// the MN-major A tile (64-feature blocks 1024 B apart, 8-row K groups 2048 B
// apart, chunk c of K row r at c ^ (r & 7)).
template <int QK, int S, int AS>
__device__ __forceinline__ void dequant_loop_pt(const Params& p, const Bars& bb, uint8_t* ws, uint8_t* a_smem,
                                                int warp, int lane, int n0, int num_kb, uint32_t a_full_remote,
                                                int kb_base, int kb_first) {
  constexpr int kWStage = BK * BM;
  constexpr int kAStage = BM * BK * 2;
  const int t = warp * 32 + lane;
  const int kr = t >> 2, grp = t & 3;
  const int nq = n0 + grp * 32;  // first feature of this thread's group
  const bool col_ok = nq < p.N;
  const int64_t gpr = p.N / 32;  // scale bytes per K row
  const uint8_t* sc = static_cast<const uint8_t*>(p.scales);
  bool ok = true;
  for (int kb = 0; kb < num_kb && ok; ++kb) {
    const int g = kb_base + kb;
    const int s = g % S;
    const uint32_t ph = (g / S) & 1;
    const int as = g % AS;
    const uint32_t aph = (g / AS) & 1;
    const int64_t k = static_cast<int64_t>(kb_first + kb) * BK + kr;  // absolute K row
    const uint32_t sbyte = col_ok ? __ldg(sc + k * gpr + nq / 32) : 0u;
    if (!mbar_wait(&bb.w_full[s], ph, bb.abort_flag, p.err)) {
      ok = false;
      break;
    }
    const uint8_t* wrow = ws + s * kWStage + kr * BM + grp * 32;
    const uint4 v0 = *reinterpret_cast<const uint4*>(wrow);
    const uint4 v1 = *reinterpret_cast<const uint4*>(wrow + 16);
    const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t o[16];
    if (QK == kMxfp8F) {
      const uint32_t s2 = e8m0_fast_scale2(sbyte);
#pragma unroll
      for (int w = 0; w < 8; ++w) deq_mxfp8_word_fast(wv[w], s2, o[2 * w], o[2 * w + 1]);
    } else {
      const float fsc = e8m0_to_f32(sbyte);
#pragma unroll
      for (int w = 0; w < 8; ++w) deq_mxfp8_word(wv[w], fsc, o[2 * w], o[2 * w + 1]);
    }
    if (!col_ok) {
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = 0u;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bb.w_empty[s]);  // packed bytes consumed
    if (!mbar_wait(&bb.a_empty[as], aph ^ 1, bb.abort_flag, p.err)) {
      ok = false;
      break;
    }
    uint8_t* abase = a_smem + as * kAStage + (kr >> 3) * 2048 + (grp >> 1) * 1024 + (kr & 7) * 128;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(abase + (((4 * (grp & 1) + i) ^ (kr & 7)) << 4)) =
          make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    fence_proxy_async_smem();  // generic-proxy writes -> the MMA's async-proxy reads
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(a_full_remote + 8u * static_cast<uint32_t>(as));
  }
}

template <int QK>
__global__ void __launch_bounds__(kPairThreads, 1)
    qgemm_pair_pt_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                         const Params p) {
  using P = PairPlanPT<QK>;
  constexpr int BN = P::BN;
  constexpr int S = P::kStages;
  constexpr int AS = P::kAStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem;
  uint8_t* as_base = smem + P::kAOff;
  uint8_t* ws = smem + P::kWOff;
  uint16_t* gtab = reinterpret_cast<uint16_t*>(smem + P::kTabOff);
  uint64_t *acc_full2, *acc_empty2;
  const Bars bb = carve_bars_pt<S, AS>(smem + P::kBarOff, acc_full2, acc_empty2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_kb = p.K / BK;
  const int n_pt = (p.N + 2 * BM - 1) / (2 * BM);
  const int m_tiles = (p.M + BN - 1) / BN;
  const int tiles = n_pt * m_tiles;
  // work unit u < dp: whole tile u; u >= dp: K range sp of tile
  // dp + (u - dp) / splits.  Every role walks the same units in the same order.
  const int dp = p.dp_tiles;
  const int splits = p.splits;
  const int units = dp + (tiles - dp) * splits;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int n_clusters = static_cast<int>(gridDim.x >> 1);
  auto unit = [&](int u, int& n0, int& m0, int& sp, int& kb_lo, int& kb_hi) {
    int tile;
    if (u < dp) {
      tile = u;
      sp = -1;
      kb_lo = 0;
      kb_hi = num_kb;
    } else {
      tile = dp + (u - dp) / splits;
      sp = (u - dp) - (tile - dp) * splits;
      kb_lo = sp * num_kb / splits;
      kb_hi = (sp + 1) * num_kb / splits;
    }
    int nt, mt;
    pair_tile_coords(tile, n_pt, m_tiles, nt, mt);
    n0 = nt * (2 * BM) + static_cast<int>(rank) * BM;
    m0 = mt * BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bb.x_full[s], 1);
      mbar_init(&bb.x_empty[s], 1);
      mbar_init(&bb.w_full[s], 1);
      mbar_init(&bb.w_empty[s], kDeqWarps);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init(&bb.a_full[s], 2 * kDeqWarps);  // both CTAs' dequant warps (the leader's copy is used)
      mbar_init(&bb.a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full2[b], 1);
      mbar_init(&acc_empty2[b], 2);  // both CTAs' epilogue groups (the leader's copy is used)
    }
    *bb.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc_pair(bb.tmem_slot, P::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialized, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *bb.tmem_slot;
  const uint32_t leader_x_full = mapa_shared(smem_u32(bb.x_full), 0);
  const uint32_t leader_a_full = mapa_shared(smem_u32(bb.a_full), 0);
  const uint32_t leader_acc_empty = mapa_shared(smem_u32(acc_empty2), 0);

  if (warp == kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      bool ok = true;
      int g0 = 0;
      for (int u = cluster_id; u < units && ok; u += n_clusters) {
        int n0, m0, sp, kb_lo, kb_hi;
        unit(u, n0, m0, sp, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          const int g = g0 + (kb - kb_lo);
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&bb.w_empty[s], ph ^ 1, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bb.w_full[s], P::kWStage);
          tma_load_2d(ws + s * P::kWStage, &tmap_w, &bb.w_full[s], n0, kb * BK);  // [K][N] bytes
          if (!mbar_wait(&bb.x_empty[s], ph ^ 1, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          // the leader expects both halves; each CTA's copy completes on the leader's barrier
          if (leader) mbar_arrive_expect_tx(&bb.x_full[s], 2 * P::kXStage);
          tma_load_2d_pair(xs + s * P::kXStage, &tmap_x, leader_x_full + 8u * s, kb * BK,
                           m0 + static_cast<int>(rank) * (BN / 2));
        }
        g0 += kb_hi - kb_lo;
      }
      if (*bb.abort_flag) {
        // give copies already in flight time to land before smem is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (leader && lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(2 * BM, BN) | (1u << 15);  // A MN-major
      bool ok = true;
      int it = 0, g0 = 0;
      for (int u = cluster_id; u < units && ok; u += n_clusters, ++it) {
        int n0, m0, sp, kb_lo, kb_hi;
        unit(u, n0, m0, sp, kb_lo, kb_hi);
        const int buf = it & 1;
        // both epilogue groups must be done with this accumulator's previous use
        if (!mbar_wait(&acc_empty2[buf], ((it >> 1) & 1) ^ 1, bb.abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          const int g = g0 + (kb - kb_lo);
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          const int as = g % AS;
          const uint32_t aph = (g / AS) & 1;
          if (!mbar_wait(&bb.a_full[as], aph, bb.abort_flag, p.err) ||
              !mbar_wait(&bb.x_full[s], ph, bb.abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xaddr = smem_u32(xs + s * P::kXStage);
          const uint32_t aaddr = smem_u32(as_base + as * P::kAStage);
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            mma_bf16_ss_pair(d, smem_desc_sw128_mn(aaddr + j * 4096, 1024, 2048),  // 16 K rows = 2 row groups
                             smem_desc_sw128(xaddr + j * 32), idesc, (kb != kb_lo || j != 0) ? 1u : 0u);
          mma_commit_pair(&bb.x_empty[s], 0x3);
          mma_commit_pair(&bb.a_empty[as], 0x3);
        }
        mma_commit_pair(&acc_full2[buf], 0x3);  // accumulator of this unit ready in both CTAs
        g0 += kb_hi - kb_lo;
      }
      if (*bb.abort_flag) {
        // give MMAs already issued time to complete before TMEM is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp < kDeqWarps) {
    int g0 = 0;
    for (int u = cluster_id; u < units && !*bb.abort_flag; u += n_clusters) {
      int n0, m0, sp, kb_lo, kb_hi;
      unit(u, n0, m0, sp, kb_lo, kb_hi);
      dequant_loop_pt<QK, S, AS>(p, bb, ws, as_base, warp, lane, n0, kb_hi - kb_lo, leader_a_full, g0, kb_lo);
      g0 += kb_hi - kb_lo;
    }
  } else {
    // ------------------------------------------------ epilogue warps 10..13
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int r = q * 32 + lane;
    const int tid = (warp - kEpiWarp0) * 32 + lane;  // 0..127
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    uint16_t* stw = reinterpret_cast<uint16_t*>(smem + P::kStgOff) + q * (32 * 32);
    const bool gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
    const bool two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
    const bool gate_bcast = p.gate.rows_per_vec == 0;
    if (p.epi == LTXQ_EPI_GELU) {
      gelu_tab_fill(gtab, tid, 128);  // while the first tile's main loop runs
      named_bar_sync(1, 128);
    }
    for (int u = cluster_id, it = 0; u < units; u += n_clusters, ++it) {
      int n0, m0, sp, kb_lo, kb_hi;
      unit(u, n0, m0, sp, kb_lo, kb_hi);
      const int buf = it & 1;
      if (!mbar_wait(&acc_full2[buf], (it >> 1) & 1, bb.abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t tacc = tmem + t_lane + static_cast<uint32_t>(buf * BN);
      const int n = n0 + r;  // register side: this thread's feature
      if (sp >= 0) {
        // fp32 partial of split sp of this tile, tile-local [token][feature]
        const int tile_i = (u - dp) / splits;
        float* dst = p.partial + (static_cast<size_t>(tile_i) * splits + sp) * (kPairTile * kPairTile) +
                     static_cast<int>(rank) * BM + r;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          if (m0 + c * 32 >= p.M) break;  // uniform
          uint32_t v[32];
          tmem_ld_32x32b_x32(tacc + c * 32, v);
          tmem_wait_ld();
          if (n < p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (m0 + c * 32 + j < p.M) dst[(c * 32 + j) * kPairTile] = __uint_as_float(v[j]);
            }
          }
        }
      } else {
        const float bias_n = (p.bias != nullptr && n < p.N) ? bf16_to_f32(__ldg(p.bias + n)) : 0.f;
        // row side: 8 features [nf, nf + 8) of token rows (lane >> 2) + 8 i
        const int nf = n0 + q * 32 + (lane & 3) * 8;
        float g8b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (gated && gate_bcast && nf < p.N) load_vec8(p.gate, vec_row(p.gate, 0), nf, g8b);
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          if (m0 + c * 32 >= p.M) break;  // uniform
          uint32_t v[2][32];
          tmem_ld_32x32b_x32(tacc + c * 32, v[0]);
          tmem_ld_32x32b_x32(tacc + (c + 1) * 32, v[1]);
          tmem_wait_ld();
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int m_c = m0 + (c + h2) * 32;
            if (m_c >= p.M) break;  // uniform
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              // bf16(acc) (the reference's first rounding point), bias, GELU
              uint32_t w = pack_bf16x2(__uint_as_float(v[h2][j]), __uint_as_float(v[h2][j + 1]));
              if (p.bias != nullptr) w = pack_bf16x2(__fadd_rn(lo_bf16(w), bias_n), __fadd_rn(hi_bf16(w), bias_n));
              if (p.epi == LTXQ_EPI_GELU) w = gelu_tab_x2(w, gtab);
              stw[j * 32 + lane] = static_cast<uint16_t>(w & 0xFFFFu);
              stw[(j + 1) * 32 + lane] = static_cast<uint16_t>(w >> 16);
            }
            __syncwarp();
#pragma unroll
            for (int pass = 0; pass < 4; ++pass) {
              const int jr = (lane >> 2) + 8 * pass;
              const uint4 a = *reinterpret_cast<const uint4*>(stw + jr * 32 + (lane & 3) * 8);
              if (m_c + jr < p.M && nf < p.N) {
                uint32_t uw[4] = {a.x, a.y, a.z, a.w};
                epi_row_store(p, uw, m_c + jr, nf, g8b, gated, two_round, gate_bcast);
              }
            }
            __syncwarp();  // transpose tile consumed
          }
        }
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (tid == 0) mbar_arrive_cluster(leader_acc_empty + 8u * static_cast<uint32_t>(buf));
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal or read it
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, P::kTmemCols);
  }
}

template <int QK, int BN>
static ltxq_status launch_cfg(const CUtensorMap& tx, const CUtensorMap& tw, const Params& p, cudaStream_t stream) {
  using PL = Plan<QK, BN, BN>;
  auto kern = qgemm_kernel<QK, BN>;
  ltxq_status st =
      cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem), "smem attribute");
  if (st) return st;
  const dim3 grid((p.N + BM - 1) / BM, (p.M + BN - 1) / BN);
  kern<<<grid, kThreads, PL::kSmem, stream>>>(tx, tw, p);
  return launch_check("qgemm launch");
}

template <int QK>
static ltxq_status launch_pair(const CUtensorMap& tx, const CUtensorMap& tw, const Params& p, cudaStream_t stream) {
  using PL = PairPlan<QK>;
  auto kern = qgemm_pair_kernel<QK>;
  ltxq_status st =
      cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem), "smem attribute");
  if (st) return st;
  const int tiles = ((p.N + 2 * BM - 1) / (2 * BM)) * ((p.M + 255) / 256);
  const int units = p.dp_tiles + (tiles - p.dp_tiles) * p.splits;
  const int max_clusters = num_sms() / 2;
  const int clusters = units < max_clusters ? units : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = PL::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, p);
  if (e == cudaSuccess) note_launch();
  if (ltxq_status st = cuda_check(e, "qgemm pair launch")) return st;
  if (p.dp_tiles >= tiles) return LTXQ_OK;
  const int64_t items = static_cast<int64_t>(tiles - p.dp_tiles) * kPairTile * (kPairTile / 8);
  const int64_t want = (items + 255) / 256;
  const int cap = num_sms() * 8;
  splitk_reduce_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, stream>>>(p);
  return launch_check("split-K reduce launch");
}

template <int QK>
static ltxq_status launch_pair_pt(const CUtensorMap& tx, const CUtensorMap& tw, const Params& p, cudaStream_t stream) {
  using PL = PairPlanPT<QK>;
  auto kern = qgemm_pair_pt_kernel<QK>;
  ltxq_status st =
      cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem), "smem attribute");
  if (st) return st;
  const int tiles = ((p.N + 2 * BM - 1) / (2 * BM)) * ((p.M + 255) / 256);
  const int units = p.dp_tiles + (tiles - p.dp_tiles) * p.splits;
  const int max_clusters = num_sms() / 2;
  const int clusters = units < max_clusters ? units : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = PL::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tx, tw, p);
  if (e == cudaSuccess) note_launch();
  if (ltxq_status st2 = cuda_check(e, "qgemm pretransposed launch")) return st2;
  if (p.dp_tiles >= tiles) return LTXQ_OK;
  const int64_t items = static_cast<int64_t>(tiles - p.dp_tiles) * kPairTile * (kPairTile / 8);
  const int64_t want = (items + 255) / 256;
  const int cap = num_sms() * 8;
  splitk_reduce_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, stream>>>(p);
  return launch_check("split-K reduce launch");
}

// Pair-kernel schedule.  The clusters take the output tiles in waves; when
// the last wave would leave at least half of the clusters idle (few tokens:
// the audio stream, or the video rows of one of several GPUs), its tiles are
// split along K so that every cluster gets a share: the first tiles stay
// whole (dp), the rest split into `splits` K ranges (>= 2 stages each).
Sched plan_schedule(int64_t M, int64_t N, int64_t K) {
  const int tiles = static_cast<int>(((N + 2 * BM - 1) / (2 * BM)) * ((M + 255) / 256));
  Sched sc{tiles, tiles, 1};
  const int clusters = num_sms() / 2;
  const int num_kb = static_cast<int>(K / BK);
  if (clusters <= 0) return sc;
  const int rem = tiles % clusters;
  if (rem == 0 || rem * 2 > clusters) return sc;
  int sp = clusters / rem;
  if (sp > num_kb / 2) sp = num_kb / 2;
  if (sp > 32) sp = 32;
  if (sp < 2) return sc;
  sc.dp = tiles - rem;
  sc.splits = sp;
  return sc;
}

size_t splitk_bytes(int64_t M, int64_t N, int64_t K) {
  const Sched sc = plan_schedule(M, N, K);
  return sc.splits > 1 ? static_cast<size_t>(sc.tiles - sc.dp) * sc.splits * kPairTile * kPairTile * 4 : 0;
}

template <int QK>
static ltxq_status launch_qk(int bn, const CUtensorMap& tx, const CUtensorMap& tw, const Params& p,
                             cudaStream_t stream) {
  if (bn == 64) return launch_cfg<QK, 64>(tx, tw, p, stream);
  if (bn == 128) return launch_cfg<QK, 128>(tx, tw, p, stream);
  return launch_pair<QK>(tx, tw, p, stream);
}

}  // namespace gemm

ltxq_status check_epilogue(const ltxq_epilogue* epi, int64_t M, int64_t N) {
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

// workspace (may be NULL): room for the split-K partials; with less than
// splitk_bytes() the GEMM runs unsplit
ltxq_status launch_qlinear(const void* x, int64_t M, const ltxq_qweight& w, const ltxq_epilogue* epi, void* out,
                           cudaStream_t stream, void* workspace, size_t workspace_bytes) {
  int64_t R, L;
  if (ltxq_status st = check_qweight(w, true, &R, &L)) return st;
  if (!x || !out) return fail(LTXQ_ERR_INVALID, "qlinear: x/out is NULL");
  if (M < 0) return fail(LTXQ_ERR_INVALID, "qlinear: M < 0");
  const bool pt = w.layout == LTXQ_LAYOUT_PRETRANSPOSED;
  if (pt && w.mode != LTXQ_MXFP8)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: pretransposed weights are mxfp8 only (the cache's only such mode)");
  const int64_t N = w.n_out, K = w.k_in;
  if (K % gemm::BK != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: K must be a multiple of 64");
  if (N % 8 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: N must be a multiple of 8");
  if (M > 0x7FFFFFFF / 2 || N > 0x7FFFFFFF / 2 || K > 0x7FFFFFFF / 2)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: dimension too large");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: x/out must be 16-byte aligned");
  if (w.bias && (reinterpret_cast<uintptr_t>(w.bias) & 15u))
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear: bias must be 16-byte aligned");
  if (ltxq_status st = check_epilogue(epi, M, N)) return st;
  if (M == 0) return LTXQ_OK;

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

  // native block-scaled fp8 path (LTXQ_COMPUTE_MX*), when it applies and the
  // workspace holds the split activations
  if (const size_t mx_bytes = mx_workspace_bytes(M, w)) {
    if (workspace && workspace_bytes >= mx_bytes && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0)
      return launch_qlinear_mx(x, M, w, p, workspace, stream);
  }

  const int qk = w.mode == LTXQ_MXFP8 ? ((w.flags & LTXQ_QW_MXFP8_FINITE) ? gemm::kMxfp8F : gemm::kMxfp8)
                                      : (w.bits == 8 ? gemm::kAffine8 : gemm::kAffine4);
  gemm::Sched sched = gemm::plan_schedule(M, N, K);
  if (sched.splits > 1 && (!workspace || workspace_bytes < gemm::splitk_bytes(M, N, K) ||
                           (reinterpret_cast<uintptr_t>(workspace) & 15u)))
    sched = gemm::Sched{sched.tiles, sched.tiles, 1};
  const int splits = sched.splits;
  const int bn = (splits > 1 || pt) ? 256 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256));
  CUtensorMap tx, tw;
  const uint32_t xbox = bn == 256 ? 128 : static_cast<uint32_t>(bn);  // the pair kernel stages half a tile per CTA
  if (ltxq_status st = encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, M, K * 2, gemm::BK, xbox,
                                      CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  if (pt) {
    // W^T: [K rows][N bytes], box of 128 features x 64 K rows, unswizzled
    if (ltxq_status st = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.weight, N, K, N, gemm::BM, gemm::BK,
                                        CU_TENSOR_MAP_SWIZZLE_NONE))
      return st;
  } else {
    const int wbytes_row = static_cast<int>(K * w.bits / 8);
    const uint32_t wbox = qk == gemm::kAffine4 ? 32 : 64;
    const CUtensorMapSwizzle wsw = qk == gemm::kAffine4 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
    if (ltxq_status st =
            encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.weight, wbytes_row, N, wbytes_row, wbox, gemm::BM, wsw))
      return st;
  }
  {
    const int64_t gpr = w.mode == LTXQ_MXFP8 ? K / 32 : K / w.group_size;
    const int64_t per_blk = w.mode == LTXQ_MXFP8 ? 16 : 8;
    const bool al = (reinterpret_cast<uintptr_t>(w.scales) & 15u) == 0 &&
                    (w.mode == LTXQ_MXFP8 || (reinterpret_cast<uintptr_t>(w.biases) & 15u) == 0);
    p.vec_groups = (gpr % per_blk == 0 && al) ? 1 : 0;
  }
  p.dp_tiles = sched.dp;
  p.splits = splits;
  p.partial = splits > 1 ? static_cast<float*>(workspace) : nullptr;
  if (pt) {
    if (qk == gemm::kMxfp8F) return gemm::launch_pair_pt<gemm::kMxfp8F>(tx, tw, p, stream);
    return gemm::launch_pair_pt<gemm::kMxfp8>(tx, tw, p, stream);
  }
  switch (qk) {
    case gemm::kAffine8: return gemm::launch_qk<gemm::kAffine8>(bn, tx, tw, p, stream);
    case gemm::kAffine4: return gemm::launch_qk<gemm::kAffine4>(bn, tx, tw, p, stream);
    case gemm::kMxfp8F: return gemm::launch_qk<gemm::kMxfp8F>(bn, tx, tw, p, stream);
    default: return gemm::launch_qk<gemm::kMxfp8>(bn, tx, tw, p, stream);
  }
}

static size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

static int mx_terms(const ltxq_qweight& w) { return w.compute == LTXQ_COMPUTE_MX2 ? 2 : 1; }

// the AdaLN pass can write this GEMM's block-scaled input (bf16 rows of at most 4096)
static bool adaln_mx_fusable(int64_t M, const ltxq_qweight& w) {
  return mx_workspace_bytes(M, w) > 0 && w.k_in <= 4096;
}

// both FF GEMMs run block-scaled; the hidden activations pass between them as MX terms
static bool ff_mx_fusable(int64_t M, const ltxq_qweight& w_in, const ltxq_qweight& w_out) {
  return adaln_mx_fusable(M, w_in) && mx_workspace_bytes(M, w_out) > 0 && w_in.n_out % 128 == 0 &&
         w_out.k_in == w_in.n_out;
}

}  // namespace ltxq

extern "C" {

// The workspace holds the fp32 partials of the GEMM's K-split tiles (a GEMM
// whose last wave of tiles would leave most clusters idle); calls given less
// run every tile whole.
size_t ltxq_qlinear_workspace_size(int64_t M, const ltxq_qweight* w) {
  if (!w || M <= 0) return 0;
  const size_t mx = ltxq::mx_workspace_bytes(M, *w);
  if (mx) return ltxq::align_up(mx);  // the native path runs unsplit
  return ltxq::align_up(ltxq::gemm::splitk_bytes(M, w->n_out, w->k_in));
}

// With block-scaled weights (and the AdaLN pass able to write MX terms:
// K <= 4096) the prologue writes the GEMM's MX input directly into the
// workspace, and in the FF the first GEMM's epilogue writes the second's.
size_t ltxq_adaln_qlinear_workspace_size(int64_t M, const ltxq_qweight* w) {
  if (!w || M <= 0) return 0;
  if (ltxq::adaln_mx_fusable(M, *w)) return ltxq::align_up(ltxq::mx_workspace_bytes(M, *w));
  return ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w->k_in) * 2) +
         ltxq_qlinear_workspace_size(M, w);
}

size_t ltxq_feed_forward_workspace_size(int64_t M, const ltxq_qweight* w_in, const ltxq_qweight* w_out) {
  if (!w_in || !w_out || M <= 0) return 0;
  if (ltxq::ff_mx_fusable(M, *w_in, *w_out))
    return ltxq::align_up(ltxq::mx_workspace_bytes(M, *w_in)) + ltxq::align_up(ltxq::mx_workspace_bytes(M, *w_out));
  const size_t a = ltxq_qlinear_workspace_size(M, w_in), b = ltxq_qlinear_workspace_size(M, w_out);
  return ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->k_in) * 2) +
         ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->n_out) * 2) + (a > b ? a : b);
}

ltxq_status ltxq_qlinear(const void* x, int64_t M, const ltxq_qweight* w, const ltxq_epilogue* epi, void* out,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!w) return ltxq::fail(LTXQ_ERR_INVALID, "qlinear: weight is NULL");
  return ltxq::launch_qlinear(x, M, *w, epi, out, static_cast<cudaStream_t>(stream), workspace, workspace_bytes);
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
  if (ltxq::adaln_mx_fusable(M, *w)) {
    const ltxq_mx_act a = ltxq::mx_workspace_act(M, w->k_in, ltxq::mx_terms(*w), workspace);
    if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w->k_in, *pro, nullptr, s, &a)) return st;
    return ltxq_qlinear_mx(&a, M, w, epi, out, nullptr, stream);
  }
  if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w->k_in, *pro, workspace, s, nullptr)) return st;
  const size_t a_bytes = ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w->k_in) * 2);
  return ltxq::launch_qlinear(workspace, M, *w, epi, out, s, static_cast<char*>(workspace) + a_bytes,
                              workspace_bytes - a_bytes);
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
  ltxq_epilogue gelu{};
  gelu.kind = LTXQ_EPI_GELU;
  if (ltxq::ff_mx_fusable(M, *w_in, *w_out)) {
    const ltxq_mx_act a = ltxq::mx_workspace_act(M, w_in->k_in, ltxq::mx_terms(*w_in), ws);
    const ltxq_mx_act h = ltxq::mx_workspace_act(M, w_out->k_in, ltxq::mx_terms(*w_out),
                                                 ws + ltxq::align_up(ltxq::mx_workspace_bytes(M, *w_in)));
    if (pro) {
      if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w_in->k_in, *pro, nullptr, s, &a)) return st;
    } else if (ltxq_status st = ltxq_mx_split(x, M, w_in->k_in, a.terms, a.hi, a.lo, a.sf_hi, a.sf_lo, stream)) {
      return st;
    }
    if (ltxq_status st = ltxq_qlinear_mx(&a, M, w_in, &gelu, nullptr, &h, stream)) return st;
    return ltxq_qlinear_mx(&h, M, w_out, epi, out, nullptr, stream);
  }
  const void* a = x;
  if (pro) {
    if (ltxq_status st = ltxq::launch_adaln_modulate(x, LTXQ_BF16, M, w_in->k_in, *pro, ws, s, nullptr)) return st;
    a = ws;
  }
  void* hidden = ws + ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->k_in) * 2);
  const size_t h_bytes = ltxq::align_up(static_cast<size_t>(M) * static_cast<size_t>(w_in->n_out) * 2);
  char* part = static_cast<char*>(hidden) + h_bytes;
  const size_t part_bytes = workspace_bytes - static_cast<size_t>(part - ws);
  if (ltxq_status st = ltxq::launch_qlinear(a, M, *w_in, &gelu, hidden, s, part, part_bytes)) return st;
  return ltxq::launch_qlinear(hidden, M, *w_out, epi, out, s, part, part_bytes);
}

}  // extern "C"
