// mx.cu -- native block-scaled fp8 path for mxfp8 weights: tcgen05.mma
// kind::mxf8f6f4 with E8M0 scale factors in tensor memory, no weight
// dequantization.
//
// The reference's mxfp8 cache (loader/transformer_cache.py:26-33, 840-848,
// 1436-1462) stores every block linear as E4M3 codes with one E8M0 scale per
// 32 consecutive K -- exactly the OCP MX operand format of the tensor cores'
// block-scaled fp8 MMA.  This path hands the packed weight to the MMA as it
// is and converts the bf16 activations to MXFP8 first, in one or two terms:
//
//   x = hi + lo,  hi = MX(x),  lo = MX(x - hi)   (two terms: the default form)
//   x ~ hi                                       (one term: faster, coarser)
//
// MX(v): per group of 32 consecutive K, the E8M0 scale 2^e with the smallest
// e for which max|v| * 2^-e <= 448 (E4M3's largest value, so nothing
// saturates) and the codes RNE_E4M3(v * 2^-e).  Both terms accumulate into
// the same fp32 TMEM accumulator (W hi + W lo), so the two-term form keeps
// each activation to about 2^-8 of its group's largest magnitude (a bf16
// input has 2^-9 relative precision); the one-term form keeps about 2^-4.
// The weight operand is exact (E4M3 times its E8M0 scale), as on the
// dequantizing path.  From the fp32 accumulator on, the epilogue is the
// dequantizing path's: bf16(acc), bias, GELU / gated residual with the
// reference's rounding points.
//
// Kernel (persistent, clusters of two CTAs, tcgen05 cta_group::2): each tile
// is 256 output features x 192 tokens; CTA r holds features [n0 + 128 r,
// +128) of the weight (A, K-major, 128-byte swizzle, straight from the cache
// by TMA) and tokens [m0 + 96 r, +96) of each activation term (B).  The
// scale factors are in the MMA's atom layout in global memory -- the
// weight's repacked once per weight (ltxq_mx_pack_weight_scales, from the
// cache's row-major [N, K/32]), the activations' written by the splitter --
// so every operand of a 128-K stage, in both CTAs, arrives by TMA with its
// completion counted on one barrier of the leader.  The leader's MMA thread
// waits on that barrier alone, copies the scale factors into TMEM
// (tcgen05.cp) and issues 4 MMAs (K = 32 each) per term.  Two 192-column
// accumulators let the epilogue of one tile run while the next accumulates.
// Every wait is bounded (common.cuh mbar_wait); no TMA load uses cluster
// multicast.
#include "common.cuh"
#include "gemm_epilogue.cuh"
#include "mx_act.cuh"

namespace ltxq {
namespace mx {

constexpr int BM = 128;      // output features per CTA (MMA M = 256 per pair)
constexpr int BN = 192;      // tokens per tile (MMA N)
constexpr int BNC = BN / 2;  // tokens per CTA
constexpr int BK = 128;      // K per stage = bytes of one fp8 row
constexpr uint32_t kTmemCols = 512;
constexpr int kGroupM = 16;  // token tiles that walk a feature tile together (L2 reuse of the weight)

// ---------------------------------------------------------------- activation splitter

// One thread per group of 32 K values of a row.  Rows run over whole
// 128-row tiles plus one spare tile (its scales are those of zero rows), so
// that every tile the GEMM reads scale atoms from exists.  Codes: [M, K]
// bytes row-major per term.  Scales: atom (k-tile j, row tile t) at
// sf + (j * tiles + t) * 512 holds the scales of rows t*128 + 32*m1 + m0 for
// groups 4j + k1 at byte m0*16 + m1*4 + k1 -- the layout tcgen05.cp.32x128b
// .warpx4 moves into TMEM for the block-scaled MMA.
template <int kTerms>
__global__ void __launch_bounds__(256) mx_split_kernel(const uint16_t* __restrict__ x, int64_t M, int K,
                                                       int64_t rows, int tiles, uint8_t* __restrict__ hi,
                                                       uint8_t* __restrict__ lo, uint8_t* __restrict__ sf_hi,
                                                       uint8_t* __restrict__ sf_lo) {
  const int G = K / kGroup;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool live = t < rows * G;
  const int64_t row = live ? t / G : 0;
  const int g = live ? static_cast<int>(t - row * G) : 0;
  const bool valid = live && row < M;
  float v[32];
  if (valid) {
    const uint4* src = reinterpret_cast<const uint4*>(x + row * K + static_cast<int64_t>(g) * kGroup);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 a = __ldg(src + q);
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[8 * q + 2 * i] = lo_bf16(w[i]);
        v[8 * q + 2 * i + 1] = hi_bf16(w[i]);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  uint32_t c[8], s0 = 0, s1 = 0;
  mx_term<kTerms == 2>(v, c, s0);
  if (valid) {
    uint4* dst = reinterpret_cast<uint4*>(hi + row * K + static_cast<int64_t>(g) * kGroup);
    dst[0] = make_uint4(c[0], c[1], c[2], c[3]);
    dst[1] = make_uint4(c[4], c[5], c[6], c[7]);
  }
  if (kTerms == 2) {
    mx_term<false>(v, c, s1);
    if (valid) {
      uint4* dst = reinterpret_cast<uint4*>(lo + row * K + static_cast<int64_t>(g) * kGroup);
      dst[0] = make_uint4(c[0], c[1], c[2], c[3]);
      dst[1] = make_uint4(c[4], c[5], c[6], c[7]);
    }
  }
  // lanes 4i..4i+3 hold the four groups of one 128-K tile of one row
  // (G % 4 == 0 and a row starts at a thread index divisible by 4)
  const int lane = threadIdx.x & 31, base = lane & ~3;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    w0 |= (__shfl_sync(0xffffffffu, s0, base + i) & 0xFFu) << (8 * i);
    w1 |= (__shfl_sync(0xffffffffu, s1, base + i) & 0xFFu) << (8 * i);
  }
  if (live && (g & 3) == 0) {
    const int64_t j = g >> 2, tile = row >> 7;
    const int mi = static_cast<int>(row & 127);
    const int64_t off = (j * tiles + tile) * kAtom + (mi & 31) * 16 + (mi >> 5) * 4;
    *reinterpret_cast<uint32_t*>(sf_hi + off) = w0;
    if (kTerms == 2) *reinterpret_cast<uint32_t*>(sf_lo + off) = w1;
  }
}

// Weight scales [N, K/32] (the cache's row-major E8M0 bytes) -> the same
// atom layout: atom (k-tile j, feature tile t) at (j * cols + t) * 512, with
// cols = 4 * ceil(N / 512) (whole 512-feature tiles; rows >= N hold 0, their
// weight rows read as zeros).  One thread per (row, k-tile): one 32-bit word.
__global__ void __launch_bounds__(256) mx_pack_scales_kernel(const uint8_t* __restrict__ s, int64_t N, int G,
                                                             int cols, uint8_t* __restrict__ out) {
  const int KT = G / 4;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(cols) * 128 * KT) return;
  const int64_t n = i / KT;
  const int j = static_cast<int>(i - n * KT);
  const uint32_t w = n < N ? __ldg(reinterpret_cast<const uint32_t*>(s + n * G) + j) : 0u;
  const int m = static_cast<int>(n & 127);
  *reinterpret_cast<uint32_t*>(out + (static_cast<int64_t>(j) * cols + (n >> 7)) * kAtom + (m & 31) * 16 +
                               (m >> 5) * 4) = w;
}

// ---------------------------------------------------------------- PTX wrappers

// Shared-memory descriptor of a scale-factor atom for tcgen05.cp: K-major,
// no swizzle, 32 rows of 16 bytes (8-row core matrices 128 bytes apart).
__device__ __forceinline__ uint64_t sf_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 32;  // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;         // descriptor version
  return d;
}

// Copies a 32-row x 128-bit shared-memory matrix into TMEM lanes 0-31,
// replicated to all four lane quarters, in both CTAs of the pair (each from
// its own shared memory at the same offset).
__device__ __forceinline__ void sf_copy_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Instruction descriptor of kind::mxf8f6f4 with E8M0 scales: E4M3 A and B,
// K-major, fp32 accumulate; sf_id picks the scale byte of the 32-bit scale
// word for both operands.
__host__ __device__ constexpr uint32_t idesc_mx(uint32_t M, uint32_t N, uint32_t sf_id) {
  return (sf_id << 4)          // B scale-factor byte
         | ((N >> 3) << 17)    // N / 8
         | (1u << 23)          // scale format: E8M0
         | ((M >> 4) << 24)    // M / 16
         | (sf_id << 29);      // A scale-factor byte
}

// D[tmem] (+)= (A * SFA) (B * SFB)^T on the CTA pair, both operands from
// shared memory.
__device__ __forceinline__ void mma_mx_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                                            uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// ---------------------------------------------------------------- GEMM

// kBlocks = 1: a tile is 256 features x 192 tokens, two accumulators per CTA
// (the epilogue of one tile overlaps the next tile's MMAs); kBlocks = 2: a
// tile is 512 features x 192 tokens -- each CTA holds 256 weight rows as two
// 128-row blocks and every activation tile feeds MMAs for both, which cuts
// the shared-cache traffic per flop by a third -- with one accumulator per
// block and eight epilogue warps.
template <int kTerms, int kBlocks>
struct Plan {
  static constexpr int kA = kBlocks * BM * BK;  // this CTA's weight rows, 16 KB per block
  static constexpr int kB = BNC * BK;           // one term's activation tile, 12 KB
  static constexpr int kSfa = kBlocks * kAtom;  // weight scale atoms (one per block)
  static constexpr int kSfb = 2 * kAtom;        // one term's scales: the two 128-token atoms a tile touches
  static constexpr int kStage = kA + kTerms * kB + kSfa + kTerms * kSfb;
  // bytes one stage lands on the leader's barrier (both CTAs)
  static constexpr uint32_t kStageTx = 2u * (kA + kSfa + kTerms * (kB + kSfb));
  static constexpr int kEpiWarps = 4 * kBlocks;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);  // epilogue warps, then the TMA and MMA warps
  static constexpr int kTmaWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1;
  static constexpr int kAccBufs = kBlocks == 1 ? 2 : 1;
  static constexpr int kStg = kEpiWarps * 32 * 32 * 2;  // per-warp 32 x 32 transpose tiles of the epilogue
  static constexpr int kFixed = 1024 + kStg + 512 + gemm::kGeluTabBytes;
  static constexpr int kStagesRaw = (227 * 1024 - kFixed) / kStage;
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kAOff = 0;
  static constexpr int kBOff = kAOff + kStages * kA;  // term t, stage s at kBOff + (t * kStages + s) * kB
  static constexpr int kSfaOff = kBOff + kTerms * kStages * kB;
  static constexpr int kSfbOff = kSfaOff + kStages * kSfa;  // stage s, term t at kSfbOff + (s * kTerms + t) * kSfb
  static constexpr int kStgOff = kSfbOff + kStages * kTerms * kSfb;
  static constexpr int kBarOff = kStgOff + kStg;
  static constexpr int kTabOff = kBarOff + 512;
  static constexpr int kSmem = 1024 + kTabOff + gemm::kGeluTabBytes;
  // TMEM columns: accumulators, then the scale factors
  static constexpr uint32_t kSfaCol = 2 * BN;                // 4 columns per weight block
  static constexpr uint32_t kSfbCol = kSfaCol + 4 * kBlocks;  // term t: 8 columns + 2 of slack at kSfbCol + 16 t
  static_assert(kSfbCol + 16 * kTerms <= kTmemCols, "TMEM columns");
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static_assert(kA % 1024 == 0 && kB % 1024 == 0 && kBOff % 1024 == 0, "128B-swizzle atoms need 1024-byte alignment");
  static_assert(2 * kStages * 8 + 4 * 8 + 8 <= 512, "barrier area");
};

template <int kTerms, int kBlocks>
__global__ void __launch_bounds__(Plan<kTerms, kBlocks>::kThreads, 1)
    qgemm_mx_pair_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_sfa,
                         const __grid_constant__ CUtensorMap tmap_hi, const __grid_constant__ CUtensorMap tmap_lo,
                         const __grid_constant__ CUtensorMap tmap_sfb_hi,
                         const __grid_constant__ CUtensorMap tmap_sfb_lo, int w_atom_cols, int x_atom_cols,
                         const gemm::Params p, const MxOut out_mx) {
  using P = Plan<kTerms, kBlocks>;
  constexpr int S = P::kStages;
  constexpr int kRows = kBlocks * BM;  // weight rows per CTA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::kBarOff);
  uint64_t* full = bars;           // leader: every operand of the stage landed in both CTAs
  uint64_t* empty = bars + S;      // stage consumed by the MMAs (commit, multicast to the pair)
  uint64_t* acc_full = bars + 2 * S;       // [kAccBufs]
  uint64_t* acc_empty = bars + 2 * S + 2;  // [kAccBufs], leader: both CTAs' epilogue groups done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint16_t* gtab = reinterpret_cast<uint16_t*>(smem + P::kTabOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int num_kb = p.K / BK;
  const int n_pt = (p.N + 2 * kRows - 1) / (2 * kRows);
  const int m_t = (p.M + BN - 1) / BN;
  const int tiles = n_pt * m_t;
  const int cluster_id = static_cast<int>(blockIdx.x >> 1);
  const int n_clusters = static_cast<int>(gridDim.x >> 1);
  // tile t -> (feature tile, token tile): groups of kGroupM token tiles walk
  // the feature tiles together, so a weight tile is read by consecutive
  // clusters while it is in L2.  n0 = this CTA's first weight row.
  auto coords = [&](int t, int& n0, int& m0) {
    const int span = kGroupM * n_pt;
    const int grp = t / span;
    const int rem_m = m_t - grp * kGroupM;
    const int gm = rem_m < kGroupM ? rem_m : kGroupM;
    const int w = t - grp * span;
    n0 = (w / gm) * (2 * kRows) + static_cast<int>(rank) * kRows;
    m0 = (grp * kGroupM + w % gm) * BN;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);  // the leader's arrive.expect_tx (its copy is the one used)
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < P::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2);  // both CTAs' epilogue groups (the leader's copy is used)
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == P::kMmaWarp) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialized, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t leader_full = mapa_shared(smem_u32(full), 0);
  const uint32_t leader_acc_empty = mapa_shared(smem_u32(acc_empty), 0);

  if (warp == P::kTmaWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      tma_prefetch_desc(&tmap_sfa);
      tma_prefetch_desc(&tmap_hi);
      tma_prefetch_desc(&tmap_sfb_hi);
      if (kTerms == 2) {
        tma_prefetch_desc(&tmap_lo);
        tma_prefetch_desc(&tmap_sfb_lo);
      }
      bool ok = true;
      int g = 0;
      for (int t = cluster_id; t < tiles && ok; t += n_clusters) {
        int n0, m0;
        coords(t, n0, m0);
        const int atom0 = m0 / 128;  // first 128-token scale atom of the tile
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, abort_flag, p.err)) {
            ok = false;
            break;
          }
          // every copy of both CTAs completes on the leader's full[s]
          if (leader) mbar_arrive_expect_tx(&full[s], P::kStageTx);
          const uint32_t bar = leader_full + 8u * s;
          tma_load_2d_pair(smem + P::kAOff + s * P::kA, &tmap_w, bar, kb * BK, n0);
          // this CTA's weight rows: one scale atom (32 rows of 16 bytes) per block
          tma_load_2d_pair(smem + P::kSfaOff + s * P::kSfa, &tmap_sfa, bar, 0, (kb * w_atom_cols + n0 / 128) * 32);
          const int m_cta = m0 + static_cast<int>(rank) * BNC;
          const int sfb_row = (kb * x_atom_cols + atom0) * 32;  // the tile's two token atoms, both CTAs
          tma_load_2d_pair(smem + P::kBOff + s * P::kB, &tmap_hi, bar, kb * BK, m_cta);
          tma_load_2d_pair(smem + P::kSfbOff + (s * kTerms) * P::kSfb, &tmap_sfb_hi, bar, 0, sfb_row);
          if (kTerms == 2) {
            tma_load_2d_pair(smem + P::kBOff + (S + s) * P::kB, &tmap_lo, bar, kb * BK, m_cta);
            tma_load_2d_pair(smem + P::kSfbOff + (s * kTerms + 1) * P::kSfb, &tmap_sfb_lo, bar, 0, sfb_row);
          }
        }
      }
      if (*abort_flag) {
        // give copies already in flight time to land before smem is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else if (warp == P::kMmaWarp) {
    if (leader && lane == 0) {
      bool ok = true;
      int it = 0, g = 0;
      for (int t = cluster_id; t < tiles && ok; t += n_clusters, ++it) {
        int n0, m0;
        coords(t, n0, m0);
        const int buf = it % P::kAccBufs;
        // both epilogue groups must be done with this accumulator's previous tile
        if (!mbar_wait(&acc_empty[buf], ((it / P::kAccBufs) & 1) ^ 1, abort_flag, p.err)) break;
        tc_fence_after();
        // a tile starting 64 tokens into a 128-token atom reads its scales 2 columns in
        const uint32_t sfb_skip = (m0 & 127) ? 2u : 0u;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!mbar_wait(&full[s], ph, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int b = 0; b < kBlocks; ++b)
            sf_copy_pair(tmem + P::kSfaCol + 4u * b, sf_desc(smem_u32(smem + P::kSfaOff + s * P::kSfa + b * kAtom)));
#pragma unroll
          for (int tm = 0; tm < kTerms; ++tm) {
            const uint32_t src = smem_u32(smem + P::kSfbOff + (s * kTerms + tm) * P::kSfb);
            sf_copy_pair(tmem + P::kSfbCol + 16u * tm, sf_desc(src));
            sf_copy_pair(tmem + P::kSfbCol + 16u * tm + 4u, sf_desc(src + kAtom));
          }
          const uint32_t aaddr = smem_u32(smem + P::kAOff + s * P::kA);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint32_t idesc = idesc_mx(2 * BM, BN, static_cast<uint32_t>(kk));
#pragma unroll
            for (int b = 0; b < kBlocks; ++b) {
              const uint64_t adesc = smem_desc_sw128(aaddr + b * (BM * BK) + kk * 32);
              const uint32_t d = tmem + static_cast<uint32_t>((kBlocks == 1 ? buf : b) * BN);
              const uint32_t sfa = (static_cast<uint32_t>(kk) << 30) | (tmem + P::kSfaCol + 4u * b);
#pragma unroll
              for (int tm = 0; tm < kTerms; ++tm) {
                const uint32_t baddr = smem_u32(smem + P::kBOff + (tm * S + s) * P::kB);
                const uint32_t sfb = (static_cast<uint32_t>(kk) << 30) | (tmem + P::kSfbCol + 16u * tm + sfb_skip);
                mma_mx_pair(d, adesc, smem_desc_sw128(baddr + kk * 32), idesc, sfa, sfb,
                            (kb != 0 || kk != 0 || tm != 0) ? 1u : 0u);
              }
            }
          }
          mma_commit_pair(&empty[s], 0x3);
        }
        if (!ok) break;
        mma_commit_pair(&acc_full[buf], 0x3);  // accumulators of this tile ready in both CTAs
      }
      if (*abort_flag) {
        // give MMAs already issued time to complete before TMEM is released
        const uint64_t t0 = globaltimer();
        while (globaltimer() - t0 < 50000ull) {
        }
      }
    }
  } else {
    // ------------------------------------------------ epilogue warps
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int blk = warp >> 2;  // weight block (kBlocks == 2)
    const int tid = threadIdx.x;  // 0 .. 128 kBlocks - 1
    const uint32_t t_lane = static_cast<uint32_t>(q * 32) << 16;
    uint16_t* stw = reinterpret_cast<uint16_t*>(smem + P::kStgOff) + warp * (32 * 32);
    const bool gated = p.epi == LTXQ_EPI_GATED_RESIDUAL || p.epi == LTXQ_EPI_GATE_THEN_ADD;
    const bool two_round = p.epi == LTXQ_EPI_GATE_THEN_ADD || p.gate.dtype == LTXQ_BF16;
    const bool gate_bcast = p.gate.rows_per_vec == 0;
    if (p.epi == LTXQ_EPI_GELU) {
      gemm::gelu_tab_fill(gtab, tid, 32 * P::kEpiWarps);  // while the first tile's main loop runs
      gemm::named_bar_sync(1, 32 * P::kEpiWarps);
    }
    for (int t = cluster_id, it = 0; t < tiles; t += n_clusters, ++it) {
      int n0, m0;
      coords(t, n0, m0);
      const int buf = it % P::kAccBufs;
      if (!mbar_wait(&acc_full[buf], (it / P::kAccBufs) & 1, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t tacc = tmem + t_lane + static_cast<uint32_t>((kBlocks == 1 ? buf : blk) * BN);
      const int nb = n0 + blk * BM;  // first feature of this warp's block
      const int n = nb + q * 32 + lane;  // register side: this thread's feature
      const float bias_n = (p.bias != nullptr && n < p.N) ? bf16_to_f32(__ldg(p.bias + n)) : 0.f;
      // row side: 8 features [nf, nf + 8) of token rows (lane >> 2) + 8 i
      const int nf = nb + q * 32 + (lane & 3) * 8;
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
            if (p.epi == LTXQ_EPI_GELU) w = gemm::gelu_tab_x2(w, gtab);
            stw[j * 32 + lane] = static_cast<uint16_t>(w & 0xFFFFu);
            stw[(j + 1) * 32 + lane] = static_cast<uint16_t>(w >> 16);
          }
          __syncwarp();
#pragma unroll
          for (int pass = 0; pass < 4; ++pass) {
            const int jr = (lane >> 2) + 8 * pass;
            const uint4 a = *reinterpret_cast<const uint4*>(stw + jr * 32 + (lane & 3) * 8);
            if (m_c + jr < p.M && nf < p.N) {  // uniform over each lane quad (one row, one 32-feature group)
              uint32_t uw[4] = {a.x, a.y, a.z, a.w};
              if (out_mx.hi != nullptr)  // the next GEMM's input form instead of bf16 rows
                mx_write8(uw, m_c + jr, nf, out_mx, 0xFu << (lane & ~3));
              else
                gemm::epi_row_store(p, uw, m_c + jr, nf, g8b, gated, two_round, gate_bcast);
            }
          }
          __syncwarp();  // transpose tile consumed
        }
      }
      tc_fence_before();
      gemm::named_bar_sync(1, 32 * P::kEpiWarps);
      if (tid == 0) mbar_arrive_cluster(leader_acc_empty + 8u * static_cast<uint32_t>(buf));
    }
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal or read it
  if (warp == P::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

static size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

// Workspace of the split activations: codes of each term, then the scale
// atoms of each term.
struct Layout {
  int64_t k_tiles, row_tiles;  // row_tiles includes the spare tile
  size_t codes, sf, total;
};

static Layout layout(int64_t M, int64_t K, int terms) {
  Layout l{};
  l.k_tiles = K / BK;
  l.row_tiles = (M + 127) / 128 + 1;
  l.codes = align_up(static_cast<size_t>(M) * static_cast<size_t>(K));
  l.sf = align_up(static_cast<size_t>(l.k_tiles * l.row_tiles) * kAtom);
  l.total = static_cast<size_t>(terms) * (l.codes + l.sf);
  return l;
}

// feature atoms per k-tile of the packed weight scales: whole 512-feature
// tiles, so that both kernel forms read only atoms that exist
static int64_t weight_atom_cols(int64_t N) { return 4 * ((N + 511) / 512); }

// weight rows per cluster tile: 512 (two blocks per CTA) where that still
// gives every cluster a tile, else 256
static int pick_blocks(int64_t M, int64_t N) {
  const int64_t m_t = (M + BN - 1) / BN;
  const int clusters = num_sms() / 2;
  if (((N + 511) / 512) * m_t >= clusters) return 2;
  if (((N + 255) / 256) * m_t >= clusters) return 1;
  return 0;
}

template <int kTerms, int kBlocks>
static ltxq_status launch_gemm(const CUtensorMap& tw, const CUtensorMap& tsfa, const CUtensorMap& thi,
                               const CUtensorMap& tlo, const CUtensorMap& tsfb_hi, const CUtensorMap& tsfb_lo,
                               int w_atom_cols, int x_atom_cols, const gemm::Params& p, const MxOut& out_mx,
                               cudaStream_t stream) {
  using PL = Plan<kTerms, kBlocks>;
  auto kern = qgemm_mx_pair_kernel<kTerms, kBlocks>;
  if (ltxq_status st = cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PL::kSmem),
                                  "smem attribute"))
    return st;
  const int tiles = ((p.N + 2 * kBlocks * BM - 1) / (2 * kBlocks * BM)) * ((p.M + BN - 1) / BN);
  const int max_clusters = num_sms() / 2;
  const int clusters = tiles < max_clusters ? tiles : max_clusters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(PL::kThreads);
  cfg.dynamicSmemBytes = PL::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, kern, tw, tsfa, thi, tlo, tsfb_hi, tsfb_lo, w_atom_cols, x_atom_cols, p, out_mx);
  if (e == cudaSuccess) note_launch();
  return cuda_check(e, "mxfp8 block-scaled GEMM launch");
}

}  // namespace mx

// Whether the native block-scaled path runs this GEMM, and its workspace.
// It needs the standard mxfp8 layout, K a multiple of 512 (the weight-scale
// rows are read as 16-byte boxes) and at least one output tile per cluster
// (fewer tokens run the dequantizing path's K-split schedule instead).
size_t mx_workspace_bytes(int64_t M, const ltxq_qweight& w) {
  if (w.compute != LTXQ_COMPUTE_MX2 && w.compute != LTXQ_COMPUTE_MX1) return 0;
  if (w.mode != LTXQ_MXFP8 || w.layout != LTXQ_LAYOUT_STD || w.group_size != 32) return 0;
  if (M <= 0 || w.k_in % 512 != 0 || w.n_out % 8 != 0 || !w.mx_scales) return 0;
  if (reinterpret_cast<uintptr_t>(w.mx_scales) & 15u) return 0;
  if (!mx::pick_blocks(M, w.n_out)) return 0;
  return mx::layout(M, w.k_in, w.compute == LTXQ_COMPUTE_MX2 ? 2 : 1).total;
}

ltxq_status launch_mx_split(const void* x, int64_t M, int64_t K, int terms, void* hi, void* lo, void* sf_hi,
                            void* sf_lo, cudaStream_t stream) {
  const mx::Layout l = mx::layout(M, K, terms);
  const int64_t rows = l.row_tiles * 128;
  const int64_t threads = rows * (K / mx::kGroup);
  const unsigned blocks = static_cast<unsigned>((threads + 255) / 256);
  if (terms == 2)
    mx::mx_split_kernel<2><<<blocks, 256, 0, stream>>>(
        static_cast<const uint16_t*>(x), M, static_cast<int>(K), rows, static_cast<int>(l.row_tiles),
        static_cast<uint8_t*>(hi), static_cast<uint8_t*>(lo), static_cast<uint8_t*>(sf_hi), static_cast<uint8_t*>(sf_lo));
  else
    mx::mx_split_kernel<1><<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(x), M, static_cast<int>(K), rows,
                                                       static_cast<int>(l.row_tiles), static_cast<uint8_t*>(hi),
                                                       nullptr, static_cast<uint8_t*>(sf_hi), nullptr);
  return launch_check("mx split launch");
}

// The block-scaled GEMM from activations already in MX form (codes and
// scale atoms of `terms` terms, M rows, row_tiles = ceil(M / 128) + 1).  With
// out_mx.hi set, the epilogue writes its result as MX terms (bias / GELU
// applied, rounded to bf16 first) instead of bf16 rows.
static ltxq_status launch_gemm_from_terms(const uint8_t* hi, const uint8_t* lo, const uint8_t* sf_hi,
                                          const uint8_t* sf_lo, int terms, int64_t M, const ltxq_qweight& w,
                                          const gemm::Params& p, const mx::MxOut& out_mx, cudaStream_t stream) {
  const int64_t K = w.k_in, N = w.n_out;
  const mx::Layout l = mx::layout(M, K, terms);
  const int blocks = mx::pick_blocks(M, N);
  CUtensorMap tw, tsfa, thi, tlo, tsbh, tsbl;
  // weight: [N rows][K E4M3 bytes], 128-byte rows of 128 features per block, 128B swizzle
  if (ltxq_status st = encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.weight, K, N, K, mx::BK,
                                      mx::BM * blocks, CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  // scale atoms as rows of 16 bytes: one weight atom (32 rows) per block, two token atoms (64 rows) per tile
  const int64_t w_cols = mx::weight_atom_cols(N);
  if (ltxq_status st = encode_tmap_2d(&tsfa, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.mx_scales, 16, l.k_tiles * w_cols * 32,
                                      16, 16, 32 * blocks, CU_TENSOR_MAP_SWIZZLE_NONE))
    return st;
  if (ltxq_status st = encode_tmap_2d(&tsbh, CU_TENSOR_MAP_DATA_TYPE_UINT8, sf_hi, 16, l.k_tiles * l.row_tiles * 32,
                                      16, 16, 64, CU_TENSOR_MAP_SWIZZLE_NONE))
    return st;
  if (ltxq_status st = encode_tmap_2d(&thi, CU_TENSOR_MAP_DATA_TYPE_UINT8, hi, K, M, K, mx::BK, mx::BNC,
                                      CU_TENSOR_MAP_SWIZZLE_128B))
    return st;
  tlo = thi;
  tsbl = tsbh;
  const int wc = static_cast<int>(w_cols), xc = static_cast<int>(l.row_tiles);
  if (terms == 2) {
    if (ltxq_status st = encode_tmap_2d(&tlo, CU_TENSOR_MAP_DATA_TYPE_UINT8, lo, K, M, K, mx::BK, mx::BNC,
                                        CU_TENSOR_MAP_SWIZZLE_128B))
      return st;
    if (ltxq_status st = encode_tmap_2d(&tsbl, CU_TENSOR_MAP_DATA_TYPE_UINT8, sf_lo, 16,
                                        l.k_tiles * l.row_tiles * 32, 16, 16, 64, CU_TENSOR_MAP_SWIZZLE_NONE))
      return st;
    return blocks == 2 ? mx::launch_gemm<2, 2>(tw, tsfa, thi, tlo, tsbh, tsbl, wc, xc, p, out_mx, stream)
                       : mx::launch_gemm<2, 1>(tw, tsfa, thi, tlo, tsbh, tsbl, wc, xc, p, out_mx, stream);
  }
  return blocks == 2 ? mx::launch_gemm<1, 2>(tw, tsfa, thi, tlo, tsbh, tsbl, wc, xc, p, out_mx, stream)
                     : mx::launch_gemm<1, 1>(tw, tsfa, thi, tlo, tsbh, tsbl, wc, xc, p, out_mx, stream);
}

// The MX terms of M rows of K values in a workspace of mx_act_bytes(M, K,
// terms) bytes: the codes of each term, then the scale atoms of each term.
size_t mx_act_bytes(int64_t M, int64_t K, int terms) { return mx::layout(M, K, terms).total; }

ltxq_mx_act mx_workspace_act(int64_t M, int64_t K, int terms, void* workspace) {
  const mx::Layout l = mx::layout(M, K, terms);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ltxq_mx_act a{};
  a.hi = ws;
  a.lo = terms == 2 ? ws + l.codes : nullptr;
  a.sf_hi = ws + terms * l.codes;
  a.sf_lo = terms == 2 ? ws + terms * l.codes + l.sf : nullptr;
  a.terms = terms;
  return a;
}

// The native path from bf16 activations: split x into MX terms in the
// workspace, then the block-scaled GEMM.  The caller checked the shapes,
// pointers, alignment and epilogue and that mx_workspace_bytes(M, w) > 0 fits
// the workspace.
ltxq_status launch_qlinear_mx(const void* x, int64_t M, const ltxq_qweight& w, const gemm::Params& p, void* workspace,
                              cudaStream_t stream) {
  const int terms = w.compute == LTXQ_COMPUTE_MX2 ? 2 : 1;
  const ltxq_mx_act a = mx_workspace_act(M, w.k_in, terms, workspace);
  auto* hi = static_cast<uint8_t*>(a.hi);
  auto* lo = static_cast<uint8_t*>(a.lo);
  auto* sf_hi = static_cast<uint8_t*>(a.sf_hi);
  auto* sf_lo = static_cast<uint8_t*>(a.sf_lo);
  if (ltxq_status st = launch_mx_split(x, M, w.k_in, terms, hi, lo, sf_hi, sf_lo, stream)) return st;
  return launch_gemm_from_terms(hi, lo, sf_hi, sf_lo, terms, M, w, p, mx::MxOut{}, stream);
}

ltxq_status check_epilogue(const ltxq_epilogue* epi, int64_t M, int64_t N);

}  // namespace ltxq

extern "C" {

int32_t ltxq_qlinear_mx_supported(int64_t M, const ltxq_qweight* w) {
  return (w && ltxq::mx_workspace_bytes(M, *w) > 0) ? 1 : 0;
}

ltxq_status ltxq_qlinear_mx(const ltxq_mx_act* x, int64_t M, const ltxq_qweight* w, const ltxq_epilogue* epi,
                            void* out, const ltxq_mx_act* out_mx, void* stream) {
  using namespace ltxq;
  if (!x || !w) return fail(LTXQ_ERR_INVALID, "qlinear_mx: NULL argument");
  if (M < 0) return fail(LTXQ_ERR_INVALID, "qlinear_mx: M < 0");
  if (!mx::act_ok(x)) return fail(LTXQ_ERR_INVALID, "qlinear_mx: x terms / pointers (16-byte aligned) invalid");
  if (M > 0 && !ltxq_qlinear_mx_supported(M, w))
    return fail(LTXQ_ERR_UNSUPPORTED,
                "qlinear_mx: the block-scaled kernels do not run this GEMM (ltxq_qlinear_mx_supported)");
  if ((w->compute == LTXQ_COMPUTE_MX2 ? 2 : 1) != x->terms)
    return fail(LTXQ_ERR_INVALID, "qlinear_mx: x's term count does not match the weight's compute mode");
  if (ltxq_status st = check_epilogue(epi, M, w->n_out)) return st;
  if (w->bias && (reinterpret_cast<uintptr_t>(w->bias) & 15u))
    return fail(LTXQ_ERR_UNSUPPORTED, "qlinear_mx: bias must be 16-byte aligned");
  const int kind = epi ? epi->kind : LTXQ_EPI_NONE;
  if (out_mx) {
    if (!mx::act_ok(out_mx)) return fail(LTXQ_ERR_INVALID, "qlinear_mx: out_mx terms / pointers invalid");
    if (kind != LTXQ_EPI_NONE && kind != LTXQ_EPI_GELU)
      return fail(LTXQ_ERR_UNSUPPORTED, "qlinear_mx: MX output takes the none / GELU epilogues only");
    if (w->n_out % 128 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "qlinear_mx: MX output needs N % 128 == 0");
  } else if (!out || (reinterpret_cast<uintptr_t>(out) & 15u)) {
    return fail(LTXQ_ERR_INVALID, "qlinear_mx: out is NULL or not 16-byte aligned");
  }
  if (M == 0) return LTXQ_OK;
  gemm::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(w->n_out);
  p.K = static_cast<int>(w->k_in);
  p.gs = w->group_size;
  p.scales = w->scales;
  p.bias = static_cast<const uint16_t*>(w->bias);
  p.epi = kind;
  if (epi && (kind == LTXQ_EPI_GATED_RESIDUAL || kind == LTXQ_EPI_GATE_THEN_ADD)) {
    p.gate = to_vec(epi->gate);
    p.residual = static_cast<const uint16_t*>(epi->residual);
  } else {
    p.gate = VecArg{nullptr, LTXQ_F32, 0, 0};
  }
  p.out = static_cast<uint16_t*>(out);
  p.err = dev_error_word();
  if (!p.err) return fail(LTXQ_ERR_CUDA, "qlinear_mx: device error word unavailable");
  const mx::MxOut om = out_mx ? mx::out_of(*out_mx, M, w->n_out) : mx::MxOut{};
  return launch_gemm_from_terms(static_cast<const uint8_t*>(x->hi), static_cast<const uint8_t*>(x->lo),
                                static_cast<const uint8_t*>(x->sf_hi), static_cast<const uint8_t*>(x->sf_lo), x->terms,
                                M, *w, p, om, static_cast<cudaStream_t>(stream));
}

size_t ltxq_mx_split_sizes(int64_t M, int64_t K, size_t* codes_bytes, size_t* scale_bytes) {
  if (M <= 0 || K <= 0 || K % 128 != 0) return 0;
  const ltxq::mx::Layout l = ltxq::mx::layout(M, K, 1);
  if (codes_bytes) *codes_bytes = static_cast<size_t>(M) * static_cast<size_t>(K);
  if (scale_bytes) *scale_bytes = static_cast<size_t>(l.k_tiles * l.row_tiles) * ltxq::mx::kAtom;
  return l.row_tiles;
}

size_t ltxq_mx_weight_scales_size(const ltxq_qweight* w) {
  if (!w || w->mode != LTXQ_MXFP8 || w->layout != LTXQ_LAYOUT_STD || w->k_in <= 0 || w->k_in % 128 != 0 ||
      w->n_out <= 0)
    return 0;
  return static_cast<size_t>(w->k_in / 128) * static_cast<size_t>(ltxq::mx::weight_atom_cols(w->n_out)) *
         ltxq::mx::kAtom;
}

ltxq_status ltxq_mx_pack_weight_scales(const ltxq_qweight* w, void* out, void* stream) {
  using namespace ltxq;
  if (!w || !out || !w->scales) return fail(LTXQ_ERR_INVALID, "mx_pack_weight_scales: NULL argument");
  const size_t bytes = ltxq_mx_weight_scales_size(w);
  if (!bytes || w->k_in % 512 != 0)
    return fail(LTXQ_ERR_UNSUPPORTED, "mx_pack_weight_scales: mxfp8 weights, standard layout, K % 512 == 0");
  if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(w->scales)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "mx_pack_weight_scales: scales / out must be 16-byte aligned");
  const int G = static_cast<int>(w->k_in / 32);
  const int cols = static_cast<int>(mx::weight_atom_cols(w->n_out));
  const int64_t threads = static_cast<int64_t>(cols) * 128 * (G / 4);
  mx::mx_pack_scales_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w->scales), w->n_out, G, cols, static_cast<uint8_t*>(out));
  return launch_check("mx pack scales launch");
}

ltxq_status ltxq_mx_split(const void* x, int64_t M, int64_t K, int32_t terms, void* hi, void* lo, void* sf_hi,
                          void* sf_lo, void* stream) {
  using namespace ltxq;
  if (!x || !hi || !sf_hi || (terms == 2 && (!lo || !sf_lo))) return fail(LTXQ_ERR_INVALID, "mx_split: NULL pointer");
  if (terms != 1 && terms != 2) return fail(LTXQ_ERR_INVALID, "mx_split: terms must be 1 or 2");
  if (M < 0 || K <= 0) return fail(LTXQ_ERR_INVALID, "mx_split: bad shape");
  if (K % 128 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "mx_split: K must be a multiple of 128");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo) |
       reinterpret_cast<uintptr_t>(sf_hi) | reinterpret_cast<uintptr_t>(sf_lo)) & 15u)
    return fail(LTXQ_ERR_UNSUPPORTED, "mx_split: pointers must be 16-byte aligned");
  if (M == 0) return LTXQ_OK;
  return launch_mx_split(x, M, K, terms, hi, lo, sf_hi, sf_lo, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
