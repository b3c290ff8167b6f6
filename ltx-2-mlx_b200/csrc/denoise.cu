// denoise.cu -- the per-step latent update of the AV denoise loop, after the
// transformer passes of a step (pipelines/av_pipeline.py:700-742): velocity
// -> denoised (X0Model, model/transformer/model.py:1519-1525), CFG and STG
// guidance (components/guiders.py:24-28, 79-83), the gradient-estimation
// velocity blend (av_pipeline.py:719-725), the denoise-mask blend
// (pipelines/common.py:169-191) and the Euler step
// (components/diffusion_steps.py:19-70), in one pass over the latent.
//
// The reference runs these as separate MLX array ops in fp32 (bf16 latents
// and velocities promote to fp32) and rounds once to bf16 at the end.  Every
// fp32 op here is the same single round-to-nearest op in the same order
// (explicit __f*_rn intrinsics: no FMA contraction), so the result is
// bit-identical to that op sequence.  HBM-bound: 2 bytes read per input
// stream and 2 written per element (+8 for the optional fp32 velocity
// history).
#include "common.cuh"

namespace ltxq {

struct DenoiseArgs {
  const uint16_t* x;
  const uint16_t* vc;
  const uint16_t* vu;   // nullptr: no CFG
  const uint16_t* vp;   // nullptr: no STG
  const float* mask;    // nullptr: uniform mask
  const uint16_t* clean;
  float* prev;          // nullptr: no gradient estimation
  uint16_t* out;
  int64_t chunks;       // elements / 8
  int64_t C;
  float sig, cfg_m1, stg, gamma, ratio;
  int have_prev;
};

__device__ __forceinline__ void load8_bf16(const uint16_t* p, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = lo_bf16(w[i]);
    v[2 * i + 1] = hi_bf16(w[i]);
  }
}

__device__ __forceinline__ float x0_of(float x, float ts, float v) { return __fsub_rn(x, __fmul_rn(ts, v)); }

__global__ void __launch_bounds__(256) denoise_update_kernel(DenoiseArgs a) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t ch = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; ch < a.chunks; ch += stride) {
    const int64_t e0 = ch * 8;
    float x[8], d[8], t[8];
    load8_bf16(a.x + e0, x);
    load8_bf16(a.vc + e0, t);
    float ts = a.sig, m = 1.f;
    if (a.mask) {
      m = __ldg(a.mask + e0 / a.C);
      ts = __fmul_rn(m, a.sig);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = x0_of(x[i], ts, t[i]);
    if (a.vu) {
      load8_bf16(a.vu + e0, t);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = __fadd_rn(d[i], __fmul_rn(a.cfg_m1, __fsub_rn(d[i], x0_of(x[i], ts, t[i]))));
    }
    if (a.vp) {
      load8_bf16(a.vp + e0, t);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = __fadd_rn(d[i], __fmul_rn(a.stg, __fsub_rn(d[i], x0_of(x[i], ts, t[i]))));
    }
    if (a.prev) {
      float4* pv = reinterpret_cast<float4*>(a.prev + e0);
      float cur[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cur[i] = __fdiv_rn(__fsub_rn(x[i], d[i]), a.sig);
      if (a.have_prev) {
        const float4 p0 = pv[0], p1 = pv[1];
        const float pr[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float total = __fadd_rn(__fmul_rn(a.gamma, __fsub_rn(cur[i], pr[i])), pr[i]);
          d[i] = __fsub_rn(x[i], __fmul_rn(total, a.sig));
        }
      }
      pv[0] = make_float4(cur[0], cur[1], cur[2], cur[3]);
      pv[1] = make_float4(cur[4], cur[5], cur[6], cur[7]);
    }
    if (a.mask) {
      load8_bf16(a.clean + e0, t);
      const float om = __fsub_rn(1.f, m);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = __fadd_rn(__fmul_rn(d[i], m), __fmul_rn(t[i], om));
    }
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float o0 = __fadd_rn(d[2 * i], __fmul_rn(a.ratio, __fsub_rn(x[2 * i], d[2 * i])));
      const float o1 = __fadd_rn(d[2 * i + 1], __fmul_rn(a.ratio, __fsub_rn(x[2 * i + 1], d[2 * i + 1])));
      r[i] = pack_bf16x2(o0, o1);
    }
    *reinterpret_cast<uint4*>(a.out + e0) = make_uint4(r[0], r[1], r[2], r[3]);
  }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace ltxq

extern "C" ltxq_status ltxq_denoise_update(const void* latent, const void* v_cond, const void* v_uncond,
                                           const void* v_perturbed, const float* denoise_mask,
                                           const void* clean_latent, float* prev_velocity, int64_t batch,
                                           int64_t tokens, int64_t channels, const ltxq_denoise_params* p,
                                           void* out, void* stream) {
  using namespace ltxq;
  if (!p) return fail(LTXQ_ERR_INVALID, "denoise_update: params is NULL");
  if (batch < 0 || tokens < 0 || channels <= 0) return fail(LTXQ_ERR_INVALID, "denoise_update: bad shape");
  if (channels % 8 != 0) return fail(LTXQ_ERR_UNSUPPORTED, "denoise_update: channels must be a multiple of 8");
  if (!(p->sigma > 0.f)) return fail(LTXQ_ERR_INVALID, "denoise_update: sigma must be > 0");
  if (!(p->sigma_next >= 0.f)) return fail(LTXQ_ERR_INVALID, "denoise_update: sigma_next must be >= 0");
  const int64_t n = batch * tokens * channels;
  if (n == 0) return LTXQ_OK;  // empty tensors may carry NULL pointers
  if (!latent || !v_cond || !out) return fail(LTXQ_ERR_INVALID, "denoise_update: latent/v_cond/out is NULL");
  const bool cfg = p->cfg_scale != 1.0;
  const bool stg = p->stg_scale != 0.0;
  const bool ge = p->ge_gamma > 0.0;
  if (cfg && !v_uncond) return fail(LTXQ_ERR_INVALID, "denoise_update: cfg_scale != 1 needs v_uncond");
  if (stg && !v_perturbed) return fail(LTXQ_ERR_INVALID, "denoise_update: stg_scale != 0 needs v_perturbed");
  if (ge && !prev_velocity) return fail(LTXQ_ERR_INVALID, "denoise_update: ge_gamma > 0 needs prev_velocity");
  if (denoise_mask && !clean_latent) return fail(LTXQ_ERR_INVALID, "denoise_update: a mask needs clean_latent");
  const void* ptrs[] = {latent, v_cond, cfg ? v_uncond : nullptr, stg ? v_perturbed : nullptr,
                        denoise_mask ? clean_latent : nullptr, ge ? prev_velocity : nullptr, out};
  for (const void* q : ptrs)
    if (q && !al16(q)) return fail(LTXQ_ERR_UNSUPPORTED, "denoise_update: tensors must be 16-byte aligned");
  if (denoise_mask && (reinterpret_cast<uintptr_t>(denoise_mask) & 3u))
    return fail(LTXQ_ERR_UNSUPPORTED, "denoise_update: mask must be 4-byte aligned");
  DenoiseArgs a;
  a.x = static_cast<const uint16_t*>(latent);
  a.vc = static_cast<const uint16_t*>(v_cond);
  a.vu = cfg ? static_cast<const uint16_t*>(v_uncond) : nullptr;
  a.vp = stg ? static_cast<const uint16_t*>(v_perturbed) : nullptr;
  a.mask = denoise_mask;
  a.clean = static_cast<const uint16_t*>(clean_latent);
  a.prev = ge ? prev_velocity : nullptr;
  a.out = static_cast<uint16_t*>(out);
  a.chunks = n / 8;
  a.C = channels;
  // scalar factors as the reference's Python floats meet fp32 arrays:
  // double arithmetic, one rounding to fp32
  a.sig = p->sigma;
  a.cfg_m1 = static_cast<float>(p->cfg_scale - 1.0);
  a.stg = static_cast<float>(p->stg_scale);
  a.gamma = static_cast<float>(p->ge_gamma);
  a.ratio = static_cast<float>(static_cast<double>(p->sigma_next) / static_cast<double>(p->sigma));
  a.have_prev = p->have_prev ? 1 : 0;
  const int threads = 256;
  const int64_t want = (a.chunks + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const unsigned blocks = static_cast<unsigned>(want < cap ? want : cap);
  denoise_update_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_check("denoise_update launch");
}
