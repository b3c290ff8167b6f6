/*
 * ltxq.h -- C ABI of the B200 (sm_100a) quantized DiT-block hot path.
 *
 * Plain pointers and sizes only.  Every device pointer is caller-owned
 * device memory; every call is asynchronous on the given CUDA stream
 * (`stream` is a cudaStream_t passed as void*; NULL = legacy default
 * stream).  Every entry point returns an ltxq_status; on a non-zero status
 * ltxq_last_error() (thread-local) holds a one-line message.  There is no
 * CPU fallback: unsupported shapes/dtypes return LTXQ_ERR_UNSUPPORTED.
 *
 * Reference interfaces replaced (paths inside dmlsrc/LTX-2-MLX):
 *   ltxq_adaln_modulate  <- LTX_2_MLX/kernels/fused_ops.py:237 adaln_norm_fused
 *                           (+ transformer.py:21-37 _adaln_inline)
 *   ltxq_gated_add       <- LTX_2_MLX/kernels/fused_ops.py:398 gated_add_fused
 *                           (+ transformer.py:40-50 _residual_gate_inline,
 *                              transformer.py:387,484 text-CA gate-then-add)
 *   ltxq_head_gate       <- LTX_2_MLX/model/transformer/attention.py:559-601
 *   ltxq_qk_norm_rope    <- attention.py:320-329, 580-587 + rope.py:53-90
 *   ltxq_attention       <- mx.fast.scaled_dot_product_attention in
 *                           attention.py:170-302 (kernels/steel_attention.py)
 *   ltxq_quantize        <- mx.quantize at loader/transformer_cache.py:1255
 *   ltxq_dequantize      <- mx.dequantize semantics of the same cache entries
 *   ltxq_qlinear         <- nn.QuantizedLinear.__call__ /
 *                           _PretransposedQuantizedLinear.__call__
 *                           (loader/transformer_cache.py:177-193) with the
 *                           block's epilogues (transformer.py:469,650,484,627)
 *   ltxq_adaln_qlinear   <- transformer.py:458 AdaLN then attention.py:573-575
 *                           projections (prologue-fused quantized linear)
 *   ltxq_feed_forward    <- model/transformer/feed_forward.py:64-112
 *                           FeedForward.__call__ + transformer.py:629-650
 *   ltxq_denoise_update  <- one step of the AV CFG denoise loop after the
 *                           transformer passes (pipelines/av_pipeline.py:
 *                           700-742): X0Model.denoise (model/transformer/
 *                           model.py:1519-1525), CFGGuider / STGGuider.guide
 *                           (components/guiders.py:24-28, 79-83), the
 *                           gradient-estimation blend (av_pipeline.py:
 *                           719-725), post_process_latent (pipelines/
 *                           common.py:169-191) and EulerDiffusionStep.step
 *                           (components/diffusion_steps.py:19-70)
 */
#ifndef LTXQ_H
#define LTXQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t ltxq_status;

enum {
  LTXQ_OK = 0,
  LTXQ_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, ...) */
  LTXQ_ERR_UNSUPPORTED = 2, /* shape/dtype/mode not implemented on this path */
  LTXQ_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  LTXQ_ERR_DEVICE = 4       /* a kernel reported a device-side error (bounded wait expired) */
};

enum { LTXQ_BF16 = 0, LTXQ_F32 = 1 };                              /* element dtypes */
enum { LTXQ_NORM_NONE = 0, LTXQ_NORM_RMS = 1, LTXQ_NORM_LAYER = 2 }; /* prologue norm */
enum { LTXQ_AFFINE = 0, LTXQ_MXFP8 = 1 };                           /* quantization mode */
enum { LTXQ_LAYOUT_STD = 0, LTXQ_LAYOUT_PRETRANSPOSED = 1 };        /* packed-weight layout */
enum {
  LTXQ_EPI_NONE = 0,           /* out = bf16(bf16(acc) + bias)                        */
  LTXQ_EPI_GELU = 1,           /* out = gelu_approx(bf16(bf16(acc) + bias))           */
  LTXQ_EPI_GATED_RESIDUAL = 2, /* out = bf16(residual + gate * branch)               */
  LTXQ_EPI_GATE_THEN_ADD = 3   /* out = bf16(residual + bf16(gate * branch))          */
};
enum { LTXQ_GATED_ADD = 0, LTXQ_GATE_THEN_ADD = 1 }; /* ltxq_gated_add modes */
/* ltxq_qweight.flags: properties of the packed data, as ltxq_qweight_scan
 * reports them.  A flag set on data that lacks the property gives wrong
 * results (never a fault). */
enum {
  /* mxfp8: no NaN code (0x7F / 0xFF) and every E8M0 scale <= 134, so each
   * element converts with integer moves and one bf16 multiply */
  LTXQ_QW_MXFP8_FINITE = 1
};

/* ltxq_qweight.compute: how a GEMM over this weight computes.
 *  DEQUANT: the weight is dequantized to bf16 in the kernel (exact) and
 *    multiplied by the bf16 activations on kind::f16 tensor cores; the only
 *    difference from the reference composition is the fp32 summation order.
 *  MX2 (mxfp8 weights): native block-scaled fp8 MMAs (kind::mxf8f6f4) on the
 *    cache's E4M3 codes and E8M0 scales, no dequantization; the activations
 *    are split into two MXFP8 terms x = hi + lo (per 32 K: E8M0 scale, E4M3
 *    codes, no saturation), which keeps each to about 2^-8 of its group's
 *    largest magnitude.
 *  MX1 (mxfp8 weights): as MX2 with one term, about 2^-4 of the group's
 *    largest magnitude: roughly twice the MMA rate of MX2, but it does not
 *    meet this path's stated tolerance against the reference (opt-in).
 * The MX modes apply to the standard layout with K a multiple of 512 and at
 * least one 256 x 192 output tile per two SMs (512 x 192 tiles where there
 * are enough of those), and need the repacked weight
 * scales (ltxq_qweight.mx_scales); other GEMMs over the same weight run the
 * DEQUANT kernels.  The MX modes need workspace for the split
 * activations (ltxq_qlinear_workspace_size accounts for it); given less,
 * the GEMM runs the DEQUANT kernels. */
enum { LTXQ_COMPUTE_DEQUANT = 0, LTXQ_COMPUTE_MX2 = 1, LTXQ_COMPUTE_MX1 = 2 };

/* A quantized linear layer in the reference's MLX cache layout
 * (loader/transformer_cache.py:1238-1267, 1436-1462).
 *  affine:  weight uint32 [N, K*bits/32], scales/biases bf16 [N, K/gs]
 *  mxfp8:   weight uint32 [N, K/4] (E4M3), scales uint8 E8M0 [N, K/32]
 *  pretransposed layout: the same arrays built from W^T, i.e. weight
 *  [K, N*bits/32] and scales [K, N/gs] (groups along N).
 *  bias: optional bf16 [N] (the Linear bias, stored unquantized). */
typedef struct {
  const void* weight;
  const void* scales;
  const void* biases; /* affine only; NULL for mxfp8 */
  const void* bias;   /* optional */
  int64_t n_out;
  int64_t k_in;
  int32_t mode;       /* LTXQ_AFFINE / LTXQ_MXFP8 */
  int32_t bits;       /* 4 or 8 */
  int32_t group_size; /* 64 (affine), 32 (mxfp8) */
  int32_t layout;     /* LTXQ_LAYOUT_STD / LTXQ_LAYOUT_PRETRANSPOSED */
  uint32_t flags;     /* LTXQ_QW_* (0 = none asserted) */
  int32_t compute;    /* LTXQ_COMPUTE_*: how the GEMM computes (0 = dequantize to bf16) */
  /* LTXQ_COMPUTE_MX*: the weight scales repacked by ltxq_mx_pack_weight_scales
   * (16-byte aligned, ltxq_mx_weight_scales_size bytes); NULL runs the
   * DEQUANT kernels */
  const void* mx_scales;
} ltxq_qweight;

/* Per-channel vectors (AdaLN scale/shift/gate).  Element (row m, channel c)
 * lives at ptr[(m / rows_per_vec) * row_stride + c] when rows_per_vec > 0,
 * and at ptr[c] when rows_per_vec == 0 (the (B,1,C) broadcast of the
 * reference's T2V path; rows_per_vec = T gives per-batch vectors,
 * rows_per_vec = 1 per-token vectors). */
typedef struct {
  const void* ptr;
  int32_t dtype; /* LTXQ_BF16 or LTXQ_F32 */
  int32_t pad_;
  int64_t rows_per_vec;
  int64_t row_stride;
} ltxq_vec;

typedef struct {
  int32_t kind;          /* LTXQ_EPI_* */
  int32_t pad_;
  ltxq_vec gate;         /* GATED_RESIDUAL / GATE_THEN_ADD */
  const void* residual;  /* bf16 [M, N] (row stride N) for the gated kinds */
} ltxq_epilogue;

typedef struct {
  int32_t norm; /* LTXQ_NORM_RMS / LTXQ_NORM_LAYER / LTXQ_NORM_NONE (modulate only) */
  float eps;
  ltxq_vec scale;
  ltxq_vec shift;
} ltxq_prologue;

/* ---- library ---------------------------------------------------------- */
const char* ltxq_last_error(void);
const char* ltxq_version(void);
/* Reads (and clears) the device-side error word written by kernels whose
 * bounded waits expired.  Synchronizes the device.  0 = no error. */
ltxq_status ltxq_device_error(int32_t* code_out);
/* Number of kernels this library has launched in this process (all devices,
 * all threads).  Host-side counter; no device synchronization. */
uint64_t ltxq_launch_count(void);
/* Failure-detection self-test (no counterpart in the reference, whose MLX
 * kernels have no device-side waits).  Launches one warp that waits, through
 * the same bounded mbarrier wait every GEMM kernel uses, on a barrier phase
 * nothing completes; after limit_ns (1 us .. 1 s) the wait gives up, writes
 * the device error word and the kernel returns normally.  Synchronizes
 * `stream`.  Returns LTXQ_ERR_DEVICE when the expiry was detected and
 * reported (the expected outcome; the word then stays set until
 * ltxq_device_error reads and clears it), LTXQ_ERR_CUDA if it was not.
 * Call it with the error word clear. */
ltxq_status ltxq_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* ---- bandwidth kernels ------------------------------------------------ */
/* out[m, :] = modulate(norm(x[m, :])) for m < rows; x/out dtype x_dtype
 * (bf16 or f32), C % 8 == 0, C <= 8192.  norm = LTXQ_NORM_NONE gives the
 * norm-free context modulation of transformer.py:379. */
ltxq_status ltxq_adaln_modulate(const void* x, int32_t x_dtype, int64_t rows, int64_t C,
                                const ltxq_prologue* pro, void* out, void* stream);

/* out = residual + gate * branch (mode LTXQ_GATED_ADD, one rounding) or
 * residual + bf16(gate * branch) (LTXQ_GATE_THEN_ADD).  bf16 tensors [rows, C]. */
ltxq_status ltxq_gated_add(const void* residual, const void* branch, const ltxq_vec* gate,
                           int64_t rows, int64_t C, int32_t mode, void* out, void* stream);

/* out[m, h*d:(h+1)*d] = o[m, ...] * (2*sigmoid(logits[m, h])), bf16. */
ltxq_status ltxq_head_gate(const void* o, const void* logits, int64_t rows, int64_t heads,
                           int64_t head_dim, void* out, void* stream);

/* QK RMSNorm + split rotary embedding of one attention operand
 * (attention.py:320-329 q_norm/k_norm, then rope.py:53-90):
 *   y = bf16(x * rsqrt(mean(x^2) + eps) * weight)   over each row of heads*head_dim,
 *   out[h] = bf16([y1 * cos - y2 * sin, y1 * sin + y2 * cos]) per head (y1/y2: halves).
 * x: bf16 rows with row stride row_stride elements (a column slice of a fused
 * projection output is fine); weight: f32 [heads*head_dim]; cos/sin: f32
 * [B, heads, pe_tokens, head_dim/2] with rows = B * pe_tokens, or both NULL
 * for the norm alone; out: contiguous bf16 [rows, heads*head_dim].
 * head_dim 64 or 128, heads <= 32. */
ltxq_status ltxq_qk_norm_rope(const void* x, int64_t rows, int64_t row_stride, int64_t heads,
                              int64_t head_dim, const float* weight, float eps, const float* cos_table,
                              const float* sin_table, int64_t pe_tokens, void* out, void* stream);

/* Attention core without a mask (the block's mx.fast.scaled_dot_product_attention,
 * model/transformer/attention.py:170-302; kernels/steel_attention.py:251-280):
 * out[b, i, h*D:(h+1)*D] = sum_j softmax_j(q_i . k_j * scale) v_j over the
 * kv_rows keys of batch b, per head h; fp32 scores and softmax, P rounded to
 * bf16 for the P.V product (fp32 accumulate), one bf16 rounding of the result.
 * q: bf16 [batch, q_rows, *] with row stride q_stride elements, head h at
 * columns [h*D, (h+1)*D); k, v: bf16 [batch, kv_rows, *] likewise (column
 * slices of fused projection outputs work as they are); out: contiguous bf16
 * [batch, q_rows, heads*D].  head_dim D 64 or 128; strides multiples of 8;
 * 16-byte aligned. */
ltxq_status ltxq_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t q_rows,
                           int64_t kv_rows, int64_t heads, int64_t head_dim, int64_t q_stride, int64_t k_stride,
                           int64_t v_stride, float scale, void* out, void* stream);

/* ltxq_qk_norm_rope for Q and K of the same rows and the same RoPE tables
 * (the self-attention's, attention.py:580-587): one pass, the tables read
 * once for both.  heads * head_dim / 16 a multiple of 32 (at most 256);
 * weights 16-byte aligned; otherwise as ltxq_qk_norm_rope. */
ltxq_status ltxq_qk_norm_rope_pair(const void* q, const void* k, int64_t rows, int64_t q_stride, int64_t k_stride,
                                   int64_t heads, int64_t head_dim, const float* q_weight, const float* k_weight,
                                   float eps, const float* cos_table, const float* sin_table, int64_t pe_tokens,
                                   void* q_out, void* k_out, void* stream);

/* ---- quantized weights ------------------------------------------------ */
/* Quantize a bf16 weight [N, K] into the MLX cache layout described by `w`
 * (w->weight/scales/biases are outputs here; w->bias is ignored). */
ltxq_status ltxq_quantize(const void* w_bf16, const ltxq_qweight* w, void* stream);
/* Dequantize `w` to bf16 [N, K] (standard layout) or [K, N] (pretransposed). */
ltxq_status ltxq_dequantize(const ltxq_qweight* w, void* out_bf16, void* stream);
/* Scans the packed data of `w` and returns the LTXQ_QW_* flags it
 * satisfies.  Synchronizes `stream` (one pass over the packed bytes). */
ltxq_status ltxq_qweight_scan(const ltxq_qweight* w, uint32_t* flags_out, void* stream);

/* ---- quantized linear ------------------------------------------------- */
/* Bytes of device workspace the calls below need for these shapes. */
size_t ltxq_qlinear_workspace_size(int64_t M, const ltxq_qweight* w);
size_t ltxq_adaln_qlinear_workspace_size(int64_t M, const ltxq_qweight* w);
size_t ltxq_feed_forward_workspace_size(int64_t M, const ltxq_qweight* w_in, const ltxq_qweight* w_out);

/* out[M, N] = epilogue(x[M, K] . dequant(W)^T); x, out bf16 row-major
 * (row strides K and N). */
ltxq_status ltxq_qlinear(const void* x, int64_t M, const ltxq_qweight* w, const ltxq_epilogue* epi,
                         void* out, void* workspace, size_t workspace_bytes, void* stream);

/* out = epilogue(modulate(norm(x)) . dequant(W)^T) -- the AdaLN prologue
 * fused in front of the quantized linear. */
ltxq_status ltxq_adaln_qlinear(const void* x, int64_t M, const ltxq_prologue* pro,
                               const ltxq_qweight* w, const ltxq_epilogue* epi, void* out,
                               void* workspace, size_t workspace_bytes, void* stream);

/* Activation quantization of the LTXQ_COMPUTE_MX* path (no counterpart in
 * the reference, whose mxfp8 matmul dequantizes the weight instead): bf16
 * x [M, K] (K % 128 == 0) -> `terms` MXFP8 terms, x = hi (+ lo).  Per group
 * of 32 consecutive K: E8M0 scale 2^e with the smallest e >= -127 for which
 * max|v| * 2^-e <= 448, E4M3 codes RNE(v * 2^-e); the second term quantizes
 * the residual x - hi the same way.  Codes: [M, K] bytes per term.  Scales:
 * in the block-scaled MMA's atom layout -- atom (k-tile j = k / 128, row
 * tile t = m / 128) at (j * row_tiles + t) * 512 holds the scale of row
 * t*128 + 32*m1 + m0, group 4j + k1 at byte m0*16 + m1*4 + k1; row_tiles
 * = ceil(M / 128) + 1 (the last tile is zero rows).  ltxq_mx_split_sizes
 * returns row_tiles and the byte sizes of one term's codes and scales. */
size_t ltxq_mx_split_sizes(int64_t M, int64_t K, size_t* codes_bytes, size_t* scale_bytes);
/* The weight side of LTXQ_COMPUTE_MX*: the cache's E8M0 scales [N, K/32]
 * repacked into the same atom layout (atom (k-tile j, feature tile t) at
 * (j * cols + t) * 512, cols = 4 * ceil(N / 512); rows >= N hold 0).  Done
 * once per weight; the caller owns the buffer and passes it as
 * ltxq_qweight.mx_scales.  Standard-layout mxfp8 weights with K % 512 == 0. */
size_t ltxq_mx_weight_scales_size(const ltxq_qweight* w);
ltxq_status ltxq_mx_pack_weight_scales(const ltxq_qweight* w, void* out, void* stream);
ltxq_status ltxq_mx_split(const void* x, int64_t M, int64_t K, int32_t terms, void* hi, void* lo, void* sf_hi,
                          void* sf_lo, void* stream);

/* Activations in the MX split form (ltxq_mx_split's codes and scale-atom
 * layout) -- the input of the block-scaled GEMMs, written directly by
 * ltxq_adaln_modulate_mx, ltxq_head_gate_mx and ltxq_qlinear_mx's out_mx. */
typedef struct {
  void* hi;      /* [M, K] E4M3 codes of the first term (16-byte aligned) */
  void* lo;      /* [M, K] codes of the second term (terms == 2) */
  void* sf_hi;   /* scale atoms of each term (ltxq_mx_split_sizes bytes) */
  void* sf_lo;
  int32_t terms; /* 1 or 2 */
  int32_t pad_;
} ltxq_mx_act;

/* 1 when the block-scaled kernels run a GEMM of M rows over `w`
 * (LTXQ_COMPUTE_MX* with its packed scales, enough output tiles). */
int32_t ltxq_qlinear_mx_supported(int64_t M, const ltxq_qweight* w);
/* ltxq_qlinear from activations already in MX form (x->terms must match
 * w->compute; ltxq_qlinear_mx_supported(M, w) must hold; no workspace).
 * With out_mx != NULL the result (bias / GELU applied, rounded to bf16) is
 * written as MX terms of the next GEMM's input instead of bf16 `out`
 * (epilogue none or GELU, N % 128 == 0); out may then be NULL.  Same bits as
 * ltxq_mx_split of the bf16 result.  The reference composition it replaces
 * is ltxq_qlinear's (transformer_cache.py:177-193 with the block's
 * epilogues). */
ltxq_status ltxq_qlinear_mx(const ltxq_mx_act* x, int64_t M, const ltxq_qweight* w, const ltxq_epilogue* epi,
                            void* out, const ltxq_mx_act* out_mx, void* stream);
/* ltxq_adaln_modulate (bf16 x, C % 128 == 0, C <= 4096) writing its result
 * as MX terms (`out` then unused, may be NULL) or both: bf16 to `out` when it
 * is not NULL.  The terms are the bits ltxq_mx_split gives for the bf16
 * result. */
ltxq_status ltxq_adaln_modulate_mx(const void* x, int64_t rows, int64_t C, const ltxq_prologue* pro, void* out,
                                   const ltxq_mx_act* out_mx, void* stream);
/* ltxq_head_gate writing MX terms (heads * head_dim % 128 == 0); `out` as
 * in ltxq_adaln_modulate_mx. */
ltxq_status ltxq_head_gate_mx(const void* o, const void* logits, int64_t rows, int64_t heads, int64_t head_dim,
                              void* out, const ltxq_mx_act* out_mx, void* stream);
/* ltxq_head_gate / ltxq_head_gate_mx with the gate logits of row m at
 * logits + m * logits_stride (elements, >= heads): the logits may be a
 * column slice of a fused projection output (this library's Q|K|V|gate
 * GEMM), where the reference computes them with their own linear
 * (attention.py:559-601).  `out_mx` NULL: bf16 `out` only. */
ltxq_status ltxq_head_gate_ex(const void* o, const void* logits, int64_t logits_stride, int64_t rows, int64_t heads,
                              int64_t head_dim, void* out, const ltxq_mx_act* out_mx, void* stream);

/* ltxq_adaln_qlinear without a workspace argument and without allocating.
 * No counterpart in the reference.  For hosts that cannot let a library
 * allocate device memory (a runtime that owns the whole GPU's memory
 * through its own pool, a plugin inside another framework's allocator, a
 * latency-critical loop where cudaMalloc/cudaFree would synchronize the
 * device).  The scratch is a fixed 8 MiB array inside the library's device
 * image, held by every GPU that loads the library until exit: M * K must be
 * <= 4194304 (else LTXQ_ERR_UNSUPPORTED, nothing launched).  All calls share
 * that array, so calls that overlap on the GPU race; serialize them.  The
 * first call on a device looks the array's address up, and so does the
 * first call after a device reset (make those before any stream capture).
 * No cudaMalloc/cudaFree or allocating routine is used. */
ltxq_status ltxq_adaln_qlinear_noalloc(const void* x, int64_t M, const ltxq_prologue* pro,
                                       const ltxq_qweight* w, const ltxq_epilogue* epi, void* out,
                                       void* stream);

/* out = x + gate * project_out(gelu(project_in(modulate(norm(x))))) -- the
 * whole FF sub-layer of transformer.py:629-668.  pro may be NULL (x is
 * already modulated) and epi may be NULL / LTXQ_EPI_NONE (plain FF). */
ltxq_status ltxq_feed_forward(const void* x, int64_t M, const ltxq_prologue* pro,
                              const ltxq_qweight* w_in, const ltxq_qweight* w_out,
                              const ltxq_epilogue* epi, void* out, void* workspace,
                              size_t workspace_bytes, void* stream);

/* ---- denoise step ----------------------------------------------------- */
/* Scalars of one step.  sigma is the schedule's current value (> 0),
 * sigma_next the next (>= 0).  cfg_scale == 1 disables CFG (v_uncond
 * unused), stg_scale == 0 disables STG (v_perturbed unused), ge_gamma <= 0
 * disables the gradient-estimation blend.  The host rounds the scalar
 * factors to fp32 after their double arithmetic (cfg_scale - 1,
 * sigma_next / sigma), as the reference's Python scalars meet its fp32
 * arrays. */
typedef struct {
  float sigma;
  float sigma_next;
  double cfg_scale;
  double stg_scale;
  double ge_gamma;
  int32_t have_prev; /* ge: prev_velocity holds the previous step's velocity */
  int32_t pad_;
} ltxq_denoise_params;

/* One stream's update after the transformer passes of a step, fused in
 * fp32 with one bf16 rounding at the end:
 *   d    = latent - ts * v_cond             (ts = sigma, or mask * sigma)
 *   d   += (cfg_scale - 1) * (d - (latent - ts * v_uncond))
 *   d   += stg_scale * (d - (latent - ts * v_perturbed))
 *   ge:  v = (latent - d) / sigma; if have_prev: d = latent - (gamma * (v - prev) + prev) * sigma;
 *        prev_velocity = v
 *   mask: d = d * mask + clean * (1 - mask)
 *   out = bf16(d + (sigma_next / sigma) * (latent - d))
 * latent, v_*, clean_latent, out: bf16 [batch, tokens, channels]
 * contiguous, 16-byte aligned, channels % 8 == 0; denoise_mask: f32
 * [batch, tokens] or NULL (uniform); clean_latent required with a mask;
 * prev_velocity: f32 [batch, tokens, channels], read and written when
 * ge_gamma > 0 (NULL otherwise).  out may alias latent. */
ltxq_status ltxq_denoise_update(const void* latent, const void* v_cond, const void* v_uncond,
                                const void* v_perturbed, const float* denoise_mask,
                                const void* clean_latent, float* prev_velocity, int64_t batch,
                                int64_t tokens, int64_t channels, const ltxq_denoise_params* p,
                                void* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LTXQ_H */
