/*
 * svla.h -- C ABI of libsvla.so, the sm_100a kernels of the quantized SmolVLA sample_actions path.
 *
 * Conventions (same status codes as the reference's launch helpers,
 * deploy/cuda/fused_rope_layout.cu:566-570):
 *   return 0 = success, 1 = bad argument / shape / alignment, 2 = CUDA launch or runtime error.
 *   svla_last_error() returns a message for the last nonzero status of the calling thread.
 * Kernels are launched with programmatic dependent launch (set SVLA_PDL=0 to disable): each one waits
 * for the previous kernel in the stream before touching data it produced, so stream order is kept while
 * kernel prologues overlap.
 * Every entry point is stream-ordered (no host synchronisation) and allocates no memory: all buffers,
 * including scratch ("workspace"), are passed in by the caller, like the TensorRT plugin enqueue it
 * replaces (deploy/cuda/smoothquant_qkv_plugin_serialized_smoke.cu:346-402).  All pointers are device
 * pointers unless stated otherwise.  Tensors are row-major; "ld" values are row strides in elements.
 * bf16 tensors are passed as void* (IEEE bfloat16 bit patterns).
 */
#ifndef SVLA_H_
#define SVLA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* svla_stream_t; /* == cudaStream_t */

#define SVLA_OK 0
#define SVLA_ERR_ARG 1
#define SVLA_ERR_CUDA 2

/* operand kinds of svla_gemm */
#define SVLA_KIND_I8 0    /* int8 x int8 -> int32 (SmoothQuant W8A8) */
#define SVLA_KIND_BF16 1  /* bf16 x bf16 -> fp32 */
#define SVLA_KIND_W8A16 2 /* bf16 activations x int8 weights dequantised to bf16(q * w_s) in shared memory */

/* epilogues of svla_gemm (v = acc * a * w_s[n] + b[n] for I8, acc + b[n] otherwise) */
#define SVLA_EPI_BF16 0      /* out = bf16(v) [then bf16(out * post_scale)] */
#define SVLA_EPI_I32 1       /* out = raw int32 accumulators (I8 only) */
#define SVLA_EPI_ROPE 2      /* out = bf16(rotate_half_rope(bf16(v), pos[m])) on segments with rope = 1 */
#define SVLA_EPI_RESID 3     /* out = bf16(bf16(v) + resid) */
#define SVLA_EPI_SILU_MUL 4  /* pair: out = bf16(bf16(silu(bf16(v_gate))) * bf16(v_up)) */
#define SVLA_EPI_GELU_QUANT 5 /* g = bf16(gelu_tanh(bf16(v))); out = g (if set); qout = round((g / q_smooth[n]) / q_act) (if set) */
#define SVLA_EPI_EULER 6     /* x_t[m, n] += dt * v (fp32), x_t_bf16 = bf16(x_t) */
#define SVLA_EPI_SILU 7      /* out = bf16(silu(bf16(v))) */
#define SVLA_EPI_F32 8       /* out = v in fp32 */

/* -------------------------------------------------------------------------------------------------
 * Library
 * ------------------------------------------------------------------------------------------------*/
const char* svla_last_error(void);
/* Version string of the build (compile flags and arch). */
const char* svla_version(void);
/* Reads (and with reset != 0 clears) the device error word that bounded waits and bounds checks
 * write (0 = none).  Synchronises the current device. */
int32_t svla_device_error(int32_t* code, int32_t reset);

/* -------------------------------------------------------------------------------------------------
 * SmoothQuant primitives
 * ------------------------------------------------------------------------------------------------*/

/* Per-output-channel int8 weight packing with optional SmoothQuant fold; replaces
 * W8A8Linear.__init__ / quantize_weight_per_out_channel (deploy/linear_only_quant.py:43-54, :140-144):
 * W' = W * smooth[None, :];  wscale[n] = max(max_k |W'[n,k]|, 1e-8) / 127;
 * qweight = round(W' / wscale[n]).clamp(-127, 127).  weight bf16 [N, K]; smooth fp32 [K] or NULL. */
int32_t svla_pack_weight_i8(const void* weight, const float* smooth, int32_t n, int32_t k, int8_t* qweight,
                            float* wscale, svla_stream_t stream);

/* The bf16 weight of a W8A16 linear: out[n,k] = bf16(float(qweight[n,k]) * wscale[n]); replaces
 * dequantize_weight(qweight, scale).to(torch.bfloat16) in W8A16Linear.__init__
 * (deploy/linear_only_quant.py:122-124, :147-148).  out bf16 [N, K]; K % 8 == 0. */
int32_t svla_dequant_weight_bf16(const int8_t* qweight, const float* wscale, int32_t n, int32_t k, void* out,
                                 svla_stream_t stream);

/* SmoothQuant activation quantisation; replaces smoothQuantActivationKernel
 * (deploy/cuda/smoothquant_linear_epilogue.cu:108-119) with bf16 input:
 * q[m,k] = round((x[m,k] / smooth[k]) / act_scale).clamp(-128, 127).  K, ldx, ldq multiples of 8 (>= K);
 * x 16-byte aligned, q 8-byte aligned; smooth fp32 [K], or NULL for no smoothing. */
int32_t svla_quantize_smooth(const void* x, int32_t ldx, const float* smooth, float act_scale, int8_t* q,
                             int32_t ldq, int32_t m, int32_t k, svla_stream_t stream);

/* Calibration statistics of `calls` linear calls of `rows` tokens each (call c = rows [c*rows, (c+1)*rows)
 * of x, bf16 [calls*rows, ldx], 2-byte aligned, ldx >= k); replaces the forward pre-hook of
 * PerChannelLinearInputCollector (deploy/calibrate_smolvla_activation_channel_scales.py:68-84).  Per call and
 * channel: a = max(max_t |x|, 1e-8) and p = max(torch.quantile(|x[:, k]|, q), 1e-8), linear interpolation,
 * bit-identical to torch.quantile on fp32 (NaN inputs are skipped, not propagated); both are max-accumulated
 * into amax / pamax fp32 [k], which the caller zero-fills before the first call of a module.
 * 1 <= rows <= 4096, 1 <= calls <= 65535, 0 <= q <= 1. */
int32_t svla_channel_percentile(const void* x, int64_t ldx, int32_t calls, int32_t rows, int32_t k, float q,
                                float* amax, float* pamax, svla_stream_t stream);

/* int8 x int8 -> int32 GEMM acc[m,n] = sum_k qx[m,k] * qw[n,k]; replaces int8GemmInt32Kernel
 * (deploy/cuda/smoothquant_linear_epilogue.cu:121-137) and the cuBLASLt CUBLAS_COMPUTE_32I call
 * (deploy/cuda/smoothquant_linear_cublaslt.cu:230-306).  tcgen05 kind::i8. */
int32_t svla_gemm_i8_i32(const int8_t* qx, const int8_t* qw, int32_t m, int32_t n, int32_t k, int32_t* acc,
                         svla_stream_t stream);

/* Scratch bytes svla_sq_linear_w8a8 needs for (m, k). */
size_t svla_sq_linear_w8a8_workspace_size(int32_t m, int32_t k);

/* SmoothQuant W8A8 linear, quantise + tcgen05 int8 GEMM + fused dequant/bias epilogue; replaces the
 * quantize -> int8GemmFusedEpilogueKernel pipeline (deploy/cuda/smoothquant_linear_epilogue.cu:108-168)
 * and W8A8Linear.forward (deploy/linear_only_quant.py:104-116):
 * y[m,n] = bf16((acc[m,n] * act_scale) * wscale[n] + bias[n]),  x / y bf16, bias bf16 or NULL.
 * workspace >= svla_sq_linear_w8a8_workspace_size(m, k) bytes, 256-byte aligned. */
int32_t svla_sq_linear_w8a8(const void* x, const float* smooth, float act_scale, const int8_t* qweight,
                            const float* wscale, const void* bias, int32_t m, int32_t n, int32_t k, void* y,
                            void* workspace, size_t workspace_bytes, svla_stream_t stream);

/* The same SmoothQuant W8A8 linear for callers that cannot allocate device memory (a fixed-rate control
 * loop that must not allocate after start-up, or a binding that only holds the pointers it was given).
 * No counterpart in the reference.  Takes no workspace: the int8 activations go to one 4 MiB
 * (4194304-byte) array built into the library, held on every GPU that loads the library until exit.
 * Rejects m*k above 4194304 with status 1.  All calls on a device share the array, so calls that overlap
 * on the GPU race; nothing needs clearing between calls.  The first call on each device looks up the
 * array's device address and should come before any stream capture. */
int32_t svla_sq_linear_w8a8_static_scratch(const void* x, const float* smooth, float act_scale,
                                           const int8_t* qweight, const float* wscale, const void* bias, int32_t m,
                                           int32_t n, int32_t k, void* y, svla_stream_t stream);

/* W8A16 linear; replaces W8A16Linear.forward (deploy/linear_only_quant.py:119-137):
 * y = bf16(x @ bf16(qweight * wscale[:,None])^T + bias). */
int32_t svla_w8a16_linear(const void* x, const int8_t* qweight, const float* wscale, const void* bias, int32_t m,
                          int32_t n, int32_t k, void* y, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * General fused GEMM (the launch the sample_actions runner uses for every linear)
 * ------------------------------------------------------------------------------------------------*/
typedef struct svla_gemm_seg {
  const void* a;          /* A operand [M, lda]: int8 (I8) or bf16 */
  int32_t lda;
  const void* b;          /* weights [n, ldb]: int8 (I8, W8A16) or bf16 (BF16) */
  int32_t ldb;
  const float* wscale;    /* [n] per-output-channel weight scale (I8, W8A16) */
  const void* bias;       /* bf16 [n] or NULL */
  const float* bias_f32;  /* fp32 [n] or NULL, added after bias */
  void* out;              /* output [M, ldo] (bf16, int32 or fp32 by epilogue) */
  int32_t ldo;
  int32_t n;              /* columns, multiple of 16 */
  float act_scale;        /* I8: activation scale a */
  int32_t rope;           /* EPI_ROPE: rotate this segment (n % 64 == 0) */
} svla_gemm_seg;

typedef struct svla_gemm_desc {
  int32_t kind, epi;
  int32_t m, k;
  int32_t nseg;           /* 1..3 segments sharing M and K, each with its own A and weights */
  int32_t pair;           /* 1: seg[0] (gate) and seg[1] (up) form one SILU_MUL tile pair */
  svla_gemm_seg seg[3];
  int32_t block_n;        /* 64 or 128; 0 = choose */
  /* output row remap: row = (m / rows_per_group) * group_stride + m % rows_per_group + row_offset */
  int32_t rows_per_group, group_stride, row_offset;
  float post_scale;       /* EPI_BF16: 0 = off */
  const void* resid;      /* EPI_RESID: bf16 residual, may alias seg[0].out */
  int32_t ldr, resid_rows; /* resid_rows > 0: residual row = m % resid_rows */
  const float* rope_cs;   /* EPI_ROPE: [max_pos][32] float2 (cos, sin) */
  const int32_t* pos;     /* EPI_ROPE: [M] */
  int32_t max_pos;
  const float* q_smooth;  /* EPI_GELU_QUANT */
  const float* q_rsmooth; /* optional 1 / q_smooth (correctly rounded, svla_reciprocal): faster, same result */
  float q_act;
  int8_t* qout;
  int32_t ldq;
  float dt;               /* EPI_EULER */
  float* xt;
  void* xt_bf16;
  uint64_t* debug_clock;  /* optional [32]: SM clock stamps of the first CTA's phases (profiling), else NULL */
  int32_t weights_resident; /* 1: every B operand was written before the previously launched kernel started
                               (packed weights), so its first tiles are fetched before waiting for that kernel */
  /* Split-K for GEMMs with few output tiles: split_k 0 = automatic (when a workspace is given and the
   * output tiles fill at most half of the SMs), 1 = off, n > 1 = n splits.  Each split stores its raw
   * accumulators in the workspace; the last one of a tile adds them in split order (int32 sums are exact,
   * so I8 results do not change) and runs the epilogue.  The workspace (256-byte aligned) starts with
   * SVLA_SPLITK_COUNTER_BYTES of tile counters that must be zero before its first use; every completed
   * launch leaves them zero.  Launches that share a workspace must be stream-ordered.  Split-K runs with
   * 64-column tiles (block_n 0 picks them for few-tile GEMMs; other block_n values cannot split). */
  int32_t split_k;
  void* workspace;
  size_t workspace_bytes;
  /* CTA pairs: 0 or 1 = one CTA per 128-row tile, 2 = two CTAs per 256-row tile (tcgen05 cta_group::2:
   * each SM loads its own A rows and half of B, 2/3 of the operand bytes per SM for the same MMA work;
   * I8 / BF16 operands, block_n 128 or 256, no split-K, m > 128).  Bit-identical results either way. */
  int32_t cta_pair;
} svla_gemm_desc;

#define SVLA_SPLITK_COUNTER_BYTES 65536

/* Alignment (checked, status 1 otherwise): A / B operands and every output 16-byte aligned with row strides that
 * are multiples of 16 bytes and >= the segment's columns (ldo, ldr, ldq).  A NULL wscale reads as all ones. */
int32_t svla_gemm(const svla_gemm_desc* desc, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * Norm + SmoothQuant quantise (RMSNorm: SmolVLM2 text / expert; LayerNorm: SigLIP).  One launch emits the
 * bf16 normalised rows and up to three int8 tensors, each with its own smooth vector and activation
 * scale (per-projection SmoothQuant of q/k/v, deploy/cuda/smoothquant_qkv_cublaslt.cu:245-247).
 * ------------------------------------------------------------------------------------------------*/
typedef struct svla_norm_desc {
  const void* x; int32_t ldx;
  const void* weight;     /* bf16 [K] */
  const void* bias;       /* bf16 [K] (LayerNorm) or NULL */
  float eps;
  int32_t layernorm;      /* 0 = RMSNorm, 1 = LayerNorm */
  int32_t m, k;
  void* y; int32_t ldy;   /* bf16 output or NULL */
  int32_t nq;
  int8_t* q[3];
  int32_t ldq;
  const float* smooth[3];
  const float* rsmooth[3]; /* optional 1 / smooth[i] (svla_reciprocal): faster, same int8 result */
  float act[3];
  int32_t pixel_shuffle;  /* 0, or the SmolVLM connector shuffle factor (remaps y and the int8 outputs) */
  int32_t ps_grid;        /* tokens per side of the input grid */
} svla_norm_desc;

int32_t svla_norm_quant(const svla_norm_desc* desc, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * Attention; replaces the fused RoPE attention plugins (deploy/cuda/fused_rope_layout.h:44-50,
 * fused_rope_layout.cu:271-543) for post-RoPE q/k (RoPE is fused into the QKV GEMM epilogue).
 * Masked GQA, head_dim 64; keys from one or two sources (cached prefix, then current suffix).
 * Unmasked single-source calls with at least 128 queries run on the tcgen05 kernel (S and O in tensor
 * memory); the rest on an mma.sync kernel that packs each kv head's query heads into its row tiles.
 * ------------------------------------------------------------------------------------------------*/
typedef struct svla_attn_desc {
  const void* q; int64_t q_bs; int32_t q_rs;
  const void* k1; const void* v1; int64_t kv1_bs; int32_t kv1_rs; int32_t l1;
  const void* k2; const void* v2; int64_t kv2_bs; int32_t kv2_rs; int32_t l2;
  const uint8_t* mask; int64_t mask_bs; int32_t mask_rs; /* bool mask [B, Lq, l1 + l2] or NULL */
  void* o; int64_t o_bs; int32_t o_rs;                   /* bf16 context or NULL */
  int8_t* qo; int64_t qo_bs; int32_t qo_rs;              /* int8 context (next W8A8 input) or NULL */
  const float* qo_smooth; const float* qo_rsmooth; float qo_act; /* qo_rsmooth optional, as in svla_norm_desc */
  int32_t batch, lq, hq, hkv;
  float scale;                                           /* 0 = head_dim^-1/2 */
  int32_t impl; /* SVLA_ATTN_AUTO (tcgen05 for unmasked calls, mma.sync for masked ones), or force
                   SVLA_ATTN_MMA_SYNC / SVLA_ATTN_TCGEN05 (the latter needs 16-byte aligned operands and strides;
                   byte masks only on a single key source with rows padded to a multiple of 16 keys) */
  void* debug_clock; /* profiling: uint64 [96] phase clock stamps of one CTA of the tcgen05 kernel, or NULL */
  /* Structured mask, instead of `mask` (same result as the equivalent byte mask, far less mask traffic):
   * query i may see key k iff k < mask_keys ? key_mask[b*key_mask_bs + k] != 0 : k - mask_keys <= i
   * (key padding over the first mask_keys keys, causal order over the rest: the action expert's masks). */
  const uint8_t* key_mask; int64_t key_mask_bs; int32_t mask_keys;
} svla_attn_desc;

enum { SVLA_ATTN_AUTO = 0, SVLA_ATTN_MMA_SYNC = 1, SVLA_ATTN_TCGEN05 = 2 };

int32_t svla_attention(const svla_attn_desc* desc, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * Plugin-semantics RoPE operators (the SmolVLAFusedRopeLayout / SmolVLAFusedRopeAttention TensorRT plugins).
 * Data and position types use TensorRT's nvinfer1::DataType numbering, so a plugin's enqueue can pass its
 * tensor descriptors' types straight through.
 * ------------------------------------------------------------------------------------------------*/
#define SVLA_DT_FLOAT 0
#define SVLA_DT_HALF 1
#define SVLA_DT_INT32 3
#define SVLA_DT_BF16 7
#define SVLA_DT_INT64 8

/* FusedRopeLayoutParams (deploy/cuda/fused_rope_layout.h:24-30): defaults 15 / 5 / 64 / 10000. */
typedef struct svla_rope_params {
  int32_t q_heads, kv_heads, head_dim;
  float max_wavelength;
} svla_rope_params;

/* RoPE + layout; replaces launchFusedRopeLayout (deploy/cuda/fused_rope_layout.h:32-34,
 * fused_rope_layout.cu:81-124, :545-571): q_raw [B, L, Hq*D] -> q_out [B, Hq, L, D];
 * k_raw [B, L, Hkv*D] -> k_out [B, Hq, D, L] (GQA-expanded and transposed); rotate-half in fp32 with
 * theta_i = pos / max_wavelength^(2i/D).  data_type FLOAT / HALF / BF16 (outputs in the same type),
 * position_type INT32 / INT64 ([B, L]); head_dim even. */
int32_t svla_fused_rope_layout(const void* q_raw, const void* k_raw, const void* position_ids, void* q_out,
                               void* k_out, int32_t batch, int32_t seq_len, const svla_rope_params* params,
                               int32_t data_type, int32_t position_type, svla_stream_t stream);

/* The bf16 / int32-position / head_dim-64 case of svla_fused_rope_layout. */
int32_t svla_rope_layout(const void* q_raw, const void* k_raw, const int32_t* pos, void* q_out, void* k_out,
                         int32_t batch, int32_t seq_len, int32_t q_heads, int32_t kv_heads,
                         float max_wavelength, svla_stream_t stream);

/* Fused RoPE attention; replaces launchFusedRopeAttention (deploy/cuda/fused_rope_layout.h:44-46,
 * fused_rope_layout.cu:271-431, :768-788; the plugin of deploy/cuda/fused_attention_v3_real.cpp:104-116):
 * raw q [B, L, Hq*D], raw k / v [B, L, Hkv*D] (data_type), position_ids [B, L] (position_type), mask bool
 * bytes [B, L, L] (nonzero = keep) -> context fp32 [B, Hq, L, D].  fp32 arithmetic throughout: rotated q / k,
 * scores * D^-1/2 over kept keys, softmax, P.V; a query with every key masked gets the mean of V.
 * head_dim a multiple of 32 up to 128. */
int32_t svla_fused_rope_attention(const void* q_raw, const void* k_raw, const void* v_raw, const void* position_ids,
                                  const void* mask, float* context, int32_t batch, int32_t seq_len,
                                  const svla_rope_params* params, int32_t data_type, int32_t position_type,
                                  svla_stream_t stream);

/* The fp32 variant with implicit positions 0..L-1 and an fp32 mask (keep = value > 0.5); replaces
 * launchFusedRopeAttentionFp32MaskImplicitPos (deploy/cuda/fused_rope_layout.h:48-50, .cu:433-543, :790-800). */
int32_t svla_fused_rope_attention_f32_mask_implicit_pos(const float* q_raw, const float* k_raw, const float* v_raw,
                                                        const float* mask, float* context, int32_t batch,
                                                        int32_t seq_len, const svla_rope_params* params,
                                                        svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * sample_actions glue
 * ------------------------------------------------------------------------------------------------*/
/* Policy-side processing around sample_actions (lerobot SmolVLA prepare_images / prepare_state and the
 * action unnormalisation of predict_action_chunk; called at
 * deploy/calibrate_smolvla_activation_channel_scales.py:138-139).
 * Images: src fp32 [N, C, H, W] in [0, 1], or (src_u8_hwc) uint8 [N, H, W, C] read as value / 255; resized
 * keeping the aspect ratio to (int(h / r), int(w / r)), r = max(w / out_w, h / out_h), by bilinear
 * interpolation with half-pixel source indices (torch interpolate, align_corners=False), padded with
 * pad_value on the top and left to out_h x out_w, then mapped to [-1, 1] (x * 2 - 1).  Output image i at
 * out + i * out_image_stride (fp32 [C, out_h, out_w]). */
int32_t svla_resize_pad_images(const void* src, int32_t src_u8_hwc, int32_t n, int32_t c, int32_t h, int32_t w,
                               float* out, int64_t out_image_stride, int32_t out_h, int32_t out_w, float pad_value,
                               svla_stream_t stream);
/* state [B, dim] (row stride ld) -> [B, out_dim], zero-padded; mode 0 MEAN_STD (x - p0) / (p1 + 1e-8),
 * mode 1 MIN_MAX ((x - p0) / (p1 - p0 + 1e-8)) * 2 - 1 (p0 = min, p1 = max). */
int32_t svla_normalize_state(const float* state, int32_t batch, int32_t dim, int32_t ld, const float* p0,
                             const float* p1, int32_t mode, int32_t out_dim, float* out, svla_stream_t stream);
/* actions [rows, ld] -> [rows, action_dim]: mode 0 x * p1 + p0 (p0 = mean, p1 = std); mode 1
 * (x + 1) / 2 * (p1 - p0) + p0 (p0 = min, p1 = max). */
int32_t svla_unnormalize_actions(const float* actions, int32_t rows, int32_t ld, int32_t action_dim, const float* p0,
                                 const float* p1, int32_t mode, float* out, svla_stream_t stream);

/* cs[p][i] = (cos, sin)(p / max_wavelength^(2i/64)), p < max_pos, i < 32 */
int32_t svla_rope_table(float* cs, int32_t max_pos, float max_wavelength, svla_stream_t stream);

/* Masks and positions of one call (deploy/diagnose_3_4_numeric_baseline.py:42-46, :117-146, :171-172).
 * img_mask0/1 bool [B], lang_mask bool [B, n_lang]; prefix length Lp = 2*n_img + n_lang + 1, Ls = chunk.
 * prefix_mask [B, Lp, ld(Lp)], self_mask [B, Ls, ld(Lp + Ls)], cross_mask [B, Ls, ld(Lp)] bytes with the
 * row stride ld(L) = L rounded up to a multiple of 16 (padding bytes 0), 16-byte aligned; prefix_pos [B, Lp],
 * suffix_pos / cross_pos [B, Ls]. */
int32_t svla_build_masks(const uint8_t* img_mask0, const uint8_t* img_mask1, const uint8_t* lang_mask,
                         int32_t batch, int32_t n_img, int32_t n_lang, int32_t chunk, uint8_t* prefix_mask,
                         int32_t* prefix_pos, uint8_t* self_mask, uint8_t* cross_mask, int32_t* suffix_pos,
                         int32_t* cross_pos, svla_stream_t stream);

/* out[b*rows_per_batch + row_offset + t] = bf16(table[tokens[b,t]] * scale); tokens int64 [B, T] */
int32_t svla_embed_tokens(const int64_t* tokens, int32_t batch, int32_t t, const void* table, int32_t vocab,
                          int32_t hidden, float scale, void* out, int32_t rows_per_batch, int32_t row_offset,
                          svla_stream_t stream);

/* images fp32 [N, C, S, S] -> bf16 patches [N*(S/P)^2, C*P*P] in Conv2d (c, kh, kw) order */
int32_t svla_im2col(const float* images, int32_t n, int32_t c, int32_t s, int32_t p, void* out,
                    svla_stream_t stream);

int32_t svla_f32_to_bf16(const float* x, void* y, int64_t n, svla_stream_t stream);
/* y[i] = 1 / x[i], correctly rounded (the reciprocal smooth vectors the quantisers accept) */
int32_t svla_reciprocal(const float* x, float* y, int64_t n, svla_stream_t stream);
int32_t svla_euler_init(const float* noise, float* xt, void* xt_bf16, int64_t n, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * Flow-matching loop as one persistent kernel, for calls with batch * chunk <= 64 action rows (batch-1
 * latency).  Runs x_t = noise, then num_steps x [action_in_proj, time MLP, every expert layer, final
 * RMSNorm, action_out_proj, x_t += dt * v] (lerobot VLAFlowMatching.sample_actions / denoise_step) in one
 * cooperative launch (one CTA per SM, grid barriers between phases, every wait bounded).  Same arithmetic
 * and rounding points as the per-layer launches (svla_gemm / svla_norm_quant / svla_attention with the
 * structured expert masks); only the fp32 summation order inside dot products differs.  The weights are
 * read in the MMA fragment order svla_flow_pack_weight writes (each warp load is one contiguous run): the
 * expert layers' W8A16 linears as int8 with their per-output-channel scales, dequantised in registers to
 * bf16(q * w_s) -- the W8A16Linear weight (deploy/linear_only_quant.py:122-124, :147-148) bit for bit at half
 * the bytes of the bf16 copy -- and the bf16 linears (action / time projections) as bf16.  No counterpart
 * launch in the reference, whose TensorRT engine runs the loop as separate layers
 * (deploy/trt_sample_actions_core_deploy.py:108-237).
 * ------------------------------------------------------------------------------------------------*/
#define SVLA_FLOW_MAX_LAYERS 32
#define SVLA_FLOW_MAX_ROWS 64

/* Bytes of the fragment-packed copy of an [n, k] weight (n, k multiples of 16): n * k * elem_bytes. */
size_t svla_flow_packed_bytes(int32_t n, int32_t k, int32_t elem_bytes);
/* Writes the fragment-packed copy of w ([n, k], row stride ld elements; elem_bytes 1 = int8, 2 = bf16) to out
 * (svla_flow_packed_bytes, 16-byte aligned): 16-row slices, each K/16 steps x 32 lanes x 8 elements in the
 * order of the mma.m16n8k16 B fragments of the slice's two 8-row tiles. */
int32_t svla_flow_pack_weight(const void* w, int32_t elem_bytes, int64_t ld, int32_t n, int32_t k, void* out,
                              svla_stream_t stream);

typedef struct svla_flow_layer {
  const void* input_norm;  /* bf16 [E] */
  const void* post_norm;   /* bf16 [E] */
  /* int8 weights, fragment-packed (svla_flow_pack_weight, elem_bytes 1), each with its fp32 per-output-channel
   * scale w_s [n] (svla_pack_weight_i8) */
  const void* wq; const float* sq;  /* [heads * 64, E] */
  const void* wk; const float* sk;  /* [kv_heads * 64, E] (self-attention layers; NULL on cross-attention layers) */
  const void* wv; const float* sv;
  const void* wo; const float* so;  /* [E, heads * 64] */
  const void* wg; const float* sg;  /* [mlp, E] */
  const void* wu; const float* su;  /* [mlp, E] */
  const void* wd; const float* sd;  /* [E, mlp] */
  const void* keys;        /* bf16 [batch * prefix_len, kv_heads * 64]: the layer's prefix KV cache (self) or */
  const void* values;      /*   its cross-attention K/V projections (cross) */
  int32_t cross;
} svla_flow_layer;

typedef struct svla_flow_desc {
  int32_t batch, chunk, prefix_len;
  int32_t hidden;          /* E (multiple of 16, <= 1024) */
  int32_t action_dim;      /* the padded action width A (multiple of 16) */
  int32_t heads, kv_heads, mlp, n_layers, num_steps;
  float eps;               /* RMSNorm epsilon */
  const float* noise;      /* fp32 [batch * chunk, A] */
  float* xt;               /* fp32 [batch * chunk, A]: the actions on return */
  void* xt_bf16;           /* bf16 [batch * chunk, A] scratch */
  /* bf16 weights, fragment-packed (svla_flow_pack_weight, elem_bytes 2); biases bf16 */
  const void* w_action_in; const void* b_action_in;       /* [E, A], [E] */
  const void* w_time_in;                                  /* the first E columns of action_time_mlp_in, [E, E] */
  const float* time_in_const;                             /* fp32 [num_steps, E]: W[:, E:] . time_emb(t_k) + b */
  const void* w_time_out; const void* b_time_out;         /* [E, E], [E] */
  const void* final_norm;                                 /* bf16 [E] */
  const void* w_action_out; const void* b_action_out;     /* [A, E], [A] */
  const uint8_t* key_mask; int64_t key_mask_bs;           /* prefix key flags of sample b at key_mask + b * bs
                                                             (16-byte aligned rows of >= prefix_len rounded up to
                                                             16 bytes), or NULL */
  const int32_t* suffix_pos; const int32_t* cross_pos;    /* [batch * chunk] RoPE positions */
  const float* rope_cs; int32_t max_pos;                  /* svla_rope_table */
  /* scratch (bf16): a_emb, a_t, eh [rows, E]; eq, ectx [rows, heads * 64]; ek, ev [rows, kv_heads * 64];
   * emlp [rows, mlp] */
  void* a_emb; void* a_t; void* eh; void* eq; void* ek; void* ev; void* ectx; void* emlp;
  float* norm_part;        /* fp32 scratch [64 * 64]: per action row and 16-column slice of E, the sum of squares
                              of the expert hidden state (the RMSNorm statistics, written by the phase that writes
                              the rows and summed in slice order by the next) */
  uint32_t* sync;          /* 8 bytes (8-byte aligned), zero before the first launch; every completed launch leaves
                              it valid.  After a device error (svla_device_error) zero it again. */
  uint32_t spin_limit;     /* polls of a grid barrier before the kernel gives up with device error 103 and returns
                              (the other CTAs return at their next barrier); 0 = the library default (about 4M
                              polls of ~32 ns: seconds) */
  uint64_t* debug_clock;   /* profiling, or NULL: 2 x 1024 (event, globaltimer ns) pairs of the first and last CTA
                              (events 1/2 barrier enter/exit, 3 rows staged, 4 products done, 5 epilogue done,
                              6 attention task done) */
  svla_flow_layer layer[SVLA_FLOW_MAX_LAYERS];
} svla_flow_desc;

int32_t svla_flow(const svla_flow_desc* desc, svla_stream_t stream);

/* -------------------------------------------------------------------------------------------------
 * Whole-path engine: the quantized sample_actions call in native code.  Replaces the TensorRT core
 * runner's engine load + execute (deploy/trt_sample_actions_core_deploy.py:108-237, called per chunk from
 * deploy/eval_libero_trt_sample_actions_core.py) with one C call over the kernels above: masks, SigLIP,
 * connector, the prefix prefill into the KV cache, the cross-layer K/V projections and the flow-matching
 * loop of the action expert.
 * The engine loads a packed-weights file (safetensors, metadata "svla_packed" = "1", "config" and
 * "linears" JSON; tensors "lin/<module>/{weight,wscale,bias,smooth,rsmooth,weight_deq}" and "t/<name>",
 * including "t/time_embedding" bf16 [num_steps, expert_hidden]), the file the Python package's save_packed
 * writes.  It owns its device memory (weights, activation buffers for max_batch samples, a split-K
 * workspace) and one launch list per batch size, recorded as a CUDA graph after its first run.
 * ------------------------------------------------------------------------------------------------*/
typedef struct svla_engine svla_engine;

typedef struct svla_engine_info {
  int32_t n_cams, channels, image_size;          /* images: n_cams x fp32 [B, channels, image_size, image_size] */
  int32_t n_lang;                                /* language tokens per sample */
  int32_t max_state_dim, max_action_dim, chunk, num_steps, action_dim;
  int32_t prefix_len;
  int32_t vis_layers, text_layers, expert_layers;
  int32_t n_linears;                             /* linears in the file */
  int32_t n_tensors;                             /* tensors in the file */
  int32_t launches_per_call;                     /* kernel launches of one sample_actions call (0 = not built) */
  int32_t max_batch;                             /* 0 for svla_engine_inspect */
  int64_t weight_bytes;                          /* device bytes of the weights */
  int64_t buffer_bytes;                          /* device bytes of activations, workspace and constants */
} svla_engine_info;

#define SVLA_ENGINE_NO_GRAPH 1    /* launch the kernels one by one on every call (no CUDA graph) */
#define SVLA_ENGINE_NO_SPLIT_K 2  /* no split-K: every sample's result is bit-identical at any batch size */
#define SVLA_ENGINE_NO_FLOW 4     /* run the flow loop as per-layer launches even when svla_flow applies */

/* Parses and validates a packed-weights file without touching the GPU (info->max_batch = 0,
 * launches_per_call = 0, buffer_bytes = 0). */
int32_t svla_engine_inspect(const char* packed_path, svla_engine_info* info);
/* Loads the file onto the current device and computes the call's constants on `stream` (synchronised
 * before returning).  max_batch >= 1; flags: SVLA_ENGINE_* bits. */
int32_t svla_engine_create(const char* packed_path, int32_t max_batch, int32_t flags, svla_stream_t stream,
                           svla_engine** out);
int32_t svla_engine_get_info(const svla_engine* engine, svla_engine_info* info);
/* sample_actions(images, img_masks, lang_tokens, lang_masks, state, noise) for `batch` samples
 * (lerobot VLAFlowMatching.sample_actions; the reference's core engine inputs,
 * deploy/trt_sample_actions_core_deploy.py:240-299):
 *   images[cam]    fp32 [batch, channels, image_size, image_size], cam < n_cams (already resized to the
 *                  model's size and mapped to [-1, 1]: svla_resize_pad_images)
 *   img_masks[cam] uint8 [batch] (0 = camera missing)
 *   lang_tokens    int64 [batch, lang_len], lang_masks uint8 [batch, lang_len]; the first n_lang tokens are
 *                  used, shorter rows are padded with masked-out zeros (match_static_shape,
 *                  deploy/trt_sample_actions_core_deploy.py:276-286)
 *   state          fp32 [batch, state_dim], state_dim <= max_state_dim (zero-padded)
 *   noise          fp32 [batch, chunk, max_action_dim]
 *   actions        fp32 [batch, chunk, max_action_dim] (out)
 * Every array may be host memory (pageable or pinned) or device memory; copies are stream-ordered on
 * `stream`, as are the kernels.  Calls share the engine's buffers: issue them on one stream, or
 * synchronise between calls on different streams. */
int32_t svla_engine_sample_actions(svla_engine* engine, const float* const* images, const uint8_t* const* img_masks,
                                   const int64_t* lang_tokens, const uint8_t* lang_masks, int32_t lang_len,
                                   const float* state, int32_t state_dim, const float* noise, int32_t batch,
                                   float* actions, svla_stream_t stream);
/* Frees the engine's device memory and graphs (synchronises the device first).  NULL is a no-op. */
int32_t svla_engine_destroy(svla_engine* engine);

#ifdef __cplusplus
}
#endif
#endif /* SVLA_H_ */
