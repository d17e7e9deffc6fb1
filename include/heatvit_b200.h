/*
 * heatvit_b200.h — C ABI of the B200 (sm_100a) integer HeatViT-T inference engine.
 *
 * Every entry point takes plain pointers and sizes; no torch or C++ types cross
 * this boundary.  Device pointers are marked `d_`, host pointers `h_`.  All
 * arithmetic is integer and bit-exact with the reference golden model
 * (verification/heatvit_ref in YOUXINYANG/HeatViT); each declaration names the
 * reference function it replaces.
 *
 * Status codes: 0 = ok; the other values mirror the golden model's Python
 * exceptions (see HV_ERR_*) so a host wrapper can raise the same exception type.
 * Warnings are a per-image bitmask: bit0 head-weight denominator zero, bit1
 * package denominator zero (verification/heatvit_ref/selector.py:31-32), bit2
 * LayerNorm negative variance (verification/heatvit_ref/nonlinear.py:127-130).
 */
#ifndef HEATVIT_B200_H
#define HEATVIT_B200_H

#include <stdint.h>
#include <stddef.h>

#if defined(__GNUC__)
#define HV_API __attribute__((visibility("default")))
#else
#define HV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- model geometry (config/heatvit_t.json:3-12) ---------------------------- */
#define HV_IMAGE_W 224
#define HV_IMAGE_H 224
#define HV_IMAGE_BYTES (224 * 224 * 3)
#define HV_PATCH 16
#define HV_PATCHES 196
#define HV_PATCH_K 768
#define HV_TOKENS 197
#define HV_EMBED 192
#define HV_HEADS 3
#define HV_HEAD_DIM 64
#define HV_QKV 576
#define HV_FFN 768
#define HV_CLASSES 1000
#define HV_BLOCKS 12
#define HV_MAX_SELECTORS 12
#define HV_LOGIT_SCALE_EXP (-14) /* verification/heatvit_ref/model.py:21 */

/* Checkpoint slots: 0 patch, 1..12 block_01..12, 13..24 selector_01..12, 25 final_ln
 * (verification/heatvit_ref/model.py:78-117). */
#define HV_CKPT_SLOTS 26
#define HV_CKPT_PATCH 0
#define HV_CKPT_BLOCK(b) (b)              /* b = 1..12 */
#define HV_CKPT_SELECTOR(s) (12 + (s))    /* s = 1..12 */
#define HV_CKPT_FINAL_LN 25

/* ---- status codes -------------------------------------------------------------- */
#define HV_OK 0
#define HV_ERR_VALUE 1     /* ValueError: shape / range / scale contract          */
#define HV_ERR_TYPE 2      /* TypeError                                           */
#define HV_ERR_OVERFLOW 3  /* OverflowError: GEMM accumulator left int32 (gemm.py:116-117) */
#define HV_ERR_CUDA 4      /* CUDA runtime error                                  */
#define HV_ERR_NOMEM 5     /* allocation failure                                  */
#define HV_ERR_STATE 6     /* wrong call order / unsupported on this device       */

/* ---- warnings -------------------------------------------------------------------- */
#define HV_WARN_HEAD_DEN_ZERO 1u
#define HV_WARN_PACKAGE_DEN_ZERO 2u
#define HV_WARN_LN_NEG_VARIANCE 4u

/* ---- parameters (host memory, golden dataclass layouts) -------------------------
 * Matrices are row-major exactly as the golden dataclasses hold them:
 * weight[k][n] for every GEMM B operand.  Scale exponents are the dataclass
 * fields of the same name. */
typedef struct hv_patch_params {           /* transformer.py:51-93 PatchParams */
    const int8_t *weight;                  /* [768][192] */
    const int32_t *bias;                   /* [192] */
    const int8_t *cls;                     /* [192] */
    const int8_t *pos;                     /* [197][192] */
    int32_t image_scale_exp, weight_scale_exp, activation_scale_exp;
    int32_t tokens_scale_exp, cls_scale_exp, pos_scale_exp;
} hv_patch_params;

typedef struct hv_block_params {           /* transformer.py:148-198, 287-325 */
    const int8_t *ln1_gamma, *ln1_beta;    /* [192] */
    const int8_t *wqkv;                    /* [192][576] */
    const int32_t *bqkv;                   /* [576] */
    const int8_t *wproj;                   /* [192][192] */
    const int32_t *bproj;                  /* [192] */
    const int8_t *ln2_gamma, *ln2_beta;    /* [192] */
    const int8_t *w1;                      /* [192][768] */
    const int32_t *b1;                     /* [768] */
    const int8_t *w2;                      /* [768][192] */
    const int32_t *b2;                     /* [192] */
    /* MhsaParams */
    int32_t x_scale_exp, gamma1_scale_exp, beta1_scale_exp, ln1_out_scale_exp;
    int32_t wqkv_scale_exp, qkv_out_scale_exp, score_scale_exp, prob_scale_exp;
    int32_t context_out_scale_exp, wproj_scale_exp, msa_out_scale_exp;
    /* FfnParams */
    int32_t ffn_x_scale_exp, gamma2_scale_exp, beta2_scale_exp, ln2_out_scale_exp;
    int32_t w1_scale_exp, hidden_out_scale_exp, w2_scale_exp, ffn_out_scale_exp;
    int32_t out_scale_exp;
} hv_block_params;

typedef struct hv_selector_params {        /* selector.py:111-221 */
    const int8_t *local_w;                 /* [3][64][32] */
    const int32_t *local_b;                /* [3][32] */
    const int8_t *score_w1;                /* [3][64][32] */
    const int32_t *score_b1;               /* [3][32] */
    const int8_t *score_w2;                /* [3][32][16] */
    const int32_t *score_b2;               /* [3][16] */
    const int8_t *score_w3;                /* [3][16][2] */
    const int32_t *score_b3;               /* [3][2] */
    const int8_t *hw_w1;                   /* [3][3] */
    const int32_t *hw_b1;                  /* [3] */
    const int8_t *hw_w2;                   /* [3][3] */
    const int32_t *hw_b2;                  /* [3] */
    int32_t in_scale_exp, local_w_scale_exp, local_out_scale_exp, concat_out_scale_exp;
    int32_t score_w1_scale_exp, score_w2_scale_exp, score_w3_scale_exp;
    int32_t h1_out_scale_exp, h2_out_scale_exp, logits_out_scale_exp;
    int32_t stats_out_scale_exp, hw_w1_scale_exp, hw_hidden_out_scale_exp, hw_w2_scale_exp;
} hv_selector_params;

typedef struct hv_params {                 /* model.py:24-46 HeatViTParams */
    hv_patch_params patch;
    hv_block_params blocks[HV_BLOCKS];
    /* selector_before[b] = index into selectors[] of the selector that runs
     * before block b+1, or -1.  model.py:81-87 assigns selectors in block order. */
    int32_t selector_before[HV_BLOCKS];
    int32_t num_selectors;
    hv_selector_params selectors[HV_MAX_SELECTORS];
    const int8_t *final_gamma, *final_beta; /* [192] */
    const int8_t *head_w;                   /* [192][1000] */
    const int32_t *head_b;                  /* [1000] */
    int32_t final_gamma_scale_exp, final_beta_scale_exp;
    int32_t final_ln_out_scale_exp, head_w_scale_exp;
} hv_params;

/* Per-selector summary (model.py:90-96) plus the warning bits. */
typedef struct hv_selector_summary {
    int32_t input_tokens, output_tokens, kept_normal, pruned_normal;
    int32_t package_present, warnings;
} hv_selector_summary;

/* ---- library / device ------------------------------------------------------------ */
/* Returns a static version string. */
HV_API const char *hv_version(void);
/* Last error message of the calling thread (never NULL). */
HV_API const char *hv_last_error(void);

/* ---- model object (replaces HeatViTModel, model.py:70-123) ------------------------ */
typedef struct hv_model hv_model;

/* Validate and pack `params` into device memory on `device` (weights are
 * transposed to K-major and per-layer epilogue tables are built once).
 * Reference: the frozen HeatViTParams (model.py:24-46) consumed by infer().
 * A partial model is allowed: leave the patch weight, a block's wqkv, or the
 * head weight NULL to omit that part (e.g. a model holding only selectors for
 * hv_token_selector); entry points that need a missing part return HV_ERR_STATE. */
HV_API int hv_model_create(const hv_params *params, int device, hv_model **out);
HV_API int hv_model_destroy(hv_model *model);

/* Batched inference, all buffers on the model's device.
 *   d_images        [batch][224*224*3] int8 NHWC (layout.py:31-72 order)
 *   d_logits        [batch][1000] int32 at 2^-14 (model.py:107-115)
 *   d_token_counts  [batch][num_selectors+1] int32 (197, then each selector's output), may be NULL
 *   d_summary       [batch][num_selectors] hv_selector_summary, may be NULL
 *   d_warnings      [batch] uint8 bitmask, may be NULL
 *   stream          cudaStream_t (NULL = legacy default stream)
 * Replaces HeatViTModel.infer (model.py:73-123) applied image by image. */
HV_API int hv_infer_batch(hv_model *model, const int8_t *d_images, int batch,
                   int32_t *d_logits, int32_t *d_token_counts,
                   hv_selector_summary *d_summary, uint8_t *d_warnings,
                   void *stream);

/* Same as hv_infer_batch, plus every golden checkpoint:
 *   d_ckpt    [batch][HV_CKPT_SLOTS][197][192] int8; slot layout HV_CKPT_*; rows
 *             beyond a slot's token count are left untouched.
 *   d_ckpt_rows [batch][HV_CKPT_SLOTS] int32 row count of each slot (0 = slot unused).
 * Reference: ModelResult.checkpoints (model.py:78-117). */
HV_API int hv_infer_batch_checkpoints(hv_model *model, const int8_t *d_images, int batch,
                               int32_t *d_logits, int32_t *d_token_counts,
                               hv_selector_summary *d_summary, uint8_t *d_warnings,
                               int8_t *d_ckpt, int32_t *d_ckpt_rows, void *stream);

/* Host-buffer convenience: copies h_images (pinned or pageable) to the device in
 * chunks on two streams overlapped with compute, runs the batch, copies logits
 * (and the optional outputs) back.  Blocks until the results are on the host.
 * The host-side counterpart of model.HeatViTModel.infer over a batch
 * (verification/heatvit_ref/model.py:70-123). */
HV_API int hv_infer_host(hv_model *model, const int8_t *h_images, int batch,
                  int32_t *h_logits, int32_t *h_token_counts,
                  hv_selector_summary *h_summary, uint8_t *h_warnings);

/* Asynchronous form of hv_infer_host for serving loops: enqueues one call's
 * uploads, inference and downloads and returns.  hv_infer_host_wait blocks until
 * the oldest submitted call has finished and its outputs are in the caller's
 * arrays, which (and h_images) must stay untouched until then.  Two calls may be
 * in flight (a third submit first waits for the oldest); the next call's uploads
 * run during this call's compute, so a call submitted behind another runs as
 * whole 1024-image chunks on one compute stream instead of the two-stream chunks
 * of hv_infer_host.  While calls are in flight the model's other
 * entry points return HV_ERR_STATE.  No counterpart in the reference (its model
 * runs one image per call). */
HV_API int hv_infer_host_submit(hv_model *model, const int8_t *h_images, int batch,
                  int32_t *h_logits, int32_t *h_token_counts,
                  hv_selector_summary *h_summary, uint8_t *h_warnings);
HV_API int hv_infer_host_wait(hv_model *model);

/* Read and clear the model's device error word (synchronises with the device).
 * *code != 0 means a kernel's bounded wait on a tensor-core completion gave up
 * and that launch's outputs are invalid.  No counterpart in the reference (its
 * RTL reports a watchdog timeout as a fatal error code). */
HV_API int hv_device_error(hv_model *model, int *code);

/* ---- kernel timing (bench and tracing) ------------------------------------------
 * Stage ids for hv_profile_*: one id per kernel of the per-block pipeline. */
#define HV_STAGE_LN1 1
#define HV_STAGE_QKV 2
#define HV_STAGE_ATTN 3
#define HV_STAGE_PROJ 4
#define HV_STAGE_LN2 5
#define HV_STAGE_FC1 6
#define HV_STAGE_FC2 7
#define HV_STAGE_SELECTOR 8
#define HV_STAGE_PATCH 9
#define HV_STAGE_HEAD 10
#define HV_STAGE_FFN 11   /* FC1 + GELU + FC2 + residual 2 in one kernel (replaces FC1 / FC2) */

/* Record a CUDA event pair around every launch of `stage` (0 disables) in the
 * following hv_infer_* calls; at most `max_launches` launches are recorded.
 * No counterpart in the reference (its only profiler is the RTL testbench
 * monitor); used to time one kernel live inside a timed region. */
HV_API int hv_profile_start(hv_model *model, int stage, int max_launches);
/* Stop recording; returns the number of recorded launches, their total GPU time
 * in milliseconds and the summed live row count of those launches (read back
 * from the device after the events complete). */
HV_API int hv_profile_stop(hv_model *model, int *launches, double *total_ms, long long *rows);
/* Kernel nodes of the CUDA graph that the last graph-replayed hv_infer_batch ran
 * (0 before any replay).  Under profiling, hv_infer_batch replays a graph that holds
 * the profiling events, and hv_profile_stop reports the launches of its last replay.
 * No counterpart in the reference. */
HV_API int hv_graph_kernels(hv_model *model, int *kernels);

/* Test hook for the bounded-wait error path of the layer GEMMs (QKV, proj, patch,
 * and the fused FFN, or FC1 and FC2 when it is unfused).  In later calls on this
 * model their pipeline waits give up after
 * `wait_iters` polls (0 = the default limit, about a second), and with
 * skip_tile >= 0 every such launch leaves the A tile of that index unloaded, so
 * the waits on it run out: the launch stops issuing work, waits (with the default
 * limit) for the copies and tensor-core operations it already issued, releases
 * its TMEM and sets the model's device error word to 3, which hv_device_error
 * reports.  Nothing faults and the context stays usable.  skip_tile = -1 with
 * wait_iters = 0 restores normal operation.  Drops the model's captured graphs.
 * No counterpart in the reference (its RTL testbench injects stalls through the
 * behavioural memory model, sim/common/behavioral_memory.sv:13, and reports a
 * watchdog timeout as a fatal error code, rtl/include/heatvit_pkg.sv:109-118). */
HV_API int hv_test_gemm_stall(hv_model *model, unsigned wait_iters, int skip_tile);

/* ---- per-operator entry points (unit configs; device buffers) --------------------- */

/* GEMM + writeback: out = requant(A·B + bias, src_exp, dst_exp, out_bits).
 *   d_a  [m][k] int8 (or uint8 when a_unsigned), row-major
 *   d_b  [k][n] int8 row-major (transpose_b = 0) or [n][k] (transpose_b = 1)
 *   d_bias [n] int32 or NULL
 *   out_bits 8 -> d_out int8 [m][n]; 32 -> d_out int32 [m][n]
 * Replaces gemm.gemm_numpy (gemm.py:93-120) + gemm.gemm_writeback (gemm.py:123-139).
 * Returns HV_ERR_OVERFLOW when a pre-bias accumulator leaves int32 (never for
 * k <= 131071, where |acc| <= k * 2^14 < 2^31). */
HV_API int hv_gemm_i8(const void *d_a, const int8_t *d_b, const int32_t *d_bias,
               int m, int n, int k, int transpose_b, int a_unsigned,
               int src_exp, int dst_exp, int out_bits, void *d_out, void *stream);

/* Raw accumulator: d_acc[m][n] int64 = A·B (+ bias).  Replaces gemm.gemm_numpy
 * (gemm.py:93-120) without the writeback. */
HV_API int hv_gemm_i8_acc(const void *d_a, const int8_t *d_b, const int32_t *d_bias,
                   int m, int n, int k, int transpose_b, int a_unsigned,
                   int64_t *d_acc, void *stream);

/* Allocation-free form of hv_gemm_i8_acc: same arguments, same result, same
 * status codes.  No counterpart in the reference (the golden model is pure
 * Python and never owns device memory); this entry point exists for callers
 * that must not allocate or free device memory while they run, e.g. a process
 * whose device memory is all reserved up front by a caching pool (a raw
 * cudaMalloc can then fail although the pool has room), or a latency-bound
 * caller that cannot afford the device-wide synchronisation cudaFree implies.
 *
 * The padded operands and the device error word live in one fixed per-device
 * array of HV_NOALLOC_SCRATCH_BYTES inside the library.  The call needs
 *   256 + roundup256(m * kp) + np * kp  bytes of it,
 * with kp = max(64, roundup64(k)) and np = roundup64(n) (the GEMM's 64-column
 * tiles); larger problems are rejected with HV_ERR_VALUE and a message naming
 * the limit, before any work is enqueued.
 *
 * The first call on each device resolves the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture starts on the device.  Each call clears the error
 * word on `stream` before use and rewrites every padded byte it reads.  Before
 * it returns, every call copies the error word to a host variable and
 * synchronises `stream` (cudaStreamSynchronize), as hv_gemm_i8_acc does, so
 * that it can report a bounded-wait timeout.
 * The array is shared by all callers on a device: calls that overlap in time
 * (two host threads, or work on another stream still reading the array) race
 * and may return wrong results.  Serialise them. */
#define HV_NOALLOC_SCRATCH_BYTES (8u << 20)
HV_API int hv_gemm_i8_acc_noalloc(const void *d_a, const int8_t *d_b, const int32_t *d_bias,
                   int m, int n, int k, int transpose_b, int a_unsigned,
                   int64_t *d_acc, void *stream);

/* Element-wise writeback requant(v, src_exp, dst_exp, out_bits) of int64 values to
 * int8 (out_bits 8) or int32 (out_bits 24 or 32; 24 saturates to Q8.16 range)
 * (gemm.py:123-139; fixed.py:37-45). */
HV_API int hv_writeback_i64(const int64_t *d_acc, int64_t count, int src_exp, int dst_exp, int out_bits,
                            void *d_out, void *stream);

/* Element-wise residual align-add of two int8 tensors
 * requant((a << (ea-c)) + (b << (eb-c)), c, eo, 8), c = min(ea, eb)
 * (transformer.py:96-101 _align_add_requant). */
HV_API int hv_align_add_i8(const int8_t *d_a, int a_exp, const int8_t *d_b, int b_exp, int out_exp,
                           int64_t count, int8_t *d_out, void *stream);

/* Image quantisation of the P2 accuracy tooling: d_images [batch][3][224][224]
 * float (CHW planes) -> d_out [batch][150528] int8 in the HWC order of the golden
 * image, q = clamp(round_half_even(x / 2^input_exp), -128, 127); NaN gives 0.
 * Replaces the first lines of tools/p2/p2_sim.py forward_image (p2_sim.py:536-541:
 * torch.round, clamp, permute to NHWC). */
HV_API int hv_quantize_images(const float *d_images, int batch, int input_exp, int8_t *d_out, void *stream);

/* Row LayerNorm over D = 192: replaces nonlinear.layernorm (nonlinear.py:136-186).
 *   d_x [rows][192] int8, d_gamma/d_beta [192] int8 -> d_out [rows][192] int8,
 *   d_negvar [rows] uint8 (1 = variance clamped), may be NULL. */
HV_API int hv_layernorm_i8(const int8_t *d_x, const int8_t *d_gamma, const int8_t *d_beta,
                    int rows, int x_scale, int gamma_scale, int beta_scale, int out_scale,
                    int8_t *d_out, uint8_t *d_negvar, void *stream);

/* Softmax over ragged rows: row r covers d_x[d_row_offsets[r] .. d_row_offsets[r+1]).
 * mode 0: attention, UQ0.8 uint8 output (nonlinear.py:130-133);
 * mode 1: selector, Q0.16 int32 output saturated at 65536 (nonlinear.py:124-127).
 * d_x is Q8.16 int32. */
HV_API int hv_softmax_rows(const int32_t *d_x, const int32_t *d_row_offsets, int rows,
                    int mode, void *d_out, void *stream);

/* Elementwise ShiftGELU, Q8.16 in/out: replaces nonlinear.gelu (nonlinear.py:60-80). */
HV_API int hv_shiftgelu(const int32_t *d_x, int64_t count, int32_t *d_out, void *stream);

/* Elementwise PLAN sigmoid: replaces nonlinear.plan_sigmoid (nonlinear.py:83-95). */
HV_API int hv_plan_sigmoid(const int32_t *d_x, int64_t count, int32_t *d_out, void *stream);

/* FFN hidden chain requant(gelu(requant(acc, src, -16, 24)), -16, dst, 8) on int32
 * accumulators (transformer.py:351-358). */
HV_API int hv_gelu_requant(const int32_t *d_acc, int64_t count, int src_exp, int dst_exp,
                    int8_t *d_out, void *stream);

/* One Pre-LN transformer block over a ragged batch of token matrices.
 *   d_x [total][192] int8, image i at rows d_offsets[i] .. d_offsets[i+1]
 *   d_z [total][192] int8 output.  Replaces transformer.transformer_block
 *   (transformer.py:401-431) applied to each image. */
HV_API int hv_transformer_block(hv_model *model, int block_index, const int8_t *d_x,
                         const int32_t *d_offsets, int images, int total_rows,
                         int8_t *d_z, void *stream);

/* Patch embedding: d_images [batch][150528] -> d_tokens [batch][197][192].
 * Replaces transformer.patch_embedding (transformer.py:104-145). */
HV_API int hv_patch_embedding(hv_model *model, const int8_t *d_images, int batch,
                       int8_t *d_tokens, void *stream);

/* Token selector over a ragged batch.
 *   d_x [total][192] int8 with offsets d_offsets[images+1]; d_pkg_in [images] uint8
 *   -> d_y (capacity total rows) packed, new offsets d_offsets_out[images+1],
 *   d_pkg_out [images], d_summary [images] (kept/pruned/warnings).
 * Optional intermediates (NULL to skip), each indexed by image at a 196-candidate
 * stride: d_fused [images][196] int32 Q0.16, d_head_scores [images][3][196] int32,
 * d_head_weights [images][196][3] int32, d_local [images][3][196][32] int8,
 * d_global [images][3][32] int8, d_stats [images][196][3] int8.
 * Replaces selector.token_selector (selector.py:503-563) and the SelectorResult
 * fields it returns (selector.py:235-250). */
HV_API int hv_token_selector(hv_model *model, int selector_index, const int8_t *d_x,
                      const int32_t *d_offsets, const uint8_t *d_pkg_in, int images,
                      int8_t *d_y, int32_t *d_offsets_out, uint8_t *d_pkg_out,
                      hv_selector_summary *d_summary, int32_t *d_fused,
                      int32_t *d_head_scores, int32_t *d_head_weights, int8_t *d_local,
                      int8_t *d_global, int8_t *d_stats, void *stream);

/* Score layer-2 outputs h2 of selector `selector_index` over a ragged batch (rows
 * d_offsets[i]..d_offsets[i+1] of d_x): d_h2 [images][3][196][16] int8, candidate c of
 * head h at [i][h][c]; entries past an image's candidates are left untouched.
 * Replaces weights._selector_h2 (weights.py:143-155), the feature the reference's
 * selector calibration (weights.py:158-204) reads. */
HV_API int hv_selector_h2(hv_model *model, int selector_index, const int8_t *d_x,
                          const int32_t *d_offsets, int images, int8_t *d_h2, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* HEATVIT_B200_H */
