// hv_internal.cuh — launch interfaces shared by the library's .cu files.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "hv_fixed.cuh"
#include "hv_gemm.cuh"
#include "../../include/heatvit_b200.h"

namespace hv {

// LayerNorm constants of one LN layer (nonlinear.py:136-186), host-derived.
struct LnParams {
    const int8_t *gamma, *beta;    // [192]
    int x_scale;                   // in [-32, 0]
    int sh_sum;                    // x_scale + 32           (left shift of Σx)
    int sq_shift;                  // 2*x_scale + 32         (>= 0: left shift of Σx², < 0: per-element rsa)
    int sh_g, sh_b;                // gamma/beta alignment left shifts
    int sh_out;                    // out_scale - common
    int fast;                      // 1: sh_g <= 16 and sh_b <= 40 (int64 output stage)
    int split;                     // 1: x_scale <= -4, so |x_q32 - mean| <= 2^36 (64-bit split product)
    int out32;                     // 1: sh_g == 0, sh_b <= 22, sh_out in [1, 30] (32-bit output stage)
    int one;                       // a runtime 1: multiply-adds by it stay on the FMA pipe
};

LnParams make_ln(const int8_t *gamma, const int8_t *beta, int x_scale, int gamma_scale, int beta_scale,
                 int out_scale);

// LN over rows [0, rows) of x (row stride 192) -> out.  rows is *rows_dev when
// non-null.  Negative-variance rows set *negvar_row (per row, may be null) and
// OR bit 2 into warn[image] where image is found from offsets (may be null).
cudaError_t launch_layernorm(const int8_t *x, int8_t *out, int rows_max, const int32_t *rows_dev,
                             const LnParams &p, uint8_t *negvar_row, const int32_t *offsets,
                             int images, uint8_t *warn, cudaStream_t st);

// LN of each image's first row (the CLS token): row offsets[i] -> out[i].
cudaError_t launch_layernorm_cls(const int8_t *x, const int32_t *offsets, int images, int8_t *out,
                                 const LnParams &p, uint8_t *warn, cudaStream_t st);

// Attention for every (image, head) of a ragged batch: qkv [T][576] -> ctx [T][192].
struct AttnParams {
    int score_shift;   // score_scale - 2*qkv_out           (int32 score writeback)
    int q16_shift;     // -(score_scale + 13)               (Q8.16 conversion, sat 24)
    int ctx_shift;     // context_out - (prob_scale + qkv_out)
    // fast = 1 when score_shift = -k (0 <= k <= 10) and q16_shift >= k: |Q.K| <= 2^20,
    // so acc << k fits int32 and q16 = rsa(acc, q16_shift - k) never saturates.
    int fast, fast_shift, fast_half, fast_negmask;
    int ctx_fast;      // ctx_shift in [1, 30]: |P.V| < 2^23, 32-bit rounding shift is exact
};
AttnParams make_attn(int qkv_out_scale, int score_scale, int prob_scale, int context_out_scale);
// err: device word set to a non-zero code when a bounded wait gave up.
// may_be_short: some image may hold at most 128 tokens (any selector has run, or
// the caller's ragged batch is arbitrary); those go to a smaller CTA shape.
// Exact lookup table of the FFN GELU chain over its reachable Q8.16 inputs
// [-qmax, qmax]: the window [wlo, wlo + wn) outside which the int8 output is
// constant (gelu_table_window; synchronises `st`), then the table itself,
// tab[i] = requant(shift_gelu(wlo + i), -16, dst, 8) (launch_gelu_table_fill).
// d_mm: two device ints of scratch.
cudaError_t gelu_table_window(int32_t qmax, int sh_out, int *d_mm, int32_t *wlo, int32_t *wn, cudaStream_t st);
cudaError_t launch_gelu_table_fill(int8_t *tab, int32_t wlo, int32_t wn, int sh_out, cudaStream_t st);

// Work-unit lists of the attention kernel for one token layout (attn_plan_kernel in
// hv_attention.cu): list_a [3 * images] (images of at most 128 tokens), list_b
// [6 * images] (longer images), cnt [2] their lengths.  An entry is {unit code, the
// image's first row << 8 | its token count}.  Rebuilt whenever the offsets change
// (batch set-up, every selector).
struct AttnPlan {
    uint2 *list_a, *list_b;
    int32_t *cnt;
};
cudaError_t launch_attn_plan(const int32_t *offsets, int images, const AttnPlan &plan, cudaStream_t st);
cudaError_t launch_attention(const int8_t *qkv, const int32_t *offsets, int images, int8_t *ctx,
                             const AttnParams &p, int may_be_short, int sms, int *err, const AttnPlan &plan,
                             cudaStream_t st);

// The fused FFN (hv_ffn.cu): A = LN2 output [rows][192] (tensor map, 16 x 128
// boxes), W1 = the K-major FC1 weights [768][192] (16 x 128 boxes), W2 = the
// K-major FC2 weights [192][768] (16 x 192 boxes).  e1: FC1 bias and GELU chain
// (fast: the persistent kernel's fast forms, gelu_chain_fast2 or the tables); e2:
// FC2 bias, writeback shift and residual 2 (res = the block's y, add).  out
// [rows][192] must not alias A or the residual.
struct FfnArgs {
    int m_host;
    const int32_t *m_dev;
    EpiParams e1, e2;
    int8_t *out;
    // FC1 / FC2 weights in the kernel's shared-memory chunk layout: six 24,576-byte
    // chunks each (w1img[j][kc 12][row 128][16 B], w2img[j][kc 8][row 192][16 B])
    const int8_t *w1img, *w2img;
    uint32_t wait_iters;  // test hooks, as in GemmArgs
    int skip_tile;
};
cudaError_t launch_ffn(const FfnArgs &f, const CUtensorMap &tmA, int m_max, int *err, int sms, cudaStream_t st);

// Device-resident selector weights and constants.
// Exact output table of one GELU chain over the Q8.16 inputs q = rsa(v, sh_in) its
// layer can reach; outside [lo, lo + n) the output is constant (clamped index):
//   mode 1: out = tab[u], u = clamp(q - lo, 0, n - 1);
//   mode 2: buckets of 2^k inputs: e = ((uint32 *)tab)[u >> k], p = e >> 16;
//           p == 0xFFFF: out = tab[fine + (e & 0xFFFF) * 2^k + (u mod 2^k)],
//           else out = (int8)(u mod 2^k >= p ? e >> 8 : e).
// mode 0: no table.  bytes: the staged size (a multiple of 16).
struct GeluTab {
    const int8_t *tab;
    int mode, lo, n, k, fine, bytes, sh_in;
};

// Shared-memory budgets of the selector GELU tables (selector_kernel layout).
constexpr int kSelTabLocalBytes = 14080;
constexpr int kSelTabH1Bytes = 18432;
constexpr int kSelTabH2Bytes = 19392;

struct SelParams {
    const int8_t *local_wt;   // [3][32][64]  (transposed local_w)
    const int32_t *local_b;   // [3][32]
    const int8_t *w1t;        // [3][32][64]  (transposed score_w1: [h][j][k], k = 0..63)
    const int32_t *b1;        // [3][32]
    const int8_t *w2t;        // [3][16][32]
    const int32_t *b2;        // [3][16]
    const int8_t *w3t;        // [3][2][16]
    const int32_t *b3;        // [3][2]
    const int8_t *hw1;        // [3][3]  (golden [i][j])
    const int32_t *hb1;       // [3]
    const int8_t *hw2;        // [3][3]
    const int32_t *hb2;       // [3]
    int local_sh_in, local_sh_out;    // GELU chain of the local MLP
    int h1_sh_in, h1_sh_out;          // score layer 1
    int h2_sh_in, h2_sh_out;          // score layer 2
    int logit_shift;                  // logits writeback (h2 + w3 -> logits)
    int logit_q16_shift;              // logits -> Q16 (24 bit)
    int hw_sh_in, hw_sh_out;          // head-weight hidden GELU chain
    int hw_q16_shift;                 // head-weight acc -> Q16 (24 bit)
    // 1 when gelu_chain_fast's ranges hold for that layer (host-checked)
    int local_fast, h1_fast, h2_fast, hw_fast;
    // 1 when gelu_chain_fast2's ranges hold (host-checked), and its constants
    int local_k2, h1_k2, h2_k2, hw_k2;
    GeluK local_k, h1_k, h2_k, hw_k;
    // exact tables of the local, score layer-1 and layer-2 chains (mode 0: none)
    GeluTab tab_local, tab_h1, tab_h2;
    int *err;                 // device error word: 3 when a bounded wait gave up
};

// Optional selector intermediates (token_selector API), image stride 196.
struct SelDebug {
    int32_t *fused;         // [B][196]
    int32_t *head_scores;   // [B][3][196]
    int32_t *head_weights;  // [B][196][3]
    int8_t *local;          // [B][3][196][32]
    int8_t *global_;        // [B][3][32]
    int8_t *stats;          // [B][196][3]
    int8_t *h2;             // [B][3][196][16] score layer-2 outputs
};

// Selector over a ragged batch: x rows offsets[i]..offsets[i+1], pkg_in[i] ->
// stage[i][0..n') (stride 197 rows), counts_out[i] = n', pkg_out[i],
// summary[i*sum_stride], warn[i] |= bits, token_counts[i*tc_stride + tc_col] = n'.
// warn is a uint8 array whose allocation is padded to a multiple of 4 bytes.
cudaError_t launch_selector(const int8_t *x, const int32_t *offsets, const uint8_t *pkg_in, int images,
                            const SelParams &p, int8_t *stage, int32_t *counts_out, uint8_t *pkg_out,
                            hv_selector_summary *summary, int sum_stride, uint8_t *warn, int32_t *token_counts,
                            int tc_stride, int tc_col, const SelDebug *dbg, cudaStream_t st);

// Pack stage[i] (count counts[i], stride 197 rows) into x at prefix-summed
// offsets; writes offsets_out[0..images] and, when plan is non-null, the attention
// unit lists of the packed layout (so no attn_plan_kernel launch follows).
cudaError_t launch_pack(const int8_t *stage, const int32_t *counts, int images, int8_t *x,
                        int32_t *offsets_out, const AttnPlan *plan, cudaStream_t st);

// Element-wise units (unit API).
cudaError_t launch_gelu(const int32_t *x, int64_t n, int32_t *out, cudaStream_t st);
cudaError_t launch_plan(const int32_t *x, int64_t n, int32_t *out, cudaStream_t st);
cudaError_t launch_gelu_requant(const int32_t *acc, int64_t n, int sh_in, int sh_out, int8_t *out,
                                cudaStream_t st);
cudaError_t launch_softmax_rows(const int32_t *x, const int32_t *offsets, int rows, int mode, void *out,
                                cudaStream_t st);
cudaError_t launch_quantize_images(const float *src, int batch, int input_exp, int8_t *dst, cudaStream_t st);
cudaError_t launch_align_add(const int8_t *a, const int8_t *b, AlignAdd k, int64_t n, int8_t *out, cudaStream_t st);
cudaError_t launch_writeback(const int64_t *acc, int64_t n, int shift, int bits, void *out, cudaStream_t st);

}  // namespace hv
