// hv_gemm.cuh — int8 GEMM with fused integer epilogues.
//
// C[M][N] = A[M][K] · Bt[N][K]ᵀ (+ bias), int32 accumulation on tcgen05 tensor
// cores (accumulator in TMEM), then one of the
// golden writebacks (gemm.py:123-139) fused with what follows it in the model:
//   EPI_I8       requant to int8                          (QKV, generic)
//   EPI_I8_RES   requant to int8, then residual align-add  (proj + residual 1,
//                FC2 + residual 2; transformer.py:415-425, 373-381)
//   EPI_GELU     requant to Q16/24 bit, ShiftGELU, requant to int8 (FC1;
//                transformer.py:351-356)
//   EPI_PATCH    requant to int8, align-add the positional row, write into the
//                197-row token layout (transformer.py:125-145)
//   EPI_I32      requant to int32 (head logits, model.py:109-115; unit API)
//   EPI_ACC64    raw int64 accumulator + bias (unit API, gemm_numpy)
//
// Weights are stored K-major (Bt[n][k], the transpose of the golden w[k][n]).
// A may be int8 or uint8 (P·V in attention uses uint8 probabilities;
// gemm.py:81-84).  The pre-bias accumulator fits int32 for K <= 131071.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include "hv_fixed.cuh"
#include "hv_launch.cuh"

namespace hv {

enum Epi { EPI_I8 = 0, EPI_I8_RES = 1, EPI_GELU = 2, EPI_PATCH = 3, EPI_I32 = 4, EPI_ACC64 = 5 };

// Largest exact GELU-chain output table (bytes) an FC1 launch keeps in shared memory.
constexpr int kGeluTableMax = 22528;

// Per-launch epilogue constants (all derived on the host from the golden
// scale exponents).
struct EpiParams {
    const int32_t *bias;      // [N] or nullptr
    int shift;                // requant shift dst - src for the first writeback
    int bits_wide;            // 1: acc + bias may leave 30 bits (64-bit arithmetic needed)
    int fast;                 // 1: the 32-bit epilogue forms are exact (see gemm_epi_fast)
    // residual (EPI_I8_RES): out = align_add(res @ e_res, y @ e_y -> e_out)
    const int8_t *res;        // [M][N]
    AlignAdd add;             // a = residual value, b = requantised GEMM value
    // GELU chain (EPI_GELU): sh_in = -16 - src, sh_out = dst + 16
    int gelu_sh_in, gelu_sh_out;
    int gelu_fast;            // host-checked ranges of gelu_chain_fast hold
    int gelu_k2;              // host-checked ranges of gelu_chain_fast2 hold (persistent kernel)
    GeluK gk;                 // constants of gelu_chain_fast2 (also the input shift of the table form)
    // exact output tables of the GELU chain (persistent kernel), q = rsa(acc + bias, sh_in),
    // u = clamp(q - gtab_lo, 0, gtab_n - 1):
    //  gtab_mode 1: out = gtab[u], exact for q in [gtab_elo, gtab_ehi); a warp whose 32
    //    values include one outside that range evaluates them with gelu_chain_fast2
    //    instead (gelu_k2 must then hold);
    //  gtab_mode 2 (buckets of 2^gtab_k inputs): e = coarse[u >> k] (uint32 at gtab),
    //    p = e >> 16; p == 0xFFFF: out = fine[(e & 0xFFFF) * 2^k + (u & (2^k - 1))]
    //    (bytes at gtab + gtab_fine), else out = (int8)(u & (2^k - 1) >= p ? e >> 8 : e)
    //  gtab_mode 3 (the table covers the whole window, so it is exact everywhere):
    //    out = gtab[clamp((x + gtab_c + sgn(x)) >> sh_in, 0, gtab_n - 1)], x = acc + bias,
    //    gtab_c = 2^(sh_in - 1) - gtab_lo * 2^sh_in, sgn(x) = -1 for x < 0 else 0: the
    //    rounding shift and the offset by gtab_lo in one add (the host checks that
    //    |x| + |gtab_c| + 1 stays below 2^31)
    const int8_t *gtab;
    int gtab_lo, gtab_n;      // gtab_n = input span; 0 = no table
    int gtab_elo, gtab_ehi;
    int gtab_mode, gtab_k, gtab_fine;
    int gtab_c;
    int gtab_bytes;           // bytes to stage in shared memory, at most kGeluTableMax
    // patch (EPI_PATCH): pos [197][192], add = (a = embed, b = pos)
    const int8_t *pos;
};

// Where A comes from.
struct ASrc {
    const void *ptr;          // row-major [M][lda] int8/uint8, or NHWC images
    int lda;
    int patch_mode;           // 1: A row r = patch (r % 196) of image r / 196
};

struct GemmArgs {
    ASrc a;
    // TMA descriptor of A (row-major int8 [rows][k]) for the persistent kernel, or
    // nullptr for cp.async loads (the patch GEMM gathers A from images)
    const CUtensorMap *tma;
    const int8_t *bt;         // [Npad][K] K-major weights (Npad: see launch_gemm)
    int n, k;                 // logical N (stores guarded), K multiple of 64
    int m_host;               // row count when m_dev == nullptr
    const int32_t *m_dev;     // device row count (ragged batches), or nullptr
    void *out;                // int8 / int32 / int64 [M][ldo]
    int ldo;
    EpiParams epi;
    // Test hooks of the persistent kernel (zero-initialised = off): the pipeline's
    // bounded waits give up after wait_iters polls (0 = the default limit), and with
    // skip_tile > 0 the A tile of index skip_tile - 1 is never loaded, so the waits
    // on it run out and the launch takes its abort path (error word 3).
    uint32_t wait_iters;
    int skip_tile;
};

// Launch helpers (defined in hv_gemm.cu).  `bt` must hold
// ceil(n / gemm_tile_n(n)) * gemm_tile_n(n) rows; k must be a multiple of 64.
// err: device word set non-zero when a bounded wait gave up.
int gemm_tile_n(int n);

// Whether the 32-bit epilogue forms are exact for these constants: acc + bias
// fits 30 bits, the first writeback shifts right by 1..30, and the align-add
// (EPI_I8_RES / EPI_PATCH) or GELU chain (EPI_GELU) fast conditions hold.
inline int gemm_epi_fast(int epi, const EpiParams &e) {
    if (e.bits_wide) return 0;
    if (epi == EPI_GELU) return e.gelu_fast;
    const int wb_ok = e.shift >= 1 && e.shift <= 30;
    if (epi == EPI_I8_RES || epi == EPI_PATCH) return wb_ok && e.add.fast;
    if (epi == EPI_I8) return wb_ok;
    return 0;
}
cudaError_t launch_gemm(const GemmArgs &g, int epi, int a_unsigned, int m_max, int *err, cudaStream_t st);

// Persistent, warp-specialised form for the model's layer shapes (signed A,
// K in {192, 768}, N in {192, 576, 768}, int8 epilogues; hv_gemm_persistent.cu).
// The weights stay resident in shared memory; `bt` needs exactly n rows.
// `sms` is the device's SM count (one CTA per SM).
bool gemm_persistent_supported(int epi, int n, int k);
// Tensor map of a row-major int8 A operand [rows][k] (k a multiple of 16) read as
// 16-byte x 128-row boxes; rows past `rows` read as zero.  Returns 0 on success.
int make_tmap_a(CUtensorMap *map, const void *base, int k, int rows);
// The same with boxes of 16 bytes x box_rows rows (box_rows <= 256).
int make_tmap_box(CUtensorMap *map, const void *base, int k, int rows, int box_rows);
// Tensor map of NHWC images [images_n][224][224][3] for the patch GEMM's TMA
// gather: 5-D boxes of one 16-byte K strip for 7 x 14 patches.  Returns 0 on
// success, non-zero when the driver entry point is missing or `images` is not
// 16-byte aligned (the caller then keeps the cp.async gather).
int make_tmap_patch(CUtensorMap *map, const void *images, int images_n);
cudaError_t launch_gemm_persistent(const GemmArgs &g, int epi, int m_max, int *err, int sms, cudaStream_t st);

}  // namespace hv
