// hv_gemm_persistent.cu — persistent, warp-specialised tcgen05 GEMM for the
// model's five layer shapes (patch, QKV, proj, FC1, FC2).
//
// One CTA per SM loops over 128-row tiles of A.  The whole weight matrix
// (N x K int8, at most 147 KB) stays resident in shared memory for the CTA's
// lifetime, so A (read once) and the output (written once) are the only DRAM
// traffic.  Roles:
//   warps 0-3   producer.  With a tensor map, one thread issues TMA copies of A
//               into a ring of S stages, completing on the stage's `full`
//               mbarrier (expect_tx): one 2-D box of 16 bytes x 128 rows per K
//               strip for row-major A, or one 5-D box of 14 x 7 patches per K
//               strip for the patch GEMM (two 98-row tiles per image).  Without
//               one, the 128 threads gather A with cp.async in the no-swizzle
//               K-major canonical layout and arrive with
//               cp.async.mbarrier.arrive.noinc.
//   warp 4      MMA issuer (one thread): tcgen05.mma kind::i8 into one of two
//               TMEM accumulators (192 columns each, 256 apart); commits free
//               the A stage (`empty`) and hand the accumulator to the epilogue
//               (`acc_full`).
//   warps 5-12  epilogue: thread = (TMEM lane, column half); reads its
//               accumulator row with tcgen05.ld, applies the fused golden
//               writeback, stores 32 contiguous bytes per step, then releases
//               the accumulator (`acc_empty`).
// For K = 192 one stage holds the whole A tile and feeds every 192-column
// chunk of N; for K = 768 (N = 192) A streams through 8 stages of 64 columns.
// Every mbarrier wait is bounded; a timeout sets the model's error word.
#include <cudaTypedefs.h>
#include <string.h>

#include "hv_epi.cuh"
#include "hv_gemm.cuh"
#include "hv_tc05.cuh"

namespace hv {

namespace {

using namespace pg;

constexpr int PT_PROD = 4;                       // producer warps
constexpr int PT_MMA_WARP = PT_PROD;
constexpr int PT_EPI0 = PT_PROD + 1;             // first epilogue warp
constexpr int PT_THREADS = (PT_PROD + 1 + 8) * 32;
constexpr int BN = 192;
constexpr uint32_t PT_TMEM_COLS = 512;
constexpr uint32_t PT_WAIT = 1u << 24;

template <int KDIM, int N, bool RES = false>
struct PLayout {
    static constexpr int NCH = N / BN;                 // n-chunks per tile
    static constexpr int AK = KDIM == 192 ? 192 : 64;  // A stage width (bytes of K)
    static constexpr int KST = KDIM / AK;              // A stages per tile
    // ring depth; FC1 (N = 768) keeps two stages to leave room for its GELU table
    static constexpr int S = KDIM == 192 ? (N == 768 ? 2 : 3) : 8;
    static constexpr int TABB = N == 768 ? kGeluTableMax : 0;  // exact GELU-chain table (EPI_GELU)
    static constexpr int A_STAGE = 128 * AK;
    // residual rows staged beside each A stage (set by the kernel for EPI_I8_RES, K = 192)
    static constexpr int R_STAGE = 128 * N;
    // An A stage is released after its tile's last n-chunk, or after its own k-step.
    static_assert(KST == 1 || NCH == 1, "streamed K with several n-chunks is not pipelined");
    static constexpr int OFF_B = 0;
    static constexpr int OFF_A = OFF_B + N * KDIM;
    static constexpr int OFF_BIAS = OFF_A + S * A_STAGE;
    static constexpr int OFF_TAB = OFF_BIAS + N * 4;
    static constexpr int OFF_R = OFF_TAB + TABB;
    static constexpr int OFF_BAR = OFF_R + (RES ? S * R_STAGE : 0);
    static constexpr int NBAR = 3 * S + 5;
    static constexpr int USED = OFF_BAR + NBAR * 8 + 16;
    // At least 116 KB so that two CTAs never share an SM: each takes all 512 TMEM columns.
    static constexpr int SMEM = USED > 116 * 1024 ? USED : 116 * 1024;
};

// Residual rows through shared memory: the proj GEMM (one 192-column chunk, K = 192)
// with a tensor-mapped A.  The producer copies a tile's 128 residual rows (contiguous,
// 24 KB) with one bulk copy into the stage beside its A, completing on the same
// `full` barrier, so they are on chip long before the epilogue needs them; the
// epilogue warps release them (`rempty`).
template <int EPI, int KDIM, int N>
constexpr bool kResStaged = EPI == EPI_I8_RES && KDIM == 192 && N == 192;

template <int EPI, bool FAST, int KDIM, int N>
__global__ void __launch_bounds__(PT_THREADS, 1) tcp_gemm_kernel(GemmArgs g, int *err,
                                                                  const __grid_constant__ CUtensorMap tmA, int use_tma) {
    constexpr bool RS = kResStaged<EPI, KDIM, N>;
    using L = PLayout<KDIM, N, RS>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sB = smem + L::OFF_B;
    uint8_t *sA = smem + L::OFF_A;
    int32_t *sbias = (int32_t *)(smem + L::OFF_BIAS);
    uint64_t *full = (uint64_t *)(smem + L::OFF_BAR);
    uint64_t *empty = full + L::S;
    uint64_t *accf = empty + L::S;
    uint64_t *acce = accf + 2;
    uint64_t *drain = acce + 2;
    uint64_t *rempty = drain + 1;  // [S]: the epilogue has read the stage's residual rows
    const uint8_t *sR = smem + L::OFF_R;
    uint32_t *tslot = (uint32_t *)(rempty + L::S);
    volatile int *abortf = (volatile int *)(tslot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // ---- prologue: resident weights and bias, barriers, TMEM ---------------------
    if (warp == 0) {
        tc05::tmem_alloc(tslot, PT_TMEM_COLS);
        tc05::tmem_relinquish();
    }
    if (tid == 0) {
        for (int s = 0; s < L::S; ++s) {
            tc05::mbar_init(&full[s], use_tma ? 1 : 32 * PT_PROD);
            tc05::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc05::mbar_init(&accf[b], 1);
            tc05::mbar_init(&acce[b], 8);
        }
        tc05::mbar_init(drain, 1);
        for (int s = 0; s < L::S; ++s) tc05::mbar_init(&rempty[s], 8);
        *abortf = 0;
        tc05::fence_mbar_init();
    }
    // B [N][KDIM] in canonical K-major layout: chunk c -> (row group, k chunk, row)
    constexpr int KC = KDIM / 16;
    for (int c = tid; c < N * KC; c += PT_THREADS) {
        const int grp = c / (8 * KC), rem = c - grp * 8 * KC;
        const int kc = rem >> 3, r8 = rem & 7;
        const int row = grp * 8 + r8;
        cp_async16(tc05::smem_u32(sB + grp * (8 * KDIM) + kc * 128 + r8 * 16), g.bt + (size_t)row * KDIM + kc * 16,
                   16);
    }
    for (int i = tid; i < N; i += PT_THREADS) sbias[i] = g.epi.bias ? g.epi.bias[i] : 0;
    int8_t *stab = (int8_t *)(smem + L::OFF_TAB);
    if (EPI == EPI_GELU && L::TABB > 0)  // the table allocation is padded to 16 bytes
        for (int i = tid; i < (g.epi.gtab_bytes + 15) / 16; i += PT_THREADS)
            ((uint4 *)stab)[i] = ((const uint4 *)g.epi.gtab)[i];
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    // Everything above touches only weights and on-chip state; from here on the
    // kernel reads activations and row counts that the previous kernel writes.
    griddep_wait();
    griddep_launch();
    const int m_lim = g.m_dev ? *g.m_dev : g.m_host;
    // Patch GEMM with TMA: tile mt holds image mt / 2's patch rows 7 * (mt & 1) ..
    // + 6, i.e. 98 A rows (TMEM lanes 98..127 hold unused rows).
    const bool ptma = EPI == EPI_PATCH && use_tma;
    const int mtiles = ptma ? 2 * (m_lim / 196) : (m_lim + 127) / 128;
    // Work units are (tile, 192-column chunk) pairs, unit u = mt * NCH + c.  Each CTA
    // takes one contiguous range of equal size (within one unit), so a tile's chunks
    // mostly stay in one CTA and share its A stage, and no CTA runs more than one
    // chunk past the others.
    const int units = mtiles * L::NCH;
    const int u_begin = (int)(((long long)blockIdx.x * units) / gridDim.x);
    const int u_end = (int)(((long long)(blockIdx.x + 1) * units) / gridDim.x);
    tc05::fence_proxy_async();
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tslot;
    const uint8_t *abase = (const uint8_t *)g.a.ptr;
    // residual rows staged in shared memory (contiguous 16-byte-aligned rows needed)
    const bool rs_on = RS && use_tma && g.ldo == N && (((uintptr_t)g.epi.res) & 15) == 0;
    const uint32_t wl = g.wait_iters ? g.wait_iters : PT_WAIT;  // pipeline waits; drains use PT_WAIT

    if (warp < PT_PROD && use_tma) {
        // ---- producer (TMA): one thread; stage = AK/16 boxes of [128 rows][16 bytes],
        // strip kc at byte offset kc * 2048 (core matrices: LBO 2048, SBO 128)
        if (tid == 0) {
            uint32_t q = 0;
            bool ok = true;
            // last ring slot whose copies were issued into each stage (-1: none)
            int last_q[L::S];
#pragma unroll
            for (int s = 0; s < L::S; ++s) last_q[s] = -1;
            for (int u = u_begin; u < u_end && ok && !*abortf; ++u) {
                const int mt = u / L::NCH;
                if (u != u_begin && u - mt * L::NCH != 0) continue;  // the tile's A is staged already
                for (int ks = 0; ks < L::KST; ++ks, ++q) {
                    const int s = q % L::S;
                    if (q >= (uint32_t)L::S && !tc05::mbar_wait(&empty[s], ((q / L::S) - 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    const bool rs = rs_on;
                    if (rs && q >= (uint32_t)L::S && !tc05::mbar_wait(&rempty[s], ((q / L::S) - 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    if (mt == g.skip_tile - 1) continue;  // test hook: this tile never arrives
                    last_q[s] = (int)q;
                    const uint32_t dst = tc05::smem_u32(sA + s * L::A_STAGE);
                    const uint32_t rbytes = rs ? (uint32_t)min(128, m_lim - mt * 128) * (uint32_t)g.ldo : 0u;
                    mbar_expect_tx(&full[s], (ptma ? 98u : 128u) * L::AK + rbytes);
                    if (rs)
                        bulk_load(tc05::smem_u32(sR + s * L::R_STAGE), g.epi.res + (size_t)mt * 128 * g.ldo, rbytes,
                                  &full[s]);
#pragma unroll
                    for (int kc = 0; kc < L::AK / 16; ++kc) {
                        if (ptma) {
                            // K byte k = ir * 48 + w (layout.py:31-72): strip kg = k / 16
                            const int kg = ks * (L::AK / 16) + kc, ir = kg / 3;
                            tma_load_patch(dst + kc * 2048, &tmA, (kg - 3 * ir) * 16, ir, 7 * (mt & 1), mt >> 1,
                                           &full[s]);
                        } else {
                            tma_load_a(dst + kc * 2048, &tmA, ks * L::AK + kc * 16, mt * 128, &full[s]);
                        }
                    }
                }
            }
            if (!ok) *abortf = 1;
            // After an abort the consumer may have stopped before some stages: wait
            // (bounded) until every box issued into them has landed, so no bulk copy
            // still writes this CTA's shared memory when it exits.
            if (*abortf) {
#pragma unroll
                for (int s = 0; s < L::S; ++s)
                    if (last_q[s] >= 0) tc05::mbar_wait(&full[s], ((uint32_t)last_q[s] / L::S) & 1u, PT_WAIT);
            }
        }
    } else if (warp < PT_PROD) {
        // ---- producer ------------------------------------------------------------
        uint32_t q = 0;
        for (int u = u_begin; u < u_end && !*abortf; ++u) {
            const int mt = u / L::NCH;
            if (u != u_begin && u - mt * L::NCH != 0) continue;  // the tile's A is staged already
            const int m0 = mt * 128;
            for (int ks = 0; ks < L::KST; ++ks, ++q) {
                const int s = q % L::S;
                if (q >= (uint32_t)L::S && !tc05::mbar_wait(&empty[s], ((q / L::S) - 1) & 1u, wl)) {
                    *abortf = 1;
                    break;
                }
                if (mt == g.skip_tile - 1) continue;  // test hook: this tile never arrives
                uint8_t *dst = sA + s * L::A_STAGE;
                constexpr int AKC = L::AK / 16;
                for (int c = tid; c < 128 * AKC; c += 32 * PT_PROD) {
                    const int grp = c / (8 * AKC), rem = c - grp * 8 * AKC;
                    const int kc = rem >> 3, r8 = rem & 7;
                    const int row = grp * 8 + r8, grow = m0 + row;
                    const uint8_t *src = abase;
                    int bytes = 0;
                    if (grow < m_lim) {
                        bytes = 16;
                        const int k = ks * L::AK + kc * 16;
                        if (g.a.patch_mode) {
                            // layout.py:31-72 patch order; a 16-byte chunk stays inside one image row
                            const int img = grow / 196, p = grow - img * 196;
                            const int pr = p / 14, pc = p - pr * 14;
                            const int ir = k / 48, w = k - ir * 48;
                            src = abase + (size_t)img * 150528 + ((pr * 16 + ir) * 224 + pc * 16) * 3 + w;
                        } else {
                            src = abase + (size_t)grow * g.a.lda + k;
                        }
                    }
                    cp_async16(tc05::smem_u32(dst + grp * (8 * L::AK) + kc * 128 + r8 * 16), src, bytes);
                }
                cp_arrive_noinc(&full[s]);
            }
        }
    } else if (warp == PT_MMA_WARP) {
        // ---- MMA issuer -------------------------------------------------------------
        if (lane == 0) {
            const uint32_t idesc = tc05::idesc_i8(128, BN, true, true);
            uint32_t q = 0, a = 0;
            bool ok = true;
            for (int u = u_begin; u < u_end && ok && !*abortf; ++u, ++a) {
                const int mt = u / L::NCH, c = u - mt * L::NCH;
                const bool first = u == u_begin || c == 0;           // the tile's stage arrives now
                const bool last = u == u_end - 1 || c == L::NCH - 1;  // and is released after this unit
                {
                    const int tb = a & 1;
                    if (a >= 2 && !tc05::mbar_wait(&acce[tb], ((a >> 1) - 1) & 1u, wl)) { ok = false; break; }
                    tc05::fence_after();
                    const uint32_t d = tbase + tb * 256;
                    for (int ks = 0; ks < L::KST; ++ks) {
                        const uint32_t qq = q + ks;
                        const int s = qq % L::S;
                        if (first || L::KST > 1) {
                            if (!tc05::mbar_wait(&full[s], (qq / L::S) & 1u, wl)) { ok = false; break; }
                            tc05::fence_proxy_async();
                            tc05::fence_after();
                        }
                        const uint32_t a0 = tc05::smem_u32(sA + s * L::A_STAGE);
                        const uint32_t b0 = tc05::smem_u32(sB) + c * BN * KDIM + ks * (L::AK / 16) * 128;
                        // A: TMA strips (LBO 2048, SBO 128) or the cp.async canonical tile
                        const uint32_t a_step = use_tma ? 4096u : 256u, a_lbo = use_tma ? 2048u : 128u,
                                       a_sbo = use_tma ? 128u : 8u * L::AK;
#pragma unroll
                        for (int j = 0; j < L::AK / 32; ++j)
                            tc05::mma_i8_ss(d, tc05::smem_desc(a0 + j * a_step, a_lbo, a_sbo),
                                            tc05::smem_desc(b0 + j * 256, 128, 8 * KDIM), idesc, (ks | j) != 0);
                        if (L::KST > 1) tc05::commit(&empty[s]);
                    }
                    if (!ok) break;
                    if (L::KST == 1 && last) tc05::commit(&empty[q % L::S]);
                    tc05::commit(&accf[tb]);
                }
                if (last) q += L::KST;
            }
            if (!ok) *abortf = 1;
            // Every MMA this thread issued has completed once `drain` flips.
            tc05::commit(drain);
            if (!tc05::mbar_wait(drain, 0, PT_WAIT)) *abortf = 1;
        }
    } else {
        // ---- epilogue (8 warps) ---------------------------------------------------------
        const int quad = warp & 3, half = (warp - PT_EPI0) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
        uint32_t a = 0;
        for (int u = u_begin; u < u_end; ++u) {
            const int mt = u / L::NCH, c = u - mt * L::NCH;
            const int grow = mt * 128 + row;
            const bool valid = ptma ? row < 98 : grow < m_lim;
            size_t orow = (size_t)grow;
            int pidx = 0;
            if (EPI == EPI_PATCH) {
                const int img = ptma ? mt >> 1 : (valid ? grow / 196 : 0);
                pidx = !valid ? 0 : (ptma ? 98 * (mt & 1) + row : grow - img * 196);
                orow = (size_t)img * 197 + 1 + pidx;
            }
            bool stop = false;
            // Residual or positional rows (N = 192: one chunk per tile): this thread's
            // 96 bytes are requested before the accumulator wait, so their latency
            // overlaps the MMA.
            constexpr bool PRE = (EPI == EPI_I8_RES || EPI == EPI_PATCH) && L::NCH == 1;
            uint32_t rpre[BN / 64][8];
            if (PRE && !rs_on) {
                const int8_t *src = EPI == EPI_PATCH ? g.epi.pos + (pidx + 1) * 192 : g.epi.res + orow * g.ldo;
#pragma unroll
                for (int i = 0; i < BN / 64; ++i) {
                    if (valid) ld_global_32B(src + half * (BN / 2) + 32 * i, rpre[i]);
                    else
#pragma unroll
                        for (int j = 0; j < 8; ++j) rpre[i][j] = 0;
                }
            }
            {
                const int tb = a & 1;
                const int rsl = RS ? (int)(a % L::S) : 0;  // stage of this tile's residual rows
                if (!tc05::mbar_wait(&accf[tb], (a >> 1) & 1u, wl) ||
                    (rs_on && !tc05::mbar_wait(&full[rsl], (a / L::S) & 1u, wl))) {
                    *abortf = 1;
                    stop = true;
                    break;
                }
                tc05::fence_after();
                // unrolled for the prefetching epilogues only (their prefetched registers
                // need compile-time indices); the others stay rolled to keep registers low
#pragma unroll (PRE ? BN / 64 : 1)
                for (int cc = 0; cc < BN / 64; ++cc) {
                    const int col0 = half * (BN / 2) + cc * 32;  // chunk-local column of v[0]
                    const int gcol0 = c * BN + col0;
                    // residual / positional bytes first, so their latency overlaps the TMEM read
                    uint32_t aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    if (RS && rs_on) {
                        const uint8_t *rr = sR + rsl * L::R_STAGE + row * N + gcol0;
                        const uint4 ra = *(const uint4 *)rr, rb = *(const uint4 *)(rr + 16);
                        aux[0] = ra.x; aux[1] = ra.y; aux[2] = ra.z; aux[3] = ra.w;
                        aux[4] = rb.x; aux[5] = rb.y; aux[6] = rb.z; aux[7] = rb.w;
                    } else if (PRE) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) aux[j] = rpre[cc][j];
                    } else if (EPI == EPI_I8_RES && valid) {
                        ld_global_32B(g.epi.res + orow * g.ldo + gcol0, aux);
                    } else if (EPI == EPI_PATCH) {
                        ld_global_32B(g.epi.pos + (pidx + 1) * 192 + gcol0, aux);
                    }
                    uint32_t v[32];
                    tc05::ld32(lane_addr + tb * 256 + col0, v);
                    int32_t bv[32];
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        const int4 b4 = *(const int4 *)(sbias + gcol0 + 4 * q4);
                        bv[4 * q4] = b4.x;
                        bv[4 * q4 + 1] = b4.y;
                        bv[4 * q4 + 2] = b4.z;
                        bv[4 * q4 + 3] = b4.w;
                    }
                    tc05::wait_ld();
                    uint32_t pk[8];
                    epi_piece32<EPI, FAST, (L::TABB > 0)>(v, bv, aux, g.epi, stab, pk);
                    if (valid) st_global_32B((int8_t *)g.out + orow * g.ldo + gcol0, pk);
                }
                tc05::fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acce[tb]);
                    if (rs_on) mbar_arrive(&rempty[rsl]);
                }
                ++a;
            }
            if (stop || *abortf) break;
        }
    }

    if (warp < PT_PROD) asm volatile("cp.async.wait_all;\n" ::: "memory");
    tc05::fence_before();
    __syncthreads();
    if (*abortf && tid == 0) atomicExch(err, 3);
    if (warp == 0) {
        tc05::fence_after();
        tc05::tmem_dealloc(tbase, PT_TMEM_COLS);
    }
}

template <int EPI, bool FAST, int KDIM, int N>
cudaError_t launch_p(const GemmArgs &g, int m_max, int *err, int sms, cudaStream_t st) {
    auto kern = tcp_gemm_kernel<EPI, FAST, KDIM, N>;
    constexpr int smem = PLayout<KDIM, N, kResStaged<EPI, KDIM, N>>::SMEM;
    static_assert(smem <= 227 * 1024, "persistent GEMM shared memory");
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    // (the patch GEMM with TMA runs two 98-row tiles per image)
    const int tiles = EPI == EPI_PATCH && g.tma ? 2 * (m_max / 196) : (m_max + 127) / 128;
    const int units = tiles * PLayout<KDIM, N>::NCH;
    const int grid = units < sms ? units : sms;
    if (grid <= 0) return cudaSuccess;
    CUtensorMap tm;
    if (g.tma) tm = *g.tma;
    else memset(&tm, 0, sizeof(tm));
    return launch_pdl(kern, dim3(grid), dim3(PT_THREADS), smem, st, g, err, tm, g.tma ? 1 : 0);
}

// The (epilogue, K, N) combinations the model uses: QKV (I8, 192 -> 576), proj and
// FC2 (I8_RES, 192 -> 192 and 768 -> 192), FC1 (GELU, 192 -> 768), patch (768 -> 192);
// plus the plain int8 writeback for every layer shape (unit API, hv_gemm_i8).
constexpr bool shape_used(int epi, int k, int n) {
    return (epi == EPI_I8 && ((k == 192 && (n == 192 || n == 576 || n == 768)) || (k == 768 && n == 192))) ||
           (epi == EPI_I8_RES && n == 192 && (k == 192 || k == 768)) || (epi == EPI_GELU && k == 192 && n == 768) ||
           (epi == EPI_PATCH && k == 768 && n == 192);
}

template <int EPI, bool FAST, int KDIM, int N>
cudaError_t launch_if_used(const GemmArgs &g, int m_max, int *err, int sms, cudaStream_t st) {
    if constexpr (shape_used(EPI, KDIM, N)) return launch_p<EPI, FAST, KDIM, N>(g, m_max, err, sms, st);
    return cudaErrorInvalidValue;
}

template <int EPI, bool FAST>
cudaError_t launch_shape(const GemmArgs &g, int m_max, int *err, int sms, cudaStream_t st) {
    if (g.k == 192 && g.n == 576) return launch_if_used<EPI, FAST, 192, 576>(g, m_max, err, sms, st);
    if (g.k == 192 && g.n == 768) return launch_if_used<EPI, FAST, 192, 768>(g, m_max, err, sms, st);
    if (g.k == 192 && g.n == 192) return launch_if_used<EPI, FAST, 192, 192>(g, m_max, err, sms, st);
    if (g.k == 768 && g.n == 192) return launch_if_used<EPI, FAST, 768, 192>(g, m_max, err, sms, st);
    return cudaErrorInvalidValue;
}

}  // namespace

bool gemm_persistent_supported(int epi, int n, int k) { return shape_used(epi, k, n); }

cudaError_t launch_gemm_persistent(const GemmArgs &g, int epi, int m_max, int *err, int sms, cudaStream_t st) {
    const bool fast = g.epi.fast != 0;
    switch (epi) {
        case EPI_I8:
            return fast ? launch_shape<EPI_I8, true>(g, m_max, err, sms, st)
                        : launch_shape<EPI_I8, false>(g, m_max, err, sms, st);
        case EPI_I8_RES:
            return fast ? launch_shape<EPI_I8_RES, true>(g, m_max, err, sms, st)
                        : launch_shape<EPI_I8_RES, false>(g, m_max, err, sms, st);
        case EPI_GELU:
            return fast ? launch_shape<EPI_GELU, true>(g, m_max, err, sms, st)
                        : launch_shape<EPI_GELU, false>(g, m_max, err, sms, st);
        case EPI_PATCH:
            return fast ? launch_shape<EPI_PATCH, true>(g, m_max, err, sms, st)
                        : launch_shape<EPI_PATCH, false>(g, m_max, err, sms, st);
        default:
            return cudaErrorInvalidValue;
    }
}

namespace {

PFN_cuTensorMapEncodeTiled tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return nullptr;
        encode = (PFN_cuTensorMapEncodeTiled)fn;
    }
    return encode;
}

}  // namespace

// NHWC images [images][224][224][3] viewed as [img][pr][ir][pc][w]: patch row pr and
// column pc (14 each), pixel row ir inside the patch (16), byte w = in_col * 3 + ch
// of the patch's 48-byte row segment (layout.py:31-72).  Box: one 16-byte strip of
// w, all 14 patch columns, one ir, 7 patch rows, one image = 98 A rows of 16 bytes
// in tile-row order (row = 14 * pr + pc), the K-major strip layout of tma_load_a.
int make_tmap_patch(CUtensorMap *map, const void *images, int images_n) {
    PFN_cuTensorMapEncodeTiled encode = tmap_encoder();
    if (!encode) return 1;
    if ((uintptr_t)images % 16 != 0 || images_n <= 0) return 3;
    const cuuint64_t dims[5] = {48, 14, 16, 14, (cuuint64_t)images_n};
    const cuuint64_t strides[4] = {48, 672, 10752, 150528};
    const cuuint32_t box[5] = {16, 14, 1, 7, 1};
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<void *>(images), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : 2;
}

int make_tmap_a(CUtensorMap *map, const void *base, int k, int rows) { return make_tmap_box(map, base, k, rows, 128); }

int make_tmap_box(CUtensorMap *map, const void *base, int k, int rows, int box_rows) {
    PFN_cuTensorMapEncodeTiled encode = tmap_encoder();
    if (!encode) return 1;
    if ((uintptr_t)base % 16 != 0 || k % 16 != 0 || box_rows < 1 || box_rows > 256) return 3;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)k};
    const cuuint32_t box[2] = {16, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : 2;
}

}  // namespace hv
