// hv_ffn.cu — the FFN of a transformer block (transformer.py:328-384) as one
// persistent tcgen05 kernel: FC1 + ShiftGELU chain, FC2 + residual 2, with the
// hidden activations kept on chip.
//
// Per 128-row tile of the LN2 output A [rows][192]:
//   for chunk j = 0..5 (128 hidden columns each):
//     D1[j & 1]  = A · W1[:, 128j : 128j + 128]        (TMEM columns 0 / 128)
//     H[j & 1]   = requant(gelu(requant(D1 + b1)))     (epilogue warps -> shared memory,
//                                                       K-major: the A operand of FC2)
//     D2        += H · W2[128j : 128j + 128, :]        (TMEM columns 256..447)
//   out = align_add(Y, requant(D2 + b2))               (residual 2)
// so the 768 hidden bytes of a row never reach HBM.  Neither weight matrix fits in
// shared memory beside the other, so both stream from L2 in 24 KB chunks (W1: 128
// hidden rows x 192; W2: 192 output rows x 128 hidden columns), each in a two-slot
// ring.  The model stores every chunk as the exact bytes of its shared-memory image
// (FfnArgs::w1img / w2img), so one bulk copy moves a chunk: 16-byte-wide tensor
// boxes would cost one copy request per row and 16-byte strip.  The tile's residual
// rows (contiguous, 24 KB) arrive the same way, ahead of the FC2 epilogue.
//
// Roles (576 threads): warp 0 lane 0 issues every copy (A tiles by TMA; W1 and W2
// chunks and residual rows by bulk copy; in consumption order); warp 1 lane 0
// issues the MMAs, FC1 of chunk j + 1
// ahead of FC2 of chunk j, so the GELU epilogue of chunk j overlaps the tensor
// work; warps 2-17 run the epilogues, four per TMEM lane quadrant (thread = TMEM
// lane; the quadrant's four warps split each chunk's 128 columns into 32-column
// pieces), so that enough warps hide the TMEM and table-lookup latencies.  Every
// mbarrier wait is bounded; a timeout sets the error word (3) and the kernel drains
// its copies and MMAs before it releases TMEM.
#include "hv_epi.cuh"
#include "hv_internal.cuh"

namespace hv {

namespace {

using namespace pg;

constexpr int FF_MMA_WARP = 1;
constexpr int FF_EPI0 = 2;
constexpr int FF_EPI_WARPS = 16;
constexpr int FF_THREADS = (FF_EPI0 + FF_EPI_WARPS) * 32;
constexpr int CH = 128;           // hidden columns per chunk (FC1 N, FC2 K)
constexpr int NCHK = 768 / CH;    // chunks per tile
constexpr uint32_t FF_WAIT = 1u << 24;

struct FLayout {
    static constexpr int A_BYTES = 128 * 192;   // A tile: 12 strips of 16 B x 128 rows
    static constexpr int W1_BYTES = CH * 192;   // W1 chunk: 12 strips of 16 B x 128 rows
    static constexpr int W2_BYTES = 192 * CH;   // W2 chunk: 8 strips of 16 B x 192 rows
    static constexpr int H_BYTES = 128 * CH;    // hidden chunk: 8 strips of 16 B x 128 rows
    static constexpr int R_BYTES = 128 * 192;   // residual rows of the tile, row-major
    static constexpr int OFF_A = 0;
    static constexpr int OFF_W1 = OFF_A + 2 * A_BYTES;
    static constexpr int OFF_W2 = OFF_W1 + 2 * W1_BYTES;
    static constexpr int OFF_H = OFF_W2 + 2 * W2_BYTES;
    static constexpr int OFF_B1 = OFF_H + 2 * H_BYTES;
    static constexpr int OFF_B2 = OFF_B1 + 768 * 4;
    static constexpr int OFF_TAB = OFF_B2 + 192 * 4;
    static constexpr int OFF_R = OFF_TAB + kGeluTableMax;
    static constexpr int OFF_BAR = OFF_R + R_BYTES;
    static constexpr int NBAR = 25;
    static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;
};
static_assert(FLayout::SMEM <= 227 * 1024, "fused FFN shared memory");

template <bool F1, bool F2, bool TAB>
__global__ void __launch_bounds__(FF_THREADS, 1)
    ffn_kernel(FfnArgs f, int *err, const __grid_constant__ CUtensorMap tmA) {
    using L = FLayout;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sA = smem + L::OFF_A, *sW1 = smem + L::OFF_W1, *sW2 = smem + L::OFF_W2, *sH = smem + L::OFF_H;
    int32_t *sb1 = (int32_t *)(smem + L::OFF_B1), *sb2 = (int32_t *)(smem + L::OFF_B2);
    int8_t *stab = (int8_t *)(smem + L::OFF_TAB);
    const uint8_t *sR = smem + L::OFF_R;
    uint64_t *bars = (uint64_t *)(smem + L::OFF_BAR);
    uint64_t *a_full = bars, *a_empty = bars + 2, *w1_full = bars + 4, *w1_empty = bars + 6;
    uint64_t *w2_full = bars + 8, *w2_empty = bars + 10, *acc1_full = bars + 12, *acc1_empty = bars + 14;
    uint64_t *hid_full = bars + 16, *hid_empty = bars + 18, *acc2_full = bars + 20, *acc2_empty = bars + 21;
    uint64_t *drain = bars + 22, *r_full = bars + 23, *r_empty = bars + 24;
    uint32_t *tslot = (uint32_t *)(bars + L::NBAR);
    volatile int *abortf = (volatile int *)(tslot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // ---- prologue: TMEM, barriers, biases and the GELU table (weights only) ------
    if (warp == 0) {
        tc05::tmem_alloc(tslot, 512);
        tc05::tmem_relinquish();
    }
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            tc05::mbar_init(&a_full[i], 1);
            tc05::mbar_init(&a_empty[i], 1);
            tc05::mbar_init(&w1_full[i], 1);
            tc05::mbar_init(&w1_empty[i], 1);
            tc05::mbar_init(&w2_full[i], 1);
            tc05::mbar_init(&w2_empty[i], 1);
            tc05::mbar_init(&acc1_full[i], 1);
            tc05::mbar_init(&acc1_empty[i], FF_EPI_WARPS);
            tc05::mbar_init(&hid_full[i], FF_EPI_WARPS);
            tc05::mbar_init(&hid_empty[i], 1);
        }
        tc05::mbar_init(acc2_full, 1);
        tc05::mbar_init(acc2_empty, FF_EPI_WARPS);
        tc05::mbar_init(drain, 1);
        tc05::mbar_init(r_full, 1);
        tc05::mbar_init(r_empty, FF_EPI_WARPS);
        *abortf = 0;
        tc05::fence_mbar_init();
    }
    for (int i = tid; i < 768; i += FF_THREADS) sb1[i] = f.e1.bias ? f.e1.bias[i] : 0;
    for (int i = tid; i < 192; i += FF_THREADS) sb2[i] = f.e2.bias ? f.e2.bias[i] : 0;
    if (TAB)  // the table allocation is padded to 16 bytes
        for (int i = tid; i < (f.e1.gtab_bytes + 15) / 16; i += FF_THREADS)
            ((uint4 *)stab)[i] = ((const uint4 *)f.e1.gtab)[i];
    griddep_wait();  // A, the residual and the row count come from earlier kernels
    griddep_launch();
    const int m_lim = f.m_dev ? *f.m_dev : f.m_host;
    const int tiles = (m_lim + 127) / 128;
    // each CTA takes one contiguous range of tiles, equal to within one tile
    const int t_begin = (int)(((long long)blockIdx.x * tiles) / gridDim.x);
    const int t_end = (int)(((long long)(blockIdx.x + 1) * tiles) / gridDim.x);
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tslot;
    const uint32_t wl = f.wait_iters ? f.wait_iters : FF_WAIT;  // pipeline waits; drains use FF_WAIT

    if (warp == 0) {
        // ---- producer: one thread issues every TMA load (no multicast) ------------------
        if (lane == 0) {
            uint32_t qa = 0, q1 = 0, q2 = 0, qr = 0;
            int la[2] = {-1, -1}, l1[2] = {-1, -1}, l2[2] = {-1, -1}, lr = -1;  // last slot issued per stage
            bool ok = true;
            for (int t = t_begin; t < t_end && ok && !*abortf; ++t) {
                {
                    const int s = qa & 1;
                    if (qa >= 2 && !tc05::mbar_wait(&a_empty[s], ((qa >> 1) - 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    if (t != f.skip_tile - 1) {  // (test hook: that tile never arrives)
                        la[s] = (int)qa;
                        mbar_expect_tx(&a_full[s], L::A_BYTES);
#pragma unroll
                        for (int kc = 0; kc < 12; ++kc)
                            tma_load_a(tc05::smem_u32(sA + s * L::A_BYTES + kc * 2048), &tmA, kc * 16, t * 128,
                                       &a_full[s]);
                    }
                    ++qa;
                }
                for (int j = 0; j < NCHK; ++j) {
                    const int s1 = q1 & 1;
                    if (q1 >= 2 && !tc05::mbar_wait(&w1_empty[s1], ((q1 >> 1) - 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    l1[s1] = (int)q1;
                    mbar_expect_tx(&w1_full[s1], L::W1_BYTES);
                    bulk_load(tc05::smem_u32(sW1 + s1 * L::W1_BYTES), f.w1img + (size_t)j * L::W1_BYTES, L::W1_BYTES,
                              &w1_full[s1]);
                    ++q1;
                    const int s2 = q2 & 1;
                    if (q2 >= 2 && !tc05::mbar_wait(&w2_empty[s2], ((q2 >> 1) - 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    l2[s2] = (int)q2;
                    mbar_expect_tx(&w2_full[s2], L::W2_BYTES);
                    bulk_load(tc05::smem_u32(sW2 + s2 * L::W2_BYTES), f.w2img + (size_t)j * L::W2_BYTES, L::W2_BYTES,
                              &w2_full[s2]);
                    ++q2;
                    if (j == 1) {
                        // the tile's residual rows, once the previous tile's FC2 epilogue
                        // has read its own (by now long done: it precedes chunk 0's GELU)
                        if (qr >= 1 && !tc05::mbar_wait(r_empty, (qr - 1) & 1u, wl)) {
                            ok = false;
                            break;
                        }
                        const uint32_t bytes = (uint32_t)min(128, m_lim - t * 128) * 192u;
                        lr = (int)qr;
                        mbar_expect_tx(r_full, bytes);
                        bulk_load(tc05::smem_u32(sR), f.e2.res + (size_t)t * L::R_BYTES, bytes, r_full);
                        ++qr;
                    }
                }
            }
            if (!ok) *abortf = 1;
            // After an abort: wait (bounded) until every box issued has landed, so no bulk
            // copy still writes this CTA's shared memory when it exits.
            if (*abortf) {
                for (int s = 0; s < 2; ++s) {
                    if (la[s] >= 0) tc05::mbar_wait(&a_full[s], ((uint32_t)la[s] >> 1) & 1u, FF_WAIT);
                    if (l1[s] >= 0) tc05::mbar_wait(&w1_full[s], ((uint32_t)l1[s] >> 1) & 1u, FF_WAIT);
                    if (l2[s] >= 0) tc05::mbar_wait(&w2_full[s], ((uint32_t)l2[s] >> 1) & 1u, FF_WAIT);
                }
                if (lr >= 0) tc05::mbar_wait(r_full, (uint32_t)lr & 1u, FF_WAIT);
            }
        }
    } else if (warp == FF_MMA_WARP) {
        // ---- MMA issuer ----------------------------------------------------------------
        if (lane == 0) {
            const uint32_t id1 = tc05::idesc_i8(128, CH, true, true), id2 = tc05::idesc_i8(128, 192, true, true);
            uint32_t qa = 0, q1 = 0, q2 = 0, c1 = 0, h = 0, tl = 0;
            bool ok = true;
            for (int t = t_begin; t < t_end && ok && !*abortf; ++t, ++tl) {
                const int sa = qa & 1;
                if (!tc05::mbar_wait(&a_full[sa], (qa >> 1) & 1u, wl)) { ok = false; break; }
                tc05::fence_proxy_async();
                tc05::fence_after();
                const uint32_t a0 = tc05::smem_u32(sA + sa * L::A_BYTES);
                // FC1 of the next chunk into D1[c1 & 1]
                auto fc1 = [&]() -> bool {
                    const int b = c1 & 1;
                    if (c1 >= 2 && !tc05::mbar_wait(&acc1_empty[b], ((c1 >> 1) - 1) & 1u, wl)) return false;
                    const int s = q1 & 1;
                    if (!tc05::mbar_wait(&w1_full[s], (q1 >> 1) & 1u, wl)) return false;
                    tc05::fence_proxy_async();
                    tc05::fence_after();
                    const uint32_t w0 = tc05::smem_u32(sW1 + s * L::W1_BYTES);
#pragma unroll
                    for (int ks = 0; ks < 6; ++ks)
                        tc05::mma_i8_ss(tbase + b * CH, tc05::smem_desc(a0 + ks * 4096, 2048, 128),
                                        tc05::smem_desc(w0 + ks * 4096, 2048, 128), id1, ks != 0);
                    tc05::commit(&w1_empty[s]);
                    tc05::commit(&acc1_full[b]);
                    ++q1;
                    ++c1;
                    return true;
                };
                if (!fc1()) { ok = false; break; }
                // D2 is free once the previous tile's epilogue has read it
                if (tl >= 1 && !tc05::mbar_wait(acc2_empty, (tl - 1) & 1u, wl)) { ok = false; break; }
                for (int j = 0; j < NCHK && ok; ++j) {
                    if (j + 1 < NCHK && !fc1()) { ok = false; break; }
                    const int hb = h & 1, s2 = q2 & 1;
                    if (!tc05::mbar_wait(&hid_full[hb], (h >> 1) & 1u, wl) ||
                        !tc05::mbar_wait(&w2_full[s2], (q2 >> 1) & 1u, wl)) {
                        ok = false;
                        break;
                    }
                    tc05::fence_proxy_async();
                    tc05::fence_after();
                    const uint32_t h0 = tc05::smem_u32(sH + hb * L::H_BYTES), v0 = tc05::smem_u32(sW2 + s2 * L::W2_BYTES);
#pragma unroll
                    for (int ks = 0; ks < CH / 32; ++ks)
                        tc05::mma_i8_ss(tbase + 256, tc05::smem_desc(h0 + ks * 4096, 2048, 128),
                                        tc05::smem_desc(v0 + ks * 6144, 3072, 128), id2, (j | ks) != 0);
                    tc05::commit(&w2_empty[s2]);
                    tc05::commit(&hid_empty[hb]);
                    ++q2;
                    ++h;
                }
                if (!ok) break;
                tc05::commit(&a_empty[sa]);  // every FC1 of the tile has been issued
                ++qa;
                tc05::commit(acc2_full);
            }
            if (!ok) *abortf = 1;
            // Every MMA this thread issued has completed once `drain` flips.
            tc05::commit(drain);
            if (!tc05::mbar_wait(drain, 0, FF_WAIT)) *abortf = 1;
        }
    } else {
        // ---- epilogue (16 warps): thread = TMEM lane; warp `sub` of its quadrant takes
        // columns [32 sub, 32 sub + 32) of each hidden chunk and the 32-column pieces
        // sub, sub + 4 of the 192 output columns
        const int quad = warp & 3, sub = (warp - FF_EPI0) >> 2;
        const int row = quad * 32 + lane;
        const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
        uint32_t c1 = 0, h = 0, tl = 0;
        const uint32_t zero8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        bool stop = false;
        for (int t = t_begin; t < t_end && !stop; ++t, ++tl) {
            const int grow = t * 128 + row;
            const bool valid = grow < m_lim;
#pragma unroll 1
            for (int j = 0; j < NCHK; ++j) {
                const int b = c1 & 1, hb = h & 1;
                // the hidden buffer is free once FC2 of chunk h - 2 has read it
                if ((h >= 2 && !tc05::mbar_wait(&hid_empty[hb], ((h >> 1) - 1) & 1u, wl)) ||
                    !tc05::mbar_wait(&acc1_full[b], (c1 >> 1) & 1u, wl)) {
                    stop = true;
                    break;
                }
                tc05::fence_after();
                const int col0 = sub * 32;  // chunk column of v[0]
                uint32_t v[32];
                tc05::ld32(lane_addr + b * CH + col0, v);
                int32_t bv[32];
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                    const int4 b4 = *(const int4 *)(sb1 + j * CH + col0 + 4 * q4);
                    bv[4 * q4] = b4.x;
                    bv[4 * q4 + 1] = b4.y;
                    bv[4 * q4 + 2] = b4.z;
                    bv[4 * q4 + 3] = b4.w;
                }
                tc05::wait_ld();
                tc05::fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc1_empty[b]);  // D1 is read: FC1 may refill it
                ++c1;
                uint32_t p8[8];
                epi_piece32<EPI_GELU, F1, TAB>(v, bv, zero8, f.e1, stab, p8);
                // this row's hidden bytes: K strips 2 sub, 2 sub + 1 of the chunk
                uint8_t *hrow = sH + hb * L::H_BYTES + row * 16 + sub * 2 * 2048;
                *(uint4 *)hrow = make_uint4(p8[0], p8[1], p8[2], p8[3]);
                *(uint4 *)(hrow + 2048) = make_uint4(p8[4], p8[5], p8[6], p8[7]);
                tc05::fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&hid_full[hb]);
                ++h;
            }
            if (stop) break;
            if (!tc05::mbar_wait(acc2_full, tl & 1u, wl) || !tc05::mbar_wait(r_full, tl & 1u, wl)) {
                stop = true;
                break;
            }
            tc05::fence_after();
            // 32-column pieces sub and sub + 4 (< 6) of the 192 output columns: 32-byte
            // stores fill whole sectors, which beats an even three-way split into
            // 16-column pieces with 16-byte stores
            const int np = sub < 2 ? 2 : 1;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                if (i < np) {
                    const int col0 = (sub + 4 * i) * 32;
                    uint32_t v[32];
                    tc05::ld32(lane_addr + 256 + col0, v);
                    int32_t bv[32];
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4) {
                        const int4 b4 = *(const int4 *)(sb2 + col0 + 4 * q4);
                        bv[4 * q4] = b4.x;
                        bv[4 * q4 + 1] = b4.y;
                        bv[4 * q4 + 2] = b4.z;
                        bv[4 * q4 + 3] = b4.w;
                    }
                    const uint4 ra = *(const uint4 *)(sR + row * 192 + col0);
                    const uint4 rb = *(const uint4 *)(sR + row * 192 + col0 + 16);
                    const uint32_t aux[8] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
                    tc05::wait_ld();
                    uint32_t p8[8];
                    epi_piece32<EPI_I8_RES, F2, false>(v, bv, aux, f.e2, stab, p8);
                    if (valid) st_global_32B(f.out + (size_t)grow * 192 + col0, p8);
                }
            }
            tc05::fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(acc2_empty);  // D2 is read: FC2 of the next tile may start
                mbar_arrive(r_empty);     // and the residual rows: the next tile's may land
            }
        }
        if (stop) *abortf = 1;
    }

    tc05::fence_before();
    __syncthreads();
    if (*abortf && tid == 0) atomicExch(err, 3);
    if (warp == 0) {
        tc05::fence_after();
        tc05::tmem_dealloc(tbase, 512);
    }
}

template <bool F1, bool F2, bool TAB>
cudaError_t launch_t(const FfnArgs &f, const CUtensorMap &tmA, int grid, int *err, cudaStream_t st) {
    auto k = ffn_kernel<F1, F2, TAB>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, FLayout::SMEM);
    if (e != cudaSuccess) return e;
    return launch_pdl(k, dim3(grid), dim3(FF_THREADS), FLayout::SMEM, st, f, err, tmA);
}

}  // namespace

cudaError_t launch_ffn(const FfnArgs &f, const CUtensorMap &tmA, int m_max, int *err, int sms, cudaStream_t st) {
    const int tiles = (m_max + 127) / 128;
    const int grid = tiles < sms ? tiles : sms;
    if (grid <= 0) return cudaSuccess;
    const bool f1 = f.e1.fast != 0, f2 = f.e2.fast != 0, tab = f1 && f.e1.gtab_n > 0;
    if (f1 && f2) return tab ? launch_t<true, true, true>(f, tmA, grid, err, st)
                             : launch_t<true, true, false>(f, tmA, grid, err, st);
    if (f1) return tab ? launch_t<true, false, true>(f, tmA, grid, err, st)
                       : launch_t<true, false, false>(f, tmA, grid, err, st);
    return f2 ? launch_t<false, true, false>(f, tmA, grid, err, st)
              : launch_t<false, false, false>(f, tmA, grid, err, st);
}

}  // namespace hv
