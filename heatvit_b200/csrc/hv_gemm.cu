// hv_gemm.cu — int8 GEMM on tcgen05 tensor cores with fused integer epilogues.
//
// One CTA computes a 128 x BN output tile (BN = 64 columns; the ragged last tile of
// N is masked in the epilogue):
//   * 256 threads stream A [128 x 64] and B [BN x 64] k-tiles with cp.async into
//     a 4-stage ring, each stage in the no-swizzle K-major canonical layout
//     (hv_tc05.cuh); 8 consecutive threads fill one 128-byte core matrix, so
//     the shared-memory writes are conflict-free.
//   * one thread issues tcgen05.mma kind::i8 (M = 128, N = BN, K = 32 per
//     instruction) into a TMEM accumulator of BN columns; each stage's MMAs
//     commit to that stage's mbarrier, which gates the refill of the stage.
//   * the epilogue reads the accumulator straight from TMEM: thread t owns row
//     t % 128 (its TMEM lane) and half of the columns, applies the golden
//     writeback and what follows it, and stores 32 contiguous bytes at a time.
// Ragged batches pass the live row count through device memory; CTAs past it
// exit before allocating anything.  TMEM: 256 columns per CTA, two CTAs per SM.
#include "hv_gemm.cuh"
#include "hv_tc05.cuh"

namespace hv {

namespace {

constexpr int THREADS = 256;
constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr uint32_t WAIT_ITERS = 1u << 24;

// TMEM columns of a BN-wide accumulator (a power of two >= 32).
template <int BN>
struct TmemCols {
    static constexpr uint32_t value = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
};

template <int BN>
struct Layout {
    static constexpr int A_ST = BM * BK;
    static constexpr int B_ST = BN * BK;
    static constexpr int STAGE = A_ST + B_ST;
    static constexpr int OFF_BIAS = STAGES * STAGE;
    static constexpr int OFF_BAR = OFF_BIAS + BN * 4;
    static constexpr int SMEM = OFF_BAR + 64;
};

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// First writeback: requant(acc + bias, shift, 8).  FAST: host-proven that
// acc + bias fits in 30 bits and shift is in [1, 30].
template <bool FAST>
__device__ __forceinline__ int32_t wb8(int32_t acc, int32_t bias, int shift) {
    if (FAST) return requant8_r(acc + bias, shift);
    return (int32_t)requant64((int64_t)acc + bias, shift, 8);
}

// Residual / positional align-add; FAST: host-proven 32-bit form applies.
template <bool FAST>
__device__ __forceinline__ int32_t add8(int32_t a, int32_t b, AlignAdd k) {
    if (FAST) return requant8_r(a * (1 << k.sa) + b * (1 << k.sb), k.sh);
    return (int32_t)requant64(((int64_t)a << k.sa) + ((int64_t)b << k.sb), k.sh, 8);
}

__device__ __forceinline__ int32_t byte_of(const uint32_t (&w)[8], int j) {
    return (int8_t)((w[j >> 2] >> (8 * (j & 3))) & 0xffu);
}

template <int EPI, bool U8, bool FAST, int BN>
__global__ void __launch_bounds__(THREADS) tc_gemm_kernel(GemmArgs g, int *err) {
    griddep_wait();
    griddep_launch();
    using L = Layout<BN>;
    extern __shared__ __align__(1024) uint8_t smem[];
    int32_t *sbias = (int32_t *)(smem + L::OFF_BIAS);
    uint64_t *bar = (uint64_t *)(smem + L::OFF_BAR);
    uint32_t *tslot = (uint32_t *)(smem + L::OFF_BAR + 8 * STAGES);
    volatile int *abortf = (volatile int *)(smem + L::OFF_BAR + 8 * STAGES + 4);

    // N tiles vary fastest so the CTAs sharing an A tile run together (L2 reuse).
    const int m_lim = g.m_dev ? *g.m_dev : g.m_host;
    const int m0 = blockIdx.y * BM;
    if (m0 >= m_lim) return;
    const int n0 = blockIdx.x * BN;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int KT = g.k / BK;
    const uint8_t *abase = (const uint8_t *)g.a.ptr;

    constexpr uint32_t TMEM_COLS = TmemCols<BN>::value;
    if (warp == 0) {
        tc05::tmem_alloc(tslot, TMEM_COLS);
        tc05::tmem_relinquish();
    }
    if (tid < STAGES) tc05::mbar_init(&bar[tid], 1);
    if (tid == 0) {
        *abortf = 0;
        tc05::fence_mbar_init();
    }
    for (int i = tid; i < BN; i += THREADS) sbias[i] = (g.epi.bias && n0 + i < g.n) ? g.epi.bias[n0 + i] : 0;

    // Chunk c of a tile: core matrix (c >> 5, (c >> 3) & 3), row c & 7 inside it.
    auto load_stage = [&](int s, int kt) {
        uint8_t *sA = smem + s * L::STAGE;
        uint8_t *sB = sA + L::A_ST;
#pragma unroll
        for (int i = 0; i < (BM * 4) / THREADS; ++i) {
            const int c = tid + i * THREADS;
            const int row = (c >> 5) * 8 + (c & 7), kc = (c >> 3) & 3;
            const int grow = m0 + row;
            const uint8_t *src = abase;
            int bytes = 0;
            if (grow < m_lim) {
                bytes = 16;
                if (g.a.patch_mode) {
                    // layout.py:31-72: patch p = (pr, pc); k = (in_row*16 + in_col)*3 + ch,
                    // so a 16-byte chunk never straddles an image row (48 = 3 * 16).
                    const int img = grow / 196, p = grow - img * 196;
                    const int pr = p / 14, pc = p - pr * 14;
                    const int k = kt * BK + kc * 16;
                    const int ir = k / 48, w = k - ir * 48;
                    src = abase + (size_t)img * 150528 + ((pr * 16 + ir) * 224 + pc * 16) * 3 + w;
                } else {
                    src = abase + (size_t)grow * g.a.lda + kt * BK + kc * 16;
                }
            }
            cp_async16(tc05::smem_u32(sA + (c >> 5) * (8 * BK) + kc * 128 + (c & 7) * 16), src, bytes);
        }
#pragma unroll
        for (int i = 0; i < (BN * 4) / THREADS; ++i) {
            const int c = tid + i * THREADS;
            const int row = (c >> 5) * 8 + (c & 7), kc = (c >> 3) & 3;
            const int8_t *src = g.bt + (size_t)(n0 + row) * g.k + kt * BK + kc * 16;
            cp_async16(tc05::smem_u32(sB + (c >> 5) * (8 * BK) + kc * 128 + (c & 7) * 16), src, 16);
        }
    };

#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
        if (s < KT) load_stage(s, s);
        cp_commit();
    }
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tslot;
    const uint32_t idesc = tc05::idesc_i8(BM, BN, !U8, true);
    uint32_t phases = 0;

    for (int kt = 0; kt < KT; ++kt) {
        const int s = kt % STAGES;
        cp_wait<STAGES - 2>();
        tc05::fence_proxy_async();
        __syncthreads();
        if (*abortf) break;
        if (tid == 0) {
            tc05::fence_after();
            const uint32_t a0 = tc05::smem_u32(smem + s * L::STAGE), b0 = a0 + L::A_ST;
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
                tc05::mma_i8_ss(tbase, tc05::smem_desc(a0 + ks * 256, 128, 8 * BK),
                                tc05::smem_desc(b0 + ks * 256, 128, 8 * BK), idesc, (kt | ks) != 0);
            tc05::commit(&bar[s]);
        }
        // Refill the stage the previous k-tile used once its MMAs completed.
        if (kt >= 1 && kt - 1 + STAGES < KT) {
            const int ps = (kt - 1) % STAGES;
            if (tc05::mbar_wait(&bar[ps], (phases >> ps) & 1u, WAIT_ITERS)) {
                phases ^= 1u << ps;
                load_stage(ps, kt - 1 + STAGES);
            } else {
                *abortf = 1;
            }
        }
        cp_commit();
    }
    // Every MMA has completed once the last stage's final phase has.
    {
        const int ls = (KT - 1) % STAGES;
        if (!*abortf) {
            if (tc05::mbar_wait(&bar[ls], (phases >> ls) & 1u, WAIT_ITERS)) phases ^= 1u << ls;
            else *abortf = 1;
        }
    }
    cp_wait<0>();
    __syncthreads();

    if (!*abortf) {
        tc05::fence_after();
        const int row = tid & 127, half = tid >> 7;
        const int grow = m0 + row;
        const bool valid = grow < m_lim;
        const uint32_t lane_addr = tbase + ((uint32_t)((warp & 3) * 32) << 16);
        size_t orow = (size_t)grow;
        int pidx = 0;
        if (EPI == EPI_PATCH) {
            const int img = valid ? grow / 196 : 0;
            pidx = valid ? grow - img * 196 : 0;
            orow = (size_t)img * 197 + 1 + pidx;
        }
#pragma unroll 1
        for (int c = 0; c < BN / 64; ++c) {
            const int col0 = half * (BN / 2) + c * 32;  // tile-local column of v[0]
            const int gcol0 = n0 + col0;
            uint32_t v[32];
            tc05::ld32(lane_addr + col0, v);
            tc05::wait_ld();
            if (EPI == EPI_I32 || EPI == EPI_ACC64) {
                if (valid) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        if (gcol0 + j >= g.n) break;
                        const int64_t x = (int64_t)(int32_t)v[j] + sbias[col0 + j];
                        if (EPI == EPI_I32)
                            ((int32_t *)g.out)[orow * g.ldo + gcol0 + j] = (int32_t)requant64(x, g.epi.shift, 32);
                        else
                            ((int64_t *)g.out)[orow * g.ldo + gcol0 + j] = x;
                    }
                }
                continue;
            }
            uint4 r0 = make_uint4(0, 0, 0, 0), r1 = r0;
            if (EPI == EPI_I8_RES && valid) {
                const uint4 *r = (const uint4 *)(g.epi.res + orow * g.ldo + gcol0);
                r0 = r[0];
                r1 = r[1];
            }
            if (EPI == EPI_PATCH) {
                const uint4 *r = (const uint4 *)(g.epi.pos + (pidx + 1) * 192 + gcol0);
                r0 = r[0];
                r1 = r[1];
            }
            const uint32_t aux[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
            uint32_t pk[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                uint32_t word = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int j = w * 4 + b;
                    const int32_t a = (int32_t)v[j];
                    const int32_t bb = sbias[col0 + j];
                    int32_t o;
                    if (EPI == EPI_GELU) {
                        o = FAST ? gelu_chain_fast(a + bb, g.epi.gelu_sh_in, g.epi.gelu_sh_out)
                                 : gelu_chain((int64_t)a + bb, g.epi.gelu_sh_in, g.epi.gelu_sh_out);
                    } else {
                        o = wb8<FAST>(a, bb, g.epi.shift);
                        if (EPI == EPI_I8_RES) o = add8<FAST>(byte_of(aux, j), o, g.epi.add);
                        else if (EPI == EPI_PATCH) o = add8<FAST>(o, byte_of(aux, j), g.epi.add);
                    }
                    word |= ((uint32_t)o & 0xffu) << (8 * b);
                }
                pk[w] = word;
            }
            if (valid) {
                int8_t *dst = (int8_t *)g.out + orow * g.ldo + gcol0;
                if (gcol0 + 32 <= g.n) {
                    ((uint4 *)dst)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    ((uint4 *)dst)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                } else {
#pragma unroll
                    for (int w = 0; w < 8; ++w)
#pragma unroll
                        for (int b = 0; b < 4; ++b)
                            if (gcol0 + w * 4 + b < g.n) dst[w * 4 + b] = (int8_t)(pk[w] >> (8 * b));
                }
            }
        }
    } else {
        if (tid == 0) atomicExch(err, 2);
        // let MMAs still in flight drain (bounded) before the TMEM is released
        for (int s = 0; s < STAGES; ++s) tc05::mbar_wait(&bar[s], (phases >> s) & 1u, WAIT_ITERS);
    }
    tc05::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc05::fence_after();
        tc05::tmem_dealloc(tbase, TMEM_COLS);
    }
}

template <int EPI, bool U8, bool FAST, int BN>
cudaError_t launch_t(const GemmArgs &g, int m_max, int *err, cudaStream_t st) {
    auto kern = tc_gemm_kernel<EPI, U8, FAST, BN>;
    // Enough shared memory that the co-resident CTAs never ask for more than the
    // SM's 512 TMEM columns (TMEM allocation then never waits).
    constexpr int min_smem = (228 * 1024) / (512 / (int)TmemCols<BN>::value) + 1024;
    const int smem = Layout<BN>::SMEM > min_smem ? Layout<BN>::SMEM : min_smem;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    dim3 grid((g.n + BN - 1) / BN, (m_max + BM - 1) / BM);
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    return launch_pdl(kern, grid, dim3(THREADS), smem, st, g, err);
}

// 64-column tiles for every N: a ragged last tile costs only its own columns, and
// narrow tiles spread small-M GEMMs over more SMs (the 192 -> 1000 head over 1024
// CLS rows runs as 128 CTAs instead of 32 with 256-column tiles).
template <int EPI, bool U8, bool FAST>
cudaError_t launch_bn(const GemmArgs &g, int m_max, int *err, cudaStream_t st) {
    return launch_t<EPI, U8, FAST, 64>(g, m_max, err, st);
}

}  // namespace

int gemm_tile_n(int) { return 64; }

cudaError_t launch_gemm(const GemmArgs &g, int epi, int a_unsigned, int m_max, int *err, cudaStream_t st) {
    const bool fast = g.epi.fast != 0;
    switch (epi) {
        case EPI_I8:
            return fast ? launch_bn<EPI_I8, false, true>(g, m_max, err, st)
                        : launch_bn<EPI_I8, false, false>(g, m_max, err, st);
        case EPI_I8_RES:
            return fast ? launch_bn<EPI_I8_RES, false, true>(g, m_max, err, st)
                        : launch_bn<EPI_I8_RES, false, false>(g, m_max, err, st);
        case EPI_GELU:
            return fast ? launch_bn<EPI_GELU, false, true>(g, m_max, err, st)
                        : launch_bn<EPI_GELU, false, false>(g, m_max, err, st);
        case EPI_PATCH:
            return fast ? launch_bn<EPI_PATCH, false, true>(g, m_max, err, st)
                        : launch_bn<EPI_PATCH, false, false>(g, m_max, err, st);
        case EPI_I32:
            return a_unsigned ? launch_bn<EPI_I32, true, false>(g, m_max, err, st)
                              : launch_bn<EPI_I32, false, false>(g, m_max, err, st);
        case EPI_ACC64:
            return a_unsigned ? launch_bn<EPI_ACC64, true, false>(g, m_max, err, st)
                              : launch_bn<EPI_ACC64, false, false>(g, m_max, err, st);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace hv
