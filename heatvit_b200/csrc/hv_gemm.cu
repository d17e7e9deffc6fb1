// hv_gemm.cu — int8 tensor-core GEMM (mma.sync m16n8k32) with fused epilogues.
//
// CTA tile 128 x 64 x 64, 8 warps (4 along M x 2 along N, warp tile 32 x 32),
// 3-stage cp.async pipeline, XOR-swizzled shared tiles (16-byte chunk c of row r
// is stored at chunk c ^ ((r >> 1) & 3), which makes every ldmatrix phase hit
// 32 distinct banks).  Ragged batches pass the live row count through device
// memory; CTAs past it exit before touching memory.
#include "hv_gemm.cuh"

namespace hv {

namespace {

constexpr int BM = 128, BN = 64, BK = 64, STAGES = 3, THREADS = 256;
constexpr int A_TILE = BM * BK;
constexpr int B_TILE = BN * BK;
constexpr int STAGE_BYTES = A_TILE + B_TILE;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ int swz(int row, int chunk) {
    return row * BK + ((chunk ^ ((row >> 1) & 3)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(src_bytes));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

template <bool U8>
__device__ __forceinline__ void mma_i8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if (U8) {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

// First writeback: requant(acc + bias, shift, 8).
template <bool WIDE>
__device__ __forceinline__ int32_t wb8(int32_t acc, int32_t bias, int shift) {
    if (!WIDE && shift >= 1 && shift <= 30) return requant8_r(acc + bias, shift);
    return (int32_t)requant64((int64_t)acc + bias, shift, 8);
}

template <int EPI, bool U8, bool WIDE>
__global__ void __launch_bounds__(THREADS) gemm_kernel(GemmArgs g) {
    extern __shared__ __align__(128) uint8_t smem[];
    // N tiles vary fastest so the CTAs that share an A tile run together and
    // read it from L2 rather than DRAM.
    const int m_lim = g.m_dev ? *g.m_dev : g.m_host;
    const int m0 = blockIdx.y * BM;
    if (m0 >= m_lim) return;
    const int n0 = blockIdx.x * BN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp & 3, wn = warp >> 2;
    const int ktiles = g.k / BK;
    const uint8_t *abase = (const uint8_t *)g.a.ptr;

    auto load_stage = [&](int stage, int kt) {
        uint8_t *sA = smem + stage * STAGE_BYTES;
        uint8_t *sB = sA + A_TILE;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int c = tid + i * THREADS;
            const int row = c >> 2, ch = c & 3;
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
                    const int k = kt * BK + ch * 16;
                    const int ir = k / 48, w = k - ir * 48;
                    src = abase + (size_t)img * 150528 + ((pr * 16 + ir) * 224 + pc * 16) * 3 + w;
                } else {
                    src = abase + (size_t)grow * g.a.lda + kt * BK + ch * 16;
                }
            }
            cp_async16(smem_u32(sA + swz(row, ch)), src, bytes);
        }
        {
            const int row = tid >> 2, ch = tid & 3;
            const int8_t *src = g.bt + (size_t)(n0 + row) * g.k + kt * BK + ch * 16;
            cp_async16(smem_u32(sB + swz(row, ch)), src, 16);
        }
    };

    int acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0;

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < ktiles) load_stage(s, s);
        cp_commit();
    }

    const int q = lane >> 3, r8 = lane & 7;
    for (int kt = 0; kt < ktiles; ++kt) {
        cp_wait<STAGES - 2>();
        __syncthreads();
        {
            const int pf = kt + STAGES - 1;
            if (pf < ktiles) load_stage(pf % STAGES, pf);
            cp_commit();
        }
        const uint8_t *sA = smem + (kt % STAGES) * STAGE_BYTES;
        const uint8_t *sB = sA + A_TILE;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t af[2][4], bf[2][4];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int row = wm * 32 + i * 16 + (q & 1) * 8 + r8;
                ldsm_x4(af[i], smem_u32(sA + swz(row, ks * 2 + (q >> 1))));
            }
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int row = wn * 32 + p * 16 + (q >> 1) * 8 + r8;
                ldsm_x4(bf[p], smem_u32(sB + swz(row, ks * 2 + (q & 1))));
            }
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    mma_i8<U8>(acc[i][j], af[i], bf[j >> 1][(j & 1) * 2], bf[j >> 1][(j & 1) * 2 + 1]);
        }
    }
    cp_wait<0>();
    __syncthreads();

    const int gid = lane >> 2, t4 = lane & 3;

    if (EPI == EPI_I32 || EPI == EPI_ACC64) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int grow = m0 + wm * 32 + i * 16 + gid + hh * 8;
                    if (grow >= m_lim) continue;
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int col = n0 + wn * 32 + j * 8 + t4 * 2 + e;
                        if (col >= g.n) continue;
                        const int64_t v = (int64_t)acc[i][j][hh * 2 + e] + (g.epi.bias ? g.epi.bias[col] : 0);
                        if (EPI == EPI_I32)
                            ((int32_t *)g.out)[(size_t)grow * g.ldo + col] = (int32_t)requant64(v, g.epi.shift, 32);
                        else
                            ((int64_t *)g.out)[(size_t)grow * g.ldo + col] = v;
                    }
                }
        return;
    }

    // int8 epilogues go through a shared tile so the global stores are 16-byte.
    int8_t *sC = (int8_t *)smem;                   // [128][64]
    const int8_t *sR = (const int8_t *)(smem + A_TILE);  // residual [128][64]
    if (EPI == EPI_I8_RES) {
        int8_t *sRw = (int8_t *)(smem + A_TILE);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int c = tid + i * THREADS;
            const int row = c >> 2, ch = c & 3;
            const int grow = m0 + row;
            int4 v = make_int4(0, 0, 0, 0);
            if (grow < m_lim) v = *(const int4 *)(g.epi.res + (size_t)grow * g.ldo + n0 + ch * 16);
            *(int4 *)(sRw + row * BN + ch * 16) = v;
        }
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int lrow = wm * 32 + i * 16 + gid + hh * 8;
                const int grow = m0 + lrow;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int lcol = wn * 32 + j * 8 + t4 * 2 + e;
                    const int col = n0 + lcol;
                    const int32_t a = acc[i][j][hh * 2 + e];
                    const int32_t b = (g.epi.bias && col < g.n) ? g.epi.bias[col] : 0;
                    int32_t o;
                    if (EPI == EPI_GELU) {
                        o = (!WIDE && g.epi.gelu_fast)
                                ? gelu_chain_fast(a + b, g.epi.gelu_sh_in, g.epi.gelu_sh_out)
                                : gelu_chain((int64_t)a + b, g.epi.gelu_sh_in, g.epi.gelu_sh_out);
                    } else {
                        o = wb8<WIDE>(a, b, g.epi.shift);
                        if (EPI == EPI_I8_RES) {
                            o = align_add8(sR[lrow * BN + lcol], o, g.epi.add);
                        } else if (EPI == EPI_PATCH) {
                            const int p = grow < m_lim ? grow % 196 : 0;
                            o = align_add8(o, g.epi.pos[(p + 1) * 192 + col], g.epi.add);
                        }
                    }
                    sC[lrow * BN + lcol] = (int8_t)o;
                }
            }
    __syncthreads();

#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = tid + i * THREADS;
        const int row = c >> 2, ch = c & 3;
        const int grow = m0 + row;
        if (grow >= m_lim) continue;
        size_t orow = (size_t)grow;
        if (EPI == EPI_PATCH) {
            const int img = grow / 196;
            orow = (size_t)img * 197 + 1 + (grow - img * 196);
        }
        int8_t *dst = (int8_t *)g.out + orow * g.ldo + n0 + ch * 16;
        if (n0 + ch * 16 + 16 <= g.n) {
            *(int4 *)dst = *(const int4 *)(sC + row * BN + ch * 16);
        } else {
            for (int e = 0; e < 16; ++e)
                if (n0 + ch * 16 + e < g.n) dst[e] = sC[row * BN + ch * 16 + e];
        }
    }
}

template <int EPI, bool U8, bool WIDE>
cudaError_t launch_t(const GemmArgs &g, int m_max, cudaStream_t st) {
    auto kern = gemm_kernel<EPI, U8, WIDE>;
    dim3 grid((g.n + BN - 1) / BN, (m_max + BM - 1) / BM);
    if (grid.x == 0) return cudaSuccess;
    kern<<<grid, THREADS, SMEM_BYTES, st>>>(g);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(const GemmArgs &g, int epi, int a_unsigned, int m_max, cudaStream_t st) {
    const bool wide = g.epi.bits_wide != 0;
    switch (epi) {
        case EPI_I8:
            return wide ? launch_t<EPI_I8, false, true>(g, m_max, st) : launch_t<EPI_I8, false, false>(g, m_max, st);
        case EPI_I8_RES:
            return wide ? launch_t<EPI_I8_RES, false, true>(g, m_max, st)
                        : launch_t<EPI_I8_RES, false, false>(g, m_max, st);
        case EPI_GELU:
            return wide ? launch_t<EPI_GELU, false, true>(g, m_max, st) : launch_t<EPI_GELU, false, false>(g, m_max, st);
        case EPI_PATCH:
            return wide ? launch_t<EPI_PATCH, false, true>(g, m_max, st)
                        : launch_t<EPI_PATCH, false, false>(g, m_max, st);
        case EPI_I32:
            return a_unsigned ? launch_t<EPI_I32, true, true>(g, m_max, st) : launch_t<EPI_I32, false, true>(g, m_max, st);
        case EPI_ACC64:
            return a_unsigned ? launch_t<EPI_ACC64, true, true>(g, m_max, st)
                              : launch_t<EPI_ACC64, false, true>(g, m_max, st);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace hv
