// hv_attention.cu — fused per-(image, head) attention on the ragged token layout.
//
// Restates transformer.py:233-268 for one image and head:
//   score = requant(Q·Kᵀ, 2q, score_scale, 32)            (int32 writeback)
//   q16   = sat24(rsa(score, -(score_scale + 13)))         (Q8.16)
//   prob  = softmax_attention(q16 row)                     (UQ0.8, nonlinear.py:130-133)
//   ctx   = requant(prob(uint8)·V, prob_scale + q, context_out, 8)
// written straight into the head-concatenated layout (layout.py:132-155).
//
// One CTA per (image, head), 4 warps; each warp owns 16-query strips.  Q, K and
// a permuted, transposed V live in shared memory; scores and probabilities
// never leave registers.  The S accumulator fragment of mma.m16n8k32 gives a
// thread columns {8j + 2t, 8j + 2t + 1}; P·V needs A fragments holding 4
// consecutive k per thread, so the token order along P·V's k axis is permuted
// (k = 32g + 16h + 4u + 2a + b  <->  token 32g + 16h + 8a + 2u + b) and V is
// stored with the same permutation.  A dot product does not depend on the
// order of its terms, so the result is exact.
#include "hv_internal.cuh"

namespace hv {

namespace {

constexpr int MAXN = 197;
constexpr int NPMAX = 224;          // MAXN rounded up to 32
constexpr int QK_STRIDE = 80;       // 64 data bytes + 16 pad: conflict-free ldmatrix
constexpr int V_STRIDE = NPMAX + 16;
constexpr int WARPS = 4;
constexpr int SMEM_Q = NPMAX * QK_STRIDE;
constexpr int SMEM_K = NPMAX * QK_STRIDE;
constexpr int SMEM_V = 64 * V_STRIDE;
constexpr int SMEM_BYTES = SMEM_Q + SMEM_K + SMEM_V;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_u8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Position along P·V's k axis of token r (see file comment).
__device__ __forceinline__ int perm_pos(int r) {
    const int g = r & ~31, h = r & 16, a = (r >> 3) & 1, u = (r >> 1) & 3, b = r & 1;
    return g + h + 4 * u + 2 * a + b;
}

__global__ void __launch_bounds__(WARPS * 32) attention_kernel(const int8_t *__restrict__ qkv,
                                                               const int32_t *__restrict__ offsets,
                                                               int8_t *__restrict__ ctx, AttnParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *sQ = smem;
    uint8_t *sK = smem + SMEM_Q;
    uint8_t *sV = smem + SMEM_Q + SMEM_K;
    const int img = blockIdx.x, head = blockIdx.y;
    const int row0 = offsets[img];
    const int n = offsets[img + 1] - row0;
    if (n <= 0) return;
    const int np = (n + 31) & ~31;
    const int tid = threadIdx.x;

    // Q and K rows: 4 x 16-byte chunks each; zero rows up to np.
    for (int c = tid; c < np * 4; c += WARPS * 32) {
        const int r = c >> 2, ch = c & 3;
        int4 qv = make_int4(0, 0, 0, 0), kv = qv;
        if (r < n) {
            const int8_t *src = qkv + (size_t)(row0 + r) * 576 + head * 64 + ch * 16;
            qv = *(const int4 *)src;
            kv = *(const int4 *)(src + 192);
        }
        *(int4 *)(sQ + r * QK_STRIDE + ch * 16) = qv;
        *(int4 *)(sK + r * QK_STRIDE + ch * 16) = kv;
    }
    // V transposed + permuted: sV[lane][perm_pos(token)].
    for (int c = tid; c < np * 16; c += WARPS * 32) {
        const int r = c >> 4, w = c & 15;
        uint32_t word = 0;
        if (r < n) word = *(const uint32_t *)(qkv + (size_t)(row0 + r) * 576 + 384 + head * 64 + w * 4);
        const int pos = perm_pos(r);
#pragma unroll
        for (int b = 0; b < 4; ++b) sV[(w * 4 + b) * V_STRIDE + pos] = (uint8_t)(word >> (8 * b));
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    const int q4 = lane >> 3, r8 = lane & 7;
    const int gid = lane >> 2, t4 = lane & 3;
    const int nt = np >> 3;           // 8-column score tiles
    const int strips = (n + 15) >> 4;

    for (int s = warp; s < strips; s += WARPS) {
        uint32_t qa[2][4];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
            ldsm_x4(qa[ks], smem_u32(sQ + (s * 16 + (q4 & 1) * 8 + r8) * QK_STRIDE + (ks * 2 + (q4 >> 1)) * 16));

        int sc[NPMAX / 8][4];
#pragma unroll
        for (int j = 0; j < NPMAX / 8; ++j) {
            sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0;
        }
#pragma unroll
        for (int jp = 0; jp < NPMAX / 16; ++jp) {
            if (2 * jp < nt) {
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    uint32_t kb[4];
                    // matrices: (tile 2jp, k lo), (2jp, k hi), (2jp+1, k lo), (2jp+1, k hi)
                    ldsm_x4(kb, smem_u32(sK + ((2 * jp + (q4 >> 1)) * 8 + r8) * QK_STRIDE + (ks * 2 + (q4 & 1)) * 16));
                    mma_s8(sc[2 * jp], qa[ks], kb[0], kb[1]);
                    mma_s8(sc[2 * jp + 1], qa[ks], kb[2], kb[3]);
                }
            }
        }

        // Softmax on rows gid (e = 0,1) and gid + 8 (e = 2,3).
        int32_t mx0 = INT32_MIN, mx1 = INT32_MIN;
#pragma unroll
        for (int j = 0; j < NPMAX / 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = j * 8 + t4 * 2 + (e & 1);
                int32_t v = INT32_MIN;
                if (col < n) {
                    const int32_t score = (int32_t)requant64(sc[j][e], p.score_shift, 32);
                    v = (int32_t)requant64(score, p.q16_shift, 24);
                }
                sc[j][e] = v;
                if (e < 2) mx0 = max(mx0, v);
                else mx1 = max(mx1, v);
            }
        }
        mx0 = max(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = max(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = max(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = max(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        uint32_t s0 = 0, s1 = 0;
#pragma unroll
        for (int j = 0; j < NPMAX / 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int32_t v = sc[j][e];
                uint32_t ex = 0;
                if (v != INT32_MIN) ex = softmax_exp_q16(v - (e < 2 ? mx0 : mx1));
                sc[j][e] = (int32_t)ex;
                if (e < 2) s0 += ex;
                else s1 += ex;
            }
        }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        const uint64_t rc0 = softmax_recip(s0 ? s0 : 1u), rc1 = softmax_recip(s1 ? s1 : 1u);
#pragma unroll
        for (int j = 0; j < NPMAX / 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                sc[j][e] = (int32_t)softmax_attn_u8(softmax_ratio((uint32_t)sc[j][e], e < 2 ? rc0 : rc1));
        }

        // ctx = P·V with P (uint8) as the A operand.
        int oc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) oc[j][0] = oc[j][1] = oc[j][2] = oc[j][3] = 0;
#pragma unroll
        for (int g = 0; g < NPMAX / 32; ++g) {
            if (4 * g < nt) {
                uint32_t pa[4];
                pa[0] = (uint32_t)sc[4 * g][0] | ((uint32_t)sc[4 * g][1] << 8) | ((uint32_t)sc[4 * g + 1][0] << 16) |
                        ((uint32_t)sc[4 * g + 1][1] << 24);
                pa[1] = (uint32_t)sc[4 * g][2] | ((uint32_t)sc[4 * g][3] << 8) | ((uint32_t)sc[4 * g + 1][2] << 16) |
                        ((uint32_t)sc[4 * g + 1][3] << 24);
                pa[2] = (uint32_t)sc[4 * g + 2][0] | ((uint32_t)sc[4 * g + 2][1] << 8) |
                        ((uint32_t)sc[4 * g + 3][0] << 16) | ((uint32_t)sc[4 * g + 3][1] << 24);
                pa[3] = (uint32_t)sc[4 * g + 2][2] | ((uint32_t)sc[4 * g + 2][3] << 8) |
                        ((uint32_t)sc[4 * g + 3][2] << 16) | ((uint32_t)sc[4 * g + 3][3] << 24);
#pragma unroll
                for (int pr = 0; pr < 4; ++pr) {
                    uint32_t vb[4];
                    // matrices: (lanes 16pr..+7, k lo), (same, k hi), (16pr+8.., k lo), (k hi)
                    ldsm_x4(vb, smem_u32(sV + (pr * 16 + (q4 >> 1) * 8 + r8) * V_STRIDE + g * 32 + (q4 & 1) * 16));
                    mma_u8(oc[2 * pr], pa, vb[0], vb[1]);
                    mma_u8(oc[2 * pr + 1], pa, vb[2], vb[3]);
                }
            }
        }
        const int ra = s * 16 + gid, rb = ra + 8;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int col = head * 64 + j * 8 + t4 * 2;
            if (ra < n) {
                const uint32_t lo = (uint32_t)requant64(oc[j][0], p.ctx_shift, 8) & 0xff;
                const uint32_t hi = (uint32_t)requant64(oc[j][1], p.ctx_shift, 8) & 0xff;
                *(uint16_t *)(ctx + (size_t)(row0 + ra) * 192 + col) = (uint16_t)(lo | (hi << 8));
            }
            if (rb < n) {
                const uint32_t lo = (uint32_t)requant64(oc[j][2], p.ctx_shift, 8) & 0xff;
                const uint32_t hi = (uint32_t)requant64(oc[j][3], p.ctx_shift, 8) & 0xff;
                *(uint16_t *)(ctx + (size_t)(row0 + rb) * 192 + col) = (uint16_t)(lo | (hi << 8));
            }
        }
    }
}

}  // namespace

cudaError_t launch_attention(const int8_t *qkv, const int32_t *offsets, int images, int8_t *ctx,
                             const AttnParams &p, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attention_kernel<<<dim3(images, 3), WARPS * 32, SMEM_BYTES, st>>>(qkv, offsets, ctx, p);
    return cudaGetLastError();
}

}  // namespace hv
