// hv_attention.cu — per-(image, head) attention on tcgen05 tensor cores and TMEM.
//
// Restates transformer.py:233-268 for one image and head:
//   score = requant(Q·Kᵀ, 2q, score_scale, 32)            (int32 writeback)
//   q16   = sat24(rsa(score, -(score_scale + 13)))         (Q8.16)
//   prob  = softmax_attention(q16 row)                     (UQ0.8, nonlinear.py:98-133)
//   ctx   = requant(prob(uint8)·V, prob_scale + q, context_out, 8)
// written straight into the head-concatenated layout (layout.py:132-155).
//
// Persistent CTAs (16 warps) walk (image, head) items, query rows in tiles of 128:
//   1. K, V and each Q tile are staged in shared memory with 16-byte copies in
//      the no-swizzle canonical layout (hv_tc05.cuh).  K and Q are K-major
//      operands; V is the same byte layout read as an MN-major B operand
//      (tokens along K, head dims along N), so no transpose is needed.
//   2. One thread issues S = Q·Kᵀ as tcgen05.mma kind::i8 (M=128, N=np, K=64)
//      into TMEM columns [0, np); completion arrives on an mbarrier.
//   3. Query row r of the tile is TMEM lane r.  Warps w, w+4, w+8, w+12 own
//      lanes 32*(w%4)..+31 and split the row's 16-column chunks round-robin;
//      each reads its chunks with tcgen05.ld, and the four parts combine the
//      row max and the exp sum through shared memory.  Exp terms are written back to
//      TMEM, then turned into UQ0.8 probabilities stored to shared memory as
//      the A operand of the next MMA.  Warps whose 32 rows all lie past the
//      image's token count skip the softmax.
//   4. ctx = P·V as tcgen05.mma kind::i8 with unsigned A (M=128, N=64, K=np)
//      into TMEM columns [0, 64), then requantised in 16-column pieces per part
//      and written out.
// TMEM: 256 columns per CTA; shared memory is padded so two CTAs share an SM.
#include <algorithm>

#include "hv_internal.cuh"
#include "hv_tc05.cuh"

namespace hv {

namespace {

constexpr uint32_t WAIT_ITERS = 1u << 24;

// Two CTA shapes.  Images of up to 128 tokens use the small one (128 TMEM
// columns, 8 warps, about 46 KB of shared memory: four CTAs per SM); longer
// images use the large one (256 TMEM columns, 16 warps, 80 KB: two per SM).
// Shared memory is padded so that TMEM is never oversubscribed.
template <int NPM, int SPL>
struct AttnCfg {
    static constexpr int NPMAX = NPM;                 // longest image rounded up to 32
    static constexpr int SPLIT = SPL;                 // warps per TMEM lane quadrant (column parts)
    static constexpr int THREADS = 128 * SPL;
    static constexpr uint32_t TMEM_COLS = NPM <= 128 ? 128 : 256;
    static constexpr int KV = NPM * 64;                        // one [NPMAX][64] K-major operand
    static constexpr int OFF_KV = 0;                           // two (K, V) buffers: item j uses j & 1
    static constexpr int OFF_P = OFF_KV + 4 * KV;              // [128][NPMAX] uint8
    static constexpr int OFF_Q = OFF_P;                        // [128][64]; Q is dead before P is written
    static constexpr int OFF_RED = OFF_P + 128 * NPM;          // [2][SPLIT][128] int32 row partials
    static constexpr int OFF_BAR = OFF_RED + 2 * SPL * 128 * 4;  // mbarrier, TMEM base, abort flag
    static constexpr int SMEM = (OFF_BAR + 64 + 1023) / 1024 * 1024;
    // Shared memory alone keeps the resident CTAs within the 512 TMEM columns, so
    // tcgen05.alloc never waits: at most 4 small (128 columns) or 2 large (256) per SM.
    static_assert(NPM <= 128 ? (5 * SMEM > 228 * 1024 && 4 * (SMEM + 2048) <= 228 * 1024)
                             : (3 * SMEM > 228 * 1024 && 2 * (SMEM + 3072) <= 228 * 1024),
                  "attention shared memory sizing");
};
using AttnSmall = AttnCfg<128, 2>;
using AttnLarge = AttnCfg<224, 4>;

// q16 of one score accumulator.  FAST: host-proven that the int32 score
// writeback and the sat24 cannot clip, so q16 = rsa(acc, fast_shift), written
// branch-free with precomputed rounding constants (fast_shift may be 0).
template <bool FAST>
__device__ __forceinline__ int32_t q16_of(int32_t acc, const AttnParams &p) {
    if (FAST) return (acc + p.fast_half + ((acc >> 31) & p.fast_negmask)) >> p.fast_shift;
    const int32_t score = (int32_t)requant64(acc, p.score_shift, 32);
    return (int32_t)requant64(score, p.q16_shift, 24);
}

// n = mx - q16(acc) >= 0 (the negated softmax argument).  FAST: q16(acc) - mx =
// (acc + cm + sign) >> s exactly with cm = half - mx*2^s, since mx*2^s is a multiple
// of 2^s; its negation is (cmn - acc - sign) >> s with cmn = 2^s - 1 - cm, computed
// once per row.  |acc| <= 2^20 and |mx*2^s| <= 2^30 + 2^20 keep the sum inside int32.
template <bool FAST>
__device__ __forceinline__ uint32_t negxt_of(int32_t acc, int32_t mx, int32_t cmn, const AttnParams &p) {
    if (FAST) return (uint32_t)((cmn - acc - ((acc >> 31) & p.fast_negmask)) >> p.fast_shift);
    return (uint32_t)(mx - q16_of<false>(acc, p));
}

template <bool FAST, bool MASK>
__device__ __forceinline__ uint32_t chunk_exp(uint32_t (&v)[16], int valid, int32_t mx, int32_t cmn,
                                              const AttnParams &p) {
    uint32_t sum = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        uint32_t e = softmax_exp_q16_n(negxt_of<FAST>((int32_t)v[j], mx, cmn, p));
        if (MASK && j >= valid) e = 0u;
        v[j] = e;
        sum += e;
    }
    return sum;
}

// Asynchronous copy of item `item`'s K and V rows into a (K, V) buffer pair, both in
// the K-major byte layout; rows n..np-1 are zero-filled (src-size 0).
template <class CFG>
__device__ __forceinline__ void attn_load_kv(const int8_t *qkv, const int32_t *offsets, int item, uint8_t *kv,
                                             int tid) {
    const int img = item / 3, head = item - img * 3;
    const int row0 = offsets[img], n = offsets[img + 1] - row0, np = (n + 31) & ~31;
    for (int c = tid; c < np * 8; c += CFG::THREADS) {
        const int r = c >> 3, ch = c & 3, isv = (c >> 2) & 1;
        const int8_t *src = qkv + (size_t)(row0 + (r < n ? r : 0)) * 576 + 192 * (1 + isv) + head * 64 + ch * 16;
        const uint32_t dst = tc05::smem_u32(kv + isv * CFG::KV + tc05::kmajor_offset(r, ch * 16, 64));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(r < n ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// Asynchronous copy of the 128-row Q tile t of item `item` (rows past the image are
// zero-filled) into the K-major Q buffer.
template <class CFG>
__device__ __forceinline__ void attn_load_q(const int8_t *qkv, const int32_t *offsets, int item, int t, uint8_t *sq,
                                            int tid) {
    const int img = item / 3, head = item - img * 3;
    const int row0 = offsets[img], n = offsets[img + 1] - row0;
    for (int c = tid; c < 128 * 4; c += CFG::THREADS) {
        const int r = c >> 2, ch = c & 3, gr = t * 128 + r;
        const int8_t *src = qkv + (size_t)(row0 + (gr < n ? gr : 0)) * 576 + head * 64 + ch * 16;
        const uint32_t dst = tc05::smem_u32(sq + tc05::kmajor_offset(r, ch * 16, 64));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(gr < n ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// Barrier of the SPLIT warps that share TMEM lane quadrant `quad` (ids 1..4).
template <class CFG>
__device__ __forceinline__ void quad_sync(int quad) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(1 + quad), "r"(32 * CFG::SPLIT) : "memory");
}

template <bool FAST, class CFG>
__global__ void __launch_bounds__(CFG::THREADS) attention_tc_kernel(const int8_t *__restrict__ qkv,
                                                               const int32_t *__restrict__ offsets,
                                                               int8_t *__restrict__ ctx, AttnParams p,
                                                               int *__restrict__ err, int items, int np_lo,
                                                               int np_hi) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sQ = smem + CFG::OFF_Q;
    uint8_t *sP = smem + CFG::OFF_P;
    int32_t *sred = (int32_t *)(smem + CFG::OFF_RED);
    uint64_t *bar = (uint64_t *)(smem + CFG::OFF_BAR);
    uint32_t *tmem_slot = (uint32_t *)(smem + CFG::OFF_BAR + 8);
    volatile int *abort_flag = (volatile int *)(smem + CFG::OFF_BAR + 12);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, part = warp >> 2;
    const int lrow = quad * 32 + lane;  // tile row = TMEM lane

    if (warp == 0) {
        tc05::tmem_alloc(tmem_slot, CFG::TMEM_COLS);
        tc05::tmem_relinquish();
    }
    if (tid == 0) {
        tc05::mbar_init(bar, 1);
        *abort_flag = 0;
        tc05::fence_mbar_init();
    }
    griddep_wait();  // QKV and the offsets come from earlier kernels
    griddep_launch();
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tmem_slot;
    const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
    uint32_t phase = 0;

    // Persistent: the CTA's items are blockIdx.x + j * gridDim.x.  Its threads test a
    // batch of THREADS candidates at once (one offsets read each) and list the items
    // of this CTA shape; the CTA then processes the list.
    __shared__ int s_items[CFG::THREADS];
    __shared__ int s_nitems;
    for (int jb = 0; blockIdx.x + jb * gridDim.x < items && !*abort_flag; jb += CFG::THREADS) {
    if (tid == 0) s_nitems = 0;
    __syncthreads();
    {
        const int it = blockIdx.x + (jb + tid) * gridDim.x;
        if (it < items) {
            const int im = it / 3;
            const int nn = offsets[im + 1] - offsets[im];
            const int npp = (nn + 31) & ~31;
            if (nn > 0 && npp > np_lo && npp <= np_hi) s_items[atomicAdd(&s_nitems, 1)] = it;
        }
    }
    __syncthreads();
    const int nlist = s_nitems;
    if (nlist > 0) {
        attn_load_kv<CFG>(qkv, offsets, s_items[0], smem + CFG::OFF_KV, tid);
        attn_load_q<CFG>(qkv, offsets, s_items[0], 0, sQ, tid);
    }
    for (int li = 0; li < nlist && !*abort_flag; ++li) {
    const int item = s_items[li];
    const int img = item / 3, head = item - img * 3;
    const int row0 = offsets[img];
    const int n = offsets[img + 1] - row0;
    const int np = (n + 31) & ~31;
    // This item's K/V copies (issued during the previous item) land; then the next
    // item's copies go to the other buffer, whose last reader (that item's P.V) has
    // completed.
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    uint8_t *sK = smem + CFG::OFF_KV + (li & 1) * 2 * CFG::KV;
    uint8_t *sV = sK + CFG::KV;
    if (li + 1 < nlist)
        attn_load_kv<CFG>(qkv, offsets, s_items[li + 1], smem + CFG::OFF_KV + ((li + 1) & 1) * 2 * CFG::KV, tid);
    const uint32_t sbo_np = (uint32_t)(np / 16) * 128;
    const int nchunks = np >> 4;       // 16-column chunks of P
    const int nvalid = (n + 15) >> 4;  // chunks holding at least one real column

    for (int t = 0; t * 128 < n; ++t) {
        // ---- Q tile: its copies were issued when the previous P.V completed --------
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        tc05::fence_proxy_async();
        tc05::fence_before();
        __syncthreads();
        if (tid == 0) {
            tc05::fence_after();
            const uint32_t idesc = tc05::idesc_i8(128, np, true, true);
#pragma unroll
            for (int s = 0; s < 2; ++s)
                tc05::mma_i8_ss(tbase, tc05::smem_desc(tc05::smem_u32(sQ) + s * 256, 128, 512),
                                tc05::smem_desc(tc05::smem_u32(sK) + s * 256, 128, 512), idesc, s);
            tc05::commit(bar);
        }
        if (tc05::mbar_wait(bar, phase, WAIT_ITERS)) phase ^= 1;
        else *abort_flag = 1;
        __syncthreads();
        if (*abort_flag) break;
        tc05::fence_after();

        // ---- softmax straight from TMEM: this warp's rows, 16-column chunks c = part + CFG::SPLIT*i
        // q16 is monotone in the accumulator, so the row max is taken on raw
        // accumulators and converted once.
        const bool live = t * 128 + quad * 32 < n;  // warp-uniform
        const int nfull = n & ~15;
        if (live) {
            int32_t mxa = INT32_MIN;
            for (int c = part; c < nvalid; c += CFG::SPLIT) {
                const int c0 = c * 16;
                uint32_t v[16];
                tc05::ld16(lane_addr + c0, v);
                tc05::wait_ld();
                if (c0 < nfull) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) mxa = max(mxa, (int32_t)v[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c0 + j < n) mxa = max(mxa, (int32_t)v[j]);
                }
            }
            sred[part * 128 + lrow] = mxa;
            quad_sync<CFG>(quad);  // the SPLIT warps of this lane quadrant (live is quad-uniform)
            int32_t mraw = sred[lrow];
#pragma unroll
            for (int q = 1; q < CFG::SPLIT; ++q) mraw = max(mraw, sred[q * 128 + lrow]);
            const int32_t mx = q16_of<FAST>(mraw, p);
            const int32_t cmn =
                (int32_t)(((int64_t)1 << p.fast_shift) - 1 - p.fast_half + ((int64_t)mx << p.fast_shift));
            uint32_t sum = 0;
            for (int c = part; c < nvalid; c += CFG::SPLIT) {
                const int c0 = c * 16;
                uint32_t v[16];
                tc05::ld16(lane_addr + c0, v);
                tc05::wait_ld();
                if (c0 < nfull) sum += chunk_exp<FAST, false>(v, 16, mx, cmn, p);
                else sum += chunk_exp<FAST, true>(v, n - c0, mx, cmn, p);
                tc05::st16(lane_addr + c0, v);
            }
            tc05::wait_st();
            sred[(CFG::SPLIT + part) * 128 + lrow] = (int32_t)sum;
            quad_sync<CFG>(quad);
            uint32_t tot = 0;
#pragma unroll
            for (int q = 0; q < CFG::SPLIT; ++q) tot += (uint32_t)sred[(CFG::SPLIT + q) * 128 + lrow];
            const uint64_t rc = softmax_recip(tot ? tot : 1u);
            for (int c = part; c < nchunks; c += CFG::SPLIT) {
                const int c0 = c * 16;
                if (c >= nvalid) {  // padding columns: zero probabilities
                    *(uint4 *)(sP + tc05::kmajor_offset(lrow, c0, np)) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                uint32_t v[16];
                tc05::ld16(lane_addr + c0, v);
                tc05::wait_ld();
                uint32_t pk[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    int32_t pr[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        // rsa(rsa(E*rc, 16), 8) in one rounding step (nested floors); <= 256,
                        // and the saturating pack applies the min(., 255)
                        const uint64_t tt = (uint64_t)v[w * 4 + b] * rc + (32768u + (1u << 23));
                        pr[b] = (int32_t)(tt >> 24);
                    }
                    pk[w] = pack_satu8(pr[0], pr[1], pr[2], pr[3]);
                }
                *(uint4 *)(sP + tc05::kmajor_offset(lrow, c0, np)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
        }

        // ---- ctx = P·V (rows of dead warps hold stale probabilities; their ctx rows are not stored)
        tc05::fence_proxy_async();
        tc05::fence_before();
        __syncthreads();
        if (tid == 0) {
            tc05::fence_after();
            const uint32_t idesc = tc05::idesc_i8(128, 64, false, true, true);
            for (int s = 0; s < np / 32; ++s)
                tc05::mma_i8_ss(tbase, tc05::smem_desc(tc05::smem_u32(sP) + s * 256, 128, sbo_np),
                                tc05::smem_desc(tc05::smem_u32(sV) + s * 2048, 512, 128), idesc, s);
            tc05::commit(bar);
        }
        if (tc05::mbar_wait(bar, phase, WAIT_ITERS)) phase ^= 1;
        else *abort_flag = 1;
        __syncthreads();
        if (*abort_flag) break;
        tc05::fence_after();
        // P (and with it the Q buffer it overlays) is free: the next tile's Q copies
        // overlap this tile's context epilogue
        if ((t + 1) * 128 < n) attn_load_q<CFG>(qkv, offsets, item, t + 1, sQ, tid);
        else if (li + 1 < nlist) attn_load_q<CFG>(qkv, offsets, s_items[li + 1], 0, sQ, tid);
        const int r = t * 128 + lrow;
        if (live) {
            for (int pc = part; pc < 4; pc += CFG::SPLIT) {  // 16-column pieces of the 64 head dims
                uint32_t o[16];
                tc05::ld16(lane_addr + pc * 16, o);
                tc05::wait_ld();
                uint32_t pk[4];
#pragma unroll
                for (int w = 0; w < 4; ++w) {
                    int32_t q[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int32_t a = (int32_t)o[w * 4 + b];
                        q[b] = p.ctx_fast ? rsa32(a, p.ctx_shift) : (int32_t)requant64(a, p.ctx_shift, 8);
                    }
                    pk[w] = pack_sat8(q[0], q[1], q[2], q[3]);
                }
                if (r < n)
                    *(uint4 *)(ctx + (size_t)(row0 + r) * 192 + head * 64 + pc * 16) =
                        make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
        }
        tc05::fence_before();
        __syncthreads();
    }
    }  // listed items
    __syncthreads();  // s_items is rewritten by the next batch
    }  // candidate batches

    asm volatile("cp.async.wait_all;\n" ::: "memory");  // a prefetch may be left after an abort
    if (*abort_flag) {
        if (tid == 0) atomicExch(err, 1);
        // let any MMA still in flight drain (bounded) before the TMEM is released
        tc05::mbar_wait(bar, phase, WAIT_ITERS);
    }
    __syncthreads();
    if (warp == 0) {
        tc05::fence_after();
        tc05::tmem_dealloc(tbase, CFG::TMEM_COLS);
    }
}

}  // namespace

AttnParams make_attn(int qkv_out_scale, int score_scale, int prob_scale, int context_out_scale) {
    AttnParams a;
    a.score_shift = score_scale - 2 * qkv_out_scale;
    a.q16_shift = -(score_scale + 13);
    a.ctx_shift = context_out_scale - (prob_scale + qkv_out_scale);
    const int k = -a.score_shift;
    a.fast = (k >= 0 && k <= 10 && a.q16_shift >= k && a.q16_shift - k <= 30) ? 1 : 0;
    a.fast_shift = a.fast ? a.q16_shift - k : 0;
    a.fast_half = a.fast_shift ? (1 << (a.fast_shift - 1)) : 0;
    a.fast_negmask = a.fast_shift ? -1 : 0;
    a.ctx_fast = (a.ctx_shift >= 1 && a.ctx_shift <= 30) ? 1 : 0;
    return a;
}

cudaError_t launch_attention(const int8_t *qkv, const int32_t *offsets, int images, int8_t *ctx,
                             const AttnParams &p, int may_be_short, int sms, int *err, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    const int items = images * 3;
    // Images of up to 128 tokens (np <= 128) go to the small shape when any may exist.
    if (may_be_short) {
        auto ks = p.fast ? attention_tc_kernel<true, AttnSmall> : attention_tc_kernel<false, AttnSmall>;
        cudaError_t e = cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnSmall::SMEM);
        if (e != cudaSuccess) return e;
        e = launch_pdl(ks, dim3(std::min(items, sms * 4)), dim3(AttnSmall::THREADS), AttnSmall::SMEM, st, qkv, offsets,
                       ctx, p, err, items, 0, 128);
        if (e != cudaSuccess) return e;
    }
    auto kl = p.fast ? attention_tc_kernel<true, AttnLarge> : attention_tc_kernel<false, AttnLarge>;
    cudaError_t e = cudaFuncSetAttribute(kl, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnLarge::SMEM);
    if (e != cudaSuccess) return e;
    return launch_pdl(kl, dim3(std::min(items, sms * 2)), dim3(AttnLarge::THREADS), AttnLarge::SMEM, st, qkv, offsets,
                      ctx, p, err, items, may_be_short ? 128 : 0, AttnLarge::NPMAX);
}

}  // namespace hv
