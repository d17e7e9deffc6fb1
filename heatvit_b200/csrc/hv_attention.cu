// hv_attention.cu — per-(image, head) attention on tcgen05 tensor cores and TMEM.
//
// Restates transformer.py:230-268 for one image and head:
//   score = requant(Q·Kᵀ, 2q, score_scale, 32)            (int32 writeback)
//   q16   = sat24(rsa(score, -(score_scale + 13)))         (Q8.16)
//   prob  = softmax_attention(q16 row)                     (UQ0.8, nonlinear.py:98-133)
//   ctx   = requant(prob(uint8)·V, prob_scale + q, context_out, 8)
// written straight into the head-concatenated layout (layout.py:132-155).
//
// Work units (hv_attn_units.cuh) are listed once per token layout by the kernel that
// makes the layout: the batch set-up, the token packer after every selector, or
// attn_plan_kernel for a layout given by the caller.  A unit is one 128-row tile of
// query rows.
//   * n > 128 tokens (list B): one unit per (head, 128-row half): 6 per image.
//   * 64 < n <= 128 (list A): one unit per head.
//   * 32 < n <= 64 (list A): heads {0, 1} packed in one tile (64 rows each), head 2
//     alone.
//   * n <= 32 (list A): the three heads packed in one tile (32 rows each).
// A packed tile stacks the heads' Q rows, K rows and V rows in slots of R = 64 or
// 32 rows; S = Q·Kᵀ then holds every head's scores in its diagonal R x R block,
// and P is written block-diagonal (zero outside the row's own block), so one
// P·V over all 128 stacked V rows gives each row its own head's context.
//
// Launches: list B's shape (SPL = 4) walks list B and, for batches of at most 3
// images per SM, list A after it in the same launch; larger batches give list A a
// launch of its own in the SPL = 1 shape.
// Per unit (CTA of 4 x SPL warps, persistent over its units):
//   1. K, V and Q are staged in shared memory with 16-byte cp.async copies in the
//      no-swizzle canonical layout (hv_tc05.cuh); K and Q are K-major operands, V is
//      the same byte layout read as an MN-major B operand (tokens along K).  Each
//      has one buffer: the next unit's K and Q are copied as soon as this unit's
//      S = Q·Kᵀ has completed (during the softmax), its V as soon as this unit's
//      P·V has (during the context writeback).
//   2. One thread issues S = Q·Kᵀ (tcgen05.mma kind::i8, M = 128) into TMEM.
//   3. Query row r is TMEM lane r.  The SPL warps of lane quadrant r / 32 read the
//      row in 16-column pieces dealt round-robin among them; each thread takes the
//      max, exp terms and sum of its share of its row, the SPL partials of a row
//      are combined through shared memory behind a named barrier of the quadrant's
//      warps (with SPL = 1 the thread owns the whole row and nothing is exchanged),
//      the exp terms go back to TMEM, then the UQ0.8 probabilities to shared memory
//      as the A operand of the next MMA.
//   4. ctx = P·V (unsigned A) into TMEM columns [0, 64), requantised and stored.
// TMEM: 128 columns per CTA in the SPL = 1 shape (4 CTAs per SM), 256 in the SPL = 4
// shape (2 per SM).
#include <algorithm>

#include "hv_attn_units.cuh"
#include "hv_internal.cuh"
#include "hv_tc05.cuh"

namespace hv {

namespace {

constexpr uint32_t WAIT_ITERS = 1u << 24;

// One CTA (1024 threads) lists every unit of the batch, image-major.  cnt[0], cnt[1]
// = lengths of list A and list B.
__global__ void __launch_bounds__(1024) attn_plan_kernel(const int32_t *__restrict__ offsets, int images,
                                                          uint2 *__restrict__ list_a,
                                                          uint2 *__restrict__ list_b, int32_t *__restrict__ cnt) {
    griddep_wait();
    griddep_launch();
    __shared__ int wsum[2][32];
    __shared__ int base[2];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) base[0] = base[1] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < images; i0 += 1024) {
        const int img = i0 + tid;
        const int n = img < images ? offsets[img + 1] - offsets[img] : 0;
        const int ca = units_a(n), cb = units_b(n);
        int sa = ca, sb = cb;  // inclusive warp scans
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ta = __shfl_up_sync(0xffffffffu, sa, o), tb = __shfl_up_sync(0xffffffffu, sb, o);
            if (lane >= o) {
                sa += ta;
                sb += tb;
            }
        }
        if (lane == 31) {
            wsum[0][warp] = sa;
            wsum[1][warp] = sb;
        }
        __syncthreads();
        int pa = base[0], pb = base[1];
        for (int w = 0; w < warp; ++w) {
            pa += wsum[0][w];
            pb += wsum[1][w];
        }
        pa += sa - ca;  // exclusive position of this image's first unit
        pb += sb - cb;
        if (img < images) write_image_units(list_a, list_b, pa, pb, img, offsets[img], n);
        __syncthreads();
        if (tid == 0) {
            int ta = 0, tb = 0;
            for (int w = 0; w < 32; ++w) {
                ta += wsum[0][w];
                tb += wsum[1][w];
            }
            base[0] += ta;
            base[1] += tb;
        }
        __syncthreads();
    }
    if (tid == 0) {
        cnt[0] = base[0];
        cnt[1] = base[1];
    }
}

// Two CTA shapes: list A units need at most 128 S columns (TMEM 128, four CTAs per
// SM), list B units at most 224 (TMEM 256, two per SM).  SPL warps share each TMEM
// lane quadrant: a row's 32-column pieces are dealt round-robin to them, and they
// combine the row max and sum through shared memory.  Shared memory is padded so
// that the resident CTAs never ask for more than the SM's 512 TMEM columns.
// Arguments n = max - q16 below kSmallN (a quarter of ln2 in Q8.16, so z = 0) read
// their exp term from a table in shared memory: softmax_exp_q16_n(n) = tab[n].
constexpr int kSmallN = 2048;

template <int NPM, int SPL, bool DBUF>
struct AttnCfg {
    static constexpr int SPLIT = SPL;
    static constexpr bool DB = DBUF;
    static constexpr int THREADS = 128 * SPL;
    static constexpr int PER_SM = NPM <= 128 ? 4 : 2;   // resident CTAs (TMEM-limited)
    static constexpr uint32_t TMEM_COLS = NPM <= 128 ? 128 : 256;
    static constexpr int KV = NPM * 64;                 // one [NPMAX][64] operand
    static constexpr int OFF_K = 0;                     // K [NPMAX][64]
    static constexpr int OFF_V = OFF_K + KV;            // V [NPMAX][64]
    static constexpr int OFF_Q = OFF_V + KV;            // Q [128][64]
    static constexpr int OFF_P = OFF_Q + 128 * 64;      // P [128][NPMAX] uint8
    static constexpr int OFF_TAB = OFF_P + 128 * NPM;   // exp terms of small arguments [kSmallN] uint32
    static constexpr int OFF_RED = OFF_TAB + kSmallN * 4;  // [2][SPL][128] int32 row partials
    static constexpr int OFF_BAR = OFF_RED + 2 * SPL * 128 * 4;  // mbarrier, TMEM base, abort flag
    static constexpr int USED = (OFF_BAR + 64 + 1023) / 1024 * 1024;
    // padded so that no more CTAs fit an SM than its 512 TMEM columns hold
    static constexpr int MIN = NPM <= 128 ? 46 * 1024 : 77 * 1024;
    static constexpr int SMEM = USED > MIN ? USED : MIN;
    static_assert(NPM <= 128 ? (5 * SMEM > 228 * 1024 && 4 * (SMEM + 1024) <= 228 * 1024)
                             : (3 * SMEM > 228 * 1024 && 2 * (SMEM + 1024) <= 228 * 1024),
                  "attention shared memory sizing");
};

// Runs f(v, c) over the 16-column pieces c = c0, c0 + step, ... < cend of a TMEM row
// (address addr + 16c).  DB: double-buffered, the next piece's tcgen05.ld is in
// flight while f works on the current one (16 more registers).  All arguments are
// warp-uniform.
template <bool DB, class F>
__device__ __forceinline__ void for_pieces(uint32_t addr, int c0, int step, int cend, F &&f) {
    if (c0 >= cend) return;
    if (!DB) {
        for (int c = c0; c < cend; c += step) {
            uint32_t a[16];
            tc05::ld16(addr + c * 16, a);
            tc05::wait_ld_regs(a);
            f(a, c);
        }
        return;
    }
    uint32_t a[16], b[16];
    int c = c0;
    tc05::ld16(addr + c * 16, a);
    while (true) {
        tc05::wait_ld_regs(a);
        const int c1 = c + step;
        if (c1 < cend) tc05::ld16(addr + c1 * 16, b);
        f(a, c);
        if (c1 >= cend) break;
        tc05::wait_ld_regs(b);
        const int c2 = c1 + step;
        if (c2 < cend) tc05::ld16(addr + c2 * 16, a);
        f(b, c1);
        if (c2 >= cend) break;
        c = c2;
    }
}

// Barrier of the SPLIT warps that share TMEM lane quadrant `quad` (ids 1..4).
template <class CFG>
__device__ __forceinline__ void quad_sync(int quad) {
    if (CFG::SPLIT > 1) asm volatile("bar.sync %0, %1;\n" ::"r"(1 + quad), "r"(32 * CFG::SPLIT) : "memory");
}

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
    // (with fast_shift = 0 the mask is 0 and cmn = mx: mx - acc)
    if (FAST) return (uint32_t)((cmn - acc - ((acc >> 31) & p.fast_negmask)) >> p.fast_shift);
    return (uint32_t)(mx - q16_of<false>(acc, p));
}

// Exp terms of one 16-column piece (columns >= valid give 0 when MASK); returns their
// sum.  When every argument of the warp's piece is below kSmallN (one vote), the terms
// come from the table `tab` instead of the arithmetic; both are exact.
template <bool FAST, bool MASK>
__device__ __forceinline__ uint32_t piece_exp(uint32_t (&v)[16], int valid, int32_t mx, int32_t cmn,
                                              const AttnParams &p, const uint32_t *tab) {
    uint32_t orv = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        uint32_t nn = negxt_of<FAST>((int32_t)v[j], mx, cmn, p);
        if (MASK && j >= valid) nn = 0u;  // (its term is zeroed below)
        v[j] = nn;
        orv |= nn;
    }
    if (__all_sync(0xffffffffu, orv < (uint32_t)kSmallN)) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = tab[v[j]];
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = softmax_exp_q16_n(v[j]);
    }
    if (MASK) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j >= valid) v[j] = 0u;
    }
    // pairwise tree: a dependency depth of 4 instead of a chain of 16 adds
    uint32_t s8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) s8[j] = v[2 * j] + v[2 * j + 1];
#pragma unroll
    for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) s8[j] += s8[j + w];
    return s8[0];
}

// Exp terms of a warp's 4 tail columns, the first `valid` of them real (the rest
// give 0); returns their sum.  Same table / arithmetic choice as piece_exp.
template <bool FAST>
__device__ __forceinline__ uint32_t tail_exp(uint32_t (&v)[4], int valid, int32_t mx, int32_t cmn,
                                             const AttnParams &p, const uint32_t *tab) {
    uint32_t orv = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t nn = negxt_of<FAST>((int32_t)v[j], mx, cmn, p);
        if (j >= valid) nn = 0u;
        v[j] = nn;
        orv |= nn;
    }
    if (__all_sync(0xffffffffu, orv < (uint32_t)kSmallN)) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = tab[v[j]];
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = softmax_exp_q16_n(v[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (j >= valid) v[j] = 0u;
    return (v[0] + v[1]) + (v[2] + v[3]);
}

// Largest of 16 values (the first `valid` when MASK), as a pairwise tree.
template <bool MASK>
__device__ __forceinline__ int32_t piece_max(const uint32_t (&v)[16], int valid) {
    int32_t m[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int32_t a = (MASK && 2 * j >= valid) ? INT32_MIN : (int32_t)v[2 * j];
        const int32_t b = (MASK && 2 * j + 1 >= valid) ? INT32_MIN : (int32_t)v[2 * j + 1];
        m[j] = max(a, b);
    }
#pragma unroll
    for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) m[j] = max(m[j], m[j + w]);
    return m[0];
}

struct Unit {
    int img, mt, glog, h0, nh;
    int row0, n;
};

// A list entry: {unit code, row0 << 8 | n} (attn_plan_kernel).
__device__ __forceinline__ Unit decode_unit(uint2 e) {
    const uint32_t code = e.x;
    Unit u;
    u.img = (int)(code >> 7);
    u.mt = (code >> 6) & 1;
    u.glog = (code >> 4) & 3;
    u.h0 = (code >> 2) & 3;
    u.nh = code & 3;
    u.row0 = (int)(e.y >> 8);
    u.n = (int)(e.y & 0xffu);
    return u;
}

// K (V = 0) or V (V = 1) rows of a unit, K-major bytes, as one cp.async group.  Slot
// j (head h0 + j) occupies rows [j*R, j*R + R) with R = 128 >> glog (G = 1: R = np);
// rows past the image are zero-filled (src-size 0).
template <class CFG, int V>
__device__ __forceinline__ void load_kv(const int8_t *qkv, const Unit &u, uint8_t *dst_buf, int tid) {
    const int R = u.glog ? (128 >> u.glog) : ((u.n + 31) & ~31);
    const int rows = R * u.nh;
    const int rsh = 7 - u.glog;  // packed slots: R = 2^rsh
    for (int c = tid; c < rows * 4; c += CFG::THREADS) {
        const int r = c >> 2, ch = c & 3;
        const int j = u.glog ? r >> rsh : 0, t = r - j * R;
        const int8_t *src = qkv + (size_t)(u.row0 + (t < u.n ? t : 0)) * 576 + 192 * (1 + V) + (u.h0 + j) * 64 + ch * 16;
        const uint32_t dst = tc05::smem_u32(dst_buf + tc05::kmajor_offset(r, ch * 16, 64));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(t < u.n ? 16 : 0)
                     : "memory");
    }
}

// The unit's 128 query rows into the K-major Q buffer (rows past the image zero-filled).
template <class CFG>
__device__ __forceinline__ void load_q(const int8_t *qkv, const Unit &u, uint8_t *sq, int tid) {
    const int rsh = 7 - u.glog;  // slot rows R = 2^rsh (128 when unpacked)
    const int R = 1 << rsh;
    for (int c = tid; c < 128 * 4; c += CFG::THREADS) {
        const int r = c >> 2, ch = c & 3;
        const int j = r >> rsh;
        const int t = u.glog ? r - j * R : u.mt * 128 + r;
        const bool ok = j < u.nh && t < u.n;
        const int8_t *src = qkv + (size_t)(u.row0 + (ok ? t : 0)) * 576 + (u.h0 + (ok ? j : 0)) * 64 + ch * 16;
        const uint32_t dst = tc05::smem_u32(sq + tc05::kmajor_offset(r, ch * 16, 64));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
                     : "memory");
    }
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
// Wait until at most one (the newest) cp.async group of this thread is pending.
__device__ __forceinline__ void cp_wait_all_but_newest() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

template <bool FAST, class CFG>
__global__ void __launch_bounds__(CFG::THREADS, CFG::PER_SM) attention_tc_kernel(const int8_t *__restrict__ qkv,
                                                               int8_t *__restrict__ ctx, AttnParams p,
                                                               int *__restrict__ err,
                                                               const uint2 *__restrict__ list1,
                                                               const int32_t *__restrict__ count1,
                                                               const uint2 *__restrict__ list2,
                                                               const int32_t *__restrict__ count2) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *sP = smem + CFG::OFF_P;
    uint8_t *sQ = smem + CFG::OFF_Q;
    uint8_t *sK = smem + CFG::OFF_K;
    uint8_t *sV = smem + CFG::OFF_V;
    uint64_t *bar = (uint64_t *)(smem + CFG::OFF_BAR);
    uint32_t *tmem_slot = (uint32_t *)(smem + CFG::OFF_BAR + 8);
    volatile int *abort_flag = (volatile int *)(smem + CFG::OFF_BAR + 12);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quad = warp & 3, part = warp >> 2;
    const int lrow = quad * 32 + lane;  // tile row = TMEM lane
    int32_t *sred = (int32_t *)(smem + CFG::OFF_RED);
    uint32_t *stab = (uint32_t *)(smem + CFG::OFF_TAB);
    for (int i = tid; i < kSmallN; i += CFG::THREADS) stab[i] = softmax_exp_q16_n((uint32_t)i);

    if (warp == 0) {
        tc05::tmem_alloc(tmem_slot, CFG::TMEM_COLS);
        tc05::tmem_relinquish();
    }
    if (tid == 0) {
        tc05::mbar_init(bar, 1);
        *abort_flag = 0;
        tc05::fence_mbar_init();
    }
    griddep_wait();  // QKV, the offsets and the unit list come from earlier kernels
    griddep_launch();
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tmem_slot;
    const uint32_t lane_addr = tbase + ((uint32_t)(quad * 32) << 16);
    uint32_t phase = 0;
    // one index space over one or two lists (list B's units, 6 per long image, come
    // first when both are walked, so the longest units start first)
    const int n1 = *count1, units = n1 + (count2 ? *count2 : 0);
    auto entry = [&](int i) { return i < n1 ? list1[i] : list2[i - n1]; };
    const int stride = gridDim.x;

    // cp.async groups, oldest first: [K, Q] of a unit (issued once the previous unit's
    // S = Q.K^T has completed), then [V] of it (once the previous unit's P.V has).
    // The entry of the unit after the next is loaded one unit ahead, so that its
    // latency hides behind a whole unit's work.
    Unit cur;
    uint2 ahead = make_uint2(0, 0);
    if ((int)blockIdx.x + stride < units) ahead = entry(blockIdx.x + stride);
    if ((int)blockIdx.x < units) {
        cur = decode_unit(entry(blockIdx.x));
        load_kv<CFG, 0>(qkv, cur, sK, tid);
        load_q<CFG>(qkv, cur, sQ, tid);
        cp_commit();
        load_kv<CFG, 1>(qkv, cur, sV, tid);
        cp_commit();
    }
    for (int ui = blockIdx.x; ui < units && !*abort_flag; ui += stride) {
        const Unit u = cur;
        cp_wait_all_but_newest();  // this unit's K and Q have landed (its V may not have)
        tc05::fence_proxy_async();
        tc05::fence_before();
        __syncthreads();
        const bool more = ui + stride < units;
        const int np = (u.n + 31) & ~31;
        const int scols = u.glog ? 128 : np;  // S columns = K rows = P columns
        // ---- S = Q.K^T ----------------------------------------------------------------
        if (tid == 0) {
            tc05::fence_after();
            const uint32_t idesc = tc05::idesc_i8(128, scols, true, true);
#pragma unroll
            for (int s = 0; s < 2; ++s)
                tc05::mma_i8_ss(tbase, tc05::smem_desc(tc05::smem_u32(sQ) + s * 256, 128, 512),
                                tc05::smem_desc(tc05::smem_u32(sK) + s * 256, 128, 512), idesc, s);
            tc05::commit(bar);
        }
        // Every thread sees the MMA complete on the mbarrier itself (the next MMA is
        // issued only after a barrier that every thread reaches after this wait, so
        // none can miss the phase); a wait that gave up is acted on at that barrier.
        if (tc05::mbar_wait(bar, phase, WAIT_ITERS)) phase ^= 1;
        else *abort_flag = 1;
        tc05::fence_after();
        // K and Q are consumed: the next unit's copies overlap this unit's softmax
        if (more) {
            cur = decode_unit(ahead);
            if (ui + 2 * stride < units) ahead = entry(ui + 2 * stride);
            load_kv<CFG, 0>(qkv, cur, sK, tid);
            load_q<CFG>(qkv, cur, sQ, tid);
        }
        cp_commit();  // (an empty group when there is no next unit)

        // ---- this thread's row: slot j (head h0 + j), local row t, S columns [cb, cb + np);
        // this part's pieces are c = part, part + SPLIT, ...
        const int R = u.glog ? (128 >> u.glog) : 128;
        const int j = lrow / R;  // quadrant-uniform (R >= 32)
        const int t = u.glog ? lrow - j * R : u.mt * 128 + lrow;
        const int cb = u.glog ? j * R : 0;
        const int t0 = u.glog ? quad * 32 - j * R : u.mt * 128 + quad * 32;  // the quadrant's first row
        const bool live = j < u.nh && t0 < u.n;                            // quadrant-uniform
        const uint32_t row_addr = lane_addr + cb;
        const int nv = (u.n + 15) >> 4, nfull = u.n >> 4;  // 16-column pieces: with a column / all full
        constexpr int SP = CFG::SPLIT;
        // With 4 warps per quadrant the full pieces are dealt round-robin and a partial
        // last piece is split instead, 4 columns per warp (13 pieces at 197 tokens
        // would otherwise give one warp 4 pieces and the others 3).
        constexpr bool TAILS = SP == 4;
        const int npc = TAILS ? nfull : nv;                    // pieces dealt round-robin
        const bool has_tail = TAILS && (u.n & 15);             // unit-uniform
        const int tcol = nfull * 16 + 4 * part;                // this warp's tail columns
        const int tval = min(4, max(0, u.n - tcol));           // real ones among them
        if (live) {
            // q16 is monotone in the accumulator: the row max is taken on raw values
            int32_t mxa = INT32_MIN;
            for_pieces<CFG::DB>(row_addr, part, SP, npc, [&](uint32_t (&v)[16], int c) {
                mxa = max(mxa, c < nfull ? piece_max<false>(v, 16) : piece_max<true>(v, u.n - c * 16));
            });
            if (has_tail) {
                uint32_t w[4];
                tc05::ld4(row_addr + tcol, w);
                tc05::wait_ld_regs(w);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < tval) mxa = max(mxa, (int32_t)w[j]);
            }
            if (SP > 1) {
                sred[part * 128 + lrow] = mxa;
                quad_sync<CFG>(quad);
#pragma unroll
                for (int q = 0; q < SP; ++q) mxa = max(mxa, sred[q * 128 + lrow]);
            }
            const int32_t mx = q16_of<FAST>(mxa, p);
            const int32_t cmn =
                (int32_t)(((int64_t)1 << p.fast_shift) - 1 - p.fast_half + ((int64_t)mx << p.fast_shift));
            uint32_t sum = 0;
            for_pieces<CFG::DB>(row_addr, part, SP, npc, [&](uint32_t (&v)[16], int c) {
                if (c < nfull) sum += piece_exp<FAST, false>(v, 16, mx, cmn, p, stab);
                else sum += piece_exp<FAST, true>(v, u.n - c * 16, mx, cmn, p, stab);
                tc05::st16(row_addr + c * 16, v);
            });
            if (has_tail) {
                uint32_t w[4];
                tc05::ld4(row_addr + tcol, w);
                tc05::wait_ld_regs(w);
                sum += tail_exp<FAST>(w, tval, mx, cmn, p, stab);
                tc05::st4(row_addr + tcol, w);
            }
            tc05::wait_st();
            if (SP > 1) {
                sred[(SP + part) * 128 + lrow] = (int32_t)sum;
                quad_sync<CFG>(quad);
                sum = 0;
#pragma unroll
                for (int q = 0; q < SP; ++q) sum += (uint32_t)sred[(SP + q) * 128 + lrow];
            }
            // S >= exp(0) = 65554 (the max element), so rc = round_div(2^32, S) <= 65519
            // and the products below fit a 32 x 32 -> 64-bit multiply
            const uint32_t rc = softmax_recip32(sum);
            // P row: the own block's probabilities, zeros in every other column
            const int cb16 = cb >> 4;
            for_pieces<CFG::DB>(row_addr, part, SP, npc, [&](uint32_t (&v)[16], int c) {
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
                *(uint4 *)(sP + tc05::kmajor_offset(lrow, (cb16 + c) * 16, scols)) =
                    make_uint4(pk[0], pk[1], pk[2], pk[3]);
            });
            if (has_tail) {  // this warp's 4 bytes of the partial piece (zeros past the row)
                uint32_t w[4];
                tc05::ld4(row_addr + tcol, w);
                tc05::wait_ld_regs(w);
                int32_t pr[4];
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    pr[b] = (int32_t)(((uint64_t)w[b] * rc + (32768u + (1u << 23))) >> 24);
                *(uint32_t *)(sP + tc05::kmajor_offset(lrow, (cb16 + nfull) * 16, scols) + 4 * part) =
                    pack_satu8(pr[0], pr[1], pr[2], pr[3]);
            }
            for (int c = part; c < scols / 16; c += SP)
                if (c < cb16 || c >= cb16 + nv)
                    *(uint4 *)(sP + tc05::kmajor_offset(lrow, c * 16, scols)) = make_uint4(0, 0, 0, 0);
        }

        // ---- ctx = P.V (rows of dead warps hold stale probabilities; their ctx rows are not stored)
        cp_wait_all_but_newest();  // this unit's V has landed (the next unit's K/Q may not have)
        tc05::fence_proxy_async();
        tc05::fence_before();
        __syncthreads();
        if (*abort_flag) break;
        if (tid == 0) {
            tc05::fence_after();
            const uint32_t idesc = tc05::idesc_i8(128, 64, false, true, true);
            const uint32_t sbo = (uint32_t)(scols / 16) * 128;
            for (int s = 0; s < scols / 32; ++s)
                tc05::mma_i8_ss(tbase, tc05::smem_desc(tc05::smem_u32(sP) + s * 256, 128, sbo),
                                tc05::smem_desc(tc05::smem_u32(sV) + s * 2048, 512, 128), idesc, s);
            tc05::commit(bar);
        }
        if (tc05::mbar_wait(bar, phase, WAIT_ITERS)) phase ^= 1;  // (as after S = Q.K^T)
        else *abort_flag = 1;
        tc05::fence_after();
        // V is consumed: the next unit's V copies overlap the rest of this unit
        if (more) load_kv<CFG, 1>(qkv, cur, sV, tid);
        cp_commit();
        if (live && SP == 4) {
            // one 16-column quarter of the row's 64 context columns per warp
            const int h = u.h0 + j;
            uint32_t o[16];
            tc05::ld16(lane_addr + part * 16, o);
            tc05::wait_ld_regs(o);
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
            if (t < u.n)
                *(uint4 *)(ctx + (size_t)(u.row0 + t) * 192 + h * 64 + part * 16) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        } else if (live) {
            const int h = u.h0 + j;
            for (int half = part; half < 2; half += CFG::SPLIT) {
                uint32_t o[32];
                tc05::ld32(lane_addr + half * 32, o);
                tc05::wait_ld();
                uint32_t pk[8];
#pragma unroll
                for (int w = 0; w < 8; ++w) {
                    int32_t q[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int32_t a = (int32_t)o[w * 4 + b];
                        q[b] = p.ctx_fast ? rsa32(a, p.ctx_shift) : (int32_t)requant64(a, p.ctx_shift, 8);
                    }
                    pk[w] = pack_sat8(q[0], q[1], q[2], q[3]);
                }
                if (t < u.n) {
                    uint4 *dst = (uint4 *)(ctx + (size_t)(u.row0 + t) * 192 + h * 64 + half * 32);
                    dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                }
            }
        }
        tc05::fence_before();
        __syncthreads();
    }

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

cudaError_t launch_attn_plan(const int32_t *offsets, int images, const AttnPlan &plan, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    return launch_pdl(attn_plan_kernel, dim3(1), dim3(1024), 0, st, offsets, images, plan.list_a, plan.list_b,
                      plan.cnt);
}

template <class CFG>
cudaError_t launch_one(const int8_t *qkv, int8_t *ctx, const AttnParams &p, int *err, const uint2 *list1,
                       const int32_t *count1, const uint2 *list2, const int32_t *count2, int grid,
                       cudaStream_t st) {
    auto k = p.fast ? attention_tc_kernel<true, CFG> : attention_tc_kernel<false, CFG>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, CFG::SMEM);
    if (e != cudaSuccess) return e;
    return launch_pdl(k, dim3(grid), dim3(CFG::THREADS), CFG::SMEM, st, qkv, ctx, p, err, list1, count1, list2,
                      count2);
}

cudaError_t launch_attention(const int8_t *qkv, const int32_t *offsets, int images, int8_t *ctx,
                             const AttnParams &p, int may_be_short, int sms, int *err, const AttnPlan &plan,
                             cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    const uint2 *la = plan.list_a, *lb = plan.list_b;
    const int32_t *ca = plan.cnt, *cb = plan.cnt + 1;
    const int gb = std::min(images * 6, sms * 2);
    // List B: four warps per TMEM lane quadrant splitting each row's pieces,
    // single-buffered (two CTAs of 16 warps per SM, 64 registers).  Up to 3 images
    // per SM, one launch of that shape walks list B and then list A (one launch
    // fewer per block); above that, list A has a launch of its own with one warp
    // per quadrant and double-buffered TMEM reads (four CTAs of 4 warps per SM),
    // which is faster per unit once its units fill the four CTAs per SM.
    if (!may_be_short || images <= 3 * sms)
        return launch_one<AttnCfg<224, 4, false>>(qkv, ctx, p, err, lb, cb, may_be_short ? la : nullptr,
                                                  may_be_short ? ca : nullptr, gb, st);
    cudaError_t e = launch_one<AttnCfg<128, 1, true>>(qkv, ctx, p, err, la, ca, nullptr, nullptr,
                                                      std::min(images * 3, sms * 4), st);
    if (e != cudaSuccess) return e;
    return launch_one<AttnCfg<224, 4, false>>(qkv, ctx, p, err, lb, cb, nullptr, nullptr, gb, st);
}

}  // namespace hv
