// hv_selector.cu — fused per-image token selector and ragged compaction.
//
// One CTA per image restates selector.py:503-563 end to end:
//   local MLP (253-270) -> global mean (273-289) -> score MLP with the global
//   half of layer 1 computed once per image (concat, 292-355) -> keep scores
//   via the 2-way selector softmax -> head stats (358-367) -> head-weight MLP
//   with PLAN (370-389) -> head fuse with its zero-denominator fallback
//   (392-418) -> inclusive 0.5 threshold, stable compaction and the package
//   token with its own zero-denominator fallback (421-500).
// Splitting layer 1 as [local ‖ global]·W1 = local·W1[0:32] + global·W1[32:64]
// is exact in integer arithmetic.
//
// The local MLP and score layers 1-2 run on tcgen05 (kind::i8, M = 128 over the
// image's token rows, one MMA per head and K step) with the exact GELU tables in
// their TMEM epilogues; the token rows and those layers' outputs are kept in the
// strip layout the tensor cores read (see STRIP).  Score layer 3, the softmaxes,
// the head statistics and head-weight MLP, the fuse and the compaction run on the
// CUDA cores.
//
// The output goes to a per-image staging slot (stride 197 rows); the pack
// kernel then prefix-sums the new counts and writes the packed ragged layout
// that every later kernel consumes.
#include "hv_attn_units.cuh"
#include "hv_internal.cuh"
#include "hv_tc05.cuh"

namespace hv {

namespace {

constexpr int THREADS = 512;
constexpr int MAXC = 196;
// Token rows and the two MLP activations live in the strip layout the tensor cores
// read: byte k of row r at (k / 16) * STRIP + r * 16 + k % 16, 197 rows per strip
// (no-swizzle K-major core matrices: LBO = STRIP, SBO = 128).
constexpr int STRIP = 197 * 16;
// Weights as B operands, per head, strip layout with 32 (16) rows per strip:
// local [h][4 strips][32][16], layer 1 (its local half) [h][2][32][16], layer 2 [h][2][16][16].
constexpr int LW_HEAD = 4 * 32 * 16, W1_HEAD = 2 * 32 * 16, W2_HEAD = 2 * 16 * 16;

constexpr int OFF_TOK = 0;
constexpr int SZ_TOK = 12 * STRIP;
constexpr int OFF_LOCAL = OFF_TOK + SZ_TOK;     // local features [6 strips][197][16]
constexpr int SZ_LOCAL = 6 * STRIP;
constexpr int OFF_LWT = OFF_LOCAL + SZ_LOCAL;
constexpr int SZ_LWT = 3 * LW_HEAD;
constexpr int OFF_W1T = OFF_LWT + SZ_LWT;
constexpr int SZ_W1T = 3 * W1_HEAD;
constexpr int OFF_W2T = OFF_W1T + SZ_W1T;
constexpr int SZ_W2T = 3 * W2_HEAD;
constexpr int OFF_W3T = OFF_W2T + SZ_W2T;
constexpr int SZ_W3T = 3 * 2 * 16;
constexpr int OFF_G1 = (OFF_W3T + SZ_W3T + 15) & ~15;
constexpr int SZ_G1 = 3 * 32 * 8;
constexpr int OFF_GLOB = OFF_G1 + SZ_G1;
constexpr int SZ_GLOB = 3 * 32;
constexpr int OFF_HS = OFF_GLOB + SZ_GLOB;
constexpr int SZ_HS = 3 * MAXC * 4;
constexpr int OFF_HW = OFF_HS + SZ_HS;
constexpr int SZ_HW = 3 * MAXC * 4;
constexpr int OFF_FUSED = OFF_HW + SZ_HW;
constexpr int SZ_FUSED = MAXC * 4;
constexpr int OFF_KIDX = OFF_FUSED + SZ_FUSED;
constexpr int SZ_KIDX = MAXC * 4;
constexpr int OFF_FLAGS = OFF_KIDX + SZ_KIDX;
constexpr int SZ_FLAGS = MAXC;  // bit0 keep, bit1 participant
constexpr int OFF_STATS = (OFF_FLAGS + SZ_FLAGS + 15) & ~15;
constexpr int SZ_STATS = MAXC * 3;
constexpr int OFF_MISC = (OFF_STATS + SZ_STATS + 15) & ~15;
constexpr int SZ_MISC = 128;  // [0] warn, [4..4+THREADS/32) scan,
                              // [24] wait status, byte 112: mbarrier, byte 120: TMEM base
constexpr int OFF_H1 = OFF_MISC + SZ_MISC;  // score layer-1 outputs [6 strips][197][16]
constexpr int SZ_H1 = 6 * STRIP;
constexpr int OFF_H2 = OFF_LOCAL;           // score layer-2 outputs [3][MAXC][16], over the dead local rows
constexpr int SZ_H2 = 3 * MAXC * 16;
static_assert(SZ_H2 <= SZ_LOCAL, "layer-2 outputs overlay the local features");
constexpr int OFF_TABL = OFF_H1 + SZ_H1;    // GELU table of the local MLP
constexpr int SMEM_BYTES = OFF_TABL + kSelTabLocalBytes;
// The score-layer tables use the token rows while those are not needed (after the
// head statistics; the rows are copied in again for the compaction).
constexpr int OFF_TAB1 = OFF_TOK;
constexpr int OFF_TAB2 = OFF_TOK + kSelTabH1Bytes;
static_assert(kSelTabH1Bytes + kSelTabH2Bytes <= SZ_TOK, "score-layer tables fit the token rows");
static_assert(OFF_TABL % 16 == 0 && OFF_TAB2 % 16 == 0, "16-byte table staging");
// (plus 128 bytes of static shared memory: the per-warp package sums)
static_assert(2 * (SMEM_BYTES + 128 + 1024) <= 228 * 1024, "two selector CTAs per SM");
static_assert(OFF_LOCAL % 16 == 0 && OFF_LWT % 16 == 0 && OFF_W1T % 16 == 0 && OFF_W2T % 16 == 0 &&
                  OFF_H1 % 16 == 0 && OFF_MISC % 16 == 0,
              "16-byte aligned tensor-core operands");
// An M = 128 tile that starts at row 128 reads strip rows up to 255: past row 196 of
// the last strip it reads the next region (garbage rows whose results are dropped),
// which must stay inside the CTA's shared memory.
static_assert(OFF_TOK + SZ_TOK + 59 * 16 <= SMEM_BYTES && OFF_LOCAL + SZ_LOCAL + 59 * 16 <= SMEM_BYTES &&
                  OFF_H1 + SZ_H1 + 59 * 16 <= SMEM_BYTES,
              "tile overrun stays in shared memory");
constexpr uint32_t SEL_WAIT = 1u << 24;
constexpr uint32_t SEL_TMEM_COLS = 256;  // two CTAs per SM

// Address of byte k of row r in a strip-layout array.
__device__ __forceinline__ int8_t *strip_at(int8_t *base, int r, int k) {
    return base + (k >> 4) * STRIP + r * 16 + (k & 15);
}

__device__ __forceinline__ int32_t sat_q016(int64_t v) { return (int32_t)(v < 0 ? 0 : (v > 65536 ? 65536 : v)); }

// Copy a GELU table (t.bytes, a multiple of 16) into shared memory.
// 16 bytes global -> shared by cp.async (both 16-byte aligned); the caller waits
// (cp.async.wait_all) before the barrier after which the bytes are read.
__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

// A GELU table into shared memory by cp.async (see cp16).
__device__ __forceinline__ void stage_tab(const GeluTab &t, int8_t *dst, int tid) {
    if (!t.mode) return;
    for (int i = tid; i < t.bytes / 16; i += THREADS) cp16(dst + 16 * i, (const int8_t *)t.tab + 16 * i);
}

// acc + a · b over W 16-byte words of packed int8 (shared memory, 16-byte aligned).
template <int W>
__device__ __forceinline__ int32_t dot16(const int8_t *a, const int8_t *b, int32_t acc) {
#pragma unroll
    for (int w = 0; w < W; ++w) {
        const int4 x = ((const int4 *)a)[w], y = ((const int4 *)b)[w];
        acc = __dp4a(x.x, y.x, acc);
        acc = __dp4a(x.y, y.y, acc);
        acc = __dp4a(x.z, y.z, acc);
        acc = __dp4a(x.w, y.w, acc);
    }
    return acc;
}

// (head, candidate) of a flattened head-major index hc = h * C + c, without a division.
__device__ __forceinline__ void split_hc(int hc, int C, int &h, int &c) {
    h = (hc >= C) + (hc >= 2 * C);
    c = hc - h * C;
}

// One selector GELU chain (selector.py:89-99) in the fastest form the host proved exact.
__device__ __forceinline__ int32_t sel_gelu(int64_t v, int k2, const GeluK &k, int fast, int sh_in, int sh_out) {
    if (k2) return sat8(gelu_chain_fast2((int32_t)v, k));
    if (fast) return gelu_chain_fast((int32_t)v, sh_in, sh_out);
    return gelu_chain(v, sh_in, sh_out);
}

// Keep score of one candidate-head: softmax_selector([q0, q1])[1]
// (selector.py:345-354, nonlinear.py:109-127).
__device__ __forceinline__ int32_t keep_score(int32_t q0, int32_t q1) {
    const int32_t mx = max(q0, q1);
    const uint32_t e0 = softmax_exp_q16(q0 - mx), e1 = softmax_exp_q16(q1 - mx);
    const uint64_t rc = softmax_recip32(e0 + e1);  // one term is exp(0): S in [65554, 131108]
    const uint32_t r1 = softmax_ratio(e1, rc);
    return (int32_t)(r1 < 65536u ? r1 : 65536u);
}

// One selector activation in a form fixed per layer (A = 1, 2: exact table of that
// mode; 0: the GELU chain), so an epilogue's 16 unrolled elements are one short
// straight-line path rather than every form inlined per element.
struct SelAct {
    const GeluTab *tab;
    const int8_t *s;  // staged table
    int k2, fast, sh_in, sh_out;
    const GeluK *k;
};
template <int A>
__device__ __forceinline__ int32_t sel_act(int64_t v, const SelAct &a) {
    if (A == 0) return sel_gelu(v, a.k2, *a.k, a.fast, a.sh_in, a.sh_out);
    const GeluTab &t = *a.tab;
    const int32_t q = t.sh_in ? rsa32((int32_t)v, t.sh_in) : (int32_t)v;
    const int u = min(max(q - t.lo, 0), t.n - 1);
    if (A == 1) return a.s[u];
    const uint32_t e = ((const uint32_t *)a.s)[u >> t.k];
    const int off = u & ((1 << t.k) - 1);
    const uint32_t pc = e >> 16;
    int32_t o = off >= (int)pc ? (int32_t)(int8_t)(e >> 8) : (int32_t)(int8_t)e;
    if (pc == 0xFFFFu) o = a.s[t.fine + (int)((e & 0xFFFFu) << t.k) + off];
    return o;
}
// 8 outputs of one TMEM piece: act(acc + bias) packed as 8 int8 bytes.
template <int A, class B>
__device__ __forceinline__ uint2 sel_piece(const uint32_t (&v)[8], B &&bias, const SelAct &a) {
    uint32_t pk[2];
#pragma unroll
    for (int w = 0; w < 2; ++w) {
        int32_t o[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) o[b] = sel_act<A>((int64_t)(int32_t)v[4 * w + b] + bias(4 * w + b), a);
        pk[w] = pack_sat8(o[0], o[1], o[2], o[3]);
    }
    return make_uint2(pk[0], pk[1]);
}
template <class B>
__device__ __forceinline__ uint2 sel_piece_any(int mode, const uint32_t (&v)[8], B &&bias, const SelAct &a) {
    if (mode == 1) return sel_piece<1>(v, bias, a);
    if (mode == 2) return sel_piece<2>(v, bias, a);
    return sel_piece<0>(v, bias, a);
}

__global__ void __launch_bounds__(THREADS, 2) selector_kernel(
    const int8_t *__restrict__ x, const int32_t *__restrict__ offsets, const uint8_t *__restrict__ pkg_in,
    SelParams p, int8_t *__restrict__ stage, int32_t *__restrict__ counts_out, uint8_t *__restrict__ pkg_out,
    hv_selector_summary *__restrict__ summary, int sum_stride, uint8_t *__restrict__ warn,
    int32_t *__restrict__ token_counts, int tc_stride, int tc_col, SelDebug dbg) {
    griddep_wait();
    griddep_launch();
    extern __shared__ __align__(16) uint8_t smem[];
    int8_t *tok = (int8_t *)(smem + OFF_TOK);
    int8_t *local = (int8_t *)(smem + OFF_LOCAL);
    int8_t *lwt = (int8_t *)(smem + OFF_LWT);
    int8_t *w1t = (int8_t *)(smem + OFF_W1T);
    int8_t *w2t = (int8_t *)(smem + OFF_W2T);
    int8_t *w3t = (int8_t *)(smem + OFF_W3T);
    int8_t *tabl = (int8_t *)(smem + OFF_TABL);
    int8_t *tab1 = (int8_t *)(smem + OFF_TAB1);
    int8_t *tab2 = (int8_t *)(smem + OFF_TAB2);
    int64_t *g1 = (int64_t *)(smem + OFF_G1);
    int8_t *glob = (int8_t *)(smem + OFF_GLOB);
    int32_t *hs = (int32_t *)(smem + OFF_HS);
    int32_t *hwt = (int32_t *)(smem + OFF_HW);
    int32_t *fused = (int32_t *)(smem + OFF_FUSED);
    int32_t *kidx = (int32_t *)(smem + OFF_KIDX);
    uint8_t *flags = (uint8_t *)(smem + OFF_FLAGS);
    int8_t *stats = (int8_t *)(smem + OFF_STATS);
    int32_t *misc = (int32_t *)(smem + OFF_MISC);  // [0] warn, [4..] scan

    const int img = blockIdx.x, tid = threadIdx.x;
    const int row0 = offsets[img];
    const int n = offsets[img + 1] - row0;
    const int C = n - 1;
    const int pkg = pkg_in ? (pkg_in[img] != 0) : 0;
    int8_t *out = stage + (size_t)img * 197 * 192;

    if (tid < 26) misc[tid] = 0;
    if (C < 1) {  // selector.py:513-514 needs CLS plus a candidate; pass the row through
        if (tid < 12) ((int4 *)out)[tid] = ((const int4 *)(x + (size_t)row0 * 192))[tid];
        if (tid == 0) {
            counts_out[img] = n;
            if (pkg_out) pkg_out[img] = (uint8_t)pkg;
        }
        return;
    }

    // ---- load tokens (strip layout) and weights (per-head B operands) --------------
    // (all by cp.async, so every thread's copies are in flight at once)
    for (int c = tid; c < n * 12; c += THREADS)
        cp16(tok + (c % 12) * STRIP + (c / 12) * 16, x + (size_t)row0 * 192 + 16 * c);
    for (int c = tid; c < 3 * 32 * 4; c += THREADS) {  // local_wt [h][j][64]: 4 chunks per row
        const int hj = c >> 2, k4 = c & 3, h = hj >> 5, j = hj & 31;
        cp16(lwt + h * LW_HEAD + k4 * 512 + j * 16, p.local_wt + 16 * c);
    }
    for (int c = tid; c < 3 * 32 * 2; c += THREADS) {  // w1t [h][j][0..31]: the local half
        const int hj = c >> 1, k2 = c & 1, h = hj >> 5, j = hj & 31;
        cp16(w1t + h * W1_HEAD + k2 * 512 + j * 16, p.w1t + 16 * (hj * 4 + k2));
    }
    for (int c = tid; c < 3 * 16 * 2; c += THREADS) {  // w2t [h][m][32]
        const int hm = c >> 1, k2 = c & 1, h = hm >> 4, m = hm & 15;
        cp16(w2t + h * W2_HEAD + k2 * 256 + m * 16, p.w2t + 16 * c);
    }
    if (tid < 24) ((int32_t *)w3t)[tid] = ((const int32_t *)p.w3t)[tid];
    stage_tab(p.tab_local, tabl, tid);
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    uint64_t *bar = (uint64_t *)((uint8_t *)misc + 112);
    uint32_t *tslot = (uint32_t *)((uint8_t *)misc + 120);
    volatile int *wstat = (volatile int *)(misc + 24);
    if (tid < 32) {
        tc05::tmem_alloc(tslot, SEL_TMEM_COLS);
        tc05::tmem_relinquish();
    }
    if (tid == 0) {
        tc05::mbar_init(bar, 1);
        tc05::fence_mbar_init();
    }
    tc05::fence_proxy_async();  // the operands written above are read by the tensor cores
    tc05::fence_before();
    __syncthreads();
    tc05::fence_after();
    const uint32_t tbase = *tslot;
    const int lane = tid & 31, warp = tid >> 5, quad = warp & 3, part = warp >> 2;
    const int tiles = (n + 127) >> 7;  // M = 128 tiles of token rows (row 0 = CLS, dropped)
    const uint32_t lane_base = tbase + ((uint32_t)(quad * 32) << 16);
    uint32_t phase = 0;
    // One layer: thread 0 issues `issue` (the tensor-core work) and commits; every
    // thread learns whether it completed in time (bounded wait, then a barrier).
    // Every thread waits on the mbarrier itself (no barrier after the wait: the next
    // layer is issued only after a barrier that every thread reaches after this wait,
    // so none can miss a phase).
    auto mma_layer = [&](auto &&issue) -> bool {
        if (tid == 0) {
            tc05::fence_after();
            issue();
            tc05::commit(bar);
        }
        const bool ok = tc05::mbar_wait(bar, phase, SEL_WAIT);
        if (!ok) {
            *wstat = 1;
            misc[25] = (int)phase;  // the parity to drain before TMEM is released
            if (p.err) atomicExch(p.err, 3);
        }
        phase ^= 1;
        tc05::fence_after();
        return ok;
    };
    const uint32_t id32 = tc05::idesc_i8(128, 32, true, true), id16 = tc05::idesc_i8(128, 16, true, true);
    const uint32_t tok_u = tc05::smem_u32(tok), loc_u = tc05::smem_u32(local), lwt_u = tc05::smem_u32(lwt);
    const uint32_t w1t_u = tc05::smem_u32(w1t), w2t_u = tc05::smem_u32(w2t);
    int8_t *h1s = (int8_t *)(smem + OFF_H1);
    int8_t *h2s = (int8_t *)(smem + OFF_H2);
    const uint32_t h1_u = tc05::smem_u32(h1s);
    bool ok = true;
    const SelAct act_l{&p.tab_local, tabl, p.local_k2, p.local_fast, p.local_sh_in, p.local_sh_out, &p.local_k};
    const SelAct act_1{&p.tab_h1, tab1, p.h1_k2, p.h1_fast, p.h1_sh_in, p.h1_sh_out, &p.h1_k};
    const SelAct act_2{&p.tab_h2, tab2, p.h2_k2, p.h2_fast, p.h2_sh_in, p.h2_sh_out, &p.h2_k};

    // ---- local MLP (selector.py:253-270): per head [n x 64] . [64 x 32] on tcgen05 ------
    ok = mma_layer([&] {
        for (int t = 0; t < tiles; ++t)
            for (int h = 0; h < 3; ++h)
                for (int k = 0; k < 2; ++k)
                    tc05::mma_i8_ss(tbase + t * 96 + h * 32,
                                    tc05::smem_desc(tok_u + (4 * h + 2 * k) * STRIP + t * 2048, STRIP, 128),
                                    tc05::smem_desc(lwt_u + h * LW_HEAD + 2 * k * 512, 512, 128), id32, k);
    });
    // epilogue: thread = token row (TMEM lane); the 12 pieces of 8 columns (head
    // pc / 4, outputs 8 (pc % 4) ..) are dealt three to each of the quadrant's warps
    if (ok)
        for (int t = 0; t < tiles; ++t) {
            const int r = t * 128 + quad * 32 + lane;
            for (int pc = part; pc < 12; pc += 4) {
                uint32_t v[8];
                tc05::ld8(lane_base + t * 96 + pc * 8, v);
                tc05::wait_ld_regs(v);
                if (r >= 1 && r < n) {
                    const int32_t *lb = p.local_b + pc * 8;
                    *(uint2 *)(local + (pc >> 1) * STRIP + r * 16 + (pc & 1) * 8) =
                        sel_piece_any(p.tab_local.mode, v, [&](int i) { return (int64_t)lb[i]; }, act_l);
                }
            }
        }
    tc05::fence_proxy_async();
    tc05::fence_before();
    __syncthreads();
    if (dbg.local)  // exported now: the layer-2 outputs overwrite these rows later
        for (int i = tid; i < 3 * C * 32; i += THREADS) {
            const int j = i & 31;
            int h, c;
            split_hc(i >> 5, C, h, c);
            dbg.local[(((size_t)img * 3 + h) * MAXC + c) * 32 + j] = *strip_at(local, 1 + c, h * 32 + j);
        }

    // ---- global mean (selector.py:273-289) and head stats (358-367), the last reads
    // of the token rows before the score-layer tables take their place ----------------
    {
        // thread (j, q) of 24 x 20 sums the 4 features of word j of the local rows (one
        // 32-bit word of a strip row) over every twentieth candidate; the 20 partials
        // of a feature meet in shared memory (the score layer-1 rows, not yet written)
        constexpr int GQ = 20;
        int32_t *gpart = (int32_t *)(smem + OFF_H1);
        if (tid < 24 * GQ) {
            const int q = tid / 24, j = tid - q * 24;
            const int8_t *col = local + (j >> 2) * STRIP + (j & 3) * 4;
            int32_t t[4] = {0, 0, 0, 0};
            for (int c = q; c < C; c += GQ) {
                const uint32_t wv = *(const uint32_t *)(col + (1 + c) * 16);
#pragma unroll
                for (int k = 0; k < 4; ++k) t[k] += (int32_t)(int8_t)(wv >> (8 * k));
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) gpart[q * 96 + 4 * j + k] = t[k];
        }
        __syncthreads();
        if (tid < 96) {
            int32_t t = 0;
#pragma unroll
            for (int q = 0; q < GQ; ++q) t += gpart[q * 96 + tid];
            glob[tid] = (int8_t)sat8((int32_t)round_div64(t, C));
        }
    }
    for (int c = tid; c < C; c += THREADS) {
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            int32_t t = 0;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const int4 x4 = *(const int4 *)(tok + (4 * h + w) * STRIP + (1 + c) * 16);
                t = __dp4a(x4.x, 0x01010101, t);
                t = __dp4a(x4.y, 0x01010101, t);
                t = __dp4a(x4.z, 0x01010101, t);
                t = __dp4a(x4.w, 0x01010101, t);
            }
            stats[c * 3 + h] = (int8_t)sat8((int32_t)round_div64(t, 64));
        }
    }
    __syncthreads();
    stage_tab(p.tab_h1, tab1, tid);  // (their copies overlap the global half below)
    stage_tab(p.tab_h2, tab2, tid);
    if (tid < 96) {
        // the global half of layer 1, once per image (W1 rows read from global memory)
        const int h = tid >> 5, j = tid & 31;
        const int4 *wrow = (const int4 *)(p.w1t + (h * 32 + j) * 64 + 32);
        const int32_t acc = dot16<2>(glob + h * 32, (const int8_t *)wrow, 0);  // (2 x 16-byte words)
        g1[h * 32 + j] = (int64_t)acc + p.b1[h * 32 + j];
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");  // the score-layer tables
    __syncthreads();

    // ---- score MLP layer 1 (selector.py:307-330): per head [n x 32] . [32 x 32] -------
    ok = ok && mma_layer([&] {
        for (int t = 0; t < tiles; ++t)
            for (int h = 0; h < 3; ++h)
                tc05::mma_i8_ss(tbase + t * 96 + h * 32, tc05::smem_desc(loc_u + 2 * h * STRIP + t * 2048, STRIP, 128),
                                tc05::smem_desc(w1t_u + h * W1_HEAD, 512, 128), id32, 0);
    });
    if (ok)
        for (int t = 0; t < tiles; ++t) {
            const int r = t * 128 + quad * 32 + lane;
            for (int pc = part; pc < 12; pc += 4) {
                uint32_t v[8];
                tc05::ld8(lane_base + t * 96 + pc * 8, v);
                tc05::wait_ld_regs(v);
                if (r >= 1 && r < n) {
                    const int64_t *gb = g1 + pc * 8;  // global half of layer 1 plus its bias
                    *(uint2 *)(h1s + (pc >> 1) * STRIP + r * 16 + (pc & 1) * 8) =
                        sel_piece_any(p.tab_h1.mode, v, [&](int i) { return gb[i]; }, act_1);
                }
            }
        }
    tc05::fence_proxy_async();
    tc05::fence_before();
    __syncthreads();

    // ---- score MLP layer 2 (selector.py:331-344): per head [n x 32] . [32 x 16] -------
    ok = ok && mma_layer([&] {
        for (int t = 0; t < tiles; ++t)
            for (int h = 0; h < 3; ++h)
                tc05::mma_i8_ss(tbase + t * 48 + h * 16, tc05::smem_desc(h1_u + 2 * h * STRIP + t * 2048, STRIP, 128),
                                tc05::smem_desc(w2t_u + h * W2_HEAD, 256, 128), id16, 0);
    });
    // layer-2 outputs [h][c][16] (one 16-byte row per candidate and head, over the dead
    // local features)
    if (ok)
        for (int t = 0; t < tiles; ++t) {
            const int r = t * 128 + quad * 32 + lane;
            for (int pc = part; pc < 6; pc += 4) {  // pieces of 8: head pc / 2, outputs 8 (pc % 2) ..
                uint32_t v[8];
                tc05::ld8(lane_base + t * 48 + pc * 8, v);
                tc05::wait_ld_regs(v);
                if (r >= 1 && r < n) {
                    const int32_t *b2 = p.b2 + pc * 8;
                    *(uint2 *)(h2s + ((pc >> 1) * MAXC + (r - 1)) * 16 + (pc & 1) * 8) =
                        sel_piece_any(p.tab_h2.mode, v, [&](int i) { return (int64_t)b2[i]; }, act_2);
                }
            }
        }
    tc05::fence_before();
    __syncthreads();
    if (dbg.h2)
        for (int i = tid; i < 3 * C * 16; i += THREADS) {
            const int m = i & 15;
            int h, c;
            split_hc(i >> 4, C, h, c);
            dbg.h2[(((size_t)img * 3 + h) * MAXC + c) * 16 + m] = h2s[(h * MAXC + c) * 16 + m];
        }
    // the token rows come back for the compaction (their copies overlap the phases below)
    if (p.tab_h1.mode || p.tab_h2.mode) {
        for (int c = tid; c < n * 12; c += THREADS) {
            const uint32_t dst = (uint32_t)__cvta_generic_to_shared(tok + (c % 12) * STRIP + (c / 12) * 16);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst),
                         "l"(x + (size_t)row0 * 192 + c * 16)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    // Layer 3 (3C items) and the head-weight MLP (C items, each costlier) are
    // independent: the last C threads take the head-weight MLP, one candidate each,
    // while the others run layer 3.
    const int nl3 = THREADS - C;  // >= THREADS - MAXC
    if (tid < nl3) {
        for (int it = tid; it < 3 * C; it += nl3) {
            int h, c;
            split_hc(it, C, h, c);
            const int8_t *hrow = h2s + (h * MAXC + c) * 16;
            int32_t q[2];
#pragma unroll
            for (int o = 0; o < 2; ++o) {
                const int32_t acc = dot16<1>(hrow, w3t + (h * 2 + o) * 16, 0);
                const int32_t logit = (int32_t)requant64((int64_t)acc + p.b3[h * 2 + o], p.logit_shift, 8);
                q[o] = (int32_t)requant64(logit, p.logit_q16_shift, 24);
            }
            hs[h * MAXC + c] = keep_score(q[0], q[1]);
        }
    } else {
        // ---- head-weight MLP per candidate (selector.py:370-389) ---------------------
        const int c = tid - nl3;
        int32_t st[3];
#pragma unroll
        for (int h = 0; h < 3; ++h) st[h] = stats[c * 3 + h];
        int32_t hid[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            int64_t acc = p.hb1[j];
#pragma unroll
            for (int i = 0; i < 3; ++i) acc += st[i] * (int32_t)p.hw1[i * 3 + j];
            hid[j] = sel_gelu(acc, p.hw_k2, p.hw_k, p.hw_fast, p.hw_sh_in, p.hw_sh_out);
        }
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            int64_t acc = p.hb2[j];
#pragma unroll
            for (int i = 0; i < 3; ++i) acc += hid[i] * (int32_t)p.hw2[i * 3 + j];
            hwt[c * 3 + j] = sat_q016(plan_sigmoid((int32_t)requant64(acc, p.hw_q16_shift, 24)));
        }
    }
    __syncthreads();

    // ---- fuse (selector.py:392-418) and keep flags ----------------------------------
    const int normals = C - pkg;
    for (int c = tid; c < C; c += THREADS) {
        int64_t num = 0, den = 0;
#pragma unroll
        for (int h = 0; h < 3; ++h) {
            num += (int64_t)hs[h * MAXC + c] * hwt[c * 3 + h];
            den += hwt[c * 3 + h];
        }
        if (den == 0) {
            num = (int64_t)hs[c] + hs[MAXC + c] + hs[2 * MAXC + c];
            den = 3;
            atomicOr(&misc[0], (int)HV_WARN_HEAD_DEN_ZERO);
        }
        const int32_t f = sat_q016(round_div64(num, den));
        fused[c] = f;
        const int keep = (c < normals) && f >= 32768;
        flags[c] = (uint8_t)(keep | ((keep ? 0 : 1) << 1));
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");  // the token rows are back
    __syncthreads();

    // ---- stable compaction index: exclusive scan of keep flags (C <= 196 < 256), and
    // the participants of the package (pruned normals plus the incoming package,
    // always) with the sum of their fused scores: per-warp ballots and reductions,
    // combined after one barrier (each fused score <= 65536, so the sums fit int32)
    __shared__ int wpart[THREADS / 32], wden[THREADS / 32];
    int kept = 0, parts = 0;
    long long pden = 0;
    {
        const int lane = tid & 31, warp = tid >> 5;
        const int fl = tid < C ? flags[tid] : 0;
        const unsigned bal = __ballot_sync(0xffffffffu, fl & 1);
        const unsigned pbal = __ballot_sync(0xffffffffu, fl & 2);
        const int dsum = __reduce_add_sync(0xffffffffu, (fl & 2) ? fused[tid] : 0);
        if (lane == 0) {
            misc[4 + warp] = __popc(bal);
            wpart[warp] = __popc(pbal);
            wden[warp] = dsum;
        }
        __syncthreads();
        int base = 0;
        for (int w = 0; w < warp; ++w) base += misc[4 + w];
        if (tid < C) kidx[tid] = base + __popc(bal & ((1u << lane) - 1u));
#pragma unroll
        for (int w = 0; w < THREADS / 32; ++w) {
            kept += misc[4 + w];
            parts += wpart[w];
            pden += wden[w];
        }
    }
    __syncthreads();  // kidx
    const int nout = 1 + kept + (parts > 0 ? 1 : 0);

    // ---- write rows: CLS, kept (stable), package --------------------------------------
    if (tid < 12) ((int4 *)out)[tid] = *(const int4 *)(tok + tid * STRIP);
    for (int idx = tid; idx < C * 12; idx += THREADS) {
        const int c = idx / 12, ch = idx - c * 12;
        if (flags[c] & 1)
            ((int4 *)(out + (size_t)(1 + kidx[c]) * 192))[ch] = *(const int4 *)(tok + ch * STRIP + (1 + c) * 16);
    }
    if (parts > 0) {
        // Σ s·x[d] (or Σ x[d]) over the participants: thread (j, q) of 48 x 10 sums
        // columns 4j..4j+3 (one 32-bit word of a token strip row) over every tenth
        // candidate (s <= 65536, |x| <= 128, at most 20 terms per thread: int32 is
        // exact); the ten partials of a column meet in shared memory (over the score
        // layer-1 rows, dead by now)
        int8_t *prow = out + (size_t)(1 + kept) * 192;
        int32_t *ppart = (int32_t *)(smem + OFF_H1);
        constexpr int PQ = 10;
        if (tid < 48 * PQ) {
            const int q = tid / 48, j = tid - q * 48;
            const int8_t *col = tok + (j >> 2) * STRIP + (j & 3) * 4;
            int32_t num[4] = {0, 0, 0, 0};
            for (int c = q; c < C; c += PQ)
                if (flags[c] & 2) {
                    const int32_t s = pden == 0 ? 1 : fused[c];
                    const uint32_t wv = *(const uint32_t *)(col + (1 + c) * 16);
#pragma unroll
                    for (int k = 0; k < 4; ++k) num[k] += s * (int32_t)(int8_t)(wv >> (8 * k));
                }
#pragma unroll
            for (int k = 0; k < 4; ++k) ppart[q * 192 + 4 * j + k] = num[k];
        }
        __syncthreads();
        if (tid < 192) {
            long long num = 0;
#pragma unroll
            for (int q = 0; q < PQ; ++q) num += ppart[q * 192 + tid];
            prow[tid] = (int8_t)sat8((int32_t)round_div64(num, pden == 0 ? parts : pden));
        }
    }
    if (tid == 0) {
        const int w = misc[0] | (parts > 0 && pden == 0 ? (int)HV_WARN_PACKAGE_DEN_ZERO : 0);
        counts_out[img] = nout;
        if (pkg_out) pkg_out[img] = (uint8_t)(parts > 0);
        if (summary) {
            hv_selector_summary s;
            s.input_tokens = n;
            s.output_tokens = nout;
            s.kept_normal = kept;
            s.pruned_normal = parts - pkg;
            s.package_present = parts > 0;
            s.warnings = w;
            summary[(size_t)img * sum_stride] = s;
        }
        if (warn && w) atomicOr((unsigned int *)(warn + (img & ~3)), (unsigned int)w << (8 * (img & 3)));
        if (token_counts) token_counts[(size_t)img * tc_stride + tc_col] = nout;
    }
    // ---- optional intermediates (token_selector API) -------------------------------
    if (dbg.fused)
        for (int c = tid; c < C; c += THREADS) dbg.fused[(size_t)img * MAXC + c] = fused[c];
    if (dbg.head_scores)
        for (int i = tid; i < 3 * C; i += THREADS) {
            int h, c;
            split_hc(i, C, h, c);
            dbg.head_scores[((size_t)img * 3 + h) * MAXC + c] = hs[h * MAXC + c];
        }
    if (dbg.head_weights)
        for (int i = tid; i < 3 * C; i += THREADS) dbg.head_weights[(size_t)img * MAXC * 3 + i] = hwt[i];
    if (dbg.global_ && tid < 96) dbg.global_[(size_t)img * 96 + tid] = glob[tid];
    if (dbg.stats)
        for (int i = tid; i < 3 * C; i += THREADS) dbg.stats[(size_t)img * MAXC * 3 + i] = stats[i];
    // release TMEM; after a wait that gave up, first let that layer's MMAs finish (bounded)
    if (tid == 0 && *wstat) tc05::mbar_wait(bar, (uint32_t)misc[25], SEL_WAIT);
    tc05::fence_before();
    __syncthreads();
    if (tid < 32) {
        tc05::fence_after();
        tc05::tmem_dealloc(tbase, SEL_TMEM_COLS);
    }
}

// One CTA per image: copies the image's kept rows from the staging buffer to their
// packed place and writes its offset and, when `plan` has lists, its attention units
// (the prefix sums over the images before it give all three positions).
__global__ void __launch_bounds__(256) pack_kernel(const int8_t *__restrict__ stage,
                                                   const int32_t *__restrict__ counts, int images,
                                                   int8_t *__restrict__ x, int32_t *__restrict__ offsets_out,
                                                   AttnPlan plan) {
    griddep_wait();
    griddep_launch();
    __shared__ int part[3][8];
    const int img = blockIdx.x, tid = threadIdx.x;
    int s = 0, sa = 0, sb = 0;
    for (int i = tid; i < img; i += 256) {
        const int n = counts[i];
        s += n;
        sa += units_a(n);
        sb += units_b(n);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        sa += __shfl_xor_sync(0xffffffffu, sa, o);
        sb += __shfl_xor_sync(0xffffffffu, sb, o);
    }
    if ((tid & 31) == 0) {
        part[0][tid >> 5] = s;
        part[1][tid >> 5] = sa;
        part[2][tid >> 5] = sb;
    }
    __syncthreads();
    int off = 0, pa = 0, pb = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        off += part[0][w];
        pa += part[1][w];
        pb += part[2][w];
    }
    const int cnt = counts[img];
    if (tid == 0) {
        offsets_out[img] = off;
        if (img == images - 1) offsets_out[images] = off + cnt;
        if (plan.cnt) {
            write_image_units(plan.list_a, plan.list_b, pa, pb, img, off, cnt);
            if (img == images - 1) {
                plan.cnt[0] = pa + units_a(cnt);
                plan.cnt[1] = pb + units_b(cnt);
            }
        }
    }
    const int4 *src = (const int4 *)(stage + (size_t)img * 197 * 192);
    int4 *dst = (int4 *)(x + (size_t)off * 192);
    for (int c = tid; c < cnt * 12; c += 256) dst[c] = src[c];
}

}  // namespace

cudaError_t launch_selector(const int8_t *x, const int32_t *offsets, const uint8_t *pkg_in, int images,
                            const SelParams &p, int8_t *stage, int32_t *counts_out, uint8_t *pkg_out,
                            hv_selector_summary *summary, int sum_stride, uint8_t *warn, int32_t *token_counts,
                            int tc_stride, int tc_col, const SelDebug *dbg, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(selector_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    SelDebug d = dbg ? *dbg : SelDebug{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    return launch_pdl(selector_kernel, dim3(images), dim3(THREADS), SMEM_BYTES, st, x, offsets, pkg_in, p, stage,
                      counts_out, pkg_out, summary, sum_stride, warn, token_counts, tc_stride, tc_col, d);
}

cudaError_t launch_pack(const int8_t *stage, const int32_t *counts, int images, int8_t *x, int32_t *offsets_out,
                        const AttnPlan *plan, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    const AttnPlan pl = plan ? *plan : AttnPlan{nullptr, nullptr, nullptr};
    return launch_pdl(pack_kernel, dim3(images), dim3(256), 0, st, stage, counts, images, x, offsets_out, pl);
}

}  // namespace hv
