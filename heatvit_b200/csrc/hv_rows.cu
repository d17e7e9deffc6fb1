// hv_rows.cu — row kernels: LayerNorm, the shift-softmax rows and element-wise units.
//
// LayerNorm (nonlinear.py:136-186) over D = 192: eight lanes per row, lane `sub`
// owning channels [24 sub, 24 sub + 24); a warp takes up to 32 rows per pass (4-row
// sub-passes for the sums, then one lane per row for the statistics, then the
// sub-passes again to normalise).  The arithmetic (hv_ln.cuh) forms the 81-bit
// product (x_q32 - mean) * inv_std_q32 exactly, through a 32-bit short form where
// the host-proven range allows.
#include <algorithm>

#include "hv_internal.cuh"
#include "hv_ln.cuh"

namespace hv {

LnParams make_ln(const int8_t *gamma, const int8_t *beta, int x_scale, int gamma_scale, int beta_scale,
                 int out_scale) {
    LnParams p;
    p.gamma = gamma;
    p.beta = beta;
    p.x_scale = x_scale;
    p.sh_sum = x_scale + 32;
    p.sq_shift = 2 * x_scale + 32;
    const int common = (gamma_scale - 16) < beta_scale ? (gamma_scale - 16) : beta_scale;
    p.sh_g = gamma_scale - 16 - common;
    p.sh_b = beta_scale - common;
    p.sh_out = out_scale - common;
    p.fast = (p.sh_g <= 16 && p.sh_b <= 40) ? 1 : 0;
    p.split = x_scale <= -4 ? 1 : 0;
    p.out32 = (p.sh_g == 0 && p.sh_b <= 22 && p.sh_out >= 1 && p.sh_out <= 30) ? 1 : 0;
    p.one = 1;
    return p;
}

namespace {

__device__ __forceinline__ int32_t warp_max_i32(int32_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Per-lane channel constants: lane `sub` owns channels [24*sub, 24*sub + 24) of
// every row it processes, so gamma and the aligned beta term are loaded once.
template <bool OUT32>
__device__ __forceinline__ void ln_lane_consts(const LnParams &p, int sub, int32_t (&gam)[24], int32_t (&bet)[24]) {
#pragma unroll
    for (int i = 0; i < 24; ++i) {
        gam[i] = p.gamma[24 * sub + i];
        const int32_t b = p.beta[24 * sub + i];
        bet[i] = OUT32 ? b * (1 << p.sh_b) : b;
    }
}

// One row per 8-lane group; lane `sub` owns channels [24*sub, 24*sub + 24).
// Returns true on negative variance.  All 32 lanes of the warp must call it.
template <bool SPLIT, bool OUT32>
__device__ __forceinline__ bool ln_row8(const int8_t *xr, int8_t *outr, const LnParams &p, int sub, bool active,
                                        const int32_t (&gam)[24], const int32_t (&bet)[24]) {
    int32_t v[24];
    uint2 w[3] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
    if (active) {
        const uint2 *src = (const uint2 *)(xr + 24 * sub);
        w[0] = src[0];
        w[1] = src[1];
        w[2] = src[2];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            v[i * 8 + b] = (int8_t)((w[i].x >> (8 * b)) & 0xffu);
            v[i * 8 + 4 + b] = (int8_t)((w[i].y >> (8 * b)) & 0xffu);
        }
    }
    int32_t s = 0;
#pragma unroll
    for (int i = 0; i < 24; ++i) s += v[i];
    int64_t s2;
    if (p.sq_shift >= 0) {
        int32_t q = 0;
#pragma unroll
        for (int i = 0; i < 24; ++i) q += v[i] * v[i];
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        s2 = (int64_t)q << p.sq_shift;
    } else {
        const int k = -p.sq_shift;  // per-element ties-away right shift (x^2 >= 0)
        int64_t q = 0;
#pragma unroll
        for (int i = 0; i < 24; ++i) q += ((int64_t)(v[i] * v[i]) + ((int64_t)1 << (k - 1))) >> k;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        s2 = q;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const LnStats st = ln_stats(s, s2, p);
    const LnAff af = ln_aff(st, p);
    int32_t o[24];
    if (af.safe) {
#pragma unroll
        for (int i = 0; i < 24; ++i) {
            const int32_t nr = ln_norm_aff(v[i], af);
            o[i] = OUT32 ? rsa32(nr * gam[i] + bet[i], p.sh_out) : ln_out<false>(nr, gam[i], bet[i], p);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 24; ++i) o[i] = ln_out<OUT32>(ln_norm<SPLIT>(v[i], st, p), gam[i], p.beta[24 * sub + i], p);
    }
    uint32_t ow[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) ow[i] = pack_sat8(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    if (active) {
        uint2 *dst = (uint2 *)(outr + 24 * sub);
        dst[0] = make_uint2(ow[0], ow[1]);
        dst[1] = make_uint2(ow[2], ow[3]);
        dst[2] = make_uint2(ow[4], ow[5]);
    }
    return st.neg;
}

// 24 bytes of a row (lane `sub` of its 8-lane group) as int32 values.
__device__ __forceinline__ void ln_load24(const int8_t *xr, int sub, bool active, int32_t (&v)[24]) {
    uint2 w[3] = {make_uint2(0, 0), make_uint2(0, 0), make_uint2(0, 0)};
    if (active) {
        const uint2 *src = (const uint2 *)(xr + 24 * sub);
        w[0] = src[0];
        w[1] = src[1];
        w[2] = src[2];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            v[i * 8 + b] = (int8_t)((w[i].x >> (8 * b)) & 0xffu);
            v[i * 8 + 4 + b] = (int8_t)((w[i].y >> (8 * b)) & 0xffu);
        }
    }
}

// 32 rows per warp and pass.  Phase 1: eight 4-row sub-passes (8 lanes per row,
// 24 channels per lane) reduce Σx and Σx² per row; lane L keeps row base + L.
// Phase 2: every lane derives the statistics and affine constants of its own row
// (one row per lane instead of eight lanes per row).  Phase 3: the sub-passes
// again, each 8-lane group taking its row's constants from the owning lane.
template <bool SPLIT, bool OUT32>
__global__ void __launch_bounds__(256, 3) ln_kernel(const int8_t *x, int8_t *out, int rows_max, const int32_t *rows_dev,
                                                 LnParams p, uint8_t *negvar_row, const int32_t *offsets,
                                                 int images, uint8_t *warn) {
    const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    // gamma and the aligned beta term per channel, in shared memory (lane stride 25
    // words: the 8 lanes of a row group hit distinct banks)
    __shared__ int32_t s_gam[8 * 25], s_bet[8 * 25];
    // the same as {gamma, beta} pairs of consecutive channels, one 16-byte load per
    // two channels (lane stride 13 x 16 bytes: the 8 row-group lanes hit distinct
    // bank quads)
    __shared__ int4 s_gb[8 * 13];
    for (int c = threadIdx.x; c < 192; c += blockDim.x) {
        const int slot = (c / 24) * 25 + c % 24;
        s_gam[slot] = p.gamma[c];
        const int32_t b = p.beta[c];
        s_bet[slot] = OUT32 ? b * (1 << p.sh_b) : b;
        int32_t *pair = (int32_t *)&s_gb[(c / 24) * 13 + (c % 24) / 2] + 2 * (c & 1);
        pair[0] = p.gamma[c];
        // (the pairs feed only the 32-bit fast form, which also takes its rounding
        // half here: 2^(sh_out - 1) with sh_out >= 1 there)
        pair[1] = OUT32 ? b * (1 << p.sh_b) + (1 << (p.sh_out - 1)) : b;
    }
    __syncthreads();
    const int4 *gb = s_gb + sub * 13;
    const int32_t *gam = s_gam + sub * 25, *bet = s_bet + sub * 25;
    griddep_wait();  // rows and their count come from earlier kernels
    griddep_launch();
    const int rows = rows_dev ? *rows_dev : rows_max;
    // Rounds of one pass per warp (the grid is one wave of resident CTAs).  Each
    // round's rows per pass, 4 * g for g 4-row sub-passes, spread the remaining rows
    // over every warp: full 32-row passes while more than one round's worth remain
    // (they amortise the per-row statistics best), then one shorter balanced round,
    // so no warp runs a pass more than the others need (the pass latency bounds the
    // launch).
    for (int done = 0; done < rows;) {
    const int g = max(1, min(8, (rows - done + 4 * warps - 1) / (4 * warps)));
    const int R = 4 * g;
    const int base = done + warp * R;
    done += warps * R;
    if (base >= rows) break;  // warp-uniform; every later round starts past the rows
    {
        int32_t my_s = 0;
        int64_t my_s2 = 0;
        // this lane's 24 bytes of sub-pass k's row (zeros past the rows); each
        // sub-pass loads the next one's words before its own arithmetic
        auto load_words = [&](int k, uint2 (&w)[3]) {
            const int r = base + 4 * k + grp;
            w[0] = w[1] = w[2] = make_uint2(0, 0);
            if (k < g && r < rows) {
                const uint2 *src = (const uint2 *)(x + (size_t)r * 192 + 24 * sub);
                w[0] = src[0];
                w[1] = src[1];
                w[2] = src[2];
            }
        };
        uint2 wn[3];
        load_words(0, wn);
        // (unrolled by two: the shuffle reductions of consecutive sub-passes overlap)
#pragma unroll 2
        for (int k = 0; k < g; ++k) {
            const int r = base + 4 * k + grp;
            const uint2 w[3] = {wn[0], wn[1], wn[2]};
            load_words(k + 1, wn);
            // Σx and Σx² of the 24 bytes with 4-way byte dot products (|Σx²| < 2^21),
            // two independent chains each
            int32_t s = 0, q = 0, s1 = 0, q1 = 0;
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                s = __dp4a((int)w[i].x, 0x01010101, s);
                s1 = __dp4a((int)w[i].y, 0x01010101, s1);
                q = __dp4a((int)w[i].x, (int)w[i].x, q);
                q1 = __dp4a((int)w[i].y, (int)w[i].y, q1);
            }
            s += s1;
            q += q1;
            int64_t s2;
            if (p.sq_shift >= 0) {
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
                s2 = (int64_t)q << p.sq_shift;
            } else {
                int32_t v[24];
                ln_load24(x + (size_t)(r < rows ? r : 0) * 192, sub, r < rows, v);
                const int kk = -p.sq_shift;  // per-element ties-away right shift (x^2 >= 0)
                int64_t q64 = 0;
#pragma unroll
                for (int i = 0; i < 24; ++i) q64 += ((int64_t)(v[i] * v[i]) + ((int64_t)1 << (kk - 1))) >> kk;
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) q64 += __shfl_xor_sync(0xffffffffu, q64, o);
                s2 = q64;
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            // lane L = 4k + g takes the totals of group g (any of its lanes)
            const int32_t ts = __shfl_sync(0xffffffffu, s, (lane & 3) * 8);
            const int64_t tq = shfl64(s2, (lane & 3) * 8);
            if ((lane >> 2) == k) {
                my_s = ts;
                my_s2 = tq;
            }
        }
        const int myrow = lane < R ? base + lane : rows;  // lanes past the pass own no row
        const LnStats st = ln_stats(my_s, my_s2, p);
        const LnAff af = ln_aff(st, p);
        if (myrow < rows) {
            if (negvar_row) negvar_row[myrow] = st.neg ? 1 : 0;
            if (st.neg && warn && offsets) {
                const int img = image_of_row(offsets, images, myrow);
                atomicOr((unsigned int *)(warn + (img & ~3)), (unsigned int)HV_WARN_LN_NEG_VARIANCE << (8 * (img & 3)));
            }
        }
        const bool all_safe = __all_sync(0xffffffffu, af.safe || myrow >= rows);
        if (OUT32 && all_safe) load_words(0, wn);
#pragma unroll 1
        for (int k = 0; k < g; ++k) {
            const int r = base + 4 * k + grp;
            const bool active = r < rows;
            const int owner = 4 * k + grp;
            // the owner's statistics, for the exact per-element form only (fetched in
            // warp-uniform branches, so the fast form skips the shuffles)
            LnStats rs;
            auto fetch_rs = [&]() {
                rs.mean = shfl64(st.mean, owner);
                rs.inv = (uint64_t)shfl64((int64_t)st.inv, owner);
                rs.neg = false;
            };
            if (OUT32 && all_safe) {
                // Short form with the output stage on the FMA pipe, per element:
                //   t  = vp*ahh + (khh + 255 + kq*2^32)   (vp = v + 128, 64-bit)
                //   nr = vp*aq + hi32(t)            (hi32(t) carries kq, mod 2^32)
                //   o  = (x + 2^(sh-1) - [x < 0]) >> sh,  x = nr*gamma + beta'
                // The +255 keeps hi32(t) equal to the short form's term exactly when the
                // low word of vp*ahh + khh lies in [1, 2^32 - 256] (no carry) and then
                // lifts it to [256, 2^32 - 1]; every other case leaves a low word below
                // 256.  The lanes track the smallest low word, and a pass with one below
                // 256 is redone with the exact per-element form.
                const uint32_t aq = __shfl_sync(0xffffffffu, af.aq, owner);
                const uint32_t ahh = __shfl_sync(0xffffffffu, af.ahh, owner);
                const int32_t kq = __shfl_sync(0xffffffffu, af.kq, owner);
                const uint64_t kh = ((uint64_t)__shfl_sync(0xffffffffu, af.khh, owner) + 255u) +
                                    ((uint64_t)(uint32_t)kq << 32);
                const int32_t half = 1 << (p.sh_out - 1);
                const uint32_t words[6] = {wn[0].x, wn[0].y, wn[1].x, wn[1].y, wn[2].x, wn[2].y};
                load_words(k + 1, wn);
                uint32_t lo_min = 0xFFFFFFFFu, ow[6];
#pragma unroll
                for (int q = 0; q < 6; ++q) {
                    const uint32_t xb = words[q] ^ 0x80808080u;  // bytes v + 128
                    const int4 g01 = gb[2 * q], g23 = gb[2 * q + 1];
                    const int32_t gg[4] = {g01.x, g01.z, g23.x, g23.z}, bb[4] = {g01.y, g01.w, g23.y, g23.w};
                    int32_t o4[4];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const uint32_t vp = __byte_perm(xb, 0u, 0x4440u + b);
                        const uint64_t t = (uint64_t)vp * ahh + kh;
                        lo_min = min(lo_min, (uint32_t)t);
                        const int32_t nr = (int32_t)(vp * aq) + (int32_t)(t >> 32);
                        // xh = x + 2^(sh-1) (the half is folded into bb): the ties-away
                        // shift of x is (xh - [x < 0]) >> sh, and x < 0 iff xh < 2^(sh-1)
                        const int32_t xh = nr * gg[b] + bb[b];
                        o4[b] = (xh - (xh < half ? 1 : 0)) >> p.sh_out;
                    }
                    ow[q] = pack_sat8(o4[0], o4[1], o4[2], o4[3]);
                }
                if (!active) lo_min = 0xFFFFFFFFu;
                if (__any_sync(0xffffffffu, lo_min < 256u)) {
                    fetch_rs();
                    LnAff f;
                    f.aq = aq;
                    f.ahh = ahh;
                    f.khh = (uint32_t)(kh - 255u);
                    f.kq = kq;
                    int32_t v[24];
                    ln_load24(x + (size_t)(active ? r : 0) * 192, sub, active, v);
#pragma unroll
                    for (int q = 0; q < 6; ++q) {
                        int32_t o4[4];
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int i = 4 * q + b;
                            bool ok;
                            int32_t nr = ln_norm_short(v[i], f, ok);
                            if (!ok) nr = ln_norm<SPLIT>(v[i], rs, p);
                            o4[b] = rsa32(nr * gam[i] + bet[i], p.sh_out);
                        }
                        ow[q] = pack_sat8(o4[0], o4[1], o4[2], o4[3]);
                    }
                }
                if (active) {
                    uint2 *dst = (uint2 *)(out + (size_t)r * 192 + 24 * sub);
                    dst[0] = make_uint2(ow[0], ow[1]);
                    dst[1] = make_uint2(ow[2], ow[3]);
                    dst[2] = make_uint2(ow[4], ow[5]);
                }
                continue;
            }
            fetch_rs();
            int32_t v[24];
            ln_load24(x + (size_t)(active ? r : 0) * 192, sub, active, v);
            int32_t o[24];
            if (all_safe) {
                LnAff f;
                f.aq = __shfl_sync(0xffffffffu, af.aq, owner);
                f.ahh = __shfl_sync(0xffffffffu, af.ahh, owner);
                f.khh = __shfl_sync(0xffffffffu, af.khh, owner);
                f.kq = __shfl_sync(0xffffffffu, af.kq, owner);
#pragma unroll
                for (int i = 0; i < 24; ++i) {
                    bool ok;
                    int32_t nr = ln_norm_short(v[i], f, ok);
                    if (!ok) nr = ln_norm<SPLIT>(v[i], rs, p);
                    o[i] = OUT32 ? rsa32(nr * gam[i] + bet[i], p.sh_out) : ln_out<false>(nr, gam[i], bet[i], p);
                }
            } else {
                LnAff f;
                f.al = __shfl_sync(0xffffffffu, af.al, owner);
                f.ah0 = __shfl_sync(0xffffffffu, af.ah0, owner);
                f.ah1 = __shfl_sync(0xffffffffu, af.ah1, owner);
                f.klo = __shfl_sync(0xffffffffu, af.klo, owner);
                f.khi = shfl64(af.khi, owner);
                f.vt = __shfl_sync(0xffffffffu, af.vt, owner);
                const bool rsafe = __shfl_sync(0xffffffffu, af.safe ? 1 : 0, owner) != 0;
#pragma unroll
                for (int i = 0; i < 24; ++i) {
                    if (rsafe) {
                        const int32_t nr = ln_norm_aff(v[i], f);
                        o[i] = OUT32 ? rsa32(nr * gam[i] + bet[i], p.sh_out) : ln_out<false>(nr, gam[i], bet[i], p);
                    } else {
                        o[i] = ln_out<OUT32>(ln_norm<SPLIT>(v[i], rs, p), gam[i], p.beta[24 * sub + i], p);
                    }
                }
            }
            if (active) {
                uint2 *dst = (uint2 *)(out + (size_t)r * 192 + 24 * sub);
                dst[0] = make_uint2(pack_sat8(o[0], o[1], o[2], o[3]), pack_sat8(o[4], o[5], o[6], o[7]));
                dst[1] = make_uint2(pack_sat8(o[8], o[9], o[10], o[11]), pack_sat8(o[12], o[13], o[14], o[15]));
                dst[2] = make_uint2(pack_sat8(o[16], o[17], o[18], o[19]), pack_sat8(o[20], o[21], o[22], o[23]));
            }
        }
    }
    }  // rounds
}

template <bool SPLIT, bool OUT32>
__global__ void __launch_bounds__(256) ln_cls_kernel(const int8_t *x, const int32_t *offsets, int images, int8_t *out,
                                                     LnParams p, uint8_t *warn) {
    griddep_wait();
    griddep_launch();
    const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
    const int i = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * 4 + grp;
    const bool active = i < images;
    int32_t gam[24], bet[24];
    ln_lane_consts<OUT32>(p, sub, gam, bet);
    const bool neg = ln_row8<SPLIT, OUT32>(x + (size_t)(active ? offsets[i] : 0) * 192, out + (size_t)(active ? i : 0) * 192, p,
                                           sub, active, gam, bet);
    if (neg && active && sub == 0 && warn)
        atomicOr((unsigned int *)(warn + (i & ~3)), (unsigned int)HV_WARN_LN_NEG_VARIANCE << (8 * (i & 3)));
}

// --- softmax rows (unit API; the attention kernel fuses its own) -------------
__device__ __forceinline__ uint32_t exp_of(int32_t x, int32_t mx) {
    int64_t xt = (int64_t)x - mx;
    if (xt < -(1ll << 30)) return 0u;   // z >= 23637 there, so E = 0
    return softmax_exp_q16((int32_t)xt);
}

__global__ void softmax_rows_kernel(const int32_t *x, const int32_t *off, int rows, int mode, void *out) {
    const int lane = threadIdx.x & 31;
    const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (r >= rows) return;
    const int a = off[r], n = off[r + 1] - a;
    if (n <= 0) return;
    int32_t mx = INT32_MIN;
    for (int i = lane; i < n; i += 32) mx = max(mx, x[a + i]);
    mx = warp_max_i32(mx);
    uint64_t s = 0;
    for (int i = lane; i < n; i += 32) s += exp_of(x[a + i], mx);
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const uint64_t rc = softmax_recip(s);
    for (int i = lane; i < n; i += 32) {
        const uint64_t e = exp_of(x[a + i], mx);
        const uint64_t ratio = (e * rc + 32768u) >> 16;
        if (mode == 0) {
            const uint64_t v = (ratio + 128u) >> 8;
            ((uint8_t *)out)[a + i] = (uint8_t)(v < 255u ? v : 255u);
        } else {
            ((int32_t *)out)[a + i] = (int32_t)(ratio < 65536u ? ratio : 65536u);
        }
    }
}

// ShiftGELU on a 64-bit argument (|x| < 2^40), for unit-API inputs outside the
// Q8.16 24-bit range; the in-range path is hv::shift_gelu.
__device__ int32_t shift_gelu_wide(int64_t x) {
    const int64_t ip = x + (x >> 1) + (x >> 3) + (x >> 4);
    const int64_t ip2 = ip + (ip >> 1) - (ip >> 4);
    const int64_t a = ip2 < 0 ? -ip2 : ip2;
    const int64_t q = a >> 16;
    const int64_t frac = ((a & 0xFFFF) * 11 + 15) >> 4;
    int64_t e;
    if (ip2 < 0) e = q <= 16 ? ((65536 - frac) >> q) : 0;
    else e = q <= 7 ? min((65536 + frac) << q, (int64_t)8388607) : (int64_t)8388607;
    const int64_t den = 65536 + e;
    const int64_t sig = ((e << 16) + (den >> 1)) / den;
    const i128 p = (i128)x * sig;
    const i128 y = (p + ((i128)1 << 15) + (p >> 127)) >> 16;
    return y > 8388607 ? 8388607 : (y < -8388608 ? -8388608 : (int32_t)y);
}

__global__ void gelu_kernel(const int32_t *x, int64_t n, int32_t *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int32_t v = x[i];
        out[i] = (v >= -(1 << 23) && v < (1 << 23)) ? shift_gelu(v) : shift_gelu_wide(v);
    }
}

__global__ void plan_kernel(const int32_t *x, int64_t n, int32_t *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = plan_sigmoid(x[i]);
}

// Four values per thread.  Groups whose values all lie in [-vlim, vlim] take the
// FMA-pipe chain (gelu_chain_fast2) and the saturating pack; the others, and the
// tail, take the exact 64-bit chain.  k2 = 0 disables the fast form.
__global__ void gelu_requant_kernel(const int32_t *acc, int64_t n, int sh_in, int sh_out, GeluK k, int k2,
                                    int32_t vlim, int8_t *out) {
    const int64_t n4 = n >> 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        int32_t w[4];
        bool ok = k2 != 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            w[j] = acc[4 * i + j];
            ok = ok && w[j] >= -vlim && w[j] <= vlim;
        }
        if (ok) {
            const uint32_t d = pack_sat8(gelu_chain_fast2(w[0], k), gelu_chain_fast2(w[1], k),
                                         gelu_chain_fast2(w[2], k), gelu_chain_fast2(w[3], k));
#pragma unroll
            for (int j = 0; j < 4; ++j) out[4 * i + j] = (int8_t)(d >> (8 * j));
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) out[4 * i + j] = (int8_t)gelu_chain(w[j], sh_in, sh_out);
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3))
        out[4 * n4 + threadIdx.x] = (int8_t)gelu_chain(acc[4 * n4 + threadIdx.x], sh_in, sh_out);
}

__global__ void writeback_kernel(const int64_t *acc, int64_t n, int shift, int bits, void *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t v = requant64(acc[i], shift, bits);
        if (bits == 8) ((int8_t *)out)[i] = (int8_t)v;
        else ((int32_t *)out)[i] = (int32_t)v;
    }
}

__global__ void align_add_kernel(const int8_t *a, const int8_t *b, AlignAdd k, int64_t n, int8_t *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int8_t)align_add8(a[i], b[i], k);
}

// Output of the GELU chain's second half for a Q8.16 input q (|q| < 2^23):
// requant(shift_gelu(q), -16, dst, 8) with sh_out = dst + 16.
__device__ __forceinline__ int32_t gelu_out_q16(int32_t q, int sh_out) {
    return (int32_t)requant64(shift_gelu(q), sh_out, 8);
}

// Change points of gelu_out_q16 over q in [qlo, qlo + n): positions i in [1, n)
// with out(qlo + i) != out(qlo + i - 1); first / last of them land in mm[0] / mm[1].
__global__ void gelu_window_kernel(int32_t qlo, int32_t n, int sh_out, int *mm) {
    for (int32_t i = 1 + blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (gelu_out_q16(qlo + i, sh_out) != gelu_out_q16(qlo + i - 1, sh_out)) {
            atomicMin(&mm[0], i);
            atomicMax(&mm[1], i);
        }
    }
}

__global__ void gelu_table_fill_kernel(int8_t *tab, int32_t wlo, int32_t wn, int sh_out) {
    for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < wn; i += gridDim.x * blockDim.x)
        tab[i] = (int8_t)gelu_out_q16(wlo + i, sh_out);
}

inline int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    return (int)(b < 148 * 16 ? (b < 1 ? 1 : b) : 148 * 16);
}

}  // namespace

cudaError_t launch_layernorm(const int8_t *x, int8_t *out, int rows_max, const int32_t *rows_dev,
                             const LnParams &p, uint8_t *negvar_row, const int32_t *offsets, int images,
                             uint8_t *warn, cudaStream_t st) {
    if (rows_max <= 0) return cudaSuccess;
    auto kern = p.split ? (p.out32 ? ln_kernel<true, true> : ln_kernel<true, false>)
                        : (p.out32 ? ln_kernel<false, true> : ln_kernel<false, false>);
    // One wave: as many CTAs as the GPU holds at once (3 per SM by the launch
    // bounds).  The live row count is read on the device, which sizes each round's
    // passes to it.
    const int variant = (p.split ? 2 : 0) + (p.out32 ? 1 : 0);
    static int s_wave[16][4];  // per device and variant; 0 = not yet queried
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int wave = dev < 16 ? s_wave[dev][variant] : 0;
    if (wave <= 0) {
        int sms = 0, per_sm = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
        if (e != cudaSuccess) return e;
        wave = std::max(1, sms * per_sm);
        if (dev < 16) s_wave[dev][variant] = wave;
    }
    // The whole wave even when fewer 32-row passes would cover the rows: the kernel
    // then picks shorter passes (4 rows per sub-pass, fewer sub-passes per warp), so a
    // small batch finishes in the latency of a shorter pass; CTAs beyond the live rows
    // exit at once.  Tiny calls (unit API) keep one CTA per 8 x 4 rows.
    const int blocks = std::min((rows_max + 31) / 32, wave);
    return launch_pdl(kern, dim3(blocks), dim3(256), 0, st, x, out, rows_max, rows_dev, p, negvar_row, offsets, images,
                      warn);
}

cudaError_t launch_layernorm_cls(const int8_t *x, const int32_t *offsets, int images, int8_t *out,
                                 const LnParams &p, uint8_t *warn, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    auto kern = p.split ? (p.out32 ? ln_cls_kernel<true, true> : ln_cls_kernel<true, false>)
                        : (p.out32 ? ln_cls_kernel<false, true> : ln_cls_kernel<false, false>);
    return launch_pdl(kern, dim3((images + 31) / 32), dim3(256), 0, st, x, offsets, images, out, p, warn);
}

// Image quantisation of the P2 tooling (tools/p2/p2_sim.py:536-545): one CTA per
// image row.  Each thread takes one pixel's three channel values from the CHW
// float planes (coalesced per plane), q = clamp(round_half_even(x * 2^-e),
// -128, 127) (the division by a power of two is exact in fp32, so the product
// equals the quotient), and the row's 672 HWC bytes leave shared memory as words.
__global__ void __launch_bounds__(224) quantize_images_kernel(const float *__restrict__ src, float scale,
                                                              int8_t *__restrict__ dst) {
    __shared__ uint32_t row[168];
    const int h = blockIdx.x, b = blockIdx.y, w = threadIdx.x;
    const float *img = src + (size_t)b * 3 * 224 * 224 + h * 224 + w;
    int8_t *srow = (int8_t *)row;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float v = rintf(img[(size_t)c * 224 * 224] * scale);
        // NaN maps to 0; fminf/fmaxf return the non-NaN operand
        srow[3 * w + c] = (int8_t)(v != v ? 0 : (int)fminf(fmaxf(v, -128.0f), 127.0f));
    }
    __syncthreads();
    if (w < 168) ((uint32_t *)(dst + (size_t)b * 150528 + h * 672))[w] = row[w];
}

cudaError_t launch_quantize_images(const float *src, int batch, int input_exp, int8_t *dst, cudaStream_t st) {
    if (batch <= 0) return cudaSuccess;
    const float scale = ldexpf(1.0f, -input_exp);
    quantize_images_kernel<<<dim3(224, batch), 224, 0, st>>>(src, scale, dst);
    return cudaGetLastError();
}

cudaError_t launch_softmax_rows(const int32_t *x, const int32_t *offsets, int rows, int mode, void *out,
                                cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    softmax_rows_kernel<<<(rows + 7) / 8, 256, 0, st>>>(x, offsets, rows, mode, out);
    return cudaGetLastError();
}

cudaError_t gelu_table_window(int32_t qmax, int sh_out, int *d_mm, int32_t *wlo, int32_t *wn, cudaStream_t st) {
    const int32_t qlo = -qmax, n = 2 * qmax + 1;
    const int init[2] = {0x7fffffff, -1};
    cudaError_t e = cudaMemcpyAsync(d_mm, init, sizeof(init), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return e;
    gelu_window_kernel<<<grid_for(n, 256), 256, 0, st>>>(qlo, n, sh_out, d_mm);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    int mm[2];
    if ((e = cudaMemcpyAsync(mm, d_mm, sizeof(mm), cudaMemcpyDeviceToHost, st)) != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(st)) != cudaSuccess) return e;
    if (mm[1] < 0) {  // constant over the whole range
        *wlo = qlo;
        *wn = 1;
    } else {
        *wlo = qlo + mm[0] - 1;
        *wn = mm[1] - mm[0] + 2;
    }
    return cudaSuccess;
}

cudaError_t launch_gelu_table_fill(int8_t *tab, int32_t wlo, int32_t wn, int sh_out, cudaStream_t st) {
    gelu_table_fill_kernel<<<grid_for(wn, 256), 256, 0, st>>>(tab, wlo, wn, sh_out);
    return cudaGetLastError();
}

cudaError_t launch_gelu(const int32_t *x, int64_t n, int32_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    gelu_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, out);
    return cudaGetLastError();
}

cudaError_t launch_plan(const int32_t *x, int64_t n, int32_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    plan_kernel<<<grid_for(n, 256), 256, 0, st>>>(x, n, out);
    return cudaGetLastError();
}

cudaError_t launch_gelu_requant(const int32_t *acc, int64_t n, int sh_in, int sh_out, int8_t *out,
                                cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int32_t vlim = 0;
    const int k2 = gelu_fast2_range(sh_in, sh_out, &vlim);
    gelu_requant_kernel<<<grid_for((n + 3) / 4, 256), 256, 0, st>>>(acc, n, sh_in, sh_out,
                                                                   make_gelu_k(k2 ? sh_in : 0, k2 ? sh_out : 0),
                                                                   k2, vlim, out);
    return cudaGetLastError();
}

cudaError_t launch_align_add(const int8_t *a, const int8_t *b, AlignAdd k, int64_t n, int8_t *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    align_add_kernel<<<grid_for(n, 256), 256, 0, st>>>(a, b, k, n, out);
    return cudaGetLastError();
}

cudaError_t launch_writeback(const int64_t *acc, int64_t n, int shift, int bits, void *out, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    writeback_kernel<<<grid_for(n, 256), 256, 0, st>>>(acc, n, shift, bits, out);
    return cudaGetLastError();
}

}  // namespace hv
