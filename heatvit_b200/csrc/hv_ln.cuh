// hv_ln.cuh — LayerNorm arithmetic of the LayerNorm kernels (hv_rows.cu): row
// statistics, the per-row affine constants of the 2^48 normalisation and its exact
// fallbacks (nonlinear.py:136-186), kept apart from the kernels so that any kernel
// that normalises rows can include them.
#pragma once
#include "hv_internal.cuh"

namespace hv {

typedef __int128 i128;
typedef unsigned __int128 u128;

namespace {

// requant of a 128-bit value (requant64 semantics).
__device__ __forceinline__ int32_t requant128_8(i128 v, int shift) {
    if (shift > 0) {
        if (shift >= 126) return 0;
        i128 r = (v + ((i128)1 << (shift - 1)) + (v >> 127)) >> shift;
        return r > 127 ? 127 : (r < -128 ? -128 : (int32_t)r);
    }
    if (shift == 0) return v > 127 ? 127 : (v < -128 ? -128 : (int32_t)v);
    if (v == 0) return 0;
    const int ls = -shift;
    if (ls >= 16) return v > 0 ? 127 : -128;
    i128 r = v << ls;
    return r > 127 ? 127 : (r < -128 ? -128 : (int32_t)r);
}

// Row statistics shared by the 8 lanes of a row group (nonlinear.py:159-172):
// mean, inv_std_q32 and the negative-variance flag.
struct LnStats {
    int64_t mean;
    uint64_t inv;
    bool neg;
};

__device__ __forceinline__ LnStats ln_stats(int32_t s, int64_t s2, const LnParams &p) {
    LnStats st;
    const int64_t sum_x = (int64_t)s << p.sh_sum;
    st.mean = round_div64(sum_x, 192);
    const int64_t e2 = round_div64(s2, 192);
    const uint64_t am = (uint64_t)(st.mean < 0 ? -st.mean : st.mean);
    const int64_t mean_sq = (int64_t)(((u128)am * am + ((u128)1 << 31)) >> 32);
    int64_t var = e2 - mean_sq;
    st.neg = var < 0;
    if (st.neg) var = 0;
    const uint64_t sd = isqrt64((uint64_t)var + 4295u);
    // inv = round_div(2^48, sd): a double-precision quotient (within 1 of the
    // floor, as 2^48 / sd < 2^42) corrected by the exact remainder.
    uint64_t inv = (uint64_t)(281474976710656.0 / (double)sd);
    int64_t rem = (int64_t)(((uint64_t)1 << 48) - inv * sd);
    if (rem < 0) { inv -= 1; rem += (int64_t)sd; }
    if (rem >= (int64_t)sd) { inv += 1; rem -= (int64_t)sd; }
    if (2 * (uint64_t)rem >= sd) inv += 1;
    st.inv = inv;
    return st;
}

// Affine form of the normalisation for one row.  With s = sh_sum and v the int8
// input, prod = (v*2^s - mean) * inv and T = prod + 2^47 = (v + 128) * A + K for
// A = inv * 2^s and K = 2^47 - mean*inv - 128*A, both fixed per row.  Then
// rsa(prod, 48) = floor((T - [prod < 0]) / 2^48), and prod < 0 iff v + 128 < vt.
// `safe`: |prod| + 2^47 < 2^71 for every int8 v, so the result needs no 24-bit
// saturation and fits 32 bits.  inv < 2^42 (sd >= 65) and s <= 32 give A < 2^74,
// |K| < 2^82.
struct LnAff {
    uint32_t al, ah0, ah1, klo;  // A = ah1*2^64 + ah0*2^32 + al, K mod 2^32
    int64_t khi;                 // floor(K / 2^32)
    int32_t vt;
    bool safe;
    // short form (safe rows): A = aq*2^48 + ahh*2^16 + (A mod 2^16),
    // K = kq*2^48 + khh*2^16 + (K mod 2^16), see ln_norm_short
    uint32_t aq, ahh, khh;
    int32_t kq;
};

__device__ __forceinline__ LnAff ln_aff(const LnStats &st, const LnParams &p) {
    LnAff f;
    const u128 A = (u128)st.inv << p.sh_sum;
    f.al = (uint32_t)A;
    const uint64_t ah = (uint64_t)(A >> 32);
    f.ah0 = (uint32_t)ah;
    f.ah1 = (uint32_t)(ah >> 32);
    const i128 K = ((i128)1 << 47) - (i128)st.mean * (i128)st.inv - (i128)128 * (i128)A;
    f.klo = (uint32_t)(u128)K;
    f.khi = (int64_t)(K >> 32);
    int64_t vt = -((-st.mean) >> p.sh_sum);  // ceil(mean / 2^s): prod >= 0 iff v >= vt
    vt = vt < -128 ? -128 : (vt > 128 ? 128 : vt);
    f.vt = (int32_t)vt + 128;
    const i128 d1 = ((i128)127 << p.sh_sum) - st.mean, d2 = st.mean + ((i128)128 << p.sh_sum);
    const u128 dm = (u128)(d1 > d2 ? d1 : d2);
    f.safe = dm * st.inv + ((u128)1 << 47) < ((u128)1 << 71);
    const u128 m48 = ((u128)1 << 48) - 1;
    f.aq = (uint32_t)(A >> 48);
    f.ahh = (uint32_t)((A & m48) >> 16);
    f.kq = (int32_t)(K >> 48);                    // floor; in int32 range on safe rows
    f.khh = (uint32_t)(((u128)K & m48) >> 16);    // K - kq*2^48 in [0, 2^48)
    return f;
}

// ln_norm_aff in 32-bit pieces, valid on safe rows.  With vp = v + 128 < 2^8,
// R = vp*(A mod 2^48) + (K mod 2^48) = 2^16*t + e, t = vp*ahh + khh and
// e = vp*(A mod 2^16) + (K mod 2^16) < 2^24, so floor(T / 2^48) =
// vp*aq + kq + floor((t + floor(e / 2^16)) / 2^32) with floor(e / 2^16) <= 255.
// When the low word of t lies in [1, 2^32 - 256] that is vp*aq + kq + (t >> 32)
// exactly, and T is no multiple of 2^48 (no tie correction).  *ok = false
// otherwise (about 2^-24 of inputs): the caller takes the exact form.
__device__ __forceinline__ int32_t ln_norm_short(int32_t v, const LnAff &f, bool &ok) {
    const uint32_t vp = (uint32_t)(v + 128);
    const uint64_t t = (uint64_t)vp * f.ahh + f.khh;
    ok = (uint32_t)t - 1u < 0xFFFFFF00u;
    return (int32_t)(vp * f.aq) + f.kq + (int32_t)(t >> 32);
}

// norm of one int8 input on a safe row (see LnAff).
__device__ __forceinline__ int32_t ln_norm_aff(int32_t v, const LnAff &f) {
    const uint32_t vp = (uint32_t)(v + 128);
    const uint64_t S = (uint64_t)vp * f.al + f.klo;                          // < 2^41
    const uint64_t Q = (uint64_t)vp * f.ah0 + ((uint64_t)(vp * f.ah1) << 32);  // < 2^50
    const int64_t U = (int64_t)Q + f.khi + (int64_t)(S >> 32);              // floor(T / 2^32)
    int32_t nr = (int32_t)(U >> 16);                                         // floor(T / 2^48)
    if ((uint32_t)S == 0u) {
        // T is a multiple of 2^48 only if its low 48 bits vanish; then a negative
        // product rounds one lower.
        if ((U & 0xFFFF) == 0 && (int32_t)vp < f.vt) nr -= 1;
    }
    return nr;
}

// norm = sat24(rsa((x_q32 - mean) * inv, 48)) (nonlinear.py:176-179).
// Split path (|d| <= 2^36, inv < 2^42): with inv = hi*2^16 + lo, T = d*inv =
// U*2^16 + B_lo where U = d*hi + floor(d*lo / 2^16) and B_lo = (d*lo) mod 2^16.
// The ties-away rounding floor((T + 2^47 - [T<0]) / 2^48) then equals
// floor((U + 2^31 - [T<0 and B_lo == 0]) / 2^32), because the dropped low part
// is a fraction in [0, 1) of the 2^16 unit.
template <bool SPLIT>
__device__ __forceinline__ int32_t ln_norm(int32_t v, const LnStats &st, const LnParams &p) {
    const int64_t d = ((int64_t)v << p.sh_sum) - st.mean;
    int64_t nr;
    if (SPLIT) {
        const int64_t hi = (int64_t)(st.inv >> 16), lo = (int64_t)(st.inv & 0xFFFFu);
        const int64_t a = d * hi;
        const int64_t b = d * lo;
        const int64_t u = a + (b >> 16);
        const int64_t adj = (d < 0 && (b & 0xFFFF) == 0) ? 1 : 0;
        nr = (u + ((int64_t)1 << 31) - adj) >> 32;
    } else {
        const i128 prod = (i128)d * (i128)st.inv;
        const i128 r = (prod + ((i128)1 << 47) + (prod >> 127)) >> 48;
        nr = r > 8388607 ? 8388607 : (r < -8388608 ? -8388608 : (int64_t)r);
    }
    return (int32_t)clamp_i64(nr, -8388608, 8388607);
}

// out = requant((norm*gamma << sh_g) + (beta << sh_b), common, out, 8) (nonlinear.py:181-186).
template <bool OUT32>
__device__ __forceinline__ int32_t ln_out(int32_t norm, int32_t g, int32_t b, const LnParams &p) {
    const int32_t prodg = norm * g;
    if (OUT32) return requant8_r(prodg + b * (1 << p.sh_b), p.sh_out);
    if (p.fast) return (int32_t)requant64(((int64_t)prodg << p.sh_g) + ((int64_t)b << p.sh_b), p.sh_out, 8);
    return requant128_8(((i128)prodg << p.sh_g) + ((i128)b << p.sh_b), p.sh_out);
}

__device__ __forceinline__ int image_of_row(const int32_t *offsets, int images, int row) {
    int lo = 0, hi = images - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= row) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ int64_t shfl64(int64_t v, int src) {
    const int32_t lo = __shfl_sync(0xffffffffu, (int32_t)v, src);
    const int32_t hi = __shfl_sync(0xffffffffu, (int32_t)(v >> 32), src);
    return (int64_t)(((uint64_t)(uint32_t)hi << 32) | (uint32_t)lo);
}

}  // namespace
}  // namespace hv
