// hv_fixed.cuh — integer fixed-point primitives for the HeatViT-T engine.
//
// Device restatements of the golden model's numeric contract
// (verification/heatvit_ref/fixed.py:15-80, nonlinear.py:60-186).  Rounding is
// ties-away-from-zero everywhere; every helper documents the operand range it
// is exact for.  No floating-point result is ever used without an exact integer
// correction step.
#pragma once
#include <stdint.h>

#define HV_DEV __device__ __forceinline__
#define HV_HD __host__ __device__ __forceinline__

namespace hv {

// ---------------------------------------------------------------------------
// Rounding shifts (fixed.py:15-25)
// ---------------------------------------------------------------------------

// Ties-away right shift of a 32-bit value by s in [1, 30], valid while
// |v| + 2^(s-1) < 2^31.  For v >= 0 it is floor((v + 2^(s-1)) / 2^s); for v < 0
// the ties-away value -floor((|v| + 2^(s-1)) / 2^s) equals
// floor((v + 2^(s-1) - 1) / 2^s), hence the (v >> 31) correction term.
HV_HD int32_t rsa32(int32_t v, int s) {
    return (v + (1 << (s - 1)) + (v >> 31)) >> s;
}

// Same on 64-bit values, s in [1, 62], |v| + 2^(s-1) < 2^63.
HV_HD int64_t rsa64(int64_t v, int s) {
    return (v + ((int64_t)1 << (s - 1)) + (v >> 63)) >> s;
}

// round_shift_away with any signed shift on a 64-bit value (negative = left
// shift); callers guarantee the left-shifted value fits in 64 bits.
HV_HD int64_t rsa64_any(int64_t v, int s) {
    if (s > 0) return s >= 63 ? 0 : rsa64(v, s);
    return v << (-s);
}

HV_HD int32_t clamp_i32(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
HV_HD int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

HV_HD int32_t sat8(int32_t v) { return clamp_i32(v, -128, 127); }
HV_HD int32_t sat24(int32_t v) { return clamp_i32(v, -(1 << 23), (1 << 23) - 1); }

// requant (fixed.py:37-45) of a 64-bit value to `bits` in {8, 24, 32} with
// shift = dst - src (any sign).  A left shift saturates by sign once the value
// is out of range, matching the unbounded Python result after saturation.
HV_HD int64_t requant64(int64_t v, int shift, int bits) {
    const int64_t hi = ((int64_t)1 << (bits - 1)) - 1, lo = -hi - 1;
    if (shift > 0) {
        if (shift >= 63) return 0;  // |v| < 2^62 in every caller
        return clamp_i64(rsa64(v, shift), lo, hi);
    }
    if (shift == 0) return clamp_i64(v, lo, hi);
    const int ls = -shift;
    if (v == 0) return 0;
    if (ls >= 40) return v > 0 ? hi : lo;
    const int64_t lim = (int64_t)1 << (62 - ls);
    if (v >= lim) return hi;
    if (v <= -lim) return lo;
    return clamp_i64(v << ls, lo, hi);
}

// Fast int8 requant of a 32-bit value with a right shift s in [1, 30]
// (|v| + 2^(s-1) < 2^31).
HV_HD int32_t requant8_r(int32_t v, int s) { return sat8(rsa32(v, s)); }

// ---------------------------------------------------------------------------
// Division helpers (fixed.py:58-72 round_div, fixed.py:75-80 isqrt)
// ---------------------------------------------------------------------------

// round_div for a non-negative denominator: nearest, ties away from zero, sign
// of the numerator.
HV_HD int64_t round_div64(int64_t n, int64_t d) {
    uint64_t an = n < 0 ? (uint64_t)(-n) : (uint64_t)n;
    uint64_t q = an / (uint64_t)d, r = an - q * (uint64_t)d;
    if (2 * r >= (uint64_t)d) q += 1;
    return n < 0 ? -(int64_t)q : (int64_t)q;
}

// Exact floor(n / d) for n < 2^32 and d in [2^16, 2^24): a float estimate of
// the quotient (relative error < 2^-21, so |estimate - q| <= 1 for q < 2^17)
// followed by an exact integer remainder correction.
HV_DEV uint32_t udiv_u32_small_q(uint32_t n, uint32_t d) {
    float fq = __fdividef(__uint2float_rz(n), __uint2float_rn(d));
    uint32_t q = __float2uint_rz(fq);
    int32_t r = (int32_t)(n - q * d);          // |true remainder| < 2d < 2^25
    if (r < 0) { q -= 1; r += (int32_t)d; }
    if (r >= (int32_t)d) { q += 1; }
    return q;
}

// Floor square root of v < 2^62 (fixed.py:75-80 isqrt): a double estimate
// corrected by exact integer comparisons.
HV_DEV uint64_t isqrt64(uint64_t v) {
    uint64_t s = (uint64_t)sqrt((double)v);
    while (s > 0 && s * s > v) --s;
    while ((s + 1) * (s + 1) <= v) ++s;
    return s;
}

// ---------------------------------------------------------------------------
// ShiftGELU (nonlinear.py:60-80): Q8.16 in [-2^23, 2^23) -> Q8.16
// ---------------------------------------------------------------------------
// The division sig = floor(((e << 16) + (den >> 1)) / den) with den = 2^16 + e
// is rewritten without 64-bit operands: e*2^16 + h = den*2^16 - (2^32 - h), so
// sig = 2^16 - ceil((2^32 - h) / den) = 65535 - floor((2^32 - 1 - h) / den),
// and 2^32 - 1 - h is ~h in 32 bits.  den lies in [2^16, 2^23 + 2^16), so the
// quotient is below 2^17 and udiv_u32_small_q is exact.  |x * sig| < 2^39 and
// |y| <= 2^23 - 128, so the final sat24 of the golden model never clips.
HV_DEV int32_t shift_gelu(int32_t x) {
    int32_t ip = x + (x >> 1) + (x >> 3) + (x >> 4);     // 1.702x
    int32_t ip2 = ip + (ip >> 1) - (ip >> 4);            // * log2(e)
    uint32_t a = (uint32_t)(ip2 < 0 ? -ip2 : ip2);
    uint32_t q = a >> 16;
    uint32_t frac = ((a & 0xFFFFu) * 11u + 15u) >> 4;    // slope 11/16
    uint32_t e;
    if (ip2 < 0) {
        e = (65536u - frac) >> (q < 31u ? q : 31u);      // q > 16 gives 0 anyway
    } else {
        uint32_t t = (65536u + frac) << (q < 8u ? q : 8u);
        e = t < 8388607u ? t : 8388607u;                  // q >= 8 saturates
    }
    uint32_t den = 65536u + e;
    uint32_t sig = 65535u - udiv_u32_small_q(~(den >> 1), den);
    int64_t p = (int64_t)x * (int64_t)sig;
    return (int32_t)rsa64(p, 16);
}

// The FFN / selector GELU post-op chain
// requant(gelu(requant(v, src, -16, 24)), -16, dst, 8)
// (transformer.py:351-356, selector.py:89-99).  sh_in = -16 - src,
// sh_out = dst + 16.
HV_DEV int32_t gelu_chain(int64_t v, int sh_in, int sh_out) {
    int32_t q16 = (int32_t)requant64(v, sh_in, 24);
    return (int32_t)requant64(shift_gelu(q16), sh_out, 8);
}

// 32-bit form of gelu_chain for host-checked ranges: |v| < 2^30, sh_in in
// [1, 30] (q16 = sat24(rsa(v, sh_in))) and sh_out in [-7, 30] (|gelu| < 2^23,
// so a left shift by at most 7 stays inside int32 before the int8 clamp).
HV_DEV int32_t gelu_chain_fast(int32_t v, int sh_in, int sh_out) {
    const int32_t q16 = sat24(rsa32(v, sh_in));
    const int32_t g = shift_gelu(q16);
    return sh_out >= 1 ? requant8_r(g, sh_out) : sat8(g * (1 << -sh_out));
}

// ---------------------------------------------------------------------------
// FMA-pipe form of the GELU chain
// ---------------------------------------------------------------------------
// The integer ALU pipe issues at half the rate of the FP32/IMAD pipes, and the
// chain above is almost all ALU work.  gelu_chain_fast2 computes the same value
// with part of the work moved to multiplier forms:
//   * mul.hi.s32(x, 2^(32-k)) = floor(x / 2^k) = x >> k  (k >= 2),
//     mul.hi.u32(x, 2^(32-k)) = x >> k for unsigned x,
//     mul.hi.s32(x, 2) = x >> 31 for |x| < 2^30;
//   * mad.lo.s32 with a multiplier of 1 or -1 in place of an add;
//   * the quotient floor(n / den) of shift_gelu from a single-precision
//     reciprocal estimate (rcp.approx.ftz.f32, at most 1 ulp from 1/den by the
//     PTX ISA), biased so that it is q or q + 1, then one exact integer
//     correction;
//   * integer <-> float conversions by exponent-bias arithmetic
//     (2^23 + e has the bit pattern 0x4B000000 + e for 0 <= e < 2^23).
// The multiplier constants are kernel arguments (GeluK) so the compiler cannot
// fold them back into shifts.  Valid for sh_in in [0, 30] when |v| + 2^(sh_in-1)
// < 2^30 and |rsa(v, sh_in)| < 2^23 (no saturation to 24 bits), and sh_out in
// [-7, 30]; the result is the unsaturated requantised value, which the caller
// saturates to int8 (pack_sat8).
struct GeluK {
    int32_t sh_in, hin, ksgn;          // x = (v + hin + mulhi(v, ksgn)) >> sh_in
    int32_t one, m1, c11, m65536;      // 1, -1, 11, -65536
    int32_t c28, c29, two;             // 2^28, 2^29, 2
    uint32_t c16u, c28u, c31u;         // 2^16, 2^28, 2^31
    int32_t so_r, hout, ksgn_o, mul_l; // requant of the GELU value to the output scale
};

inline GeluK make_gelu_k(int sh_in, int sh_out) {
    GeluK k;
    k.sh_in = sh_in;
    k.hin = sh_in > 0 ? 1 << (sh_in - 1) : 0;
    k.ksgn = sh_in > 0 ? 2 : 0;
    k.one = 1;
    k.m1 = -1;
    k.c11 = 11;
    k.m65536 = -65536;
    k.c28 = 1 << 28;
    k.c29 = 1 << 29;
    k.two = 2;
    k.c16u = 1u << 16;
    k.c28u = 1u << 28;
    k.c31u = 1u << 31;
    if (sh_out >= 1) {
        k.so_r = sh_out;
        k.hout = 1 << (sh_out - 1);
        k.ksgn_o = 2;
        k.mul_l = 1;
    } else {
        k.so_r = 0;
        k.hout = 0;
        k.ksgn_o = 0;
        k.mul_l = 1 << (-sh_out);
    }
    return k;
}

// Whether gelu_chain_fast2 applies for these shifts, and the largest |v| it
// accepts: |v| + 2^(sh_in-1) < 2^30 and |rsa(v, sh_in)| < 2^23.
inline int gelu_fast2_range(int sh_in, int sh_out, int32_t *vlim) {
    if (sh_in < 0 || sh_in > 30 || sh_out < -7 || sh_out > 30) return 0;
    const int64_t hin = sh_in > 0 ? (int64_t)1 << (sh_in - 1) : 0;
    int64_t lim = ((int64_t)1 << 30) - hin - 1;
    const int64_t sat = ((int64_t)1 << (23 + sh_in)) - hin - 1;
    if (sat < lim) lim = sat;
    *vlim = (int32_t)lim;
    return 1;
}

HV_DEV int32_t mulhi_s(int32_t a, int32_t b) {
    int32_t r;
    asm("mul.hi.s32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
HV_DEV uint32_t mulhi_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
HV_DEV int32_t mad_s(int32_t a, int32_t b, int32_t c) {
    int32_t r;
    asm("mad.lo.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

HV_DEV int32_t gelu_chain_fast2(int32_t v, const GeluK &k) {
    // q16 = rsa(v, sh_in), no saturation by the caller's range check.
    const int32_t x = (v + k.hin + mulhi_s(v, k.ksgn)) >> k.sh_in;
    // shift_gelu (nonlinear.py:60-80): ip = 1.702x, ip2 = ip * log2(e)
    const int32_t ip = x + (x >> 1) + mulhi_s(x, k.c29) + mulhi_s(x, k.c28);
    const int32_t ip2 = ip + (ip >> 1) - mulhi_s(ip, k.c28);
    const uint32_t a = (uint32_t)(ip2 < 0 ? -ip2 : ip2);
    const uint32_t q = mulhi_u(a, k.c16u);
    const uint32_t lo = (uint32_t)mad_s((int32_t)q, k.m65536, (int32_t)a);
    const uint32_t frac = mulhi_u((uint32_t)mad_s((int32_t)lo, k.c11, 15), k.c28u);
    uint32_t en;
    asm("shr.b32 %0, %1, %2;" : "=r"(en) : "r"(65536u - frac), "r"(q));  // shifts >= 32 give 0
    const uint32_t tp = (65536u + frac) << (q < 8u ? q : 8u);
    const uint32_t e = ip2 < 0 ? en : (tp < 8388607u ? tp : 8388607u);
    // sig = 65535 - floor(n / den), den = 2^16 + e, n = 2^32 - 1 - floor(den / 2)
    const float fe = __int_as_float(mad_s((int32_t)e, k.one, 0x4B000000)) - 8388608.0f;
    float rc;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rc) : "f"(fe + 65536.0f));
    // n / den = 2^32 / den - (floor(den/2) + 1) / den, the last term in (0.5, 0.5 + 2^-16]:
    // the estimate below lies within 0.03 of n / den + 0.25, so it rounds to q or q + 1.
    const float fq = fmaf(4294967296.0f, rc, -0.25f);
    int32_t qe = mad_s(__float_as_int(fq + 12582912.0f), k.one, -0x4B400000);
    const int32_t nh = mad_s((int32_t)mulhi_u(e, k.c31u), k.m1, -32769);    // ~(den >> 1)
    const int32_t r = mad_s(qe, mad_s((int32_t)e, k.m1, -65536), nh);       // n - qe * den
    qe += mulhi_s(r, k.two);                                                 // r < 0: q + 1 -> q
    const int32_t sig = 65535 - qe;
    const int64_t p = (int64_t)x * sig;
    const int32_t g = (int32_t)((p + 32768 + (x >> 31)) >> 16);             // rsa(x * sig, 16)
    // requant to the output scale (saturated by the caller)
    return ((g + k.hout + mulhi_s(g, k.ksgn_o)) >> k.so_r) * k.mul_l;
}

// Saturate four int32 values to int8 and pack them (w0 in the low byte):
// cvt.pack.sat.s8.s32.b32 d, a, b, c puts sat(b) in byte 0, sat(a) in byte 1 and
// the low half of c in bytes 2-3.
HV_DEV uint32_t pack_sat8(int32_t w0, int32_t w1, int32_t w2, int32_t w3) {
    uint32_t hi, d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(w3), "r"(w2));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(w1), "r"(w0), "r"(hi));
    return d;
}

// Saturate four non-negative int32 values to [0, 255] and pack them (w0 low).
HV_DEV uint32_t pack_satu8(int32_t w0, int32_t w1, int32_t w2, int32_t w3) {
    uint32_t hi, d;
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(w3), "r"(w2));
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(w1), "r"(w0), "r"(hi));
    return d;
}

// PLAN sigmoid (nonlinear.py:83-95), unsigned Q0.16.
HV_HD int32_t plan_sigmoid(int32_t x) {
    int32_t ax = x < 0 ? -x : x, y;
    if (ax >= 327680) y = 65536;
    else if (ax >= 155648) y = (ax >> 5) + 55296;
    else if (ax >= 65536) y = (ax >> 3) + 40960;
    else y = (ax >> 2) + 32768;
    return x < 0 ? 65536 - y : y;
}

// ---------------------------------------------------------------------------
// Shift-softmax pieces (nonlinear.py:98-133)
// ---------------------------------------------------------------------------
// exp of a non-positive Q8.16 argument xt = x - max, |xt| < 2^31.
// z = floor(-xt / 45426) is a multiply-high by the invariant reciprocal
// m = ceil(2^47 / 45426) = 3098170395 followed by a 15-bit shift (division by an
// invariant integer, Granlund & Montgomery 1994): m * 45426 - 2^47 < 2^16, so the
// quotient is exact for every n < 2^31 (checked exhaustively).  Then
// p = xt + z*45426 = -r with r the remainder.  A shift by z >= 32 gives 0 under
// PTX shr semantics, and e < 2^17 makes z = 31 give 0 as well.
HV_DEV uint32_t softmax_exp_q16(int32_t xt) {
    const uint32_t n = (uint32_t)(-xt);
    const uint32_t z = __umulhi(n, 3098170395u) >> 15;
    const uint32_t r = n - z * 45426u;
    const uint32_t sh = 88670u - r;                                   // p + 88670, in (43244, 88670]
    const uint64_t sq = ((uint64_t)sh * sh + 32768u) >> 16;           // rsa(sh^2, 16), <= 119970
    const uint32_t e = ((uint32_t)(23495u * (uint32_t)sq + 32768u) >> 16) + 22544u;
    uint32_t out;
    asm("shr.b32 %0, %1, %2;" : "=r"(out) : "r"(e), "r"(z));
    return out;
}

// softmax_exp_q16 of xt = -n, in 32-bit pieces.  With sh' = 88670 - r - 65536 =
// z*45426 + 23134 - n in [-22291, 23134]: rsa(sh^2, 16) = 65536 + 2*sh' + t,
// t = (sh'^2 + 32768) >> 16, so e = 46039 + floor((46990*sh' + 23495*t + 32768) / 2^16)
// (the 2^32 and 2^17*sh' parts are whole multiples of 2^16).  Equal to
// softmax_exp_q16(-n) for every n in [0, 2^31), checked exhaustively on the host.
HV_DEV uint32_t softmax_exp_q16_n(uint32_t n) {
    const uint32_t z = __umulhi(n, 3098170395u) >> 15;
    const int32_t shp = (int32_t)(z * 45426u + 23134u - n);
    const int32_t t = (int32_t)(((uint32_t)(shp * shp) + 32768u) >> 16);
    const int32_t u = 46990 * shp + 23495 * t + 32768;
    const uint32_t e = (uint32_t)((u >> 16) + 46039);
    uint32_t out;
    asm("shr.b32 %0, %1, %2;" : "=r"(out) : "r"(e), "r"(z));
    return out;
}

// recip = round_div(2^32, S) for S >= 1.
HV_DEV uint64_t softmax_recip(uint64_t s) {
    uint64_t q = ((uint64_t)1 << 32) / s, r = ((uint64_t)1 << 32) - q * s;
    if (2 * r >= s) q += 1;
    return q;
}

// round_div(2^32, S) for a softmax row sum S in [65554, 2^25) (every term <= 65554
// and the row maximum's term equal to it, at most 224 columns): q0 from a single-precision quotient
// (relative error below 2^-21, so within 1 of the true quotient, which is < 65520),
// then the exact remainder r = 2^32 - q*S fixes q to floor(2^32 / S) and the
// ties-away rounding adds one when 2r >= S.
__device__ __forceinline__ uint32_t softmax_recip32(uint32_t S) {
    int32_t q = (int32_t)__fdividef(4294967296.0f, __uint2float_rn(S));
    int64_t r = ((int64_t)1 << 32) - (int64_t)q * S;
    if (r < 0) { q -= 1; r += S; }
    if (r >= (int64_t)S) { q += 1; r -= S; }
    return (uint32_t)(2 * r >= (int64_t)S ? q + 1 : q);
}

// ratio = rsa(E * recip, 16); scaled = rsa(ratio * 65536, 16) == ratio.
HV_DEV uint32_t softmax_ratio(uint32_t e, uint64_t recip) {
    return (uint32_t)(((uint64_t)e * recip + 32768u) >> 16);
}

// Attention narrowing: min(rsa(scaled, 8), 255) (nonlinear.py:130-133).
HV_DEV uint32_t softmax_attn_u8(uint32_t ratio) {
    uint32_t v = (ratio + 128u) >> 8;
    return v < 255u ? v : 255u;
}

// ---------------------------------------------------------------------------
// Residual align-add (transformer.py:96-101)
// ---------------------------------------------------------------------------
// out = requant((a << (ea - c)) + (b << (eb - c)), c, eo, 8), c = min(ea, eb).
struct AlignAdd {
    int sa, sb, sh;   // left shifts of a and b, requant shift eo - c
    int fast;         // sa, sb <= 22 and sh in [1, 30]: the sum fits int32
};

HV_HD AlignAdd make_align_add(int ea, int eb, int eo) {
    int c = ea < eb ? ea : eb;
    AlignAdd r;
    r.sa = ea - c;
    r.sb = eb - c;
    r.sh = eo - c;
    r.fast = (r.sa <= 22 && r.sb <= 22 && r.sh >= 1 && r.sh <= 30) ? 1 : 0;
    return r;
}

// Exact for shifts up to 54 (int8 << 54 stays below 2^62).
HV_HD int32_t align_add8(int32_t a, int32_t b, AlignAdd k) {
    if (k.fast) return requant8_r(a * (1 << k.sa) + b * (1 << k.sb), k.sh);
    int64_t v = ((int64_t)a << k.sa) + ((int64_t)b << k.sb);
    return (int32_t)requant64(v, k.sh, 8);
}

}  // namespace hv
