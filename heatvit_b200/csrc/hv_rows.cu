// hv_rows.cu — warp-per-row LayerNorm and shift-softmax, element-wise units.
//
// LayerNorm (nonlinear.py:136-186) over D = 192: one warp per row, each lane
// owns 6 channels (bytes 4l..4l+3 and 128+2l..129+2l, so every load and
// store is aligned and the warp touches the row with two coalesced accesses).
// The 81-bit product (x_q32 - mean) * inv_std_q32 is formed in 128 bits.
#include "hv_internal.cuh"

namespace hv {

typedef __int128 i128;
typedef unsigned __int128 u128;

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
    return p;
}

namespace {

__device__ __forceinline__ int32_t warp_sum_i32(int32_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int64_t warp_sum_i64(int64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int32_t warp_max_i32(int32_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

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

// One row; returns true on negative variance.  Whole warp participates.
__device__ __forceinline__ bool ln_row(const int8_t *xr, int8_t *outr, const LnParams &p, int lane) {
    const int w4 = *(const int32_t *)(xr + 4 * lane);
    const int16_t w2 = *(const int16_t *)(xr + 128 + 2 * lane);
    int32_t v[6];
    v[0] = (int8_t)(w4 & 0xff);
    v[1] = (int8_t)((w4 >> 8) & 0xff);
    v[2] = (int8_t)((w4 >> 16) & 0xff);
    v[3] = (int8_t)((w4 >> 24) & 0xff);
    v[4] = (int8_t)(w2 & 0xff);
    v[5] = (int8_t)((w2 >> 8) & 0xff);
    int32_t s = 0;
#pragma unroll
    for (int i = 0; i < 6; ++i) s += v[i];
    s = warp_sum_i32(s);
    int64_t s2;
    if (p.sq_shift >= 0) {
        int32_t q = 0;
#pragma unroll
        for (int i = 0; i < 6; ++i) q += v[i] * v[i];
        s2 = (int64_t)warp_sum_i32(q) << p.sq_shift;
    } else {
        const int k = -p.sq_shift;  // per-element ties-away right shift (x^2 >= 0)
        int64_t q = 0;
#pragma unroll
        for (int i = 0; i < 6; ++i) q += ((int64_t)(v[i] * v[i]) + ((int64_t)1 << (k - 1))) >> k;
        s2 = warp_sum_i64(q);
    }
    const int64_t sum_x = (int64_t)s << p.sh_sum;
    const int64_t mean = round_div64(sum_x, 192);
    const int64_t e2 = round_div64(s2, 192);
    const uint64_t am = (uint64_t)(mean < 0 ? -mean : mean);
    const int64_t mean_sq = (int64_t)(((u128)am * am + ((u128)1 << 31)) >> 32);
    int64_t var = e2 - mean_sq;
    const bool neg = var < 0;
    if (neg) var = 0;
    const uint64_t sd = isqrt64((uint64_t)var + 4295u);
    uint64_t inv = ((uint64_t)1 << 48) / sd;
    if (2 * (((uint64_t)1 << 48) - inv * sd) >= sd) inv += 1;

    int32_t o[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
        const int ch = i < 4 ? 4 * lane + i : 128 + 2 * lane + (i - 4);
        const int64_t d = ((int64_t)v[i] << p.sh_sum) - mean;
        const i128 prod = (i128)d * (i128)inv;
        i128 nr = (prod + ((i128)1 << 47) + (prod >> 127)) >> 48;
        const int32_t norm = nr > 8388607 ? 8388607 : (nr < -8388608 ? -8388608 : (int32_t)nr);
        const int32_t prodg = norm * (int32_t)p.gamma[ch];
        const int32_t b = p.beta[ch];
        if (p.fast) {
            const int64_t aligned = ((int64_t)prodg << p.sh_g) + ((int64_t)b << p.sh_b);
            o[i] = (int32_t)requant64(aligned, p.sh_out, 8);
        } else {
            const i128 aligned = ((i128)prodg << p.sh_g) + ((i128)b << p.sh_b);
            o[i] = requant128_8(aligned, p.sh_out);
        }
    }
    const uint32_t ow = (uint32_t)(o[0] & 0xff) | ((uint32_t)(o[1] & 0xff) << 8) |
                        ((uint32_t)(o[2] & 0xff) << 16) | ((uint32_t)(o[3] & 0xff) << 24);
    const uint16_t oh = (uint16_t)((o[4] & 0xff) | ((o[5] & 0xff) << 8));
    *(uint32_t *)(outr + 4 * lane) = ow;
    *(uint16_t *)(outr + 128 + 2 * lane) = oh;
    return neg;
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

__global__ void __launch_bounds__(256) ln_kernel(const int8_t *x, int8_t *out, int rows_max, const int32_t *rows_dev,
                                                 LnParams p, uint8_t *negvar_row, const int32_t *offsets,
                                                 int images, uint8_t *warn) {
    const int rows = rows_dev ? *rows_dev : rows_max;
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
        const bool neg = ln_row(x + (size_t)r * 192, out + (size_t)r * 192, p, lane);
        if (lane == 0) {
            if (negvar_row) negvar_row[r] = neg ? 1 : 0;
            if (neg && warn && offsets) {
                const int img = image_of_row(offsets, images, r);
                atomicOr((unsigned int *)(warn + (img & ~3)), (unsigned int)HV_WARN_LN_NEG_VARIANCE << (8 * (img & 3)));
            }
        }
    }
}

__global__ void __launch_bounds__(256) ln_cls_kernel(const int8_t *x, const int32_t *offsets, int images, int8_t *out,
                                                     LnParams p, uint8_t *warn) {
    const int lane = threadIdx.x & 31;
    const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (i >= images) return;
    const bool neg = ln_row(x + (size_t)offsets[i] * 192, out + (size_t)i * 192, p, lane);
    if (neg && lane == 0 && warn)
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

__global__ void gelu_requant_kernel(const int32_t *acc, int64_t n, int sh_in, int sh_out, int8_t *out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (int8_t)gelu_chain(acc[i], sh_in, sh_out);
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

inline int grid_for(int64_t n, int threads) {
    int64_t b = (n + threads - 1) / threads;
    return (int)(b < 148 * 16 ? (b < 1 ? 1 : b) : 148 * 16);
}

}  // namespace

cudaError_t launch_layernorm(const int8_t *x, int8_t *out, int rows_max, const int32_t *rows_dev,
                             const LnParams &p, uint8_t *negvar_row, const int32_t *offsets, int images,
                             uint8_t *warn, cudaStream_t st) {
    if (rows_max <= 0) return cudaSuccess;
    const int warps_per_block = 8;
    int blocks = (rows_max + warps_per_block - 1) / warps_per_block;
    if (blocks > 148 * 8) blocks = 148 * 8;
    ln_kernel<<<blocks, 32 * warps_per_block, 0, st>>>(x, out, rows_max, rows_dev, p, negvar_row, offsets, images,
                                                       warn);
    return cudaGetLastError();
}

cudaError_t launch_layernorm_cls(const int8_t *x, const int32_t *offsets, int images, int8_t *out,
                                 const LnParams &p, uint8_t *warn, cudaStream_t st) {
    if (images <= 0) return cudaSuccess;
    ln_cls_kernel<<<(images + 7) / 8, 256, 0, st>>>(x, offsets, images, out, p, warn);
    return cudaGetLastError();
}

cudaError_t launch_softmax_rows(const int32_t *x, const int32_t *offsets, int rows, int mode, void *out,
                                cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    softmax_rows_kernel<<<(rows + 7) / 8, 256, 0, st>>>(x, offsets, rows, mode, out);
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
    gelu_requant_kernel<<<grid_for(n, 256), 256, 0, st>>>(acc, n, sh_in, sh_out, out);
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
