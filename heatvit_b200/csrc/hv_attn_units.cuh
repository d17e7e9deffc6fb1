// hv_attn_units.cuh — the attention kernel's work-unit lists (hv_attention.cu),
// written by every kernel that lays out a batch's tokens: attn_plan_kernel, the
// batch set-up (all images 197 tokens) and the token packer after a selector.
//
// A unit is one 128-row tile of an image's query rows for one or more heads:
//   * n > 128 tokens (list B): one unit per (head, 128-row half): 6 per image;
//   * 64 < n <= 128 (list A): one unit per head;
//   * 32 < n <= 64 (list A): heads {0, 1} packed in one tile, head 2 alone;
//   * n <= 32 (list A): the three heads packed in one tile.
// An entry is {unit code, the image's first row << 8 | its token count}; both
// lists are image-major, and cnt[0], cnt[1] hold their lengths.
#pragma once
#include <stdint.h>

namespace hv {

// Unit code: image << 7 | mtile << 6 | log2(G) << 4 | first head << 2 | heads.
__host__ __device__ __forceinline__ uint32_t unit_code(int img, int mt, int glog, int h0, int nh) {
    return ((uint32_t)img << 7) | ((uint32_t)mt << 6) | ((uint32_t)glog << 4) | ((uint32_t)h0 << 2) | (uint32_t)nh;
}

// Units of an image of n tokens on list A (n <= 128) and list B (n > 128).
__host__ __device__ __forceinline__ int units_a(int n) { return n <= 0 || n > 128 ? 0 : (n <= 32 ? 1 : (n <= 64 ? 2 : 3)); }
// (an image longer than 224 tokens has no units: the model never makes one, and the
// kernel's buffers hold 224 rows)
__host__ __device__ __forceinline__ int units_b(int n) { return n > 128 && n <= 224 ? 6 : 0; }

// Writes the units of image `img` (first row row0 < 2^24, n tokens) at positions
// pa of list A and pb of list B.
__device__ __forceinline__ void write_image_units(uint2 *list_a, uint2 *list_b, int pa, int pb, int img, int row0,
                                                  int n) {
    const uint32_t rn = ((uint32_t)row0 << 8) | (uint32_t)n;
    const int ca = units_a(n), cb = units_b(n);
    if (ca == 1) {
        list_a[pa] = make_uint2(unit_code(img, 0, 2, 0, 3), rn);
    } else if (ca == 2) {
        list_a[pa] = make_uint2(unit_code(img, 0, 1, 0, 2), rn);
        list_a[pa + 1] = make_uint2(unit_code(img, 0, 1, 2, 1), rn);
    } else if (ca == 3) {
        for (int h = 0; h < 3; ++h) list_a[pa + h] = make_uint2(unit_code(img, 0, 0, h, 1), rn);
    }
    for (int u = 0; u < cb; ++u) list_b[pb + u] = make_uint2(unit_code(img, u / 3, 0, u % 3, 1), rn);
}

}  // namespace hv
