// hv_epi.cuh — device helpers shared by the persistent layer GEMM
// (hv_gemm_persistent.cu) and the fused FFN kernel (hv_ffn.cu): 32-byte global
// accesses, TMA tile loads (no multicast), mbarrier arrivals, and the fused golden
// writebacks of one 32-column accumulator piece.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "hv_gemm.cuh"
#include "hv_tc05.cuh"

namespace hv {
namespace pg {

// 32 contiguous bytes in one 256-bit store: whole 32-byte sectors, half the store
// instructions of two 16-byte stores.  The address must be 32-byte aligned (row
// strides of 192, 576 and 768 bytes, 32-column pieces).
__device__ __forceinline__ void st_global_32B(void *p, const uint32_t (&w)[8]) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"l"(p), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

// 32 contiguous bytes in one 256-bit read-only load (32-byte aligned address).
__device__ __forceinline__ void ld_global_32B(const void *p, uint32_t (&w)[8]) {
    asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void *g, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(saddr), "l"(g), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(tc05::smem_u32(mbar)), "r"(bytes)
                 : "memory");
}
// One 16-byte-wide box of a row-major matrix at (x = k byte, y = row) into shared
// memory, completing on `mbar` (no multicast).  The box height is the tensor map's.
__device__ __forceinline__ void tma_load_a(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
            "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc05::smem_u32(mbar))
        : "memory");
}

// One 16-byte K strip of 7 patch rows x 14 patches (98 A rows, 1568 bytes) from the
// NHWC images (5-D map [img][pr][ir][pc][48 bytes], see make_tmap_patch), no multicast.
__device__ __forceinline__ void tma_load_patch(uint32_t dst, const CUtensorMap *map, int w0, int ir, int pr0, int img,
                                               uint64_t *mbar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
        "%6}], [%7];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(w0), "r"(0), "r"(ir), "r"(pr0), "r"(img), "r"(tc05::smem_u32(mbar))
        : "memory");
}

// One contiguous run of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from global into shared memory by the bulk-copy engine, completing on `mbar` (no
// multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint64_t *mbar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(tc05::smem_u32(mbar))
                 : "memory");
}

__device__ __forceinline__ void cp_arrive_noinc(uint64_t *mbar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(tc05::smem_u32(mbar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *mbar) {
    asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(tc05::smem_u32(mbar))
                 : "memory");
}

// One output element before the final int8 saturation (pack_sat8 applies it).
// FAST: the 32-bit forms (gemm_epi_fast; for EPI_GELU, gelu_chain_fast2).
template <int EPI, bool FAST>
__device__ __forceinline__ int32_t epi_elem(int32_t acc, int32_t bb, int32_t ax, const EpiParams &e) {
    if (EPI == EPI_GELU)
        return FAST ? gelu_chain_fast2(acc + bb, e.gk) : gelu_chain((int64_t)acc + bb, e.gelu_sh_in, e.gelu_sh_out);
    if (FAST) {
        const int32_t y = rsa32(acc + bb, e.shift);
        if (EPI == EPI_I8) return y;
        const int32_t ys = sat8(y);
        if (EPI == EPI_I8_RES) return rsa32(ax * (1 << e.add.sa) + ys * (1 << e.add.sb), e.add.sh);
        return rsa32(ys * (1 << e.add.sa) + ax * (1 << e.add.sb), e.add.sh);  // patch: a = embedding, b = pos
    }
    const int32_t y = (int32_t)requant64((int64_t)acc + bb, e.shift, 8);
    if (EPI == EPI_I8) return y;
    if (EPI == EPI_I8_RES) return (int32_t)requant64(((int64_t)ax << e.add.sa) + ((int64_t)y << e.add.sb), e.add.sh, 8);
    return (int32_t)requant64(((int64_t)y << e.add.sa) + ((int64_t)ax << e.add.sb), e.add.sh, 8);
}

// The fused writeback of one 32-column piece of a row: v = accumulators, bv = biases,
// aux = residual / positional bytes (EPI_I8_RES, EPI_PATCH); pk = the 32 int8 outputs.
// EPI_GELU with TAB uses the exact GELU-chain tables staged at `stab` (see EpiParams);
// a table-1 piece with an input outside the exact range falls back, for the whole
// warp (every lane must call this), to the arithmetic form.
template <int EPI, bool FAST, bool TAB>
__device__ __forceinline__ void epi_piece32(const uint32_t (&v)[32], const int32_t (&bv)[32], const uint32_t (&aux)[8],
                                            const EpiParams &e, const int8_t *stab, uint32_t (&pk)[8]) {
    bool slow = true;
    if (EPI == EPI_GELU && FAST && TAB && e.gtab_mode == 3) {
        // whole-window table (see EpiParams): five integer operations and one byte load
        const GeluK &k = e.gk;
        const int last = e.gtab_n - 1, c = e.gtab_c;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            int32_t o[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int32_t x = (int32_t)v[w * 4 + b] + bv[w * 4 + b];
                const int32_t u = (x + c + mulhi_s(x, k.ksgn)) >> k.sh_in;
                o[b] = stab[min(max(u, 0), last)];
            }
            pk[w] = pack_sat8(o[0], o[1], o[2], o[3]);
        }
        slow = false;
    } else if (EPI == EPI_GELU && FAST && TAB && e.gtab_mode == 2) {
        // exact bucket table over the whole window (see EpiParams)
        const GeluK &k = e.gk;
        const int lo = e.gtab_lo, last = e.gtab_n - 1, kb = e.gtab_k;
        const int msk = (1 << kb) - 1;
        const uint32_t *coarse = (const uint32_t *)stab;
        const int8_t *fine = stab + e.gtab_fine;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            int32_t o[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int32_t x = (int32_t)v[w * 4 + b] + bv[w * 4 + b];
                const int32_t q = (x + k.hin + mulhi_s(x, k.ksgn)) >> k.sh_in;
                const int u = min(max(q - lo, 0), last);
                const uint32_t en = coarse[u >> kb];
                const int off = u & msk;
                const uint32_t pcut = en >> 16;
                o[b] = off >= (int)pcut ? (int32_t)(int8_t)(en >> 8) : (int32_t)(int8_t)en;
                if (pcut == 0xFFFFu) o[b] = fine[(int)((en & 0xFFFFu) << kb) + off];
            }
            pk[w] = pack_sat8(o[0], o[1], o[2], o[3]);
        }
        slow = false;
    } else if (EPI == EPI_GELU && FAST && TAB && e.gtab_mode == 1) {
        // exact table of the GELU chain, valid for q in [elo, ehi)
        const GeluK &k = e.gk;
        const int lo = e.gtab_lo, last = e.gtab_n - 1;
        const int elo = e.gtab_elo, ehi = e.gtab_ehi;
        bool esc = false;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            int32_t o[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int32_t x = (int32_t)v[w * 4 + b] + bv[w * 4 + b];
                const int32_t q = (x + k.hin + mulhi_s(x, k.ksgn)) >> k.sh_in;
                esc |= (q < elo) | (q >= ehi);
                o[b] = stab[min(max(q - lo, 0), last)];
            }
            pk[w] = pack_sat8(o[0], o[1], o[2], o[3]);
        }
        slow = __any_sync(0xffffffffu, esc);
    }
    if (slow) {
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            int32_t o[4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int j = w * 4 + b;
                const int32_t ax = (int8_t)((aux[w] >> (8 * b)) & 0xffu);
                o[b] = epi_elem<EPI, FAST>((int32_t)v[j], bv[j], ax, e);
            }
            pk[w] = pack_sat8(o[0], o[1], o[2], o[3]);
        }
    }
}

}  // namespace pg
}  // namespace hv
