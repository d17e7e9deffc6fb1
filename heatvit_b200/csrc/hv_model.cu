// hv_model.cu — the C ABI: model packing, the batched pipeline and per-op entry points.
//
// Pipeline of one batch (HeatViTModel.infer, model.py:73-123, for every image):
//   patch GEMM (+pos, CLS rows) -> for block b in 1..12:
//       [selector + pack when a selector precedes b]
//       LN1 -> QKV GEMM -> attention -> proj GEMM + residual -> LN2
//       -> FC1 GEMM + GELU -> FC2 GEMM + residual
//   -> LN of each CLS row -> head GEMM (int32 logits at 2^-14).
// Tokens live in one packed ragged buffer: image i owns rows offsets[i] ..
// offsets[i+1].  Kernels take the live row count from device memory, so the
// host never synchronises on data-dependent token counts.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>
#include <algorithm>

#include "hv_attn_units.cuh"
#include "hv_internal.cuh"

using namespace hv;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

#define CUDA_TRY(expr)                                                                      \
    do {                                                                                    \
        cudaError_t _e = (expr);                                                            \
        if (_e != cudaSuccess) return fail(HV_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
    } while (0)

// Entry points that use the model's workspaces refuse to run while host calls are
// in flight (their kernels would share the buffers).
#define HOST_IDLE(m)                                                                              \
    do {                                                                                          \
        if ((m)->host_pending)                                                                    \
            return fail(HV_ERR_STATE, "host calls in flight: call hv_infer_host_wait first");     \
    } while (0)

constexpr int64_t kNarrowLimit = (int64_t)1 << 30;

// Largest |bias| of a vector.
int64_t max_abs(const int32_t *b, int n) {
    int64_t m = 0;
    for (int i = 0; i < n; ++i) m = std::max<int64_t>(m, b[i] < 0 ? -(int64_t)b[i] : b[i]);
    return m;
}

// acc + bias fits the 32-bit epilogue path: |acc| <= K * 2^14.
int needs_wide(const int32_t *bias, int n, int k) {
    return max_abs(bias, n) + (int64_t)k * 16384 >= kNarrowLimit ? 1 : 0;
}

// Host copy of align-add for the CLS row (transformer.py:96-101).
int8_t host_align_add(int a, int ea, int b, int eb, int eo) {
    AlignAdd k = make_align_add(ea, eb, eo);
    return (int8_t)requant64(((int64_t)a << k.sa) + ((int64_t)b << k.sb), k.sh, 8);
}

bool align_ok(int ea, int eb, int eo) {
    AlignAdd k = make_align_add(ea, eb, eo);
    return k.sa <= 54 && k.sb <= 54;
}

struct Arena {
    std::vector<uint8_t> host;
    size_t add(const void *src, size_t bytes) {
        size_t off = (host.size() + 255) & ~(size_t)255;
        host.resize(off + bytes);
        if (src) memcpy(host.data() + off, src, bytes);
        else memset(host.data() + off, 0, bytes);
        return off;
    }
    // transposed copy of an int8 [rows][cols] matrix into [cols_pad][rows]
    size_t add_t(const int8_t *src, int rows, int cols, int cols_pad) {
        std::vector<int8_t> t((size_t)cols_pad * rows, 0);
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c) t[(size_t)c * rows + r] = src[(size_t)r * cols + c];
        return add(t.data(), t.size());
    }
};

struct BlockDev {
    size_t ln1_g, ln1_b, wqkv, bqkv, wproj, bproj, ln2_g, ln2_b, w1, b1, w2, b2;
    int ln1_xs, ln1_gs, ln1_bs, ln1_os, ln2_xs, ln2_gs, ln2_bs, ln2_os;
    int qkv_shift, qkv_wide, proj_shift, proj_wide, fc2_shift, fc2_wide;
    int fc1_sh_in, fc1_sh_out, fc1_wide, fc1_fast, fc1_k2;
    GeluK fc1_gk;
    size_t fc1_tab;            // exact GELU-chain table in the arena (fc1_tab_n > 0)
    int fc1_tab_lo, fc1_tab_n;
    int fc1_tab_elo, fc1_tab_ehi;  // the table is exact for q in [elo, ehi)
    int fc1_tab_mode, fc1_tab_k, fc1_tab_fine, fc1_tab_bytes;  // EpiParams gtab_* fields
    AlignAdd res1, res2;
    AttnParams attn;
    int fc1_tab_c;             // EpiParams gtab_c (table mode 3)
    // FC1 / FC2 weights in the fused FFN's shared-memory chunk layout (hv_ffn.cu): per
    // 128-column hidden chunk j, 24,576 contiguous bytes that one bulk copy moves
    //   w1img[j][kc][r][b] = w1[16 kc + b][128 j + r]   (kc < 12, r < 128)
    //   w2img[j][kc][r][b] = w2[128 j + 16 kc + b][r]   (kc < 8, r < 192)
    size_t w1img, w2img;
};

struct SelDev {
    size_t lwt, lb, w1t, b1, w2t, b2, w3t, b3, hw1, hb1, hw2, hb2;
    size_t tab_local, tab_h1, tab_h2;  // GELU tables in the arena (when their mode is set)
    SelParams p;  // shifts only until bind()
};

}  // namespace

// One set of activation scratch (ragged token buffers, offsets, counts, package
// flags, warnings and the device error word).  The model holds two, so two
// inferences can be in flight on two streams at once (hv_infer_host).
struct Workspace {
    int cap = 0;
    uint8_t *scratch = nullptr;
    int8_t *X = nullptr, *Y = nullptr, *LN = nullptr, *QKV = nullptr, *CTX = nullptr, *HID = nullptr, *STAGE = nullptr,
           *CLSLN = nullptr;
    int32_t *off[2] = {nullptr, nullptr}, *counts = nullptr;
    uint8_t *pkg[2] = {nullptr, nullptr}, *warn = nullptr;
    int *err = nullptr;
    AttnPlan plan{};  // attention work units of the current token layout
    // TMA descriptors of the GEMM A operands LN, CTX ([rows][192]) and HID ([rows][768])
    CUtensorMap tm_ln, tm_ctx, tm_hid;
    int tm_ok = 0;
    // outputs of graph-replayed batches (copied to the caller's buffers after the replay)
    int32_t *o_logits = nullptr, *o_tc = nullptr;
    hv_selector_summary *o_sum = nullptr;
    uint8_t *o_warn = nullptr;
};

// A captured inference (hv_infer_batch / one hv_infer_host chunk) and what it was
// captured for: input, batch, workspace and output buffers.
struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    const int8_t *img = nullptr;
    int batch = 0, ws = 0;
    int32_t *lg = nullptr, *tc = nullptr;
    hv_selector_summary *sum = nullptr;
    uint8_t *warn = nullptr;
    unsigned long long stamp = 0;
    int prof_stage = 0;  // stage whose launches the graph brackets with profiling events
    int prof_n = 0;      // profiling event pairs recorded by one replay
    int kernels = 0;     // kernel nodes in the graph
    int prof_max = 0;    // launch limit of the profiling bracket it was captured with
};

struct hv_model {
    int device = 0;
    int sms = 148;         // SM count: one persistent GEMM CTA per SM
    int persistent = 1;    // layer GEMMs on the persistent kernel (HV_GEMM_TILED=1 selects the per-tile one)
    int fused_ffn = 1;     // FC1 + FC2 in one kernel (HV_FFN_UNFUSED=1: two persistent GEMMs)
    int has_patch = 0, has_head = 0, has_block[HV_BLOCKS] = {0};
    int used_sel = 0;  // selectors that actually run (strides of token counts / summaries)
    uint8_t *weights = nullptr;
    size_t weights_bytes = 0;
    // patch
    size_t patch_wt = 0, patch_b = 0, pos = 0, cls_row = 0;
    int patch_shift = 0, patch_wide = 0;
    AlignAdd patch_add{};
    BlockDev blocks[HV_BLOCKS];
    int sel_before[HV_BLOCKS];
    int num_sel = 0;
    SelDev sels[HV_MAX_SELECTORS];
    size_t fin_g = 0, fin_b = 0, head_wt = 0, head_b = 0;
    int fin_xs = 0, fin_gs = 0, fin_bs = 0, fin_os = 0, head_shift = 0;
    // scratch: two workspaces; the fields below point into the one that the next
    // enqueued work uses (use_workspace)
    Workspace ws[2];
    int8_t *X = nullptr, *Y = nullptr, *LN = nullptr, *QKV = nullptr, *CTX = nullptr, *HID = nullptr, *STAGE = nullptr,
           *CLSLN = nullptr;
    int32_t *off[2] = {nullptr, nullptr}, *counts = nullptr;
    uint8_t *pkg[2] = {nullptr, nullptr}, *warn = nullptr;
    int *err = nullptr;  // device error word (bounded waits that gave up)
    AttnPlan plan{};
    const CUtensorMap *tm_ln = nullptr, *tm_ctx = nullptr, *tm_hid = nullptr;  // nullptr: cp.async loads
    // host-pipeline staging
    int host_cap = 0;
    int8_t *himg[4] = {nullptr, nullptr, nullptr, nullptr};  // device image chunks (chunk g uses g % 4)
    // pinned host staging of the host entry: the outputs of each call in flight
    // (one slot per call), and two image chunks for pageable image buffers
    uint8_t *pin_out[2] = {nullptr, nullptr};
    size_t pin_out_cap[2] = {0, 0};
    int8_t *pin_in[2] = {nullptr, nullptr};
    int pin_in_cap = 0;
    // host calls in flight (hv_infer_host_submit), a ring of two slots
    struct HostCall {
        int batch = 0, ns = 0;
        int32_t *logits = nullptr, *tc = nullptr;
        hv_selector_summary *sum = nullptr;
        uint8_t *warn = nullptr;
        bool pinned_out = false;
        size_t o_tc = 0, o_sum = 0, o_warn = 0;
        cudaEvent_t done[2] = {nullptr, nullptr};  // recorded on both compute streams
    } host_calls[2];
    int host_head = 0, host_pending = 0;
    unsigned long long host_chunks = 0;  // chunks enqueued so far: chunk g uses buffer g & 1
    int32_t *hlogits = nullptr, *htc = nullptr;
    hv_selector_summary *hsum = nullptr;
    uint8_t *hwarn = nullptr;
    cudaStream_t copy_stream = nullptr, compute_stream[2] = {nullptr, nullptr};
    // CUDA graphs of whole inferences (HV_NO_GRAPH=1 launches kernel by kernel)
    int use_graphs = 1;
    GraphEntry graphs[16];
    unsigned long long graph_clock = 0;
    cudaStream_t graph_stream = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
    // per device image chunk: upload finished / compute on it finished; per pinned
    // staging buffer: the upload out of it finished
    cudaEvent_t ev_in[4] = {}, ev_done[4] = {}, ev_pin[2] = {};

    // kernel timing (hv_profile_*)
    int prof_stage = 0, prof_max = 0, prof_n = 0;
    int last_graph_kernels = 0;  // kernel nodes of the last replayed graph
    // test hook of the layer GEMMs (hv_test_gemm_stall): wait limit and skipped tile
    uint32_t test_wait_iters = 0;
    int test_skip_tile = 0;
    std::vector<cudaEvent_t> prof_ev;
    int32_t *prof_rows = nullptr;  // device [prof_max] live row counts

    template <class T>
    const T *w(size_t off_) const { return (const T *)(weights + off_); }
};

namespace {

LnParams ln_of(const hv_model *m, size_t g, size_t b, int xs, int gs, int bs, int os) {
    return make_ln(m->w<int8_t>(g), m->w<int8_t>(b), xs, gs, bs, os);
}

SelParams bind_sel(const hv_model *m, const SelDev &s) {
    SelParams p = s.p;
    p.local_wt = m->w<int8_t>(s.lwt);
    p.local_b = m->w<int32_t>(s.lb);
    p.w1t = m->w<int8_t>(s.w1t);
    p.b1 = m->w<int32_t>(s.b1);
    p.w2t = m->w<int8_t>(s.w2t);
    p.b2 = m->w<int32_t>(s.b2);
    p.w3t = m->w<int8_t>(s.w3t);
    p.b3 = m->w<int32_t>(s.b3);
    p.hw1 = m->w<int8_t>(s.hw1);
    p.hb1 = m->w<int32_t>(s.hb1);
    p.hw2 = m->w<int8_t>(s.hw2);
    p.hb2 = m->w<int32_t>(s.hb2);
    p.tab_local.tab = p.tab_local.mode ? m->w<int8_t>(s.tab_local) : nullptr;
    p.tab_h1.tab = p.tab_h1.mode ? m->w<int8_t>(s.tab_h1) : nullptr;
    p.tab_h2.tab = p.tab_h2.mode ? m->w<int8_t>(s.tab_h2) : nullptr;
    p.err = m->err;
    return p;
}

// Point the model's working fields at workspace i.  Kernels capture these
// pointers when they are enqueued, so switching between enqueues is safe.
void use_workspace(hv_model *m, int i) {
    const Workspace &w = m->ws[i];
    m->X = w.X;
    m->Y = w.Y;
    m->LN = w.LN;
    m->QKV = w.QKV;
    m->CTX = w.CTX;
    m->HID = w.HID;
    m->STAGE = w.STAGE;
    m->CLSLN = w.CLSLN;
    m->off[0] = w.off[0];
    m->off[1] = w.off[1];
    m->counts = w.counts;
    m->pkg[0] = w.pkg[0];
    m->pkg[1] = w.pkg[1];
    m->warn = w.warn;
    m->err = w.err;
    m->plan = w.plan;
    m->tm_ln = w.tm_ok ? &w.tm_ln : nullptr;
    m->tm_ctx = w.tm_ok ? &w.tm_ctx : nullptr;
    m->tm_hid = w.tm_ok ? &w.tm_hid : nullptr;
}

// Workspace i holds at least `images` images; it becomes the current one.
int ensure_capacity(hv_model *m, int images, int i = 0) {
    Workspace &w = m->ws[i];
    if (images > w.cap) {
        if (w.scratch) {
            // Captured graphs hold this workspace's addresses: wait for the device,
            // then drop them with the buffers.
            CUDA_TRY(cudaDeviceSynchronize());
            for (GraphEntry &g : m->graphs)
                if (g.exec && g.ws == i) {
                    cudaGraphExecDestroy(g.exec);
                    g = GraphEntry();
                }
            cudaFree(w.scratch);
            w = Workspace();
        }
        const size_t rows = (size_t)images * HV_TOKENS;
        size_t total = 0;
        auto take = [&](size_t bytes) {
            size_t o = total;
            total += (bytes + 255) & ~(size_t)255;
            return o;
        };
        const size_t oX = take(rows * 192), oY = take(rows * 192), oLN = take(rows * 192), oQKV = take(rows * 576),
                     oCTX = take(rows * 192), oHID = take(rows * 768), oSTAGE = take(rows * 192),
                     oCLS = take((size_t)images * 192), oOff0 = take((size_t)(images + 1) * 4),
                     oOff1 = take((size_t)(images + 1) * 4), oCnt = take((size_t)images * 4), oPkg0 = take(images),
                     oPkg1 = take(images), oWarn = take(((size_t)images + 3) & ~(size_t)3), oErr = take(16),
                     oOL = take((size_t)images * HV_CLASSES * 4), oOT = take((size_t)images * (HV_MAX_SELECTORS + 1) * 4),
                     oOS = take((size_t)images * HV_MAX_SELECTORS * sizeof(hv_selector_summary)), oOW = take(images),
                     oLA = take((size_t)images * 3 * 8), oLB = take((size_t)images * 6 * 8), oPC = take(16);
        uint8_t *base = nullptr;
        if (cudaMalloc(&base, total) != cudaSuccess)
            return fail(HV_ERR_NOMEM, "cannot allocate %zu bytes of scratch", total);
        w.scratch = base;
        w.X = (int8_t *)(base + oX);
        w.Y = (int8_t *)(base + oY);
        w.LN = (int8_t *)(base + oLN);
        w.QKV = (int8_t *)(base + oQKV);
        w.CTX = (int8_t *)(base + oCTX);
        w.HID = (int8_t *)(base + oHID);
        w.STAGE = (int8_t *)(base + oSTAGE);
        w.CLSLN = (int8_t *)(base + oCLS);
        w.off[0] = (int32_t *)(base + oOff0);
        w.off[1] = (int32_t *)(base + oOff1);
        w.counts = (int32_t *)(base + oCnt);
        w.pkg[0] = base + oPkg0;
        w.pkg[1] = base + oPkg1;
        w.warn = base + oWarn;
        w.err = (int *)(base + oErr);
        w.o_logits = (int32_t *)(base + oOL);
        w.o_tc = (int32_t *)(base + oOT);
        w.o_sum = (hv_selector_summary *)(base + oOS);
        w.o_warn = base + oOW;
        w.plan.list_a = (uint2 *)(base + oLA);
        w.plan.list_b = (uint2 *)(base + oLB);
        w.plan.cnt = (int32_t *)(base + oPC);
        if (cudaMemset(w.err, 0, 16) != cudaSuccess) return fail(HV_ERR_CUDA, "cannot clear the error word");
        const int r = (int)rows;
        w.tm_ok = make_tmap_a(&w.tm_ln, w.LN, 192, r) == 0 && make_tmap_a(&w.tm_ctx, w.CTX, 192, r) == 0 &&
                  make_tmap_a(&w.tm_hid, w.HID, HV_FFN, r) == 0;
        w.cap = images;
    }
    use_workspace(m, i);
    return HV_OK;
}

// ---- small pipeline kernels ----------------------------------------------------
__global__ void init_batch_kernel(int images, int32_t *off, uint8_t *pkg, uint8_t *warn, int32_t *tc, int tc_stride,
                                  int8_t *x, const int8_t *cls_row, AttnPlan plan) {
    griddep_wait();  // the previous inference may still read these buffers
    griddep_launch();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i <= images; i += gridDim.x * blockDim.x) {
        off[i] = i * HV_TOKENS;
        if (i < images) {
            pkg[i] = 0;
            if (tc) tc[(size_t)i * tc_stride] = HV_TOKENS;
            // the attention units of the full layout: 6 per image on list B
            write_image_units(plan.list_a, plan.list_b, 0, 6 * i, i, i * HV_TOKENS, HV_TOKENS);
        }
        if (i < ((images + 3) & ~3)) warn[i] = 0;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        plan.cnt[0] = 0;
        plan.cnt[1] = 6 * images;
    }
    // CLS rows (row 0 of every image): 12 x 16 bytes each.
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < images * 12; c += gridDim.x * blockDim.x) {
        const int i = c / 12, ch = c - i * 12;
        ((int4 *)(x + (size_t)i * HV_TOKENS * 192))[ch] = ((const int4 *)cls_row)[ch];
    }
}

__global__ void ckpt_copy_kernel(const int8_t *x, const int32_t *off, int8_t *ckpt, int32_t *ckpt_rows, int slot) {
    const int i = blockIdx.x;
    const int a = off[i], n = off[i + 1] - a;
    const int4 *src = (const int4 *)(x + (size_t)a * 192);
    int4 *dst = (int4 *)(ckpt + ((size_t)i * HV_CKPT_SLOTS + slot) * HV_TOKENS * 192);
    for (int c = threadIdx.x; c < n * 12; c += blockDim.x) dst[c] = src[c];
    if (threadIdx.x == 0) ckpt_rows[(size_t)i * HV_CKPT_SLOTS + slot] = n;
}

GemmArgs gemm_args(const void *a, int lda, int patch_mode, const int8_t *bt, int n, int k, int m_host,
                   const int32_t *m_dev, void *out, int ldo) {
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.a.ptr = a;
    g.a.lda = lda;
    g.a.patch_mode = patch_mode;
    g.bt = bt;
    g.n = n;
    g.k = k;
    g.m_host = m_host;
    g.m_dev = m_dev;
    g.out = out;
    g.ldo = ldo;
    return g;
}

// A layer GEMM of the model: the persistent kernel for the layer shapes it covers.
cudaError_t model_gemm(const hv_model *m, GemmArgs &g, int epi, int m_max, cudaStream_t st) {
    g.epi.fast = gemm_epi_fast(epi, g.epi);
    // (the persistent epilogue stores and reads 32-byte pieces: 32-byte aligned rows)
    const bool al32 = (uintptr_t)g.out % 32 == 0 && g.ldo % 32 == 0 && (uintptr_t)g.epi.res % 32 == 0 &&
                      (uintptr_t)g.epi.pos % 32 == 0;
    if (m->persistent && gemm_persistent_supported(epi, g.n, g.k) && al32) {
        if (epi == EPI_GELU) g.epi.fast = g.epi.gelu_k2 || g.epi.gtab_n > 0;  // the persistent kernel's fast forms
        g.wait_iters = m->test_wait_iters;
        g.skip_tile = m->test_skip_tile;
        return launch_gemm_persistent(g, epi, m_max, m->err, m->sms, st);
    }
    return launch_gemm(g, epi, 0, m_max, m->err, st);
}

__global__ void copy_rows_kernel(const int32_t *src, int32_t *dst) { *dst = *src; }
__global__ void set_rows_kernel(int32_t v, int32_t *dst) { *dst = v; }

// Record a profiling event; under stream capture it becomes an external event
// record node, so the host can time it after each replay.
inline void prof_record(cudaEvent_t e, cudaStream_t st) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    cudaEventRecordWithFlags(e, st, cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault);
}

// Profiling bracket: begin/end around one launch of `stage` when enabled.
struct Prof {
    hv_model *m;
    int on;
    Prof(hv_model *m_, int stage, cudaStream_t st) : m(m_), on(0) {
        if (m->prof_stage == stage && m->prof_n < m->prof_max) {
            on = 1;
            prof_record(m->prof_ev[2 * m->prof_n], st);
        }
    }
    void end(cudaStream_t st, const int32_t *rows_dev, int rows_host) {
        if (!on) return;
        prof_record(m->prof_ev[2 * m->prof_n + 1], st);
        // a kernel, not a host copy, so that a captured graph holds the value itself
        if (rows_dev) copy_rows_kernel<<<1, 1, 0, st>>>(rows_dev, m->prof_rows + m->prof_n);
        else set_rows_kernel<<<1, 1, 0, st>>>(rows_host, m->prof_rows + m->prof_n);
        m->prof_n++;
    }
};

// One transformer block over the ragged batch in m->X (in place).
// may_be_short: some image may hold fewer than 197 tokens (after a selector, or a
// caller-supplied ragged batch).
int run_block(hv_model *m, int b, int images, const int32_t *off, int may_be_short, cudaStream_t st) {
    const BlockDev &d = m->blocks[b];
    const int rows_max = images * HV_TOKENS;
    const int32_t *rows_dev = off + images;
    LnParams ln1 = ln_of(m, d.ln1_g, d.ln1_b, d.ln1_xs, d.ln1_gs, d.ln1_bs, d.ln1_os);
    LnParams ln2 = ln_of(m, d.ln2_g, d.ln2_b, d.ln2_xs, d.ln2_gs, d.ln2_bs, d.ln2_os);
    {
        Prof pr(m, HV_STAGE_LN1, st);
        CUDA_TRY(launch_layernorm(m->X, m->LN, rows_max, rows_dev, ln1, nullptr, off, images, m->warn, st));
        pr.end(st, rows_dev, 0);
    }
    {
        Prof pr(m, HV_STAGE_QKV, st);
        GemmArgs g = gemm_args(m->LN, 192, 0, m->w<int8_t>(d.wqkv), HV_QKV, 192, 0, rows_dev, m->QKV, HV_QKV);
        g.tma = m->tm_ln;
        g.epi.bias = m->w<int32_t>(d.bqkv);
        g.epi.shift = d.qkv_shift;
        g.epi.bits_wide = d.qkv_wide;
        CUDA_TRY(model_gemm(m, g, EPI_I8, rows_max, st));
        pr.end(st, rows_dev, 0);
    }
    {
        Prof pr(m, HV_STAGE_ATTN, st);
        CUDA_TRY(launch_attention(m->QKV, off, images, m->CTX, d.attn, may_be_short, m->sms, m->err, m->plan, st));
        pr.end(st, rows_dev, 0);
    }
    {
        Prof pr(m, HV_STAGE_PROJ, st);
        GemmArgs g = gemm_args(m->CTX, 192, 0, m->w<int8_t>(d.wproj), HV_EMBED, 192, 0, rows_dev, m->Y, HV_EMBED);
        g.tma = m->tm_ctx;
        g.epi.bias = m->w<int32_t>(d.bproj);
        g.epi.shift = d.proj_shift;
        g.epi.bits_wide = d.proj_wide;
        g.epi.res = m->X;
        g.epi.add = d.res1;
        CUDA_TRY(model_gemm(m, g, EPI_I8_RES, rows_max, st));
        pr.end(st, rows_dev, 0);
    }
    {
        Prof pr(m, HV_STAGE_LN2, st);
        CUDA_TRY(launch_layernorm(m->Y, m->LN, rows_max, rows_dev, ln2, nullptr, off, images, m->warn, st));
        pr.end(st, rows_dev, 0);
    }
    if (m->fused_ffn && m->tm_ln) {
        // FC1 + GELU + FC2 + residual 2 in one kernel (hv_ffn.cu); HID stays on chip
        Prof pr(m, HV_STAGE_FFN, st);
        FfnArgs f;
        memset(&f, 0, sizeof(f));
        f.m_dev = rows_dev;
        f.e1.bias = m->w<int32_t>(d.b1);
        f.e1.bits_wide = d.fc1_wide;
        f.e1.gelu_sh_in = d.fc1_sh_in;
        f.e1.gelu_sh_out = d.fc1_sh_out;
        f.e1.gelu_fast = d.fc1_fast;
        f.e1.gelu_k2 = d.fc1_k2;
        f.e1.gk = d.fc1_gk;
        f.e1.gtab = d.fc1_tab_n > 0 ? m->w<int8_t>(d.fc1_tab) : nullptr;
        f.e1.gtab_lo = d.fc1_tab_lo;
        f.e1.gtab_n = d.fc1_tab_n;
        f.e1.gtab_elo = d.fc1_tab_elo;
        f.e1.gtab_ehi = d.fc1_tab_ehi;
        f.e1.gtab_mode = d.fc1_tab_n > 0 ? d.fc1_tab_mode : 0;
        f.e1.gtab_k = d.fc1_tab_k;
        f.e1.gtab_fine = d.fc1_tab_fine;
        f.e1.gtab_bytes = d.fc1_tab_bytes;
        f.e1.gtab_c = d.fc1_tab_c;
        f.e1.fast = d.fc1_k2 || d.fc1_tab_n > 0;  // the persistent kernels' fast GELU forms
        f.e2.bias = m->w<int32_t>(d.b2);
        f.e2.shift = d.fc2_shift;
        f.e2.bits_wide = d.fc2_wide;
        f.e2.res = m->Y;
        f.e2.add = d.res2;
        f.e2.fast = gemm_epi_fast(EPI_I8_RES, f.e2);
        f.out = m->X;
        f.w1img = m->w<int8_t>(d.w1img);
        f.w2img = m->w<int8_t>(d.w2img);
        f.wait_iters = m->test_wait_iters;
        f.skip_tile = m->test_skip_tile;
        CUDA_TRY(launch_ffn(f, *m->tm_ln, rows_max, m->err, m->sms, st));
        pr.end(st, rows_dev, 0);
        return HV_OK;
    }
    {
        Prof pr(m, HV_STAGE_FC1, st);
        GemmArgs g = gemm_args(m->LN, 192, 0, m->w<int8_t>(d.w1), HV_FFN, 192, 0, rows_dev, m->HID, HV_FFN);
        g.tma = m->tm_ln;
        g.epi.bias = m->w<int32_t>(d.b1);
        g.epi.bits_wide = d.fc1_wide;
        g.epi.gelu_sh_in = d.fc1_sh_in;
        g.epi.gelu_sh_out = d.fc1_sh_out;
        g.epi.gelu_fast = d.fc1_fast;
        g.epi.gelu_k2 = d.fc1_k2;
        g.epi.gk = d.fc1_gk;
        g.epi.gtab = d.fc1_tab_n > 0 ? m->w<int8_t>(d.fc1_tab) : nullptr;
        g.epi.gtab_lo = d.fc1_tab_lo;
        g.epi.gtab_n = d.fc1_tab_n;
        g.epi.gtab_elo = d.fc1_tab_elo;
        g.epi.gtab_ehi = d.fc1_tab_ehi;
        g.epi.gtab_mode = d.fc1_tab_n > 0 ? d.fc1_tab_mode : 0;
        g.epi.gtab_k = d.fc1_tab_k;
        g.epi.gtab_fine = d.fc1_tab_fine;
        g.epi.gtab_bytes = d.fc1_tab_bytes;
        g.epi.gtab_c = d.fc1_tab_c;
        CUDA_TRY(model_gemm(m, g, EPI_GELU, rows_max, st));
        pr.end(st, rows_dev, 0);
    }
    {
        Prof pr(m, HV_STAGE_FC2, st);
        GemmArgs g = gemm_args(m->HID, HV_FFN, 0, m->w<int8_t>(d.w2), HV_EMBED, HV_FFN, 0, rows_dev, m->X, HV_EMBED);
        g.tma = m->tm_hid;
        g.epi.bias = m->w<int32_t>(d.b2);
        g.epi.shift = d.fc2_shift;
        g.epi.bits_wide = d.fc2_wide;
        g.epi.res = m->Y;
        g.epi.add = d.res2;
        CUDA_TRY(model_gemm(m, g, EPI_I8_RES, rows_max, st));
        pr.end(st, rows_dev, 0);
    }
    return HV_OK;
}

int run_patch(hv_model *m, const int8_t *images, int count, int8_t *out, cudaStream_t st) {
    GemmArgs g = gemm_args(images, 0, 1, m->w<int8_t>(m->patch_wt), HV_EMBED, HV_PATCH_K, count * HV_PATCHES, nullptr,
                           out, HV_EMBED);
    g.epi.bias = m->w<int32_t>(m->patch_b);
    g.epi.shift = m->patch_shift;
    g.epi.bits_wide = m->patch_wide;
    g.epi.pos = m->w<int8_t>(m->pos);
    g.epi.add = m->patch_add;
    // TMA gather of the patches (two 98-row tiles per image) when the map can be made
    CUtensorMap tm;
    if (make_tmap_patch(&tm, images, count) == 0) g.tma = &tm;
    CUDA_TRY(model_gemm(m, g, EPI_PATCH, count * HV_PATCHES, st));
    return HV_OK;
}

int infer_impl(hv_model *m, const int8_t *d_images, int batch, int32_t *d_logits, int32_t *d_tc,
               hv_selector_summary *d_summary, uint8_t *d_warnings, int8_t *d_ckpt, int32_t *d_ckpt_rows,
               cudaStream_t st, int wsi = 0) {
    if (batch <= 0) return fail(HV_ERR_VALUE, "batch must be positive");
    if (!d_images || !d_logits) return fail(HV_ERR_VALUE, "images and logits are required");
    if (!m->has_patch || !m->has_head) return fail(HV_ERR_STATE, "model has no patch embedding or head");
    for (int b = 0; b < HV_BLOCKS; ++b)
        if (!m->has_block[b]) return fail(HV_ERR_STATE, "model has no block %d", b + 1);
    CUDA_TRY(cudaSetDevice(m->device));
    int rc = ensure_capacity(m, batch, wsi);
    if (rc) return rc;
    const int ns = m->used_sel;
    const int tc_stride = ns + 1;
    if (d_ckpt_rows) CUDA_TRY(cudaMemsetAsync(d_ckpt_rows, 0, sizeof(int32_t) * (size_t)batch * HV_CKPT_SLOTS, st));
    int cur = 0;
    CUDA_TRY(launch_pdl(init_batch_kernel, dim3(std::min(148 * 4, (batch * 12 + 255) / 256 + 1)), dim3(256), 0, st, 
        batch, m->off[0], m->pkg[0], m->warn, d_tc, tc_stride, m->X, m->w<int8_t>(m->cls_row), m->plan));
    CUDA_TRY(cudaGetLastError());
    {
        Prof pr(m, HV_STAGE_PATCH, st);
        rc = run_patch(m, d_images, batch, m->X, st);
        if (rc) return rc;
        pr.end(st, nullptr, batch * HV_PATCHES);
    }
    if (d_ckpt) {
        ckpt_copy_kernel<<<batch, 256, 0, st>>>(m->X, m->off[cur], d_ckpt, d_ckpt_rows, HV_CKPT_PATCH);
        CUDA_TRY(cudaGetLastError());
    }
    int sel_no = 0;  // (init_batch_kernel wrote the attention units of the full layout)
    for (int b = 0; b < HV_BLOCKS; ++b) {
        const int si = m->sel_before[b];
        if (si >= 0) {
            SelParams sp = bind_sel(m, m->sels[si]);
            Prof pr(m, HV_STAGE_SELECTOR, st);
            CUDA_TRY(launch_selector(m->X, m->off[cur], m->pkg[cur], batch, sp, m->STAGE, m->counts, m->pkg[cur ^ 1],
                                     d_summary ? d_summary + sel_no : nullptr, ns, m->warn, d_tc, tc_stride,
                                     sel_no + 1, nullptr, st));
            pr.end(st, m->off[cur] + batch, 0);
            CUDA_TRY(launch_pack(m->STAGE, m->counts, batch, m->X, m->off[cur ^ 1], &m->plan, st));
            cur ^= 1;
            ++sel_no;
            if (d_ckpt) {
                ckpt_copy_kernel<<<batch, 256, 0, st>>>(m->X, m->off[cur], d_ckpt, d_ckpt_rows,
                                                        HV_CKPT_SELECTOR(sel_no));
                CUDA_TRY(cudaGetLastError());
            }
        }
        rc = run_block(m, b, batch, m->off[cur], sel_no > 0, st);
        if (rc) return rc;
        if (d_ckpt) {
            ckpt_copy_kernel<<<batch, 256, 0, st>>>(m->X, m->off[cur], d_ckpt, d_ckpt_rows, HV_CKPT_BLOCK(b + 1));
            CUDA_TRY(cudaGetLastError());
        }
    }
    LnParams fin = ln_of(m, m->fin_g, m->fin_b, m->fin_xs, m->fin_gs, m->fin_bs, m->fin_os);
    if (d_ckpt) {
        CUDA_TRY(launch_layernorm(m->X, m->LN, batch * HV_TOKENS, m->off[cur] + batch, fin, nullptr, nullptr, 0,
                                  nullptr, st));
        ckpt_copy_kernel<<<batch, 256, 0, st>>>(m->LN, m->off[cur], d_ckpt, d_ckpt_rows, HV_CKPT_FINAL_LN);
        CUDA_TRY(cudaGetLastError());
    }
    CUDA_TRY(launch_layernorm_cls(m->X, m->off[cur], batch, m->CLSLN, fin, m->warn, st));
    {
        GemmArgs g = gemm_args(m->CLSLN, 192, 0, m->w<int8_t>(m->head_wt), HV_CLASSES, 192, batch, nullptr, d_logits,
                               HV_CLASSES);
        g.epi.bias = m->w<int32_t>(m->head_b);
        g.epi.shift = m->head_shift;
        g.epi.bits_wide = 1;
        Prof pr(m, HV_STAGE_HEAD, st);
        CUDA_TRY(launch_gemm(g, EPI_I32, 0, batch, m->err, st));
        pr.end(st, nullptr, batch);
    }
    if (d_warnings) CUDA_TRY(cudaMemcpyAsync(d_warnings, m->warn, batch, cudaMemcpyDeviceToDevice, st));
    return HV_OK;
}

// ---- parameter validation and packing -------------------------------------------
bool ln_scale_ok(int xs) { return xs >= -32 && xs <= 0; }

// A GELU-chain table [lo, lo + n) in Q8.16 input units, exact for inputs in [elo, ehi).
struct TabWindow {
    int32_t lo, n, elo, ehi;
};

// Smallest escape distance (in Q8.16 input units, one real unit = 65536) a central
// table must reach on both sides of 0 before it replaces the FMA form: inputs
// beyond it would take the slower escape path.
constexpr int64_t kEscapeRadiusMin = 65536;

// The int8 output of the GELU chain for every Q8.16 input in [-qmax, qmax] (index
// i is q = i - qmax), from the device functions the exhaustive tests cover.
int gelu_scan(int32_t qmax, int sh_out, std::vector<int8_t> &f) {
    const int64_t total = 2 * (int64_t)qmax + 1;
    int8_t *d_f = nullptr;
    f.resize((size_t)total);
    cudaError_t e = cudaMalloc(&d_f, (size_t)total);
    if (e == cudaSuccess) e = launch_gelu_table_fill(d_f, -qmax, (int32_t)total, sh_out, nullptr);
    if (e == cudaSuccess) e = cudaMemcpy(f.data(), d_f, (size_t)total, cudaMemcpyDeviceToHost);
    if (d_f) cudaFree(d_f);
    if (e != cudaSuccess) return fail(HV_ERR_CUDA, "GELU table scan: %s", cudaGetErrorString(e));
    return HV_OK;
}

// Choose a table of at most kGeluTableMax entries for a GELU chain whose output
// varies over more than that across the reachable inputs [-qmax, qmax].  The table
// [t0, t1) must contain q = 0; with its first and last entries repeated by the
// clamp, it is exact from the start of the constant run holding t0 to the end of
// the run holding t1 - 1.  Among the tables that start at the end of a run, the one
// whose exact range reaches farthest from 0 on its nearer side is taken, if that
// distance is at least kEscapeRadiusMin.  *ok = false when none qualifies.
void gelu_escape_window(const std::vector<int8_t> &f, int32_t qmax, TabWindow *tw, bool *ok) {
    *ok = false;
    const int64_t total = (int64_t)f.size();
    // run r covers indices [starts[r], starts[r + 1]); index i is q = i - qmax
    std::vector<int64_t> starts{0};
    for (int64_t i = 1; i < total; ++i)
        if (f[(size_t)i] != f[(size_t)i - 1]) starts.push_back(i);
    starts.push_back(total);
    const int64_t nruns = (int64_t)starts.size() - 1, i0 = qmax;
    auto run_of = [&](int64_t i) {  // run holding index i
        return (int64_t)(std::upper_bound(starts.begin(), starts.end(), i) - starts.begin()) - 1;
    };
    const int64_t inf = INT64_MAX / 4;
    int64_t best = -1;
    for (int64_t r = 0; r < nruns; ++r) {
        const int64_t t0 = starts[(size_t)r + 1] - 1;  // the table starts at the run's last index
        if (t0 > i0) break;
        const int64_t t1 = std::min(t0 + (int64_t)kGeluTableMax, total);
        if (t1 <= i0) continue;
        const int64_t rr = run_of(t1 - 1);
        const int64_t f0 = starts[(size_t)r], f1 = starts[(size_t)rr + 1];
        const int64_t left = f0 == 0 ? inf : i0 - f0, right = f1 == total ? inf : f1 - 1 - i0;
        const int64_t reach = std::min(left, right);
        if (reach > best) {
            best = reach;
            tw->lo = (int32_t)(t0 - qmax);
            tw->n = (int32_t)(std::max(starts[(size_t)rr], t0) + 1 - t0);  // to the last run's first index
            tw->elo = f0 == 0 ? INT32_MIN : (int32_t)(f0 - qmax);
            tw->ehi = f1 == total ? INT32_MAX : (int32_t)(f1 - qmax);
        }
    }
    *ok = best >= kEscapeRadiusMin;
}

// Two-level exact table of the whole window [w0, w1] outside which the output is
// constant (clamped indices repeat its end values).  The window is cut into buckets
// of 2^k inputs.  A bucket whose output changes at most once is one uint32
// coarse entry: v0 | v1 << 8 | p << 16 (v0 before offset p, v1 from it; p = 0x8000
// when constant).  A bucket with more changes gets p = 0xFFFF, and its low 16 bits
// index a 2^k-byte fine table stored after the coarse entries.  The smallest k in
// [3, 10] whose table fits `budget` bytes is taken; *ok = false when none does.
struct BucketTable {
    int32_t lo, n;
    int k, fine_off;
    std::vector<uint8_t> blob;
};
void gelu_bucket_table(const std::vector<int8_t> &f, int32_t qmax, BucketTable *bt, bool *ok,
                       int budget = kGeluTableMax) {
    *ok = false;
    const int64_t total = (int64_t)f.size();
    int64_t w0 = -1, w1 = -1;
    for (int64_t i = 1; i < total; ++i)
        if (f[(size_t)i] != f[(size_t)i - 1]) {
            if (w0 < 0) w0 = i - 1;
            w1 = i;
        }
    if (w0 < 0) return;  // constant: the plain window table applies
    const int64_t W = w1 - w0 + 1;
    auto at = [&](int64_t u) { return f[(size_t)(w0 + std::min(u, W - 1))]; };
    for (int k = 3; k <= 10; ++k) {
        const int64_t B = (int64_t)1 << k, nb = (W + B - 1) / B;
        int64_t nfine = 0;
        for (int64_t b = 0; b < nb; ++b) {
            int ch = 0;
            for (int64_t j = 1; j < B; ++j) ch += at(b * B + j) != at(b * B + j - 1);
            if (ch >= 2) ++nfine;
        }
        const int64_t fine_off = 4 * nb, bytes = fine_off + nfine * B;
        if (bytes > budget || nfine > 0xFFFF) continue;
        bt->lo = (int32_t)(w0 - qmax);
        bt->n = (int32_t)W;
        bt->k = k;
        bt->fine_off = (int)fine_off;
        bt->blob.assign((size_t)bytes, 0);
        int64_t fi = 0;
        for (int64_t b = 0; b < nb; ++b) {
            int ch = 0, pos = 0;
            for (int64_t j = 1; j < B; ++j)
                if (at(b * B + j) != at(b * B + j - 1)) {
                    ++ch;
                    pos = (int)j;
                }
            uint32_t e;
            if (ch >= 2) {
                for (int64_t j = 0; j < B; ++j) bt->blob[(size_t)(fine_off + fi * B + j)] = (uint8_t)at(b * B + j);
                e = (uint32_t)fi | (0xFFFFu << 16);
                ++fi;
            } else {
                const uint32_t v0 = (uint8_t)at(b * B), v1 = (uint8_t)at(b * B + (ch ? pos : 0));
                e = v0 | v1 << 8 | (uint32_t)(ch ? pos : 0x8000) << 16;
            }
            memcpy(bt->blob.data() + 4 * b, &e, 4);
        }
        *ok = true;
        return;
    }
}

// Exact table of a selector GELU chain with input v = acc + bias, |v| <= vmax, and
// q = rsa(v, sh_in): a byte table of the whole non-constant window when it fits
// `budget`, else a bucket table (gelu_bucket_table) when one fits, else none
// (t->mode = 0).  The table bytes go to the arena at *off.
int sel_gelu_table(int sh_in, int sh_out, int64_t vmax, int budget, Arena &A, GeluTab *t, size_t *off) {
    memset(t, 0, sizeof(*t));
    if (sh_in < 0 || sh_in > 30) return HV_OK;
    const int64_t hin = sh_in > 0 ? (int64_t)1 << (sh_in - 1) : 0;
    if (vmax + hin >= ((int64_t)1 << 31)) return HV_OK;
    const int64_t qmax = (vmax + hin) >> sh_in;
    if (qmax >= ((int64_t)1 << 23)) return HV_OK;  // no 24-bit saturation of the GELU input
    std::vector<int8_t> f;
    int rc = gelu_scan((int32_t)qmax, sh_out, f);
    if (rc != HV_OK) return rc;
    int64_t w0 = -1, w1 = -1;
    for (int64_t i = 1; i < (int64_t)f.size(); ++i)
        if (f[(size_t)i] != f[(size_t)i - 1]) {
            if (w0 < 0) w0 = i - 1;
            w1 = i;
        }
    if (w0 < 0) w0 = w1 = 0;  // constant: a one-entry table
    const int64_t W = w1 - w0 + 1;
    std::vector<uint8_t> blob;
    if (W <= budget) {
        blob.assign(f.begin() + w0, f.begin() + w1 + 1);
        t->mode = 1;
        t->lo = (int32_t)(w0 - qmax);
        t->n = (int32_t)W;
    } else {
        BucketTable bt;
        bool ok = false;
        gelu_bucket_table(f, (int32_t)qmax, &bt, &ok, budget - 15);  // room for the 16-byte padding
        if (!ok) return HV_OK;
        blob = bt.blob;
        t->mode = 2;
        t->lo = bt.lo;
        t->n = bt.n;
        t->k = bt.k;
        t->fine = bt.fine_off;
    }
    blob.resize((blob.size() + 15) & ~(size_t)15, 0);
    if ((int)blob.size() > budget) {
        t->mode = 0;
        return HV_OK;
    }
    t->bytes = (int)blob.size();
    t->sh_in = sh_in;
    *off = A.add(blob.data(), blob.size());
    return HV_OK;
}

int pack_model(hv_model *m, const hv_params *P) {
    // two device ints of scratch for the GELU table window search, freed on every return
    struct ScratchInts {
        int *p = nullptr;
        ~ScratchInts() {
            if (p) cudaFree(p);
        }
    } mm_hold;
    int *&mm = mm_hold.p;
    Arena A;
    const hv_patch_params &pp = P->patch;
    m->has_patch = pp.weight != nullptr;
    if (m->has_patch) {
    if (!pp.bias || !pp.cls || !pp.pos) return fail(HV_ERR_VALUE, "patch parameters missing");
    m->patch_wt = A.add_t(pp.weight, HV_PATCH_K, HV_EMBED, HV_EMBED);
    m->patch_b = A.add(pp.bias, HV_EMBED * 4);
    m->pos = A.add(pp.pos, HV_TOKENS * HV_EMBED);
    const int src_patch = pp.image_scale_exp + pp.weight_scale_exp;
    m->patch_shift = pp.activation_scale_exp - src_patch;
    m->patch_wide = needs_wide(pp.bias, HV_EMBED, HV_PATCH_K);
    if (!align_ok(pp.activation_scale_exp, pp.pos_scale_exp, pp.tokens_scale_exp) ||
        !align_ok(pp.cls_scale_exp, pp.pos_scale_exp, pp.tokens_scale_exp))
        return fail(HV_ERR_VALUE, "patch align-add exponent gap above 54 is not supported");
    m->patch_add = make_align_add(pp.activation_scale_exp, pp.pos_scale_exp, pp.tokens_scale_exp);
    int8_t cls_row[HV_EMBED];
    for (int c = 0; c < HV_EMBED; ++c)
        cls_row[c] = host_align_add(pp.cls[c], pp.cls_scale_exp, pp.pos[c], pp.pos_scale_exp, pp.tokens_scale_exp);
    m->cls_row = A.add(cls_row, HV_EMBED);
    }

    for (int b = 0; b < HV_BLOCKS; ++b) {
        const hv_block_params &q = P->blocks[b];
        BlockDev &d = m->blocks[b];
        m->has_block[b] = q.wqkv != nullptr;
        if (!m->has_block[b]) continue;
        if (!q.ln1_gamma || !q.ln1_beta || !q.wqkv || !q.bqkv || !q.wproj || !q.bproj || !q.ln2_gamma ||
            !q.ln2_beta || !q.w1 || !q.b1 || !q.w2 || !q.b2)
            return fail(HV_ERR_VALUE, "block %d parameters missing", b + 1);
        if (!ln_scale_ok(q.x_scale_exp) || !ln_scale_ok(q.ffn_x_scale_exp))
            return fail(HV_ERR_VALUE, "layernorm input scale must be in [-32, 0] (block %d)", b + 1);
        d.ln1_g = A.add(q.ln1_gamma, 192);
        d.ln1_b = A.add(q.ln1_beta, 192);
        d.wqkv = A.add_t(q.wqkv, 192, HV_QKV, HV_QKV);
        d.bqkv = A.add(q.bqkv, HV_QKV * 4);
        d.wproj = A.add_t(q.wproj, 192, 192, 192);
        d.bproj = A.add(q.bproj, 192 * 4);
        d.ln2_g = A.add(q.ln2_gamma, 192);
        d.ln2_b = A.add(q.ln2_beta, 192);
        d.w1 = A.add_t(q.w1, 192, HV_FFN, HV_FFN);
        d.b1 = A.add(q.b1, HV_FFN * 4);
        d.w2 = A.add_t(q.w2, HV_FFN, 192, 192);
        {
            std::vector<int8_t> i1((size_t)192 * HV_FFN), i2((size_t)192 * HV_FFN);
            for (int j = 0; j < HV_FFN / 128; ++j) {
                int8_t *c1 = i1.data() + (size_t)j * 24576, *c2 = i2.data() + (size_t)j * 24576;
                for (int kc = 0; kc < 12; ++kc)
                    for (int r = 0; r < 128; ++r)
                        for (int b = 0; b < 16; ++b)
                            c1[kc * 2048 + r * 16 + b] = q.w1[(size_t)(16 * kc + b) * HV_FFN + 128 * j + r];
                for (int kc = 0; kc < 8; ++kc)
                    for (int r = 0; r < 192; ++r)
                        for (int b = 0; b < 16; ++b)
                            c2[kc * 3072 + r * 16 + b] = q.w2[(size_t)(128 * j + 16 * kc + b) * 192 + r];
            }
            d.w1img = A.add(i1.data(), i1.size());
            d.w2img = A.add(i2.data(), i2.size());
        }
        d.b2 = A.add(q.b2, 192 * 4);
        d.ln1_xs = q.x_scale_exp;
        d.ln1_gs = q.gamma1_scale_exp;
        d.ln1_bs = q.beta1_scale_exp;
        d.ln1_os = q.ln1_out_scale_exp;
        d.ln2_xs = q.ffn_x_scale_exp;
        d.ln2_gs = q.gamma2_scale_exp;
        d.ln2_bs = q.beta2_scale_exp;
        d.ln2_os = q.ln2_out_scale_exp;
        d.qkv_shift = q.qkv_out_scale_exp - (q.ln1_out_scale_exp + q.wqkv_scale_exp);
        d.qkv_wide = needs_wide(q.bqkv, HV_QKV, 192);
        d.proj_shift = q.msa_out_scale_exp - (q.context_out_scale_exp + q.wproj_scale_exp);
        d.proj_wide = needs_wide(q.bproj, 192, 192);
        d.fc1_sh_in = -16 - (q.ln2_out_scale_exp + q.w1_scale_exp);
        d.fc1_sh_out = q.hidden_out_scale_exp + 16;
        d.fc1_wide = needs_wide(q.b1, HV_FFN, 192);
        d.fc1_fast = (!d.fc1_wide && d.fc1_sh_in >= 1 && d.fc1_sh_in <= 30 && d.fc1_sh_out >= -7 &&
                      d.fc1_sh_out <= 30) ? 1 : 0;
        {
            // |acc + bias| <= 192 * 2^14 + max|b1| must stay inside gelu_chain_fast2's input range
            int32_t vlim = 0;
            const int64_t vmax = max_abs(q.b1, HV_FFN) + (int64_t)192 * 16384;
            d.fc1_k2 = (!d.fc1_wide && gelu_fast2_range(d.fc1_sh_in, d.fc1_sh_out, &vlim) && vmax <= vlim) ? 1 : 0;
            d.fc1_gk = make_gelu_k(d.fc1_k2 ? d.fc1_sh_in : 0, d.fc1_k2 ? d.fc1_sh_out : 0);
            // Exact table form when the output varies only over a short window of the
            // reachable Q8.16 inputs [-qmax, qmax], qmax = rsa(vmax, sh_in).
            d.fc1_tab_n = 0;
            d.fc1_tab_elo = INT32_MIN;
            d.fc1_tab_ehi = INT32_MAX;
            d.fc1_tab_mode = d.fc1_tab_k = d.fc1_tab_fine = d.fc1_tab_bytes = d.fc1_tab_c = 0;
            if (!d.fc1_wide && d.fc1_sh_in >= 0 && d.fc1_sh_in <= 30 && vmax < ((int64_t)1 << 30)) {
                const int64_t hin = d.fc1_sh_in > 0 ? (int64_t)1 << (d.fc1_sh_in - 1) : 0;
                const int64_t qmax = (vmax + hin) >> d.fc1_sh_in;
                if (qmax < ((int64_t)1 << 23)) {
                    if (!mm) CUDA_TRY(cudaMalloc(&mm, 2 * sizeof(int)));
                    int32_t wlo = 0, wn = 0;
                    CUDA_TRY(gelu_table_window((int32_t)qmax, d.fc1_sh_out, mm, &wlo, &wn, nullptr));
                    TabWindow tw{wlo, wn, INT32_MIN, INT32_MAX};
                    bool ok = wn <= kGeluTableMax;
                    BucketTable bt;
                    bool bucket = false;
                    if (!ok) {
                        // too wide for a whole-window table: a central table whose clamped
                        // ends cover long constant runs, with gelu_chain_fast2 outside them
                        // (needs the FMA form), else a two-level bucket table
                        std::vector<int8_t> f;
                        int rc = gelu_scan((int32_t)qmax, d.fc1_sh_out, f);
                        if (rc != HV_OK) return rc;
                        if (d.fc1_k2) gelu_escape_window(f, (int32_t)qmax, &tw, &ok);
                        if (!ok) gelu_bucket_table(f, (int32_t)qmax, &bt, &bucket);
                    }
                    if (ok) {
                        d.fc1_tab_mode = 1;
                        d.fc1_tab = A.add(nullptr, ((size_t)tw.n + 15) & ~(size_t)15);
                        d.fc1_tab_lo = tw.lo;
                        d.fc1_tab_n = tw.n;
                        d.fc1_tab_elo = tw.elo;
                        d.fc1_tab_ehi = tw.ehi;
                        d.fc1_tab_bytes = tw.n;
                        d.fc1_gk = make_gelu_k(d.fc1_sh_in, d.fc1_k2 ? d.fc1_sh_out : 0);
                        // a table over the whole window is exact everywhere: fold the
                        // offset into the rounding add when that stays in int32
                        const int64_t c = hin - ((int64_t)tw.lo << d.fc1_sh_in);
                        if (tw.elo == INT32_MIN && tw.ehi == INT32_MAX &&
                            vmax + (c < 0 ? -c : c) + 1 < ((int64_t)1 << 31)) {
                            d.fc1_tab_mode = 3;
                            d.fc1_tab_c = (int32_t)c;
                        }
                    } else if (bucket) {
                        bt.blob.resize((bt.blob.size() + 15) & ~(size_t)15, 0);
                        d.fc1_tab_mode = 2;
                        d.fc1_tab = A.add(bt.blob.data(), bt.blob.size());
                        d.fc1_tab_lo = bt.lo;
                        d.fc1_tab_n = bt.n;
                        d.fc1_tab_k = bt.k;
                        d.fc1_tab_fine = bt.fine_off;
                        d.fc1_tab_bytes = (int)bt.blob.size();
                        d.fc1_gk = make_gelu_k(d.fc1_sh_in, d.fc1_k2 ? d.fc1_sh_out : 0);
                    }
                }
            }
        }
        d.fc2_shift = q.ffn_out_scale_exp - (q.hidden_out_scale_exp + q.w2_scale_exp);
        d.fc2_wide = needs_wide(q.b2, 192, HV_FFN);
        if (!align_ok(q.x_scale_exp, q.msa_out_scale_exp, q.ffn_x_scale_exp) ||
            !align_ok(q.ffn_x_scale_exp, q.ffn_out_scale_exp, q.out_scale_exp))
            return fail(HV_ERR_VALUE, "residual exponent gap above 54 is not supported (block %d)", b + 1);
        d.res1 = make_align_add(q.x_scale_exp, q.msa_out_scale_exp, q.ffn_x_scale_exp);
        d.res2 = make_align_add(q.ffn_x_scale_exp, q.ffn_out_scale_exp, q.out_scale_exp);
        d.attn = make_attn(q.qkv_out_scale_exp, q.score_scale_exp, q.prob_scale_exp, q.context_out_scale_exp);
    }
    m->has_head = P->head_w != nullptr;
    if (m->has_head && !ln_scale_ok(P->blocks[HV_BLOCKS - 1].out_scale_exp))
        return fail(HV_ERR_VALUE, "layernorm input scale must be in [-32, 0] (final LN)");

    if (P->num_selectors < 0 || P->num_selectors > HV_MAX_SELECTORS)
        return fail(HV_ERR_VALUE, "num_selectors out of range");
    m->used_sel = 0;
    for (int b = 0; b < HV_BLOCKS; ++b) {
        m->sel_before[b] = P->selector_before[b];
        if (m->sel_before[b] >= P->num_selectors) return fail(HV_ERR_VALUE, "selector index out of range");
        if (m->sel_before[b] >= 0) m->used_sel++;
    }
    m->num_sel = P->num_selectors;
    for (int s = 0; s < P->num_selectors; ++s) {
        const hv_selector_params &q = P->selectors[s];
        SelDev &d = m->sels[s];
        if (!q.local_w || !q.local_b || !q.score_w1 || !q.score_b1 || !q.score_w2 || !q.score_b2 || !q.score_w3 ||
            !q.score_b3 || !q.hw_w1 || !q.hw_b1 || !q.hw_w2 || !q.hw_b2)
            return fail(HV_ERR_VALUE, "selector %d parameters missing", s + 1);
        std::vector<int8_t> t(3 * 32 * 64);
        for (int h = 0; h < 3; ++h)
            for (int k = 0; k < 64; ++k)
                for (int j = 0; j < 32; ++j) t[(h * 32 + j) * 64 + k] = q.local_w[(h * 64 + k) * 32 + j];
        d.lwt = A.add(t.data(), t.size());
        for (int h = 0; h < 3; ++h)
            for (int k = 0; k < 64; ++k)
                for (int j = 0; j < 32; ++j) t[(h * 32 + j) * 64 + k] = q.score_w1[(h * 64 + k) * 32 + j];
        d.w1t = A.add(t.data(), t.size());
        std::vector<int8_t> t2(3 * 16 * 32);
        for (int h = 0; h < 3; ++h)
            for (int j = 0; j < 32; ++j)
                for (int mm = 0; mm < 16; ++mm) t2[(h * 16 + mm) * 32 + j] = q.score_w2[(h * 32 + j) * 16 + mm];
        d.w2t = A.add(t2.data(), t2.size());
        std::vector<int8_t> t3(3 * 2 * 16);
        for (int h = 0; h < 3; ++h)
            for (int mm = 0; mm < 16; ++mm)
                for (int o = 0; o < 2; ++o) t3[(h * 2 + o) * 16 + mm] = q.score_w3[(h * 16 + mm) * 2 + o];
        d.w3t = A.add(t3.data(), t3.size());
        d.lb = A.add(q.local_b, 96 * 4);
        d.b1 = A.add(q.score_b1, 96 * 4);
        d.b2 = A.add(q.score_b2, 48 * 4);
        d.b3 = A.add(q.score_b3, 6 * 4);
        d.hw1 = A.add(q.hw_w1, 9);
        d.hb1 = A.add(q.hw_b1, 12);
        d.hw2 = A.add(q.hw_w2, 9);
        d.hb2 = A.add(q.hw_b2, 12);
        SelParams &p = d.p;
        memset(&p, 0, sizeof(p));
        p.local_sh_in = -16 - (q.in_scale_exp + q.local_w_scale_exp);
        p.local_sh_out = q.local_out_scale_exp + 16;
        p.h1_sh_in = -16 - (q.concat_out_scale_exp + q.score_w1_scale_exp);
        p.h1_sh_out = q.h1_out_scale_exp + 16;
        p.h2_sh_in = -16 - (q.h1_out_scale_exp + q.score_w2_scale_exp);
        p.h2_sh_out = q.h2_out_scale_exp + 16;
        p.logit_shift = q.logits_out_scale_exp - (q.h2_out_scale_exp + q.score_w3_scale_exp);
        p.logit_q16_shift = -16 - q.logits_out_scale_exp;
        p.hw_sh_in = -16 - (q.stats_out_scale_exp + q.hw_w1_scale_exp);
        p.hw_sh_out = q.hw_hidden_out_scale_exp + 16;
        p.hw_q16_shift = -16 - (q.hw_hidden_out_scale_exp + q.hw_w2_scale_exp);
        auto fast = [](int sh_in, int sh_out, int64_t bound) {
            return (sh_in >= 1 && sh_in <= 30 && sh_out >= -7 && sh_out <= 30 && bound < kNarrowLimit) ? 1 : 0;
        };
        p.local_fast = fast(p.local_sh_in, p.local_sh_out, max_abs(q.local_b, 96) + 64 * 16384);
        p.h1_fast = fast(p.h1_sh_in, p.h1_sh_out, max_abs(q.score_b1, 96) + 64 * 16384);
        p.h2_fast = fast(p.h2_sh_in, p.h2_sh_out, max_abs(q.score_b2, 48) + 32 * 16384);
        p.hw_fast = fast(p.hw_sh_in, p.hw_sh_out, max_abs(q.hw_b1, 3) + 3 * 16384);
        // FMA-pipe GELU chain: |acc + bias| must stay inside its input range
        auto k2 = [](int sh_in, int sh_out, int64_t bound, int wide_ok, GeluK *k) {
            int32_t vlim = 0;
            const int ok = (wide_ok && gelu_fast2_range(sh_in, sh_out, &vlim) && bound <= vlim) ? 1 : 0;
            *k = make_gelu_k(ok ? sh_in : 0, ok ? sh_out : 0);
            return ok;
        };
        p.local_k2 = k2(p.local_sh_in, p.local_sh_out, max_abs(q.local_b, 96) + 64 * 16384, 1, &p.local_k);
        p.h1_k2 = k2(p.h1_sh_in, p.h1_sh_out, max_abs(q.score_b1, 96) + 64 * 16384, 1, &p.h1_k);
        p.h2_k2 = k2(p.h2_sh_in, p.h2_sh_out, max_abs(q.score_b2, 48) + 32 * 16384, 1, &p.h2_k);
        p.hw_k2 = k2(p.hw_sh_in, p.hw_sh_out, max_abs(q.hw_b1, 3) + 3 * 16384, 1, &p.hw_k);
        // exact tables (selector_kernel's shared-memory budgets: local in its own
        // region, layers 1 and 2 together in the token region)
        int trc = sel_gelu_table(p.local_sh_in, p.local_sh_out, max_abs(q.local_b, 96) + 64 * 16384,
                                 kSelTabLocalBytes, A, &p.tab_local, &d.tab_local);
        if (trc == HV_OK)
            trc = sel_gelu_table(p.h1_sh_in, p.h1_sh_out, max_abs(q.score_b1, 96) + 64 * 16384, kSelTabH1Bytes, A,
                                 &p.tab_h1, &d.tab_h1);
        if (trc == HV_OK)
            trc = sel_gelu_table(p.h2_sh_in, p.h2_sh_out, max_abs(q.score_b2, 48) + 32 * 16384, kSelTabH2Bytes, A,
                                 &p.tab_h2, &d.tab_h2);
        if (trc != HV_OK) return trc;
    }
    if (m->has_head) {
    if (!P->final_gamma || !P->final_beta || !P->head_b) return fail(HV_ERR_VALUE, "head parameters missing");
    m->fin_g = A.add(P->final_gamma, 192);
    m->fin_b = A.add(P->final_beta, 192);
    m->fin_xs = P->blocks[HV_BLOCKS - 1].out_scale_exp;
    m->fin_gs = P->final_gamma_scale_exp;
    m->fin_bs = P->final_beta_scale_exp;
    m->fin_os = P->final_ln_out_scale_exp;
    m->head_wt = A.add_t(P->head_w, 192, HV_CLASSES, 1024);
    m->head_b = A.add(P->head_b, HV_CLASSES * 4);
    m->head_shift = HV_LOGIT_SCALE_EXP - (P->final_ln_out_scale_exp + P->head_w_scale_exp);
    }
    if (A.host.empty()) A.add(nullptr, 256);

    CUDA_TRY(cudaMalloc(&m->weights, A.host.size()));
    m->weights_bytes = A.host.size();
    CUDA_TRY(cudaMemcpy(m->weights, A.host.data(), A.host.size(), cudaMemcpyHostToDevice));
    for (int b = 0; b < HV_BLOCKS; ++b) {
        const BlockDev &d = m->blocks[b];
        if (m->has_block[b] && d.fc1_tab_n > 0 && (d.fc1_tab_mode == 1 || d.fc1_tab_mode == 3))
            CUDA_TRY(launch_gelu_table_fill((int8_t *)(m->weights + d.fc1_tab), d.fc1_tab_lo, d.fc1_tab_n, d.fc1_sh_out,
                                            nullptr));
    }
    CUDA_TRY(cudaDeviceSynchronize());
    return HV_OK;
}

}  // namespace

// Enqueue one inference on `st` (a non-default stream) as a CUDA graph: replay the
// cached capture for the same input, batch, workspace and outputs, else capture
// and instantiate one (the least recently used entry is replaced).  The kernels
// read the live token counts from device memory, so a capture is valid for any
// input contents.
int run_graph(hv_model *m, const int8_t *img, int batch, int32_t *lg, int32_t *tc, hv_selector_summary *sum,
              uint8_t *warn, int wsi, cudaStream_t st) {
    GraphEntry *hit = nullptr, *victim = &m->graphs[0];
    for (GraphEntry &g : m->graphs) {
        if (g.exec && g.img == img && g.batch == batch && g.ws == wsi && g.lg == lg && g.tc == tc && g.sum == sum &&
            g.warn == warn && g.prof_stage == m->prof_stage && (!m->prof_stage || g.prof_max == m->prof_max))
            hit = &g;
        if (!g.exec || g.stamp < victim->stamp) victim = &g;
    }
    if (!hit) {
        int rc = ensure_capacity(m, batch, wsi);  // allocations stay outside the capture
        if (rc) return rc;
        // Under profiling, the capture records the event pairs 0..n-1 around the
        // stage's launches; every replay records the same events again.
        m->prof_n = 0;
        cudaGraph_t graph = nullptr;
        CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = infer_impl(m, img, batch, lg, tc, sum, warn, nullptr, nullptr, st, wsi);
        const cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return rc;
        }
        if (ce != cudaSuccess) return fail(HV_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
        int kernels = 0;
        size_t nn = 0;
        if (cudaGraphGetNodes(graph, nullptr, &nn) == cudaSuccess && nn > 0) {
            std::vector<cudaGraphNode_t> nodes(nn);
            if (cudaGraphGetNodes(graph, nodes.data(), &nn) == cudaSuccess)
                for (size_t i = 0; i < nn; ++i) {
                    cudaGraphNodeType ty;
                    if (cudaGraphNodeGetType(nodes[i], &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
                }
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return fail(HV_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
        if (victim->exec) cudaGraphExecDestroy(victim->exec);
        *victim = GraphEntry{exec, img, batch, wsi, lg, tc, sum, warn, 0, m->prof_stage, m->prof_n, kernels, m->prof_max};
        hit = victim;
    }
    hit->stamp = ++m->graph_clock;
    if (m->prof_stage) m->prof_n = hit->prof_n;
    m->last_graph_kernels = hit->kernels;
    use_workspace(m, wsi);
    CUDA_TRY(cudaGraphLaunch(hit->exec, st));
    return HV_OK;
}

// =============================================================================
// C ABI
// =============================================================================
extern "C" {

const char *hv_version(void) { return "heatvit_b200 0.1 (sm_100a)"; }

const char *hv_last_error(void) { return g_err; }

int hv_model_create(const hv_params *params, int device, hv_model **out) {
    if (!params || !out) return fail(HV_ERR_VALUE, "null argument");
    *out = nullptr;
    CUDA_TRY(cudaSetDevice(device));
    int sms = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    hv_model *m = new hv_model();
    m->device = device;
    m->sms = sms;
    {
        const char *t = getenv("HV_GEMM_TILED");
        m->persistent = (t && t[0] == '1') ? 0 : 1;
        const char *u = getenv("HV_FFN_UNFUSED");
        m->fused_ffn = (m->persistent && !(u && u[0] == '1')) ? 1 : 0;
        const char *g = getenv("HV_NO_GRAPH");
        m->use_graphs = (g && g[0] == '1') ? 0 : 1;
    }
    int rc = pack_model(m, params);
    if (rc) {
        hv_model_destroy(m);
        return rc;
    }
    *out = m;
    return HV_OK;
}

int hv_model_destroy(hv_model *m) {
    if (!m) return HV_OK;
    cudaSetDevice(m->device);
    for (int i = 0; i < 2; ++i)
        for (int k = 0; k < 2; ++k)
            if (m->host_calls[i].done[k]) {
                cudaEventSynchronize(m->host_calls[i].done[k]);  // calls never waited for
                cudaEventDestroy(m->host_calls[i].done[k]);
            }
    for (GraphEntry &g : m->graphs)
        if (g.exec) cudaGraphExecDestroy(g.exec);
    if (m->graph_stream) cudaStreamDestroy(m->graph_stream);
    if (m->ev_fork) cudaEventDestroy(m->ev_fork);
    if (m->ev_join) cudaEventDestroy(m->ev_join);
    if (m->weights) cudaFree(m->weights);
    for (int i = 0; i < 2; ++i)
        if (m->ws[i].scratch) cudaFree(m->ws[i].scratch);
    for (int i = 0; i < 2; ++i) {
        if (m->ev_pin[i]) cudaEventDestroy(m->ev_pin[i]);
    }
    for (int i = 0; i < 4; ++i) {
        if (m->himg[i]) cudaFree(m->himg[i]);
        if (m->ev_in[i]) cudaEventDestroy(m->ev_in[i]);
        if (m->ev_done[i]) cudaEventDestroy(m->ev_done[i]);
    }
    if (m->hlogits) cudaFree(m->hlogits);
    if (m->htc) cudaFree(m->htc);
    if (m->hsum) cudaFree(m->hsum);
    if (m->hwarn) cudaFree(m->hwarn);
    for (int i = 0; i < 2; ++i) {
        if (m->pin_out[i]) cudaFreeHost(m->pin_out[i]);
        if (m->pin_in[i]) cudaFreeHost(m->pin_in[i]);
    }
    for (auto e : m->prof_ev) cudaEventDestroy(e);
    if (m->prof_rows) cudaFree(m->prof_rows);
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    for (int i = 0; i < 2; ++i)
        if (m->compute_stream[i]) cudaStreamDestroy(m->compute_stream[i]);
    delete m;
    return HV_OK;
}

int hv_infer_batch(hv_model *m, const int8_t *d_images, int batch, int32_t *d_logits, int32_t *d_token_counts,
                   hv_selector_summary *d_summary, uint8_t *d_warnings, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    cudaStream_t st = (cudaStream_t)stream;
    if (!m->use_graphs || batch <= 0 || !d_images || !d_logits)
        return infer_impl(m, d_images, batch, d_logits, d_token_counts, d_summary, d_warnings, nullptr, nullptr, st);
    // Replay on the model's own stream, ordered after and before the caller's work on
    // `stream`; outputs go to workspace buffers and are copied out on `stream`.
    CUDA_TRY(cudaSetDevice(m->device));
    if (!m->graph_stream) {
        CUDA_TRY(cudaStreamCreateWithFlags(&m->graph_stream, cudaStreamNonBlocking));
        CUDA_TRY(cudaEventCreateWithFlags(&m->ev_fork, cudaEventDisableTiming));
        CUDA_TRY(cudaEventCreateWithFlags(&m->ev_join, cudaEventDisableTiming));
    }
    int rc = ensure_capacity(m, batch, 0);
    if (rc) return rc;
    const Workspace &w = m->ws[0];
    const int ns = m->used_sel;
    CUDA_TRY(cudaEventRecord(m->ev_fork, st));
    CUDA_TRY(cudaStreamWaitEvent(m->graph_stream, m->ev_fork, 0));
    rc = run_graph(m, d_images, batch, w.o_logits, d_token_counts ? w.o_tc : nullptr, d_summary ? w.o_sum : nullptr,
                   d_warnings ? w.o_warn : nullptr, 0, m->graph_stream);
    if (rc) return rc;
    CUDA_TRY(cudaEventRecord(m->ev_join, m->graph_stream));
    CUDA_TRY(cudaStreamWaitEvent(st, m->ev_join, 0));
    CUDA_TRY(cudaMemcpyAsync(d_logits, w.o_logits, (size_t)batch * HV_CLASSES * 4, cudaMemcpyDeviceToDevice, st));
    if (d_token_counts)
        CUDA_TRY(cudaMemcpyAsync(d_token_counts, w.o_tc, (size_t)batch * (ns + 1) * 4, cudaMemcpyDeviceToDevice, st));
    if (d_summary && ns)
        CUDA_TRY(cudaMemcpyAsync(d_summary, w.o_sum, (size_t)batch * ns * sizeof(hv_selector_summary),
                                 cudaMemcpyDeviceToDevice, st));
    if (d_warnings) CUDA_TRY(cudaMemcpyAsync(d_warnings, w.o_warn, (size_t)batch, cudaMemcpyDeviceToDevice, st));
    return HV_OK;
}

int hv_infer_batch_checkpoints(hv_model *m, const int8_t *d_images, int batch, int32_t *d_logits,
                               int32_t *d_token_counts, hv_selector_summary *d_summary, uint8_t *d_warnings,
                               int8_t *d_ckpt, int32_t *d_ckpt_rows, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (!d_ckpt || !d_ckpt_rows) return fail(HV_ERR_VALUE, "checkpoint buffers are required");
    return infer_impl(m, d_images, batch, d_logits, d_token_counts, d_summary, d_warnings, d_ckpt, d_ckpt_rows,
                      (cudaStream_t)stream);
}

namespace {

int host_wait_oldest(hv_model *m) {
    hv_model::HostCall &c = m->host_calls[m->host_head];
    const int slot = m->host_head;
    for (int k = 0; k < 2; ++k) CUDA_TRY(cudaEventSynchronize(c.done[k]));
    m->host_head = (m->host_head + 1) % 2;
    m->host_pending -= 1;
    const uint8_t *st = m->pin_out[slot];
    if (!c.pinned_out) memcpy(c.logits, st, (size_t)c.batch * HV_CLASSES * 4);
    if (c.tc) memcpy(c.tc, st + c.o_tc, (size_t)c.batch * (c.ns + 1) * 4);
    if (c.sum && c.ns) memcpy(c.sum, st + c.o_sum, (size_t)c.batch * c.ns * sizeof(hv_selector_summary));
    if (c.warn) memcpy(c.warn, st + c.o_warn, (size_t)c.batch);
    for (int i = 0; i < 2; ++i) {
        if (!m->ws[i].err) continue;
        int code = 0;
        CUDA_TRY(cudaMemcpy(&code, m->ws[i].err, sizeof(int), cudaMemcpyDeviceToHost));
        if (code) return fail(HV_ERR_STATE, "a device-side bounded wait gave up (code %d)", code);
    }
    return HV_OK;
}

// Let the device work of every call in flight finish; the calls stay pending
// (their outputs reach the caller at their waits).
int host_quiesce(hv_model *m) {
    for (int k = 0; k < m->host_pending; ++k) {
        const hv_model::HostCall &c = m->host_calls[(m->host_head + k) % 2];
        for (int j = 0; j < 2; ++j) CUDA_TRY(cudaEventSynchronize(c.done[j]));
    }
    return HV_OK;
}

}  // namespace

int hv_infer_host_submit(hv_model *m, const int8_t *h_images, int batch, int32_t *h_logits, int32_t *h_token_counts,
                         hv_selector_summary *h_summary, uint8_t *h_warnings) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    if (batch <= 0 || !h_images || !h_logits) return fail(HV_ERR_VALUE, "bad arguments");
    CUDA_TRY(cudaSetDevice(m->device));
    if (m->host_pending == 2) {
        const int rc = host_wait_oldest(m);
        if (rc) return rc;
    }
    if (!m->host_pending) m->host_chunks = 0;  // every earlier chunk has finished
    // Chunk schedule.  Consecutive chunks run on two streams and every upload but
    // the first overlaps compute; a tail of less than a quarter chunk joins the
    // chunk before it.  The first chunk stays as large as the others: measured on
    // B200, one inference costs about 0.9 ms plus 3.2 us per image (64 images
    // 1.10 ms, 512 images 2.53 ms, 1024 images 4.19 ms), so a smaller first chunk
    // adds more fixed cost than the 2.7 us per image of upload it hides (1024
    // images: first chunk 512 -> 6.16 ms, 256 -> 6.75 ms, 128 -> 6.93 ms).
    // A call submitted behind another has its upload hidden behind that call's
    // compute already, so it runs as 1024-image chunks, all on one compute stream:
    // inferences on two streams at once compete for the SMs and the L2 (measured
    // pipelined at 1024 images per call: 1024-image chunks alternating between two
    // streams 4.97 ms per call, 512-image chunks on two streams 4.40 ms).
    // HV_HOST_CHUNK_FIRST / HV_HOST_CHUNK_MAX override the sizes; later chunks
    // grow by at most 1.5x.
    const bool behind = m->host_pending > 0;
    int first_chunk = behind ? 1024 : 512, max_chunk = first_chunk;
    if (const char *e = getenv("HV_HOST_CHUNK_FIRST")) first_chunk = std::max(1, atoi(e));
    if (const char *e = getenv("HV_HOST_CHUNK_MAX")) max_chunk = std::max(1, atoi(e));
    std::vector<int> starts(1, 0);
    int chunk = 0;
    for (int f = 0, next = std::min(first_chunk, max_chunk); f < batch;) {
        int cnt = std::min(next, batch - f);
        if (batch - f - cnt < cnt / 4) cnt = batch - f;
        f += cnt;
        starts.push_back(f);
        chunk = std::max(chunk, cnt);
        next = std::min(max_chunk, cnt + cnt / 2);
    }
    const int ns = m->used_sel;
    if (!m->copy_stream) {
        CUDA_TRY(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking));
        for (int i = 0; i < 2; ++i) CUDA_TRY(cudaStreamCreateWithFlags(&m->compute_stream[i], cudaStreamNonBlocking));
        for (int i = 0; i < 4; ++i) {
            CUDA_TRY(cudaEventCreateWithFlags(&m->ev_in[i], cudaEventDisableTiming));
            CUDA_TRY(cudaEventCreateWithFlags(&m->ev_done[i], cudaEventDisableTiming));
        }
        for (int i = 0; i < 2; ++i) {
            CUDA_TRY(cudaEventCreateWithFlags(&m->ev_pin[i], cudaEventDisableTiming));
            for (int k = 0; k < 2; ++k)
                CUDA_TRY(cudaEventCreateWithFlags(&m->host_calls[i].done[k], cudaEventDisableTiming));
        }
    }
    // Workspaces this call uses (chunk g takes g & 1).  Growing a device buffer
    // frees the old one, which calls in flight may still use: finish them first.
    bool use_ws[2] = {false, false};
    for (size_t c = 0; c + 1 < starts.size(); ++c) use_ws[behind ? 0 : (m->host_chunks + c) & 1] = true;
    if ((chunk > m->host_cap || (use_ws[0] && chunk > m->ws[0].cap) || (use_ws[1] && chunk > m->ws[1].cap)) &&
        m->host_pending) {
        const int rc = host_quiesce(m);
        if (rc) return rc;
    }
    if (chunk > m->host_cap) {
        for (int i = 0; i < 4; ++i)
            if (m->himg[i]) cudaFree(m->himg[i]);
        if (m->hlogits) cudaFree(m->hlogits);
        if (m->htc) cudaFree(m->htc);
        if (m->hsum) cudaFree(m->hsum);
        if (m->hwarn) cudaFree(m->hwarn);
        m->host_cap = 0;
        for (int i = 0; i < 4; ++i) CUDA_TRY(cudaMalloc(&m->himg[i], (size_t)chunk * HV_IMAGE_BYTES));
        CUDA_TRY(cudaMalloc(&m->hlogits, (size_t)chunk * HV_CLASSES * 4 * 2));
        CUDA_TRY(cudaMalloc(&m->htc, (size_t)chunk * (HV_MAX_SELECTORS + 1) * 4 * 2));
        CUDA_TRY(cudaMalloc(&m->hsum, (size_t)chunk * HV_MAX_SELECTORS * sizeof(hv_selector_summary) * 2));
        CUDA_TRY(cudaMalloc(&m->hwarn, (size_t)chunk * 2));
        m->host_cap = chunk;
    }
    // Chunks alternate between two workspaces.  The chunks of a call with nothing in
    // flight also alternate between two compute streams, so one chunk's kernels fill
    // the idle tails of the other's while the later uploads land.
    int rc = HV_OK;
    for (int i = 0; i < 2; ++i)
        if (use_ws[i] && (rc = ensure_capacity(m, chunk, i)) != 0) return rc;
    // Outputs land in the call's pinned staging slot (an asynchronous copy into
    // pageable memory would block this thread until the chunk's compute finished)
    // and reach the caller's arrays at the wait.
    const int slot = (m->host_head + m->host_pending) % 2;
    hv_model::HostCall &call = m->host_calls[slot];
    const size_t o_log = 0, o_tc = o_log + (size_t)batch * HV_CLASSES * 4,
                 o_sum = o_tc + (size_t)batch * (ns + 1) * 4,
                 o_warn = o_sum + (size_t)batch * ns * sizeof(hv_selector_summary),
                 o_end = o_warn + (size_t)batch;
    if (o_end > m->pin_out_cap[slot]) {
        if (m->pin_out[slot]) cudaFreeHost(m->pin_out[slot]);
        m->pin_out[slot] = nullptr;
        m->pin_out_cap[slot] = 0;
        CUDA_TRY(cudaHostAlloc((void **)&m->pin_out[slot], o_end, cudaHostAllocDefault));
        m->pin_out_cap[slot] = o_end;
    }
    uint8_t *stage = m->pin_out[slot];
    // Pageable images are staged through two pinned chunk buffers; the host copy of
    // chunk c + 1 overlaps the device work on chunk c.
    cudaPointerAttributes pa;
    const bool pinned_in = cudaPointerGetAttributes(&pa, h_images) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();  // clear a possible error from the query
    // Page-locked logits take the device copies directly (no staging copy at the end).
    const bool pinned_out = cudaPointerGetAttributes(&pa, h_logits) == cudaSuccess && pa.type == cudaMemoryTypeHost;
    cudaGetLastError();
    if (!pinned_in && chunk > m->pin_in_cap) {
        for (int i = 0; i < 2; ++i) {
            if (m->pin_in[i]) {
                CUDA_TRY(cudaEventSynchronize(m->ev_pin[i]));  // its last upload has finished
                cudaFreeHost(m->pin_in[i]);
            }
            m->pin_in[i] = nullptr;
        }
        m->pin_in_cap = 0;
        for (int i = 0; i < 2; ++i)
            CUDA_TRY(cudaHostAlloc((void **)&m->pin_in[i], (size_t)chunk * HV_IMAGE_BYTES, cudaHostAllocDefault));
        m->pin_in_cap = chunk;
    }
    const int nchunks = (int)starts.size() - 1;
    for (int c = 0; c < nchunks; ++c) {
        // chunk g: device images g % 4, pinned staging g % 2; workspace, device outputs
        // and compute stream g % 2, or all 0 for a call behind another (stream order
        // then follows every earlier user of workspace 0 and its outputs, and the
        // earlier call's chunks on workspace 1 / stream 1 are left alone)
        const unsigned long long g = m->host_chunks++;
        const int buf = (int)(g & 1), ib = (int)(g & 3), wsb = behind ? 0 : buf;
        const int first = starts[c], cnt = starts[c + 1] - starts[c];
        const int8_t *src = h_images + (size_t)first * HV_IMAGE_BYTES;
        if (!pinned_in) {
            // the upload out of pin_in[buf] issued two chunks back must have finished
            CUDA_TRY(cudaEventSynchronize(m->ev_pin[buf]));
            memcpy(m->pin_in[buf], src, (size_t)cnt * HV_IMAGE_BYTES);
            src = m->pin_in[buf];
        }
        // The upload into himg[ib] waits until the chunk four back has computed on it
        // (an event never recorded is complete), so uploads run up to three chunks
        // ahead of the compute.
        CUDA_TRY(cudaStreamWaitEvent(m->copy_stream, m->ev_done[ib], 0));
        CUDA_TRY(cudaMemcpyAsync(m->himg[ib], src, (size_t)cnt * HV_IMAGE_BYTES, cudaMemcpyHostToDevice,
                                 m->copy_stream));
        CUDA_TRY(cudaEventRecord(m->ev_in[ib], m->copy_stream));
        if (!pinned_in) CUDA_TRY(cudaEventRecord(m->ev_pin[buf], m->copy_stream));
        cudaStream_t cst = m->compute_stream[wsb];
        use_workspace(m, wsb);
        CUDA_TRY(cudaStreamWaitEvent(cst, m->ev_in[ib], 0));
        int32_t *dl = m->hlogits + (size_t)wsb * m->host_cap * HV_CLASSES;
        int32_t *dtc = m->htc + (size_t)wsb * m->host_cap * (HV_MAX_SELECTORS + 1);
        hv_selector_summary *dsum = m->hsum + (size_t)wsb * m->host_cap * HV_MAX_SELECTORS;
        uint8_t *dw = m->hwarn + (size_t)wsb * m->host_cap;
        if (m->use_graphs && !m->prof_stage)
            rc = run_graph(m, m->himg[ib], cnt, dl, h_token_counts ? dtc : nullptr, h_summary ? dsum : nullptr,
                           h_warnings ? dw : nullptr, wsb, cst);
        else
            rc = infer_impl(m, m->himg[ib], cnt, dl, h_token_counts ? dtc : nullptr, h_summary ? dsum : nullptr,
                            h_warnings ? dw : nullptr, nullptr, nullptr, cst, wsb);
        if (rc) {
            use_workspace(m, 0);
            return rc;
        }
        CUDA_TRY(cudaEventRecord(m->ev_done[ib], cst));
        CUDA_TRY(cudaMemcpyAsync(pinned_out ? (uint8_t *)(h_logits + (size_t)first * HV_CLASSES)
                                            : stage + o_log + (size_t)first * HV_CLASSES * 4,
                                 dl, (size_t)cnt * HV_CLASSES * 4, cudaMemcpyDeviceToHost, cst));
        if (h_token_counts)
            CUDA_TRY(cudaMemcpyAsync(stage + o_tc + (size_t)first * (ns + 1) * 4, dtc, (size_t)cnt * (ns + 1) * 4,
                                     cudaMemcpyDeviceToHost, cst));
        if (h_summary && ns)
            CUDA_TRY(cudaMemcpyAsync(stage + o_sum + (size_t)first * ns * sizeof(hv_selector_summary), dsum,
                                     (size_t)cnt * ns * sizeof(hv_selector_summary), cudaMemcpyDeviceToHost, cst));
        if (h_warnings) CUDA_TRY(cudaMemcpyAsync(stage + o_warn + first, dw, cnt, cudaMemcpyDeviceToHost, cst));
    }
    use_workspace(m, 0);
    for (int k = 0; k < 2; ++k) CUDA_TRY(cudaEventRecord(call.done[k], m->compute_stream[k]));
    call.batch = batch;
    call.ns = ns;
    call.logits = h_logits;
    call.tc = h_token_counts;
    call.sum = h_summary;
    call.warn = h_warnings;
    call.pinned_out = pinned_out;
    call.o_tc = o_tc;
    call.o_sum = o_sum;
    call.o_warn = o_warn;
    m->host_pending += 1;
    return HV_OK;
}

int hv_infer_host_wait(hv_model *m) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    if (!m->host_pending) return fail(HV_ERR_STATE, "no host call in flight");
    CUDA_TRY(cudaSetDevice(m->device));
    return host_wait_oldest(m);
}

int hv_infer_host(hv_model *m, const int8_t *h_images, int batch, int32_t *h_logits, int32_t *h_token_counts,
                  hv_selector_summary *h_summary, uint8_t *h_warnings) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    CUDA_TRY(cudaSetDevice(m->device));
    const int rc = hv_infer_host_submit(m, h_images, batch, h_logits, h_token_counts, h_summary, h_warnings);
    if (rc) return rc;
    return host_wait_oldest(m);
}

int hv_device_error(hv_model *m, int *code) {
    if (!m || !code) return fail(HV_ERR_VALUE, "null argument");
    *code = 0;
    CUDA_TRY(cudaSetDevice(m->device));
    for (int i = 0; i < 2; ++i) {
        if (!m->ws[i].err) continue;
        int c = 0;
        CUDA_TRY(cudaMemcpy(&c, m->ws[i].err, sizeof(int), cudaMemcpyDeviceToHost));
        if (c) {
            CUDA_TRY(cudaMemset(m->ws[i].err, 0, sizeof(int)));
            if (!*code) *code = c;
        }
    }
    return HV_OK;
}

int hv_profile_start(hv_model *m, int stage, int max_launches) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (max_launches < 0) return fail(HV_ERR_VALUE, "negative launch count");
    CUDA_TRY(cudaSetDevice(m->device));
    if ((int)m->prof_ev.size() < 2 * max_launches) {
        while ((int)m->prof_ev.size() < 2 * max_launches) {
            cudaEvent_t e;
            CUDA_TRY(cudaEventCreate(&e));
            m->prof_ev.push_back(e);
        }
        if (m->prof_rows) cudaFree(m->prof_rows);
        m->prof_rows = nullptr;
        CUDA_TRY(cudaMalloc(&m->prof_rows, sizeof(int32_t) * (size_t)std::max(1, max_launches)));
    }
    if (!m->prof_rows) CUDA_TRY(cudaMalloc(&m->prof_rows, sizeof(int32_t) * (size_t)std::max(1, max_launches)));
    m->prof_stage = stage;
    m->prof_max = max_launches;
    m->prof_n = 0;
    return HV_OK;
}

int hv_profile_stop(hv_model *m, int *launches, double *total_ms, long long *rows) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    CUDA_TRY(cudaSetDevice(m->device));
    const int n = m->prof_n;
    double tot = 0.0;
    long long rsum = 0;
    if (n > 0) {
        CUDA_TRY(cudaEventSynchronize(m->prof_ev[2 * n - 1]));
        for (int i = 0; i < n; ++i) {
            float ms = 0.f;
            CUDA_TRY(cudaEventElapsedTime(&ms, m->prof_ev[2 * i], m->prof_ev[2 * i + 1]));
            tot += ms;
        }
        std::vector<int32_t> r(n);
        CUDA_TRY(cudaMemcpy(r.data(), m->prof_rows, sizeof(int32_t) * n, cudaMemcpyDeviceToHost));
        for (int i = 0; i < n; ++i) rsum += r[i];
    }
    m->prof_stage = 0;
    m->prof_n = 0;
    if (launches) *launches = n;
    if (total_ms) *total_ms = tot;
    if (rows) *rows = rsum;
    return HV_OK;
}

int hv_test_gemm_stall(hv_model *m, unsigned wait_iters, int skip_tile) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (skip_tile < -1) return fail(HV_ERR_VALUE, "skip_tile must be -1 (off) or a tile index");
    CUDA_TRY(cudaSetDevice(m->device));
    // Captured graphs hold the launch arguments: drop them so the next calls capture
    // (or launch) with the new settings.
    CUDA_TRY(cudaDeviceSynchronize());
    for (GraphEntry &g : m->graphs)
        if (g.exec) {
            cudaGraphExecDestroy(g.exec);
            g = GraphEntry();
        }
    m->test_wait_iters = wait_iters;
    m->test_skip_tile = skip_tile + 1;  // GemmArgs: 0 = off, t + 1 = tile t
    return HV_OK;
}

int hv_graph_kernels(hv_model *m, int *kernels) {
    if (!m || !kernels) return fail(HV_ERR_VALUE, "null argument");
    *kernels = m->last_graph_kernels;
    return HV_OK;
}

// ---- per-operator entry points ------------------------------------------------------

int hv_gemm_i8_acc(const void *d_a, const int8_t *d_b, const int32_t *d_bias, int m, int n, int k, int transpose_b,
                   int a_unsigned, int64_t *d_acc, void *stream);

namespace {
__global__ void pad_a_kernel(const uint8_t *a, int m, int k, int kp, uint8_t *out) {
    const int64_t total = (int64_t)m * kp;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kp), c = (int)(i - (int64_t)r * kp);
        out[i] = c < k ? a[(size_t)r * k + c] : 0;
    }
}
// Bt[np][kp]: from b [k][n] (transpose_b = 0) or [n][k] (transpose_b = 1).
__global__ void pad_b_kernel(const int8_t *b, int n, int k, int transpose_b, int np, int kp, int8_t *out) {
    const int64_t total = (int64_t)np * kp;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / kp), c = (int)(i - (int64_t)r * kp);
        int8_t v = 0;
        if (r < n && c < k) v = transpose_b ? b[(size_t)r * k + c] : b[(size_t)c * n + r];
        out[i] = v;
    }
}
}  // namespace

int hv_gemm_i8_acc(const void *d_a, const int8_t *d_b, const int32_t *d_bias, int m, int n, int k, int transpose_b,
                   int a_unsigned, int64_t *d_acc, void *stream) {
    if (m < 0 || n < 0 || k < 0) return fail(HV_ERR_VALUE, "negative dimension");
    if (m == 0 || n == 0) return HV_OK;
    if (!d_a || !d_b || !d_acc) return fail(HV_ERR_VALUE, "null buffer");
    if (k > (a_unsigned ? 65793 : 131071))
        return fail(HV_ERR_VALUE, "k=%d can overflow the int32 accumulator; not supported", k);
    cudaStream_t st = (cudaStream_t)stream;
    const int tn = gemm_tile_n(n);
    const int kp = std::max(64, (k + 63) / 64 * 64), np = (n + tn - 1) / tn * tn;
    uint8_t *ap = nullptr;
    int8_t *bp = nullptr;
    int *err = nullptr;
    CUDA_TRY(cudaMalloc(&ap, (size_t)m * kp + 16));
    if (cudaMalloc(&bp, (size_t)np * kp) != cudaSuccess || cudaMalloc(&err, 16) != cudaSuccess) {
        cudaFree(ap);
        cudaFree(bp);
        return fail(HV_ERR_NOMEM, "cannot allocate padded operands");
    }
    int rc = HV_OK;
    cudaMemsetAsync(err, 0, 16, st);
    pad_a_kernel<<<148 * 4, 256, 0, st>>>((const uint8_t *)d_a, m, k, kp, ap);
    pad_b_kernel<<<148 * 4, 256, 0, st>>>(d_b, n, k, transpose_b, np, kp, bp);
    GemmArgs g = gemm_args(ap, kp, 0, bp, n, kp, m, nullptr, d_acc, n);
    g.epi.bias = d_bias;
    g.epi.bits_wide = 1;
    cudaError_t e = launch_gemm(g, EPI_ACC64, a_unsigned, m, err, st);
    if (e != cudaSuccess) rc = fail(HV_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
    cudaStreamSynchronize(st);
    int code = 0;
    cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (!rc && code) rc = fail(HV_ERR_STATE, "a device-side bounded wait gave up (code %d)", code);
    cudaFree(ap);
    cudaFree(bp);
    cudaFree(err);
    return rc;
}

int hv_gemm_i8(const void *d_a, const int8_t *d_b, const int32_t *d_bias, int m, int n, int k, int transpose_b,
               int a_unsigned, int src_exp, int dst_exp, int out_bits, void *d_out, void *stream) {
    if (out_bits != 8 && out_bits != 32) return fail(HV_ERR_VALUE, "output_bits must be 8 or 32");
    if (m < 0 || n < 0 || k < 0) return fail(HV_ERR_VALUE, "negative dimension");
    if (m == 0 || n == 0) return HV_OK;
    if (!d_a || !d_b || !d_out) return fail(HV_ERR_VALUE, "null buffer");
    if (k > (a_unsigned ? 65793 : 131071))
        return fail(HV_ERR_VALUE, "k=%d can overflow the int32 accumulator; not supported", k);
    cudaStream_t st = (cudaStream_t)stream;
    // The tiled kernel's int8 epilogue stores 16-byte pieces of a row: it needs
    // 16-byte aligned output rows (n a multiple of 16, d_out 16-byte aligned).
    const bool i8_rows_ok = n % 16 == 0 && (uintptr_t)d_out % 16 == 0;
    if (k == 0 || (out_bits == 8 && (a_unsigned || !i8_rows_ok))) {
        // the raw accumulator, then the element-wise writeback
        int64_t *acc = nullptr;
        CUDA_TRY(cudaMalloc(&acc, (size_t)m * n * 8));
        int rc = HV_OK;
        if (k == 0) {
            cudaMemsetAsync(acc, 0, (size_t)m * n * 8, st);
            if (d_bias) rc = fail(HV_ERR_VALUE, "k = 0 with a bias: use hv_gemm_i8_acc");
        } else {
            rc = hv_gemm_i8_acc(d_a, d_b, d_bias, m, n, k, transpose_b, a_unsigned, acc, stream);
        }
        if (!rc) {
            cudaError_t e = launch_writeback(acc, (int64_t)m * n, dst_exp - src_exp, out_bits, d_out, st);
            if (e != cudaSuccess) rc = fail(HV_ERR_CUDA, "writeback: %s", cudaGetErrorString(e));
            cudaStreamSynchronize(st);
        }
        cudaFree(acc);
        return rc;
    }
    // Fused writeback in the GEMM epilogue (gemm.py:123-139): EPI_I8 requantises
    // acc + bias to int8, EPI_I32 to int32.  The 32-bit epilogue form needs the
    // host-side bias bound (|acc| <= k * 2^14 plus |bias| below 2^30).
    std::vector<int32_t> hb(n, 0);
    if (d_bias) CUDA_TRY(cudaMemcpy(hb.data(), d_bias, sizeof(int32_t) * (size_t)n, cudaMemcpyDeviceToHost));
    int dev = 0, sms = 148;
    CUDA_TRY(cudaGetDevice(&dev));
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int epi = out_bits == 8 ? EPI_I8 : EPI_I32;
    // The model's layer shapes (signed A, K in {192, 768}) run on the persistent
    // kernel: weights resident in shared memory, A by TMA, 32-byte output stores.
    const bool persistent = epi == EPI_I8 && gemm_persistent_supported(EPI_I8, n, k) &&
                            (uintptr_t)d_a % 16 == 0 && (uintptr_t)d_out % 32 == 0;
    const int tn = gemm_tile_n(n);
    const int kp = persistent ? k : std::max(64, (k + 63) / 64 * 64);
    const int np = persistent ? n : (n + tn - 1) / tn * tn;
    const bool pad_a = !persistent && (kp != k || (uintptr_t)d_a % 16 != 0);
    uint8_t *ap = nullptr;
    int8_t *bp = nullptr;
    int *err = nullptr;
    if ((pad_a && cudaMalloc(&ap, (size_t)m * kp + 16) != cudaSuccess) ||
        cudaMalloc(&bp, (size_t)np * kp) != cudaSuccess || cudaMalloc(&err, 16) != cudaSuccess) {
        cudaFree(ap);
        cudaFree(bp);
        cudaFree(err);
        return fail(HV_ERR_NOMEM, "cannot allocate padded operands");
    }
    int rc = HV_OK;
    cudaMemsetAsync(err, 0, 16, st);
    if (pad_a) pad_a_kernel<<<148 * 4, 256, 0, st>>>((const uint8_t *)d_a, m, k, kp, ap);
    pad_b_kernel<<<148 * 4, 256, 0, st>>>(d_b, n, k, transpose_b, np, kp, bp);
    GemmArgs g = gemm_args(pad_a ? (const void *)ap : d_a, kp, 0, bp, n, kp, m, nullptr, d_out, n);
    g.epi.bias = d_bias;
    g.epi.shift = dst_exp - src_exp;
    g.epi.bits_wide = needs_wide(hb.data(), n, k);
    g.epi.fast = gemm_epi_fast(epi, g.epi);
    cudaError_t e;
    if (persistent) {
        CUtensorMap tm;
        if (make_tmap_a(&tm, d_a, k, m) != 0) {
            rc = fail(HV_ERR_CUDA, "cannot encode the tensor map of A");
            e = cudaSuccess;
        } else {
            g.tma = &tm;
            e = launch_gemm_persistent(g, EPI_I8, m, err, sms, st);
        }
    } else {
        e = launch_gemm(g, epi, a_unsigned, m, err, st);
    }
    if (!rc && e != cudaSuccess) rc = fail(HV_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
    cudaStreamSynchronize(st);
    int code = 0;
    cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (!rc && code) rc = fail(HV_ERR_STATE, "a device-side bounded wait gave up (code %d)", code);
    cudaFree(ap);
    cudaFree(bp);
    cudaFree(err);
    return rc;
}

int hv_writeback_i64(const int64_t *d_acc, int64_t count, int src_exp, int dst_exp, int out_bits, void *d_out,
                     void *stream) {
    if (out_bits != 8 && out_bits != 24 && out_bits != 32) return fail(HV_ERR_VALUE, "output_bits must be 8 or 32");
    if (count < 0) return fail(HV_ERR_VALUE, "negative count");
    CUDA_TRY(launch_writeback(d_acc, count, dst_exp - src_exp, out_bits, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_align_add_i8(const int8_t *d_a, int a_exp, const int8_t *d_b, int b_exp, int out_exp, int64_t count,
                    int8_t *d_out, void *stream) {
    if (count < 0) return fail(HV_ERR_VALUE, "negative count");
    if (!align_ok(a_exp, b_exp, out_exp)) return fail(HV_ERR_VALUE, "align-add exponent gap above 54 is not supported");
    CUDA_TRY(launch_align_add(d_a, d_b, make_align_add(a_exp, b_exp, out_exp), count, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_quantize_images(const float *d_images, int batch, int input_exp, int8_t *d_out, void *stream) {
    if (batch < 0) return fail(HV_ERR_VALUE, "negative batch");
    if (input_exp < -100 || input_exp > 100) return fail(HV_ERR_VALUE, "input exponent outside [-100, 100]");
    if (batch && (!d_images || !d_out)) return fail(HV_ERR_VALUE, "null buffer");
    if (((uintptr_t)d_images & 3) || ((uintptr_t)d_out & 3))
        return fail(HV_ERR_VALUE, "image buffers must be 4-byte aligned");
    CUDA_TRY(launch_quantize_images(d_images, batch, input_exp, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_layernorm_i8(const int8_t *d_x, const int8_t *d_gamma, const int8_t *d_beta, int rows, int x_scale,
                    int gamma_scale, int beta_scale, int out_scale, int8_t *d_out, uint8_t *d_negvar, void *stream) {
    if (x_scale < -32 || x_scale > 0) return fail(HV_ERR_VALUE, "layernorm input scale must be in [-32, 0]");
    if (rows < 0) return fail(HV_ERR_VALUE, "negative row count");
    const int common = std::min(gamma_scale - 16, beta_scale);
    if (gamma_scale - 16 - common > 100 || beta_scale - common > 100)
        return fail(HV_ERR_VALUE, "gamma/beta exponent gap above 100 is not supported");
    LnParams p = make_ln(d_gamma, d_beta, x_scale, gamma_scale, beta_scale, out_scale);
    CUDA_TRY(launch_layernorm(d_x, d_out, rows, nullptr, p, d_negvar, nullptr, 0, nullptr, (cudaStream_t)stream));
    return HV_OK;
}

int hv_softmax_rows(const int32_t *d_x, const int32_t *d_row_offsets, int rows, int mode, void *d_out, void *stream) {
    if (mode != 0 && mode != 1) return fail(HV_ERR_VALUE, "mode must be 0 (attention) or 1 (selector)");
    CUDA_TRY(launch_softmax_rows(d_x, d_row_offsets, rows, mode, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_shiftgelu(const int32_t *d_x, int64_t count, int32_t *d_out, void *stream) {
    CUDA_TRY(launch_gelu(d_x, count, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_plan_sigmoid(const int32_t *d_x, int64_t count, int32_t *d_out, void *stream) {
    CUDA_TRY(launch_plan(d_x, count, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_gelu_requant(const int32_t *d_acc, int64_t count, int src_exp, int dst_exp, int8_t *d_out, void *stream) {
    CUDA_TRY(launch_gelu_requant(d_acc, count, -16 - src_exp, dst_exp + 16, d_out, (cudaStream_t)stream));
    return HV_OK;
}

int hv_transformer_block(hv_model *m, int block_index, const int8_t *d_x, const int32_t *d_offsets, int images,
                         int total_rows, int8_t *d_z, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (block_index < 0 || block_index >= HV_BLOCKS) return fail(HV_ERR_VALUE, "block index out of range");
    if (!m->has_block[block_index]) return fail(HV_ERR_STATE, "model has no block %d", block_index + 1);
    if (images <= 0 || total_rows < 0 || total_rows > images * HV_TOKENS)
        return fail(HV_ERR_VALUE, "bad ragged batch (each image holds at most 197 tokens)");
    CUDA_TRY(cudaSetDevice(m->device));
    int rc = ensure_capacity(m, images);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemcpyAsync(m->X, d_x, (size_t)total_rows * 192, cudaMemcpyDeviceToDevice, st));
    CUDA_TRY(cudaMemsetAsync(m->warn, 0, ((size_t)images + 3) & ~(size_t)3, st));
    CUDA_TRY(launch_attn_plan(d_offsets, images, m->plan, st));
    rc = run_block(m, block_index, images, d_offsets, 1, st);
    if (rc) return rc;
    CUDA_TRY(cudaMemcpyAsync(d_z, m->X, (size_t)total_rows * 192, cudaMemcpyDeviceToDevice, st));
    return HV_OK;
}

int hv_patch_embedding(hv_model *m, const int8_t *d_images, int batch, int8_t *d_tokens, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (batch <= 0) return fail(HV_ERR_VALUE, "batch must be positive");
    if (!m->has_patch) return fail(HV_ERR_STATE, "model has no patch embedding");
    CUDA_TRY(cudaSetDevice(m->device));
    int rc = ensure_capacity(m, batch);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(launch_pdl(init_batch_kernel, dim3(std::min(148 * 4, (batch * 12 + 255) / 256 + 1)), dim3(256), 0, st, 
        batch, m->off[0], m->pkg[0], m->warn, nullptr, 0, d_tokens, m->w<int8_t>(m->cls_row), m->plan));
    CUDA_TRY(cudaGetLastError());
    return run_patch(m, d_images, batch, d_tokens, st);
}

int hv_token_selector(hv_model *m, int selector_index, const int8_t *d_x, const int32_t *d_offsets,
                      const uint8_t *d_pkg_in, int images, int8_t *d_y, int32_t *d_offsets_out, uint8_t *d_pkg_out,
                      hv_selector_summary *d_summary, int32_t *d_fused, int32_t *d_head_scores,
                      int32_t *d_head_weights, int8_t *d_local, int8_t *d_global, int8_t *d_stats, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (selector_index < 0 || selector_index >= m->num_sel) return fail(HV_ERR_VALUE, "selector index out of range");
    if (images <= 0) return fail(HV_ERR_VALUE, "images must be positive");
    CUDA_TRY(cudaSetDevice(m->device));
    int rc = ensure_capacity(m, images);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemsetAsync(m->warn, 0, ((size_t)images + 3) & ~(size_t)3, st));
    SelDebug dbg{d_fused, d_head_scores, d_head_weights, d_local, d_global, d_stats, nullptr};
    SelParams sp = bind_sel(m, m->sels[selector_index]);
    CUDA_TRY(launch_selector(d_x, d_offsets, d_pkg_in, images, sp, m->STAGE, m->counts, d_pkg_out, d_summary, 1,
                             m->warn, nullptr, 0, 0, &dbg, st));
    CUDA_TRY(launch_pack(m->STAGE, m->counts, images, d_y, d_offsets_out, nullptr, st));
    return HV_OK;
}

int hv_selector_h2(hv_model *m, int selector_index, const int8_t *d_x, const int32_t *d_offsets, int images,
                   int8_t *d_h2, void *stream) {
    if (!m) return fail(HV_ERR_VALUE, "null model");
    HOST_IDLE(m);
    if (!m || !d_x || !d_offsets || !d_h2) return fail(HV_ERR_VALUE, "null argument");
    if (selector_index < 0 || selector_index >= m->num_sel) return fail(HV_ERR_VALUE, "selector index out of range");
    if (images <= 0) return fail(HV_ERR_VALUE, "images must be positive");
    CUDA_TRY(cudaSetDevice(m->device));
    int rc = ensure_capacity(m, images);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    CUDA_TRY(cudaMemsetAsync(m->warn, 0, ((size_t)images + 3) & ~(size_t)3, st));
    SelDebug dbg{nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, d_h2};
    SelParams sp = bind_sel(m, m->sels[selector_index]);
    CUDA_TRY(launch_selector(d_x, d_offsets, nullptr, images, sp, m->STAGE, m->counts, nullptr, nullptr, 1, m->warn,
                             nullptr, 0, 0, &dbg, st));
    return HV_OK;
}

}  // extern "C"

// ---- allocation-free accumulator GEMM ------------------------------------------------
// hv_gemm_i8_acc_noalloc has no counterpart in the reference.  It serves callers that
// must not call the device allocator mid-run: a process whose device memory is handed
// out up front to a caching pool (a raw cudaMalloc can fail with memory free inside
// the pool), or a latency-bound caller sharing the device with in-flight work, where
// cudaFree's implicit device-wide synchronisation would stall everything.  It does the
// work of hv_gemm_i8_acc with the padded operands and the error word placed in a fixed
// __device__ array (one instance per device context) instead of cudaMalloc'd buffers.
#include <mutex>

static __device__ __align__(256) uint8_t g_noalloc_scratch[HV_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_base[kNoallocDevices];

// Device address of g_noalloc_scratch on the current device, resolved once per
// device with that device current and cached afterwards.
int noalloc_scratch(uint8_t **base) {
    int dev = -1;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoallocDevices)
        return fail(HV_ERR_VALUE, "device %d is beyond the %d devices the allocation-free GEMM tracks", dev,
                    kNoallocDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_base[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(HV_ERR_CUDA, "cudaGetSymbolAddress of the GEMM scratch on device %d: %s", dev,
                        cudaGetErrorString(e));
        g_noalloc_base[dev] = (uint8_t *)p;
    }
    *base = g_noalloc_base[dev];
    return HV_OK;
}

}  // namespace

extern "C" int hv_gemm_i8_acc_noalloc(const void *d_a, const int8_t *d_b, const int32_t *d_bias, int m, int n,
                                      int k, int transpose_b, int a_unsigned, int64_t *d_acc, void *stream) {
    if (m < 0 || n < 0 || k < 0) return fail(HV_ERR_VALUE, "negative dimension");
    if (m == 0 || n == 0) return HV_OK;
    if (!d_a || !d_b || !d_acc) return fail(HV_ERR_VALUE, "null buffer");
    if (k > (a_unsigned ? 65793 : 131071))
        return fail(HV_ERR_VALUE, "k=%d can overflow the int32 accumulator; not supported", k);
    const int tn = gemm_tile_n(n);
    const int64_t kp = std::max(64, (k + 63) / 64 * 64), np = ((int64_t)n + tn - 1) / tn * tn;
    const int64_t a_bytes = ((int64_t)m * kp + 255) / 256 * 256;
    const int64_t need = 256 + a_bytes + np * kp;
    if (need > (int64_t)HV_NOALLOC_SCRATCH_BYTES)
        return fail(HV_ERR_VALUE,
                    "m=%d n=%d k=%d needs %lld bytes of scratch; the allocation-free GEMM holds at most %u "
                    "(HV_NOALLOC_SCRATCH_BYTES); use hv_gemm_i8_acc",
                    m, n, k, (long long)need, (unsigned)HV_NOALLOC_SCRATCH_BYTES);
    uint8_t *base = nullptr;
    int rc = noalloc_scratch(&base);
    if (rc) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    int *err = (int *)base;                        // bounded-wait status: must start at zero
    uint8_t *ap = base + 256;                      // [m][kp], fully rewritten by pad_a_kernel
    int8_t *bp = (int8_t *)(base + 256 + a_bytes); // [np][kp], fully rewritten by pad_b_kernel
    CUDA_TRY(cudaMemsetAsync(err, 0, sizeof(int), st));
    pad_a_kernel<<<148 * 4, 256, 0, st>>>((const uint8_t *)d_a, m, k, (int)kp, ap);
    pad_b_kernel<<<148 * 4, 256, 0, st>>>(d_b, n, k, transpose_b, (int)np, (int)kp, bp);
    CUDA_TRY(cudaGetLastError());
    GemmArgs g = gemm_args(ap, (int)kp, 0, bp, n, (int)kp, m, nullptr, d_acc, n);
    g.epi.bias = d_bias;
    g.epi.bits_wide = 1;
    cudaError_t e = launch_gemm(g, EPI_ACC64, a_unsigned, m, err, st);
    if (e != cudaSuccess) return fail(HV_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
    int code = 0;
    CUDA_TRY(cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, st));
    CUDA_TRY(cudaStreamSynchronize(st));
    if (code) return fail(HV_ERR_STATE, "a device-side bounded wait gave up (code %d)", code);
    return HV_OK;
}
