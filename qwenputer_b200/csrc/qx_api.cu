// qx_api.cu -- the C ABI of include/qx.h: plan validation, device buffers, launches.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <new>
#include <thread>
#include <vector>

#include "qx.h"
#include "qx_exec.cuh"

template <int RUN, int QH, int TC, int R>
__global__ void qx_token_kernel(const __grid_constant__ QxDev d, int32_t n_tokens, int32_t *tokens);
// the token kernel instantiation for the plan: run or step mode, query rows per read (2 or 4),
// tensor-core form phases or none, record slots a warp (32 / machines a CTA)
template <int RUN, int R>
void *token_kernel_qh(const QxDev &d) {
    return d.qhot_max <= 2 ? reinterpret_cast<void *>(qx_token_kernel<RUN, 2, 0, R>)
                           : reinterpret_cast<void *>(qx_token_kernel<RUN, 4, 0, R>);
}
template <int RUN>
void *token_kernel_for(const QxDev &d) {
    if (d.has_mma)
        return d.qhot_max <= 2 ? reinterpret_cast<void *>(qx_token_kernel<RUN, 2, 1, 1>)
                               : reinterpret_cast<void *>(qx_token_kernel<RUN, 4, 1, 1>);
    switch (d.group) {
    case 16: return token_kernel_qh<RUN, 2>(d);
    case 8: return token_kernel_qh<RUN, 4>(d);
    case 4: return token_kernel_qh<RUN, 8>(d);
    default: return token_kernel_qh<RUN, 1>(d);
    }
}
// CTAs of one token-kernel launch: a CTA (or a cluster of d.cluster CTAs) per group of machines
unsigned token_ctas(int B, const QxDev &d) {
    return (unsigned)((B + d.group - 1) / d.group) * (unsigned)d.cluster;
}
__global__ void qx_embed_kernel(const __grid_constant__ QxDev d, int32_t row0, int32_t n, const int32_t *tok);
__global__ void qx_predecode_kernel(const QxImage *img, uint32_t *pool, int32_t n);
__global__ void qx_load_kernel(const __grid_constant__ QxDev d, const QxImage *img, const uint32_t *pool,
                               int32_t row0, int32_t n);
__global__ void qx_load_cover_kernel(const __grid_constant__ QxDev d, uint8_t *cover);
__global__ void qx_readback_kernel(const __grid_constant__ QxDev d, int32_t row0, int32_t n, qx_state *out);
__global__ void qx_checksum_kernel(const qx_state *st, int32_t n, uint64_t *out);
__global__ void qx_reset_kernel(float *H, uint32_t ne, uint32_t bpad, int32_t row0, int32_t n);
cudaError_t qx_gdn_launch(int64_t BH, float *S, const float *q, const float *k, const float *v, const float *alpha,
                          const float *beta, float *o, uint32_t *work, cudaStream_t st);
cudaError_t qx_gdn_prepare();
cudaError_t qx_gdn_prepare_current();
cudaError_t qx_gdn_noalloc_scratch(uint32_t **out);

namespace {

thread_local char g_err[512] = "";

qx_status fail(qx_status s, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return s;
}

#define CU(call)                                                                                  \
    do {                                                                                          \
        cudaError_t e_ = (call);                                                                  \
        if (e_ != cudaSuccess) return fail(QX_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

}  // namespace

struct qx_executor {
    int device = 0, B = 0, Bpad = 0;
    qx_plan_header hdr{};
    std::vector<uint8_t> host_plan;
    void *dplan = nullptr;
    QxDev d{};
    int n_hl = 0;
    size_t smem = 0;
    int max_clusters = 0;         // clusters of the token kernel that fit on the device at once
    int32_t *dtok = nullptr;      // [B] scratch for qx_set_tokens
    qx_state *dstate = nullptr;   // readback staging
    int32_t state_cap = 0;
    uint32_t *err_host = nullptr;
    std::vector<void *> allocs;
    // machine-image upload staging (qx_load_machines), two of each so that packing the next
    // chunk on the host overlaps the copy and the loader kernels of the previous one
    void *pin[2] = {nullptr, nullptr};
    void *dstage[2] = {nullptr, nullptr};
    size_t stage_bytes = 0;
    cudaEvent_t staged[2] = {nullptr, nullptr};
    // the image copies run on their own stream, so that chunk k+1 crosses PCIe while the loader
    // kernels build chunk k
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t copied[2] = {nullptr, nullptr};
    // shared read-only tables (qx_set_table_images): the content of each image slot in use
    int table_slots = 0;
    std::vector<std::vector<uint32_t>> slot_rom;
    std::vector<std::vector<uint8_t>> slot_drom;
    ~qx_executor() {
        for (void *p : allocs) cudaFree(p);
        if (dplan) cudaFree(dplan);
        if (err_host) cudaFreeHost(err_host);
        if (dstate) cudaFree(dstate);
        for (int i = 0; i < 2; i++) {
            if (pin[i]) cudaFreeHost(pin[i]);
            if (dstage[i]) cudaFree(dstage[i]);
            if (staged[i]) cudaEventDestroy(staged[i]);
            if (copied[i]) cudaEventDestroy(copied[i]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
    }
};

namespace {

// One launch of the token kernel: a CTA per group of machines, or a cluster of d.cluster CTAs
// per group of 32 (launched with the cluster-dimension attribute).
template <int RUN>
cudaError_t launch_token(const qx_t *ex, const QxDev &d, int32_t n_tokens, int32_t *tokens, cudaStream_t st) {
    const int C = d.cluster;
    const unsigned grid = token_ctas(ex->B, d);
    void *args[] = {const_cast<QxDev *>(&d), &n_tokens, &tokens};
    if (C == 1) return cudaLaunchKernel(token_kernel_for<RUN>(d), dim3(grid), dim3(QX_NT), args, ex->smem, st);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(QX_NT);
    cfg.dynamicSmemBytes = ex->smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)C;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, token_kernel_for<RUN>(d), args);
}

qx_status dev_alloc(qx_t *ex, void **p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(e == cudaErrorMemoryAllocation ? QX_ERR_OOM : QX_ERR_CUDA, "cudaMalloc(%zu): %s", bytes,
                    cudaGetErrorString(e));
    }
    ex->allocs.push_back(*p);
    return QX_OK;
}

template <class T>
const T *sec(const qx_executor *ex, int s) {
    return reinterpret_cast<const T *>(static_cast<const uint8_t *>(ex->dplan) + ex->hdr.off[s]);
}

struct SecSpec {
    int id;
    size_t elem;
};

qx_status validate(const qx_plan_header &h, size_t bytes) {
    if (bytes < sizeof(qx_plan_header)) return fail(QX_ERR_INVALID_PLAN, "plan shorter than its header");
    if (h.magic != QX_PLAN_MAGIC) return fail(QX_ERR_INVALID_PLAN, "bad plan magic");
    if (h.version != QX_PLAN_VERSION)
        return fail(QX_ERR_INVALID_PLAN, "plan version %u, expected %d", h.version, QX_PLAN_VERSION);
    if (h.qhot_max > 4) return fail(QX_ERR_INVALID_PLAN, "queries read at most 4 rows");
    if (h.nw != QX_NW) return fail(QX_ERR_INVALID_PLAN, "plan balanced for %u warps, kernel has %d", h.nw, QX_NW);
    if (h.cluster < 1 || h.cluster > 8) return fail(QX_ERR_INVALID_PLAN, "cluster of %u CTAs (1 to 8)", h.cluster);
    if (h.group != 32 && h.group != 16 && h.group != 8 && h.group != 4)
        return fail(QX_ERR_INVALID_PLAN, "groups of %u machines (32, 16, 8 or 4)", h.group);
    if (h.group != 32 && (h.cluster != 1 || (h.flags & QX_PLAN_FLAG_MMA)))
        return fail(QX_ERR_INVALID_PLAN, "a group of %u machines runs on one CTA, without tensor-core phases", h.group);
    if ((h.flags & QX_PLAN_FLAG_DIRECT_OUT) && h.cluster != 1)
        return fail(QX_ERR_INVALID_PLAN, "direct value-head outputs need one CTA a group");
    if (h.table_bytes % 16 || h.table_bytes > 65536 || (h.group == 32 && h.table_bytes))
        return fail(QX_ERR_INVALID_PLAN, "plan-table area of %u bytes", h.table_bytes);
    if (h.n_head_levels > QX_MAX_HL) return fail(QX_ERR_INVALID_PLAN, "too many head sublayers");
    if (h.n_pay > 16 || h.n_fam > 16) return fail(QX_ERR_INVALID_PLAN, "output code too wide");
    if (h.n_born0 > h.n_feat) return fail(QX_ERR_INVALID_PLAN, "embedding dims mismatch");
    const SecSpec specs[] = {
        {QX_S_RUN_PROG, sizeof(qx_phase)}, {QX_S_STEP_PROG, sizeof(qx_phase)}, {QX_S_ROWS, 4},
        {QX_S_PAIRS, 8}, {QX_S_STREAM, 16}, {QX_S_VHSUM_ROWS, 4}, {QX_S_WARP_PTR, 4},
        {QX_S_STAGES, sizeof(qx_stage)}, {QX_S_VHEADS, sizeof(qx_vhead)},
        {QX_S_VFORM, sizeof(qx_colform)}, {QX_S_ZFORM, sizeof(qx_colform)}, {QX_S_OUT_ROW, 4}, {QX_S_OUT_W, 4},
        {QX_S_HL_V, 4}, {QX_S_HL_NE, 4}, {QX_S_FAM_ROW, 4}, {QX_S_PAY_ROW, 4}, {QX_S_FEAT_ROW, 4},
        {QX_S_FAM_IDS, 4}, {QX_S_FAM_SIZE, 4}, {QX_S_FAM_ROW0, 4}, {QX_S_EMB_BASE, 4}, {QX_S_EMB_BITS, 4},
        {QX_S_EMB_TABLE, 4}, {QX_S_TABLES, 4}, {QX_S_REG_COLS, 4},
        {QX_S_FAM_TOUCH_PTR, 4}, {QX_S_FAM_TOUCH, 4}, {QX_S_MMA_PHASES, sizeof(qx_mma_phase)},
        {QX_S_MMA_TILES, sizeof(qx_mma_tile)}, {QX_S_TILEDATA, 2}, {QX_S_FEAT_DIM, 4}, {QX_S_CODE_ROW, 4},
        {QX_S_TEXT_WORDS, 4}, {QX_S_TEXT_BASE, 4}, {QX_S_TEXT_BITS, 4}, {QX_S_PRINTABLE, 4},
        {QX_S_TEXT_TOUCH, 4}, {QX_S_MERGED_INFO, 4}};
    for (const SecSpec &s : specs) {
        if (h.off[s.id] % 16 || h.off[s.id] + h.cnt[s.id] * s.elem > bytes)
            return fail(QX_ERR_INVALID_PLAN, "section %d out of bounds", s.id);
    }
    if (h.cnt[QX_S_FAM_TOUCH_PTR] != (uint64_t)h.n_families + 1)
        return fail(QX_ERR_INVALID_PLAN, "touched-feature offsets missing");
    if (h.cnt[QX_S_TABLES] != 198 || h.cnt[QX_S_REG_COLS] != 256)
        return fail(QX_ERR_INVALID_PLAN, "snapshot tables missing");
    if (h.cnt[QX_S_FEAT_DIM] != h.n_feat || h.cnt[QX_S_MERGED_INFO] != 8)
        return fail(QX_ERR_INVALID_PLAN, "feature dims or merged-readout facts missing");
    if (h.cnt[QX_S_HL_V] != h.n_head_levels || h.cnt[QX_S_FEAT_ROW] != h.n_feat ||
        h.cnt[QX_S_FAM_ROW] < h.n_fam || h.cnt[QX_S_PAY_ROW] < h.n_pay)
        return fail(QX_ERR_INVALID_PLAN, "section counts disagree with the header");
    return QX_OK;
}

// The pieces of one stream phase's warp ranges: each a header line and n body lines of 32 / group
// quads inside one ring chunk; every slot of a line agrees on n, on the first / last flags and on
// R_SPLIT (which only form phases of bundled plans use, and which the whole warp then takes);
// every row a header names lies inside the rows (the zero row included).
bool stream_ranges_ok(const qx_plan_header &h, const uint8_t *plan, uint32_t kind, const uint32_t *wp) {
    const uint4 *st = reinterpret_cast<const uint4 *>(plan + h.off[QX_S_STREAM]);
    const uint32_t R = 32 / h.group, chunk = QX_RING_QUADS * R;
    const uint64_t rows_end = (uint64_t)(h.n_slots + h.n_scratch + 1) * (h.group + 1) * 4;
    for (uint32_t w = 0; w < h.nw * h.cluster; w++) {
        const uint32_t start = wp[w], end = wp[w + 1];
        uint32_t i = start;
        while (i < end) {
            const uint32_t fl = st[i].w >> 24, n = st[i].w & 0xFFFFFFu;
            if (fl & QX_R_SKIP) {
                i = start + ((i - start) / chunk + 1) * chunk;
                continue;
            }
            if (n + 1 > (uint32_t)QX_RING_QUADS || (i - start) / chunk != (i - start + R * (n + 1) - 1) / chunk ||
                i + R * (n + 1) > end)
                return false;
            if ((fl & QX_R_SPLIT) && (kind != QX_PH_FORMS || R == 1)) return false;
            const uint32_t nc = st[i].y;  // (units: the piece's constant-gate quads)
            for (uint32_t k = 0; k < R; k++) {
                const uint4 hk = st[i + k];
                if ((hk.w & 0xFFFFFFu) != n || ((hk.w >> 24) ^ fl) & (QX_R_FIRST | QX_R_LAST | QX_R_SPLIT | QX_R_SKIP))
                    return false;
                if (kind == QX_PH_FORMS && (hk.x >= rows_end || hk.y >= rows_end)) return false;
                if (kind == QX_PH_UNITS && (hk.x >= rows_end || hk.y != nc || nc > n || (n - nc) % 2)) return false;
                if (kind == QX_PH_KSEL &&
                    ((hk.x & 0xFFFFu) >= h.n_ksel_slots || hk.y >= rows_end || hk.z >= rows_end))
                    return false;
            }
            for (uint32_t j = 0; j < n; j++) {
                for (uint32_t k = 0; k < R; k++) {
                    const uint4 b = st[i + R * (1 + j) + k];
                    const bool second = kind == QX_PH_UNITS && j >= nc && (j - nc) % 2;  // a unit's constants
                    if (!second && b.x >= rows_end) return false;
                    if (kind == QX_PH_FORMS && b.z >= rows_end) return false;
                    if (kind == QX_PH_UNITS && j >= nc && !second && b.y >= rows_end) return false;
                }
            }
            i += R * (n + 1);
        }
    }
    return true;
}

// every snapshot table names head state, every program ends, and every value-head phase names at most QX_VH_CHUNK heads of the section
qx_status validate_programs(const qx_plan_header &h, const uint8_t *plan) {
    {
        // every snapshot table names a head sublayer and value heads inside it (tables 0-6, the
        // counter and register heads, use their first value head; the rest use two)
        const uint32_t *tab = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_TABLES]);
        const uint32_t *hlv = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_HL_V]);
        for (int t = 0; t < 99; t++) {
            const uint32_t hl = tab[2 * t], vh0 = tab[2 * t + 1], need = t < 7 ? 1 : 2;
            if (hl >= h.n_head_levels || hl >= QX_MAX_HL || vh0 > hlv[hl] || hlv[hl] - vh0 < need)
                return fail(QX_ERR_INVALID_PLAN, "snapshot table %d names no head state", t);
        }
    }
    for (int id : {QX_S_RUN_PROG, QX_S_STEP_PROG}) {
        const qx_phase *p = reinterpret_cast<const qx_phase *>(plan + h.off[id]);
        bool ended = false;
        for (uint64_t i = 0; i < h.cnt[id] && !ended; i++) {
            const uint32_t kind = p[i].kind & 0xFFu;
            if (kind > QX_PH_MMA) return fail(QX_ERR_INVALID_PLAN, "unknown phase kind %u", kind);
            if (kind == QX_PH_MMA) {
                if (!(h.flags & QX_PLAN_FLAG_MMA) || p[i].a >= h.cnt[QX_S_MMA_PHASES])
                    return fail(QX_ERR_INVALID_PLAN, "tensor-core phase %u names no phase record", p[i].a);
                if (p[i].kind & QX_PH_NOSYNC)
                    return fail(QX_ERR_INVALID_PLAN, "a tensor-core phase ends with a barrier");
            }
            ended = kind == QX_PH_END;
            if ((kind == QX_PH_FORMS || kind == QX_PH_UNITS || kind == QX_PH_KSEL) &&
                (uint64_t)p[i].c + (uint64_t)h.nw * h.cluster >= h.cnt[QX_S_WARP_PTR])
                return fail(QX_ERR_INVALID_PLAN, "stream phase %llu: warp ranges beyond the section",
                            (unsigned long long)i);
            if (kind == QX_PH_FORMS || kind == QX_PH_UNITS || kind == QX_PH_KSEL) {
                // every warp range inside the stream, in whole lines of 32 / group quads
                const uint32_t *wp = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_WARP_PTR]);
                const uint32_t ways = 32 / h.group;
                for (uint32_t w = 0; w <= h.nw * h.cluster; w++) {
                    const uint32_t v = wp[p[i].c + w];
                    if (v > h.cnt[QX_S_STREAM] || v % ways || (w && v < wp[p[i].c + w - 1]))
                        return fail(QX_ERR_INVALID_PLAN, "stream phase %llu: a warp range outside the stream",
                                    (unsigned long long)i);
                }
                if (!stream_ranges_ok(h, plan, kind, wp + p[i].c))
                    return fail(QX_ERR_INVALID_PLAN, "stream phase %llu: a malformed piece", (unsigned long long)i);
            }
            if ((kind == QX_PH_VH || kind == QX_PH_VHRUN) &&
                (p[i].b < p[i].a || p[i].b - p[i].a > QX_VH_CHUNK || p[i].b > h.cnt[QX_S_VHEADS] ||
                 p[i].c > QX_DELTA_ROWS || (size_t)(p[i].b - p[i].a) * h.group * 8 > QX_RING_BYTES))
                return fail(QX_ERR_INVALID_PLAN, "value-head phase [%u, %u) with %u delta rows exceeds its buffers",
                            p[i].a, p[i].b, p[i].c);
            if (kind == QX_PH_VHSUM && (p[i].b > QX_DELTA_ROWS || (uint64_t)p[i].a + p[i].b > h.cnt[QX_S_VHSUM_ROWS]))
                return fail(QX_ERR_INVALID_PLAN, "delta-sum phase beyond its rows");
        }
        if (!ended) return fail(QX_ERR_INVALID_PLAN, "program without an END phase");
    }
    if (h.flags & QX_PLAN_FLAG_MMA) {
        // tensor-core phases: source and destination rows inside the rows (plus the zero row),
        // K and form blocks within the staging area and the accumulator columns, every tile's
        // data and blocks inside its phase
        const qx_mma_phase *mp = reinterpret_cast<const qx_mma_phase *>(plan + h.off[QX_S_MMA_PHASES]);
        const qx_mma_tile *mt = reinterpret_cast<const qx_mma_tile *>(plan + h.off[QX_S_MMA_TILES]);
        const uint32_t *rows = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_ROWS]);
        const uint64_t zero_row = (uint64_t)(h.n_slots + h.n_scratch) * QX_RP * 4;  // (groups of 32)
        const uint64_t n_tiles = h.cnt[QX_S_TILEDATA] / (128 * 16);
        for (uint64_t i = 0; i < h.cnt[QX_S_MMA_PHASES]; i++) {
            const qx_mma_phase &m = mp[i];
            if (m.n_kb < 1 || m.n_kb > QX_MMA_MAX_KB || m.n_fb < 1 || m.n_fb > QX_MMA_MAX_FB ||
                (uint64_t)m.kr0 + 16ull * m.n_kb > h.cnt[QX_S_ROWS] ||
                (uint64_t)m.dst0 + 128ull * m.n_fb > h.cnt[QX_S_ROWS] || m.t0 > m.t1 ||
                m.t1 > h.cnt[QX_S_MMA_TILES])
                return fail(QX_ERR_INVALID_PLAN, "tensor-core phase %llu out of bounds", (unsigned long long)i);
            for (uint32_t r = 0; r < 16 * m.n_kb; r++)
                if (rows[m.kr0 + r] > zero_row || rows[m.kr0 + r] % (QX_RP * 4))
                    return fail(QX_ERR_INVALID_PLAN, "tensor-core phase %llu: a source row outside the rows",
                                (unsigned long long)i);
            for (uint32_t r = 0; r < 128 * m.n_fb; r++)
                if (rows[m.dst0 + r] != QX_NONE32 && (rows[m.dst0 + r] >= zero_row || rows[m.dst0 + r] % (QX_RP * 4)))
                    return fail(QX_ERR_INVALID_PLAN, "tensor-core phase %llu: a destination outside the rows",
                                (unsigned long long)i);
            for (uint32_t t = m.t0; t < m.t1; t++)
                if (mt[t].data >= n_tiles || mt[t].fb >= m.n_fb || mt[t].kb >= m.n_kb)
                    return fail(QX_ERR_INVALID_PLAN, "tensor-core tile %u out of bounds", t);
        }
    }
    {
        // features: rows inside the rows, deferred ones naming dims below D; merged readout:
        // code rows inside the rows, the text tables' sizes, printable tokens inside the vocabulary
        const uint32_t *fr = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_FEAT_ROW]);
        const uint32_t *fd = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_FEAT_DIM]);
        const uint64_t zero_row = (uint64_t)(h.n_slots + h.n_scratch) * (h.group + 1) * 4;
        for (uint32_t f = 0; f < h.n_feat; f++) {
            if (fd[f] >= h.D) return fail(QX_ERR_INVALID_PLAN, "feature %u names no dim", f);
            if (fr[f] & QX_FEAT_DEFERRED ? (fr[f] & ~QX_FEAT_DEFERRED) != fd[f] : fr[f] >= zero_row)
                return fail(QX_ERR_INVALID_PLAN, "feature %u: row out of range", f);
        }
        const uint32_t *mi = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_MERGED_INFO]);
        if (h.flags & QX_PLAN_FLAG_MERGED) {
            const uint32_t q_fid = mi[0], n_text = mi[1], n_pr = mi[2], n_touch = mi[3], n_code = mi[4],
                           n_bits = mi[5];
            if (n_code < 1 || n_code > 32 || n_code <= 16 || h.cnt[QX_S_CODE_ROW] < n_code || n_bits != 152 ||
                h.cnt[QX_S_TEXT_WORDS] != 5ull * n_text || h.cnt[QX_S_TEXT_BASE] != h.n_feat ||
                h.cnt[QX_S_TEXT_BITS] != (uint64_t)n_bits * h.n_feat || h.cnt[QX_S_PRINTABLE] < n_pr ||
                h.cnt[QX_S_TEXT_TOUCH] < n_touch || n_text < 1 || n_pr < 1 || q_fid >= 32)
                return fail(QX_ERR_INVALID_PLAN, "merged readout tables inconsistent");
            const uint32_t *cr = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_CODE_ROW]);
            for (uint32_t i = 0; i < n_code; i++)
                if (cr[i] >= zero_row) return fail(QX_ERR_INVALID_PLAN, "code row out of range");
            const int32_t *pr = reinterpret_cast<const int32_t *>(plan + h.off[QX_S_PRINTABLE]);
            for (uint32_t i = 0; i < n_pr; i++)
                if (pr[i] < 0 || (uint32_t)pr[i] >= n_text) return fail(QX_ERR_INVALID_PLAN, "printable token out of range");
            const uint32_t *tt = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_TEXT_TOUCH]);
            for (uint32_t i = 0; i < n_touch; i++)
                if (tt[i] >= h.n_feat) return fail(QX_ERR_INVALID_PLAN, "text feature out of range");
        }
    }
    const uint32_t *tp = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_FAM_TOUCH_PTR]);
    const uint32_t *tf = reinterpret_cast<const uint32_t *>(plan + h.off[QX_S_FAM_TOUCH]);
    for (uint32_t f = 0; f < h.n_families; f++)
        if (tp[f] > tp[f + 1] || tp[f + 1] > h.cnt[QX_S_FAM_TOUCH])
            return fail(QX_ERR_INVALID_PLAN, "touched-feature offsets out of order");
    for (uint32_t i = 0; i < tp[h.n_families]; i++)
        if (tf[i] >= h.n_feat) return fail(QX_ERR_INVALID_PLAN, "touched feature beyond the features");
    return QX_OK;
}

}  // namespace

namespace {

// Runs pack(lo, hi) over [0, n) split into contiguous ranges on up to 8 threads (one copy stream
// into pinned memory does not reach the host's memory bandwidth); serially when n is small or a
// thread cannot be started.
template <class F>
void pack_parallel(int n, const F &pack) {
    const unsigned hw = std::thread::hardware_concurrency();
    const int T = n < 64 ? 1 : (int)std::min(8u, std::max(1u, hw));
    if (T == 1) {
        pack(0, n);
        return;
    }
    std::vector<std::thread> th;
    int done = 0;  // ranges below this index run on threads
    try {
        for (int t = 1; t < T; t++) {
            th.emplace_back([&pack, n, T, t] { pack((int)((int64_t)n * t / T), (int)((int64_t)n * (t + 1) / T)); });
            done = t;
        }
    } catch (...) {
    }
    pack(0, (int)((int64_t)n / T));
    if (done + 1 < T) pack((int)((int64_t)n * (done + 1) / T), n);  // ranges no thread took
    for (std::thread &x : th) x.join();
}

}  // namespace

extern "C" {

const char *qx_last_error(void) { return g_err; }

qx_status qx_create(const void *plan, size_t plan_bytes, int32_t batch, int32_t device, qx_t **out) {
    g_err[0] = 0;
    if (!plan || !out || batch < 1) return fail(QX_ERR_INVALID_ARG, "qx_create: bad arguments");
    *out = nullptr;
    qx_plan_header h;
    if (plan_bytes < sizeof(h)) return fail(QX_ERR_INVALID_PLAN, "plan too short");
    memcpy(&h, plan, sizeof(h));
    qx_status s = validate(h, plan_bytes);
    if (s == QX_OK) s = validate_programs(h, static_cast<const uint8_t *>(plan));
    if (s != QX_OK) return s;
    CU(cudaSetDevice(device));
    qx_executor *ex = new (std::nothrow) qx_executor();
    if (!ex) return fail(QX_ERR_OOM, "host allocation failed");
    ex->device = device;
    ex->hdr = h;
    ex->B = batch;
    ex->Bpad = (batch + 31) / 32 * 32;
    ex->host_plan.assign(static_cast<const uint8_t *>(plan), static_cast<const uint8_t *>(plan) + plan_bytes);
    auto bail = [&](qx_status st) {
        delete ex;
        return st;
    };
    cudaError_t e = cudaMalloc(&ex->dplan, plan_bytes);
    if (e != cudaSuccess) return bail(fail(QX_ERR_OOM, "plan upload: %s", cudaGetErrorString(e)));
    e = cudaMemcpy(ex->dplan, plan, plan_bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return bail(fail(QX_ERR_CUDA, "plan upload: %s", cudaGetErrorString(e)));

    QxDev &d = ex->d;
    d.run_prog = sec<qx_phase>(ex, QX_S_RUN_PROG);
    d.step_prog = sec<qx_phase>(ex, QX_S_STEP_PROG);
    d.rows = sec<uint32_t>(ex, QX_S_ROWS);
    d.pairs = sec<uint2>(ex, QX_S_PAIRS);
    d.stream = sec<uint4>(ex, QX_S_STREAM);
    d.vhsum_rows = sec<uint32_t>(ex, QX_S_VHSUM_ROWS);
    d.warp_ptr = sec<uint32_t>(ex, QX_S_WARP_PTR);
    d.stages = sec<qx_stage>(ex, QX_S_STAGES);
    d.vheads = sec<qx_vhead>(ex, QX_S_VHEADS);
    d.vform = sec<qx_colform>(ex, QX_S_VFORM);
    d.zform = sec<qx_colform>(ex, QX_S_ZFORM);
    d.out_row = sec<uint32_t>(ex, QX_S_OUT_ROW);
    d.out_w = sec<float>(ex, QX_S_OUT_W);
    d.fam_row = sec<uint32_t>(ex, QX_S_FAM_ROW);
    d.pay_row = sec<uint32_t>(ex, QX_S_PAY_ROW);
    d.feat_row = sec<uint32_t>(ex, QX_S_FEAT_ROW);
    d.fam_ids = sec<int32_t>(ex, QX_S_FAM_IDS);
    d.fam_size = sec<int32_t>(ex, QX_S_FAM_SIZE);
    d.fam_row0 = sec<int32_t>(ex, QX_S_FAM_ROW0);
    d.emb_base = sec<float>(ex, QX_S_EMB_BASE);
    d.emb_bits = sec<float>(ex, QX_S_EMB_BITS);
    d.fam_touch_ptr = sec<uint32_t>(ex, QX_S_FAM_TOUCH_PTR);
    d.fam_touch = sec<uint32_t>(ex, QX_S_FAM_TOUCH);
    d.emb_table = sec<float>(ex, QX_S_EMB_TABLE);
    d.tables = sec<uint32_t>(ex, QX_S_TABLES);
    d.reg_cols = sec<int32_t>(ex, QX_S_REG_COLS);
    d.mma_phases = sec<qx_mma_phase>(ex, QX_S_MMA_PHASES);
    d.mma_tiles = sec<qx_mma_tile>(ex, QX_S_MMA_TILES);
    d.tiledata = sec<uint4>(ex, QX_S_TILEDATA);
    d.has_mma = (h.flags & QX_PLAN_FLAG_MMA) ? 1 : 0;
    d.direct_out = (h.flags & QX_PLAN_FLAG_DIRECT_OUT) ? 1 : 0;
    d.feat_dim = sec<uint32_t>(ex, QX_S_FEAT_DIM);
    d.code_row = sec<uint32_t>(ex, QX_S_CODE_ROW);
    d.text_words = sec<uint32_t>(ex, QX_S_TEXT_WORDS);
    d.text_base = sec<float>(ex, QX_S_TEXT_BASE);
    d.text_bits = sec<float>(ex, QX_S_TEXT_BITS);
    d.printable = sec<int32_t>(ex, QX_S_PRINTABLE);
    d.text_touch = sec<uint32_t>(ex, QX_S_TEXT_TOUCH);
    {
        const uint32_t *mi = reinterpret_cast<const uint32_t *>(ex->host_plan.data() + h.off[QX_S_MERGED_INFO]);
        d.merged = (h.flags & QX_PLAN_FLAG_MERGED) ? 1 : 0;
        d.q_fid = (int32_t)mi[0];
        d.n_text = (int32_t)mi[1];
        d.n_printable = (int32_t)mi[2];
        d.n_text_touch = (int32_t)mi[3];
        d.n_code = (int32_t)mi[4];
        d.n_text_bits = (int32_t)mi[5];
    }
    d.B = batch;
    d.Bpad = ex->Bpad;
    d.D = (int32_t)h.D;
    d.smem_rows = (int32_t)(h.n_slots + h.n_scratch);
    d.group = (int32_t)h.group;
    d.n_run_prog = (int32_t)h.cnt[QX_S_RUN_PROG];
    d.n_step_prog = (int32_t)h.cnt[QX_S_STEP_PROG];
    d.n_warp_ptr = (int32_t)h.cnt[QX_S_WARP_PTR];
    {
        // plan tables into the shared-memory table area, in order, while they fit
        d.table_bytes = h.table_bytes;
        const uint64_t words[6] = {(uint64_t)std::max(d.n_run_prog, d.n_step_prog) * (sizeof(qx_phase) / 4),
                                   h.cnt[QX_S_WARP_PTR], h.cnt[QX_S_VHEADS] * (sizeof(qx_vhead) / 4),
                                   h.cnt[QX_S_ROWS], h.cnt[QX_S_VHSUM_ROWS], h.cnt[QX_S_STAGES] * (sizeof(qx_stage) / 4)};
        uint64_t at = 0;
        for (int t = 0; t < 6; t++) {
            const uint64_t bytes = (words[t] * 4 + 15) & ~15ull;
            d.tab_words[t] = (uint32_t)words[t];
            if (d.group < 32 && at + bytes <= d.table_bytes) {
                d.tab_off[t] = (uint32_t)at;
                at += bytes;
            } else {
                d.tab_off[t] = QX_NONE32;
            }
        }
    }
    d.zero_row = (uint32_t)d.smem_rows * (d.group + 1) * 4;
    d.cluster = (int32_t)h.cluster;
    d.one_row = (int32_t)h.one_row;
    d.n_fam = (int32_t)h.n_fam;
    d.n_pay = (int32_t)h.n_pay;
    d.n_feat = (int32_t)h.n_feat;
    d.n_families = (int32_t)h.n_families;
    d.n_emb_rows = (int32_t)h.n_emb_rows;
    d.n_born0 = (int32_t)h.n_born0;
    d.qhot_max = (int32_t)h.qhot_max;
    d.ksel_slots = (int32_t)h.n_ksel_slots;
    d.n_hl = (int32_t)h.n_head_levels;
    {
        // the HALT control token: the family whose first id is the largest below the vocab end is
        // a control; HALT is the sixth control (spec.py:67)
        const int32_t *ids = reinterpret_cast<const int32_t *>(ex->host_plan.data() + h.off[QX_S_FAM_IDS]);
        const int32_t *sz = reinterpret_cast<const int32_t *>(ex->host_plan.data() + h.off[QX_S_FAM_SIZE]);
        int32_t ctrl = -1;
        for (uint32_t f = 0; f < h.n_families; f++)
            if (sz[f] == 1 && (ctrl < 0 || ids[f] < ctrl)) ctrl = ids[f];
        d.halt_tok = ctrl < 0 ? -1 : ctrl + 5;
    }
    ex->n_hl = (int)h.n_head_levels;
    const uint32_t *hlv = reinterpret_cast<const uint32_t *>(ex->host_plan.data() + h.off[QX_S_HL_V]);
    const uint32_t *hne = reinterpret_cast<const uint32_t *>(ex->host_plan.data() + h.off[QX_S_HL_NE]);
    void *p;
    for (int i = 0; i < ex->n_hl; i++) {
        d.V[i] = hlv[i];
        d.NE[i] = hne[i];
        size_t sb = (size_t)batch * hlv[i] * QX_HD * QX_HD * 4;
        if ((s = dev_alloc(ex, &p, sb)) != QX_OK) return bail(s);
        d.S[i] = static_cast<float *>(p);
        if (cudaMemset(p, 0, sb) != cudaSuccess) return bail(fail(QX_ERR_CUDA, "memset S"));
        size_t hb = (size_t)3 * hne[i] * ex->Bpad * 4;
        if ((s = dev_alloc(ex, &p, hb)) != QX_OK) return bail(s);
        d.hist[i] = static_cast<float *>(p);
        if (cudaMemset(p, 0, hb) != cudaSuccess) return bail(fail(QX_ERR_CUDA, "memset hist"));
    }
    size_t xb = (size_t)batch * h.D * 4;
    if ((s = dev_alloc(ex, &p, xb)) != QX_OK) return bail(s);
    d.x = static_cast<float *>(p);
    if ((s = dev_alloc(ex, &p, (size_t)batch * 4)) != QX_OK) return bail(s);
    d.err = static_cast<uint32_t *>(p);
    if ((s = dev_alloc(ex, &p, (size_t)batch * 8)) != QX_OK) return bail(s);
    d.hash = static_cast<uint64_t *>(p);
    if ((s = dev_alloc(ex, &p, (size_t)batch * 8)) != QX_OK) return bail(s);
    d.count = static_cast<int64_t *>(p);
    if ((s = dev_alloc(ex, &p, (size_t)batch * 8)) != QX_OK) return bail(s);
    d.halt_at = static_cast<int64_t *>(p);
    if ((s = dev_alloc(ex, &p, (size_t)batch * 4)) != QX_OK) return bail(s);
    ex->dtok = static_cast<int32_t *>(p);
    if ((s = dev_alloc(ex, &p, 64)) != QX_OK) return bail(s);
    d.state_bytes = static_cast<unsigned long long *>(p);
    {
        const size_t vb = (size_t)token_ctas(batch, d) / d.cluster * 2 * QX_DELTA_ROWS * 32 * 4;
        if ((s = dev_alloc(ex, &p, vb)) != QX_OK) return bail(s);
        d.vdelta = static_cast<float *>(p);
        if (cudaMemset(p, 0, vb) != cudaSuccess) return bail(fail(QX_ERR_CUDA, "delta init"));
    }
    if (cudaMemset(d.state_bytes, 0, 64) != cudaSuccess) return bail(fail(QX_ERR_CUDA, "counter init"));
#ifdef QX_PHASE_CLOCKS
    if ((s = dev_alloc(ex, &p, 256 * 16)) != QX_OK) return bail(s);
    d.phase_clk = static_cast<unsigned long long *>(p);
    if (cudaMemset(p, 0, 256 * 16) != cudaSuccess) return bail(fail(QX_ERR_CUDA, "phase clocks"));
#endif
    if (cudaMemset(d.x, 0, xb) != cudaSuccess || cudaMemset(d.err, 0, (size_t)batch * 4) != cudaSuccess ||
        cudaMemset(d.count, 0, (size_t)batch * 8) != cudaSuccess ||
        cudaMemset(d.halt_at, 0xFF, (size_t)batch * 8) != cudaSuccess ||
        cudaMemset(d.hash, 0, (size_t)batch * 8) != cudaSuccess)
        return bail(fail(QX_ERR_CUDA, "buffer init"));
    {
        // the head-state rows of a machine that no load task writes: qx_load_machines writes zeros
        // there, so that a load leaves every row of the machine's state written once
        size_t rows = 0;
        for (int i = 0; i < ex->n_hl; i++) rows += (size_t)d.V[i] * QX_HD;
        uint8_t *cover = nullptr;
        if (cudaMalloc(&cover, rows) != cudaSuccess) {
            cudaGetLastError();
            return bail(fail(QX_ERR_OOM, "row coverage scratch"));
        }
        std::vector<uint8_t> hc(rows);
        cudaError_t e = cudaMemset(cover, 0, rows);
        if (e == cudaSuccess) {
            qx_load_cover_kernel<<<32, 256>>>(d, cover);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaMemcpy(hc.data(), cover, rows, cudaMemcpyDeviceToHost);
        cudaFree(cover);
        if (e != cudaSuccess) return bail(fail(QX_ERR_CUDA, "row coverage: %s", cudaGetErrorString(e)));
        std::vector<uint32_t> zl;
        size_t base = 0;
        for (int i = 0; i < ex->n_hl; i++) {
            for (uint32_t r = 0; r < d.V[i] * QX_HD; r++)
                if (!hc[base + r]) { zl.push_back((uint32_t)i); zl.push_back(r); }
            base += (size_t)d.V[i] * QX_HD;
        }
        d.n_zero_rows = (int32_t)(zl.size() / 2);
        d.zero_rows = nullptr;
        if (d.n_zero_rows) {
            if ((s = dev_alloc(ex, &p, zl.size() * 4)) != QX_OK) return bail(s);
            if (cudaMemcpy(p, zl.data(), zl.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                return bail(fail(QX_ERR_CUDA, "zero-row list"));
            d.zero_rows = static_cast<const uint2 *>(p);
        }
    }
    if (cudaMallocHost(&ex->err_host, (size_t)batch * 4) != cudaSuccess)
        return bail(fail(QX_ERR_OOM, "pinned error buffer"));
    ex->smem = qx_smem_bytes(d);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if ((int)ex->smem > optin)
        return bail(fail(QX_ERR_INVALID_PLAN, "plan needs %zu B of shared memory per CTA, device has %d", ex->smem,
                         optin));
    if (cudaFuncSetAttribute(token_kernel_for<0>(d), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ex->smem) !=
            cudaSuccess ||
        cudaFuncSetAttribute(token_kernel_for<1>(d), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ex->smem) !=
            cudaSuccess || qx_gdn_prepare_current() != cudaSuccess)
        return bail(fail(QX_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(cudaGetLastError())));
    {
        // how many clusters (or CTAs) of the token kernel the device holds at once
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(token_ctas(batch, d));
        cfg.blockDim = dim3(QX_NT);
        cfg.dynamicSmemBytes = ex->smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)d.cluster;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        cudaError_t e2 = cudaOccupancyMaxActiveClusters(&ex->max_clusters, token_kernel_for<1>(d), &cfg);
        if (e2 != cudaSuccess || ex->max_clusters < 1)
            return bail(fail(QX_ERR_CUDA, "a cluster of %d CTAs with %zu B of shared memory each does not fit: %s",
                             d.cluster, ex->smem, cudaGetErrorString(e2)));
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return bail(fail(QX_ERR_CUDA, "init sync"));
    *out = ex;
    return QX_OK;
}

qx_status qx_destroy(qx_t *ex) {
    if (!ex) return QX_OK;
    cudaSetDevice(ex->device);
    cudaDeviceSynchronize();
    delete ex;
    return QX_OK;
}

qx_status qx_buffer(qx_t *ex, int32_t kind, int32_t i, void **ptr, size_t *bytes) {
    if (!ex || !ptr || !bytes) return fail(QX_ERR_INVALID_ARG, "qx_buffer: null argument");
    const QxDev &d = ex->d;
    switch (kind) {
    case 0: *ptr = d.x; *bytes = (size_t)ex->B * d.D * 4; return QX_OK;
    case 1:
    case 2:
        if (i < 0 || i >= ex->n_hl) return fail(QX_ERR_INVALID_ARG, "qx_buffer: head sublayer %d", i);
        if (kind == 1) {
            const size_t copies = (d.shared_hl >> i & 1u) ? (size_t)ex->table_slots : (size_t)ex->B;
            *ptr = d.S[i];
            *bytes = copies * d.V[i] * QX_HD * QX_HD * 4;
        }
        else { *ptr = d.hist[i]; *bytes = (size_t)3 * d.NE[i] * ex->Bpad * 4; }
        return QX_OK;
    case 3: *ptr = d.err; *bytes = (size_t)ex->B * 4; return QX_OK;
    case 4: *ptr = d.hash; *bytes = (size_t)ex->B * 8; return QX_OK;
    case 5: *ptr = d.count; *bytes = (size_t)ex->B * 8; return QX_OK;
    case 6: *ptr = d.halt_at; *bytes = (size_t)ex->B * 8; return QX_OK;
    case 7: *ptr = d.state_bytes; *bytes = 8; return QX_OK;
    case 8:
        if (!d.img) return fail(QX_ERR_INVALID_ARG, "qx_buffer: the executor shares no tables");
        *ptr = d.img; *bytes = (size_t)ex->B * 4; return QX_OK;
#ifdef QX_PHASE_CLOCKS
    case 9: *ptr = d.phase_clk; *bytes = 256 * 16; return QX_OK;  // per-phase cycle counters
#endif
    default: return fail(QX_ERR_INVALID_ARG, "qx_buffer: kind %d", kind);
    }
}

qx_status qx_reset(qx_t *ex, int32_t row0, int32_t n, void *stream) {
    if (!ex || row0 < 0 || n < 0 || row0 + n > ex->B) return fail(QX_ERR_INVALID_ARG, "qx_reset: rows");
    if (n == 0) return QX_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < ex->n_hl; i++)
        qx_reset_kernel<<<256, 256, 0, st>>>(ex->d.hist[i], ex->d.NE[i], ex->Bpad, row0, n);
    CU(cudaGetLastError());
    return QX_OK;
}

qx_status qx_set_table_images(qx_t *ex, int32_t slots) {
    if (!ex || slots < 1 || slots > ex->B) return fail(QX_ERR_INVALID_ARG, "qx_set_table_images: %d slots", slots);
    CU(cudaSetDevice(ex->device));
    // the head sublayers every value head of which is a ROM or DROM table (read-only: no key
    // writes them, no decay): tables T_ROM .. T_ROM + 31 and T_DROM .. T_DROM + 15, two value
    // heads each
    const uint32_t *tab = reinterpret_cast<const uint32_t *>(ex->host_plan.data() + ex->hdr.off[QX_S_TABLES]);
    std::vector<int> table_vh(ex->n_hl, 0);
    for (int t = 11; t < 59; t++) table_vh[tab[2 * t]] += 2;
    uint32_t shared = 0;
    for (int hl = 0; hl < ex->n_hl; hl++)
        if (table_vh[hl] == (int)ex->d.V[hl]) shared |= 1u << hl;
    if (!shared) return fail(QX_ERR_INVALID_PLAN, "qx_set_table_images: no head sublayer holds only tables");
    CU(cudaDeviceSynchronize());
    QxDev &d = ex->d;
    for (int hl = 0; hl < ex->n_hl; hl++) {
        if (!(shared >> hl & 1u)) continue;
        const size_t bytes = (size_t)slots * d.V[hl] * QX_HD * QX_HD * 4;
        void *p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) {
            cudaGetLastError();
            return fail(QX_ERR_OOM, "qx_set_table_images: %zu B", bytes);
        }
        if (cudaMemset(p, 0, bytes) != cudaSuccess) {
            cudaFree(p);
            return fail(QX_ERR_CUDA, "qx_set_table_images: memset");
        }
        auto it = std::find(ex->allocs.begin(), ex->allocs.end(), static_cast<void *>(d.S[hl]));
        if (it != ex->allocs.end()) {
            cudaFree(*it);
            ex->allocs.erase(it);
        }
        ex->allocs.push_back(p);
        d.S[hl] = static_cast<float *>(p);
    }
    if (!d.img) {
        void *p = nullptr;
        qx_status st = dev_alloc(ex, &p, (size_t)ex->Bpad * 4);
        if (st != QX_OK) return st;
        d.img = static_cast<int32_t *>(p);
    }
    CU(cudaMemset(d.img, 0, (size_t)ex->Bpad * 4));
    d.shared_hl = shared;
    ex->table_slots = slots;
    ex->slot_rom.clear();
    ex->slot_drom.clear();
    return QX_OK;
}

qx_status qx_load_machines(qx_t *ex, int32_t row0, int32_t n, const qx_machine *images, void *stream) {
    if (!ex || !images || row0 < 0 || n < 0 || row0 + n > ex->B)
        return fail(QX_ERR_INVALID_ARG, "qx_load_machines: rows");
    if (n == 0) return QX_OK;
    for (int i = 0; i < n; i++) {
        const qx_machine &m = images[i];
        if (m.rom_words > 65536 || m.drom_bytes > 131072 || (!m.rom && m.rom_words) || !m.ram)
            return fail(QX_ERR_INVALID_ARG, "qx_load_machines: image %d", i);
    }
    // shared tables: each image's slot (an existing one with the same ROM and DROM content, or a
    // new one, written by the first machine that brings it)
    std::vector<uint32_t> slot(n, 0), writes(n, 0);
    if (ex->d.shared_hl) {
        for (int i = 0; i < n; i++) {
            const qx_machine &m = images[i];
            size_t k = 0;
            for (; k < ex->slot_rom.size(); k++)
                if (ex->slot_rom[k].size() == m.rom_words && ex->slot_drom[k].size() == m.drom_bytes &&
                    (m.rom_words == 0 || !memcmp(ex->slot_rom[k].data(), m.rom, (size_t)m.rom_words * 4)) &&
                    (m.drom_bytes == 0 || !memcmp(ex->slot_drom[k].data(), m.drom, m.drom_bytes)))
                    break;
            if (k == ex->slot_rom.size()) {
                if ((int)k == ex->table_slots)
                    return fail(QX_ERR_INVALID_ARG, "qx_load_machines: more distinct firmware images than the %d table slots",
                                ex->table_slots);
                ex->slot_rom.emplace_back(m.rom, m.rom + m.rom_words);
                ex->slot_drom.emplace_back(m.drom, m.drom + m.drom_bytes);
                writes[i] = 1;
            }
            slot[i] = (uint32_t)k;
        }
    }
    CU(cudaSetDevice(ex->device));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // chunks of machines: [QxImage x cn][word pool], packed into pinned memory, one copy each
    const int chunk = 512;
    auto pool_words = [&](const qx_machine &m) {
        return (size_t)m.rom_words + (m.drom_bytes + 3) / 4 + 8192 + (m.bn ? 256 : 0);
    };
    size_t need = 0;
    for (int c0 = 0; c0 < n; c0 += chunk) {
        const int cn = n - c0 < chunk ? n - c0 : chunk;
        size_t b = (size_t)cn * sizeof(QxImage);
        for (int i = 0; i < cn; i++) b += 4 * pool_words(images[c0 + i]);
        need = b > need ? b : need;
    }
    if (!ex->copy_stream) CU(cudaStreamCreateWithFlags(&ex->copy_stream, cudaStreamNonBlocking));
    if (need > ex->stage_bytes) {
        for (int i = 0; i < 2; i++) {
            if (ex->staged[i]) CU(cudaEventSynchronize(ex->staged[i]));
            if (ex->pin[i]) cudaFreeHost(ex->pin[i]);
            if (ex->dstage[i]) cudaFree(ex->dstage[i]);
            ex->pin[i] = ex->dstage[i] = nullptr;
        }
        ex->stage_bytes = 0;
        for (int i = 0; i < 2; i++) {
            if (cudaHostAlloc(&ex->pin[i], need, cudaHostAllocDefault) != cudaSuccess ||
                cudaMalloc(&ex->dstage[i], need) != cudaSuccess)
                return fail(QX_ERR_OOM, "qx_load_machines: %zu B of staging", need);
            if (!ex->staged[i]) CU(cudaEventCreateWithFlags(&ex->staged[i], cudaEventDisableTiming));
            if (!ex->copied[i]) CU(cudaEventCreateWithFlags(&ex->copied[i], cudaEventDisableTiming));
        }
        ex->stage_bytes = need;
    }
    for (int c0 = 0, k = 0; c0 < n; c0 += chunk, k ^= 1) {
        const int cn = n - c0 < chunk ? n - c0 : chunk;
        CU(cudaEventSynchronize(ex->staged[k]));  // the copy that last used this buffer is done
        QxImage *img = static_cast<QxImage *>(ex->pin[k]);
        uint32_t *pool = reinterpret_cast<uint32_t *>(img + cn);
        uint32_t w = 0;
        for (int i = 0; i < cn; i++) {  // the pool offsets first, then the copies (several threads)
            img[i].rom_off = w;
            w += (uint32_t)pool_words(images[c0 + i]);
        }
        auto pack = [&](int lo, int hi) {
            for (int i = lo; i < hi; i++) {
                const qx_machine &m = images[c0 + i];
                QxImage &q = img[i];
                uint32_t o = q.rom_off;
                q.rom_len = m.rom_words;
                if (m.rom_words) memcpy(pool + o, m.rom, (size_t)m.rom_words * 4);
                o += m.rom_words;
                q.drom_off = o;
                q.drom_words = (m.drom_bytes + 3) / 4;
                if (q.drom_words) {
                    pool[o + q.drom_words - 1] = 0;
                    memcpy(pool + o, m.drom, m.drom_bytes);  // little-endian words of the bytes
                }
                o += q.drom_words;
                q.ram_off = o;
                memcpy(pool + o, m.ram, 8192 * 4);
                o += 8192;
                if (m.bn) {
                    q.bn_off = o;
                    memcpy(pool + o, m.bn, 1024);
                } else {
                    q.bn_off = 0xFFFFFFFFu;
                }
                memcpy(q.x, m.x, sizeof(q.x));
                q.x[0] = 0;
                q.anchor = m.anchor;
                q.n = m.n;
                q.img = slot[c0 + i];
                q.write_tables = writes[c0 + i];
            }
        };
        pack_parallel(cn, pack);
        const size_t bytes = (size_t)cn * sizeof(QxImage) + (size_t)w * 4;
        QxImage *dimg = static_cast<QxImage *>(ex->dstage[k]);
        uint32_t *dpool = reinterpret_cast<uint32_t *>(dimg + cn);
        // the loader writes every head-state row of the machines, so nothing is cleared first; the
        // staging buffer's last reader (the loader two chunks back) has finished (staged[k])
        cudaError_t e = cudaMemcpyAsync(dimg, img, bytes, cudaMemcpyHostToDevice, ex->copy_stream);
        if (e == cudaSuccess) e = cudaEventRecord(ex->copied[k], ex->copy_stream);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(st, ex->copied[k], 0);
        if (e == cudaSuccess) {
            qx_predecode_kernel<<<dim3(4, cn), 256, 0, st>>>(dimg, dpool, cn);
            qx_load_kernel<<<dim3(64, cn), 256, 0, st>>>(ex->d, dimg, dpool, row0 + c0, cn);
            e = cudaGetLastError();
        }
        if (e == cudaSuccess) e = cudaEventRecord(ex->staged[k], st);
        if (e != cudaSuccess) return fail(QX_ERR_CUDA, "qx_load_machines: %s", cudaGetErrorString(e));
    }
    CU(cudaStreamSynchronize(st));
    return QX_OK;
}

qx_status qx_step(qx_t *ex, float *x, void *stream) {
    if (!ex || !x) return fail(QX_ERR_INVALID_ARG, "qx_step: null argument");
    QxDev d = ex->d;
    d.x = x;
    CU(launch_token<0>(ex, d, 1, nullptr, static_cast<cudaStream_t>(stream)));
    return QX_OK;
}

qx_status qx_run(qx_t *ex, int32_t n_tokens, int32_t *tokens, void *stream) {
    if (!ex || n_tokens < 0) return fail(QX_ERR_INVALID_ARG, "qx_run: bad arguments");
    if (n_tokens == 0) return QX_OK;
    CU(launch_token<1>(ex, ex->d, n_tokens, tokens, static_cast<cudaStream_t>(stream)));
    return QX_OK;
}

qx_status qx_set_tokens(qx_t *ex, int32_t row0, int32_t n, const int32_t *tok, void *stream) {
    if (!ex || !tok || row0 < 0 || n < 0 || row0 + n > ex->B) return fail(QX_ERR_INVALID_ARG, "qx_set_tokens");
    if (n == 0) return QX_OK;
    for (int i = 0; i < n; i++) {
        // a chip token, or (merged graphs) a text token of the graph's vocabulary
        const bool text = ex->d.merged && tok[i] >= QX_TEXT_TOKEN && tok[i] - QX_TEXT_TOKEN < ex->d.n_text;
        if (!text && (tok[i] < 0 || (uint32_t)tok[i] >= ex->hdr.vocab))
            return fail(QX_ERR_INVALID_ARG, "token %d is neither a chip token nor a text token of the graph", tok[i]);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CU(cudaMemcpyAsync(ex->dtok, tok, (size_t)n * 4, cudaMemcpyHostToDevice, st));
    qx_embed_kernel<<<n, 256, 0, st>>>(ex->d, row0, n, ex->dtok);
    CU(cudaGetLastError());
    CU(cudaStreamSynchronize(st));
    return QX_OK;
}

static qx_status ensure_states(qx_t *ex, int32_t n) {
    if (ex->state_cap >= n) return QX_OK;
    if (ex->dstate) cudaFree(ex->dstate);
    ex->dstate = nullptr;
    ex->state_cap = 0;
    cudaError_t e = cudaMalloc(&ex->dstate, (size_t)n * sizeof(qx_state));
    if (e != cudaSuccess) return fail(QX_ERR_OOM, "state staging: %s", cudaGetErrorString(e));
    ex->state_cap = n;
    return QX_OK;
}

qx_status qx_readback(qx_t *ex, int32_t row, qx_state *out, void *stream) {
    if (!ex || !out || row < 0 || row >= ex->B) return fail(QX_ERR_INVALID_ARG, "qx_readback");
    qx_status s = ensure_states(ex, 1);
    if (s != QX_OK) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    qx_readback_kernel<<<1, 256, 0, st>>>(ex->d, row, 1, ex->dstate);
    CU(cudaGetLastError());
    CU(cudaMemcpyAsync(out, ex->dstate, sizeof(qx_state), cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    return QX_OK;
}

qx_status qx_checksums(qx_t *ex, uint64_t *out, void *stream) {
    if (!ex || !out) return fail(QX_ERR_INVALID_ARG, "qx_checksums");
    const int chunk = ex->B < 1024 ? ex->B : 1024;
    qx_status s = ensure_states(ex, chunk);
    if (s != QX_OK) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int r0 = 0; r0 < ex->B; r0 += chunk) {
        const int n = ex->B - r0 < chunk ? ex->B - r0 : chunk;
        qx_readback_kernel<<<n, 256, 0, st>>>(ex->d, r0, n, ex->dstate);
        qx_checksum_kernel<<<(n + 127) / 128, 128, 0, st>>>(ex->dstate, n, out + r0);
    }
    CU(cudaGetLastError());
    return QX_OK;
}

qx_status qx_errors(qx_t *ex, uint32_t *any, void *stream) {
    if (!ex || !any) return fail(QX_ERR_INVALID_ARG, "qx_errors");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CU(cudaMemcpyAsync(ex->err_host, ex->d.err, (size_t)ex->B * 4, cudaMemcpyDeviceToHost, st));
    CU(cudaStreamSynchronize(st));
    uint32_t acc = 0;
    for (int i = 0; i < ex->B; i++) acc |= ex->err_host[i];
    *any = acc;
    return QX_OK;
}

qx_status qx_cluster_capacity(const void *plan, size_t plan_bytes, int32_t device, int32_t cluster,
                              int32_t *max_clusters) {
    if (!plan || !max_clusters || cluster < 1 || cluster > 8)
        return fail(QX_ERR_INVALID_ARG, "qx_cluster_capacity: bad arguments");
    qx_plan_header h;
    if (plan_bytes < sizeof(h)) return fail(QX_ERR_INVALID_PLAN, "plan too short");
    memcpy(&h, plan, sizeof(h));
    qx_status st = validate(h, plan_bytes);
    if (st != QX_OK) return st;
    if (h.group != 32) return fail(QX_ERR_INVALID_ARG, "qx_cluster_capacity: clusters run groups of 32 machines");
    QxDev d{};
    d.smem_rows = (int32_t)(h.n_slots + h.n_scratch);
    d.qhot_max = (int32_t)h.qhot_max;
    d.ksel_slots = (int32_t)h.n_ksel_slots;
    d.group = 32;
    d.cluster = 1;
    const size_t smem = qx_smem_bytes(d);
    CU(cudaSetDevice(device));
    CU(cudaFuncSetAttribute(token_kernel_for<1>(d), cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cluster);
    cfg.blockDim = dim3(QX_NT);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)cluster;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    CU(cudaOccupancyMaxActiveClusters(&n, token_kernel_for<1>(d), &cfg));
    *max_clusters = n;
    return QX_OK;
}

qx_status qx_info(qx_t *ex, int32_t what, int64_t *out) {
    if (!ex || !out) return fail(QX_ERR_INVALID_ARG, "qx_info: null argument");
    switch (what) {
    case QX_INFO_CLUSTER: *out = ex->d.cluster; return QX_OK;
    case QX_INFO_MAX_CLUSTERS: *out = ex->max_clusters; return QX_OK;
    case QX_INFO_CTAS: *out = (int64_t)token_ctas(ex->B, ex->d); return QX_OK;
    case QX_INFO_SMEM: *out = (int64_t)ex->smem; return QX_OK;
    default: return fail(QX_ERR_INVALID_ARG, "qx_info: unknown item %d", what);
    }
}

size_t qx_gdn_work_bytes(int64_t BH) { return 8 + 4 * (size_t)(BH > 0 ? BH : 0); }

qx_status qx_gdn_step(int64_t BH, float *S, const float *q, const float *k, const float *v, const float *alpha,
                      const float *beta, float *o, void *work, void *stream) {
    if (BH < 0 || BH > (int64_t)1 << 30) return fail(QX_ERR_INVALID_ARG, "qx_gdn_step: BH %lld", (long long)BH);
    if (BH == 0) return QX_OK;
    if (!S || !q || !k || !v || !alpha || !beta || !o || !work)
        return fail(QX_ERR_INVALID_ARG, "qx_gdn_step: null argument");
    CU(qx_gdn_prepare_current());  // once per device: the matrix kernel's shared-memory limit
    CU(qx_gdn_launch(BH, S, q, k, v, alpha, beta, o, static_cast<uint32_t *>(work), static_cast<cudaStream_t>(stream)));
    return QX_OK;
}

qx_status qx_gdn_step_noalloc(int64_t BH, float *S, const float *q, const float *k, const float *v,
                              const float *alpha, const float *beta, float *o, uint32_t *err, void *stream) {
    if (BH < 0 || BH > QX_GDN_NOALLOC_MAX_BH)
        return fail(QX_ERR_INVALID_ARG,
                    "qx_gdn_step_noalloc: %lld heads; its built-in scratch holds at most %d "
                    "(qx_gdn_step takes a caller buffer for more)",
                    (long long)BH, QX_GDN_NOALLOC_MAX_BH);
    if (BH == 0) return QX_OK;
    if (!S || !q || !k || !v || !alpha || !beta || !o)
        return fail(QX_ERR_INVALID_ARG, "qx_gdn_step_noalloc: null argument");
    uint32_t *work = nullptr;
    CU(qx_gdn_noalloc_scratch(&work));  // the first call on a device sets it up
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    CU(qx_gdn_launch(BH, S, q, k, v, alpha, beta, o, work, st));  // clears the count and error word first
    if (err) CU(cudaMemcpyAsync(err, work + 1, 4, cudaMemcpyDeviceToDevice, st));
    return QX_OK;
}

}  // extern "C"
