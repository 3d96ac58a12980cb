// qx_exec.cuh -- device-side view of a plan and of an executor's buffers (shared by the kernels).
#pragma once
#include <cstdint>

#include "qx.h"

#define QX_NW 16                 // warps per CTA
#define QX_NT (QX_NW * 32)       // threads per CTA
#define QX_RP 33                 // floats per smem row of a 32-machine group (32 machines + 1 pad)
#define QX_MAX_HL 16             // head sublayers a plan may have
#define QX_HD 128

// the float at a byte offset from a (shared-memory) base
#define QX_AT(base, off) (*reinterpret_cast<float *>(reinterpret_cast<char *>(base) + (off)))
#define QX_ATC(base, off) (*reinterpret_cast<const float *>(reinterpret_cast<const char *>(base) + (off)))

struct QxDev {
    // plan sections (device)
    const qx_phase *run_prog, *step_prog;
    const uint32_t *rows;
    const uint2 *pairs;
    const uint4 *stream;
    const uint32_t *vhsum_rows;  // residual rows the cluster's output deltas add into
    float *vdelta;  // [groups][2][QX_DELTA_ROWS][32] value-head output deltas (L2-resident)
    const uint32_t *warp_ptr;
    const qx_stage *stages;
    const qx_vhead *vheads;
    const qx_colform *vform, *zform;
    const uint32_t *out_row;
    const float *out_w;
    const uint32_t *fam_row, *pay_row, *feat_row;
    const int32_t *fam_ids, *fam_size, *fam_row0;
    const float *emb_base, *emb_bits, *emb_table;
    const uint32_t *fam_touch_ptr, *fam_touch;  // per family: the features its embeddings touch
    const uint32_t *tables;     // [99][2]
    const int32_t *reg_cols;    // [32][8]
    const uint2 *zero_rows;     // [n_zero_rows] (head sublayer, row) of the rows no load task writes
    // executor buffers
    float *S[QX_MAX_HL];        // [B][V][128][128]
    float *hist[QX_MAX_HL];     // [3][NE][Bpad]
    uint32_t V[QX_MAX_HL], NE[QX_MAX_HL];
    float *x;                   // [B][D]
    uint32_t *err;              // [B]
    uint64_t *hash;             // [B]
    int64_t *count;             // [B] tokens generated
    int64_t *halt_at;           // [B] index (1-based) of the first HALT token, -1 none
    unsigned long long *state_bytes;  // [1] head-state bytes the kernel read or wrote (512 B rows)
    unsigned long long *phase_clk;    // [256][2] per program position: SM cycles, visits (builds
                                      // with QX_PHASE_CLOCKS only; null otherwise)
    // sizes
    int32_t B, Bpad, D;
    int32_t smem_rows, one_row, n_fam, n_pay, n_feat, n_families, n_emb_rows, n_born0;
    int32_t qhot_max, ksel_slots, n_hl, halt_tok;
    uint32_t zero_row;  // byte offset of the row kept at zero
    int32_t cluster;    // CTAs sharing one group of 32 machines (a thread-block cluster)
    int32_t group;      // machines a CTA runs: 32, or 16 / 8 / 4 (a warp's lanes then run
                        // 32 / group records side by side; rows are group + 1 floats)
    int32_t n_zero_rows;
    int32_t n_run_prog, n_step_prog, n_warp_ptr;  // entries of the programs and of WARP_PTR
    // shared-memory copies of plan tables (bundled plans): bytes reserved after the rings, and per
    // table (QX_TAB_*) its byte offset there, or QX_NONE32 where it stays in global memory
    uint32_t table_bytes;
    uint32_t tab_off[6], tab_words[6];
    // tensor-core form phases
    const qx_mma_phase *mma_phases;
    const qx_mma_tile *mma_tiles;
    const uint4 *tiledata;  // [tiles][128 rows][2] (a row: 16 bf16 weights)
    int32_t has_mma;        // the kernel allocates tensor memory
    int32_t direct_out;     // value-head outputs add into the residual rows (no delta rows)
    // merged readout and text tokens (QX_PLAN_FLAG_MERGED)
    const uint32_t *feat_dim, *code_row, *text_words, *text_touch;
    const float *text_base, *text_bits;
    const int32_t *printable;
    int32_t merged, q_fid, n_text, n_printable, n_text_touch, n_code, n_text_bits;
    // shared read-only tables (qx_set_table_images): head sublayers whose every value head is a
    // ROM / DROM table hold one copy per firmware image; a machine's copy is img[machine]
    uint32_t shared_hl;  // bit hl: sublayer hl is shared
    int32_t *img;        // [Bpad] image slot of each machine
};

// per-machine error bits
#define QX_E_CODE 1u        // the output code names no token
#define QX_E_KEY 2u         // a key with more than one positive channel
#define QX_E_QUERY 4u       // a query with more positive channels than the head reads
#define QX_E_BUSY 8u        // a bounded wait gave up
#define QX_E_INEXACT 16u    // a value a tensor-core form phase read is not exact in bf16

struct QxImage {  // one machine inside a packed image upload (offsets into the word pool)
    uint32_t rom_off, rom_len, drom_off, drom_words, ram_off, bn_off;  // bn_off: ~0 = none
    uint32_t x[32];
    uint32_t anchor, n;
    uint32_t img, write_tables;  // shared tables: the machine's image slot; 1: this machine writes it
};

// The state copy of machine m in head sublayer hl: m, or its image slot where hl is shared.
__device__ __forceinline__ size_t qx_copy(const QxDev &d, uint32_t hl, int m) {
    return (d.shared_hl >> hl & 1u) ? (size_t)d.img[m] : (size_t)m;
}

// shared memory: the rows (byte offsets row * 132; row smem_rows is kept at zero), then the
// key-select slots, the decode area ([2][32] ints, [16][32] payload floats), a 64-byte counter
// block and the per-warp stream rings ([NW][2][32] quads)
// value heads one VH phase may list (the record packs the phase-local index in 8 bits); its
// 8-byte (value head, machine) records live in the stream rings
#define QX_VH_CHUNK 64
// plan tables a bundled plan's token loop may read from shared memory, in the order they are placed
enum { QX_TAB_PROG = 0, QX_TAB_WARP_PTR, QX_TAB_VHEADS, QX_TAB_ROWS, QX_TAB_VHSUM, QX_TAB_STAGES };
// stream piece flags (header quad .w >> 24)
#define QX_R_FIRST 1u
#define QX_R_LAST 2u
#define QX_R_STORE 4u
#define QX_R_QUERY 8u
#define QX_R_MERGE 0x10u  // a part of a split key / query record: merged into the slot words
#define QX_R_NOP 0x20u    // a bundle's padding record: computes on the zero row, stores nothing
#define QX_R_SPLIT 0x40u  // a bundle that is one form pair over every record slot (warp-reduced)
#define QX_R_SKIP 0x80u
#define QX_RING_BYTES (QX_NW * 2 * QX_RING_QUADS * 16)

__host__ __device__ inline size_t qx_ring_offset(const QxDev &d) {
    // rows (plus the zero row) of group + 1 floats, key-select slots, decode area, counters
    size_t o = (size_t)(d.smem_rows + 1) * (d.group + 1) * 4 + (size_t)d.ksel_slots * 32 * (1 + d.qhot_max) * 4 +
               (size_t)32 * (2 + 16) * 4 + 64;
    return (o + 15) & ~(size_t)15;
}
// the per-warp stream rings: two chunks of QX_RING_QUADS lines of 32 / group quads
__host__ __device__ inline size_t qx_ring_bytes(const QxDev &d) {
    return (size_t)QX_NW * 2 * QX_RING_QUADS * 16 * (32 / d.group);
}
// bundled plans (groups of fewer than 32 machines) keep the plan tables the token loop reads in
// shared memory after the rings, as many as fit the plan's table_bytes (tab_off)
__host__ __device__ inline size_t qx_table_bytes(const QxDev &d) { return d.table_bytes; }
__host__ __device__ inline size_t qx_smem_bytes(const QxDev &d) {
    return qx_ring_offset(d) + qx_ring_bytes(d) + qx_table_bytes(d);
}
