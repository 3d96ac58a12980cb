/*
 * qx.h -- C ABI of libqx, the B200 executor for compiled RV32IM transformer circuits.
 *
 * The reference drives this path from Python through one class, Executor2
 * (experimental/riscv/chipformer/rv/tritonexec.py:173-289), plus the free-running decode of
 * FreeRun (experimental/riscv/chipformer/rv/fastexec.py:236-340).  The reference has no C ABI
 * of its own; the entry points below are the calls a binding of that class needs, each mapped
 * to the method it replaces.  Plain pointers and sizes only; every call returns a qx_status and
 * never aborts the process.  Device pointers are marked `dev`, host pointers `host`.
 *
 * Threading: one host thread per qx_t at a time.  Calls that take a cudaStream_t (passed as
 * void*) only enqueue work on it; qx_step / qx_run allocate nothing and never synchronise, so
 * they can be captured in a CUDA graph (as Executor2.step is, fastexec.py:418-428).
 */
#ifndef QX_H
#define QX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define QX_API __attribute__((visibility("default")))
#else
#define QX_API
#endif

typedef enum {
    QX_OK = 0,
    QX_ERR_INVALID_PLAN = 1,   /* the plan blob failed validation */
    QX_ERR_INVALID_ARG = 2,    /* a null pointer, a size out of range, a bad row index */
    QX_ERR_CUDA = 3,           /* a CUDA runtime call failed (qx_last_error has the text) */
    QX_ERR_OOM = 4,            /* device memory could not be allocated */
    QX_ERR_DEVICE_FLAG = 5     /* the kernel set a per-machine error word (see qx_errors) */
} qx_status;

typedef struct qx_executor qx_t;

/* ---- the plan blob (written by qwenputer_b200/plan.py) ------------------------------------- */

#define QX_PLAN_MAGIC 0x314E414C50585151ull /* "QQXPLAN1" */
#define QX_MPC 32                          /* machines per CTA: one per lane */
#define QX_NONE32 0xFFFFFFFFu              /* "no row" in row fields */

enum { /* phase kinds of the per-token program */
    QX_PH_ZERO = 1,     /* rows [a, a + b) of the row list: set to 0 */
    QX_PH_LOADX = 2,    /* step mode: X[row] = x[machine][dim] for (row, dim) pairs [a, a + b) */
    QX_PH_STAGE = 3,    /* lag history of head sublayer c: entries [a, a + b) */
    QX_PH_FORMS = 4,    /* form records of the stream; warp w reads quads warp_ptr[c + w ..] */
    QX_PH_UNITS = 5,    /* FFN node records of the stream; warp ranges at warp_ptr[c] */
    QX_PH_KSEL = 6,     /* key-head records of the stream: key argmax, query top-k per machine */
    QX_PH_VH = 7,       /* value heads [a, b): list every (value head, machine) with row work;
                           c: output delta rows of the phase (at most QX_DELTA_ROWS) */
    QX_PH_VHRUN = 12,   /* value heads [a, b): serve the listed work: decay, write, read, output */
    QX_PH_VHSUM = 13,   /* rows VHSUM_ROWS[a, a + b) += the group's output delta rows 0..b-1 */
    QX_PH_APPLY = 8,    /* X[dst] += X[src] for pairs [a, a + b) */
    QX_PH_WRITEOUT = 9, /* step mode: x[machine][dim] = X[row] for pairs [a, a + b) */
    QX_PH_DECODE = 10,  /* run mode: output code -> token; next embedding into X */
    QX_PH_MMA = 14,     /* linear forms on the tensor cores: qx_mma_phase a of MMA_PHASES */
    QX_PH_END = 11,
    QX_PH_NOSYNC = 0x100 /* flag on a phase kind: no barrier after the phase */
};

typedef struct {
    uint32_t kind, a, b, c;  /* kind: QX_PH_* (low 8 bits) | QX_PH_NOSYNC */
} qx_phase;

/* Stream records (uint4 quads), consumed per warp in order.  Every row field is a shared-memory
 * byte offset (row * 132); the row after the last one is kept at zero and stands for "no form".
 *   form      [dst, n entry quads, 0, 0] + quads of two entries [row, w, row, w] (fp32 w):
 *             F[dst] = sum w X[row]
 *   FFN node  [out, n groups, n quads, 0] + groups of units sharing their forms (a, b):
 *             constant a: [a, b, n, 0] + (n + 1) / 2 quads [k, cb, k, cb]: each unit
 *                         k x0 relu(F[b] + cb x0), k = coef * ca (a padding unit has k = 0)
 *             a form:     [a, b, n | 1 << 31, 0] + n quads [coef, ca, cb, 0]: each unit
 *                         coef (F[a] + ca x0) relu(F[b] + cb x0); X[out] += the sum
 *   key head  [slot | qhot << 16, k common, q common, nk | nq << 16], [k lag-ONE row, q lag-ONE
 *             row, 0, 0], then nk key-channel quads and nq query-channel quads
 *             [row | exists << 31, c0, c1, 0]:
 *             channel = relu(F[row] + (exists ? F[common] : 0) + c0 x0 + c1 x0(t - lag)) */

typedef struct {        /* lag history entry of a head sublayer */
    uint32_t e;         /* index into that sublayer's history rows */
    uint32_t x_row;     /* byte offset of the dim's row (the value that becomes lag 1) */
    uint32_t ml;        /* deepest lag kept (1..3) */
    uint32_t stage[3];  /* byte offset of the row receiving lag 1, 2, 3 (~0u: not read) */
} qx_stage;

typedef struct {        /* value head task */
    uint32_t hl;        /* head sublayer (which S buffer) */
    uint32_t vh;        /* value-head index within that sublayer */
    uint32_t col;       /* offset into the per-column tables ([128] each) */
    uint16_t slot;      /* KSEL slot of its key head */
    uint16_t nrows;     /* decaying rows (0: the head never decays) */
    uint32_t a_row, b_row;  /* byte offsets of the decay selector and write gate forms */
    float ca, cb, bconst;
    uint32_t nout;      /* distinct output rows when at most 4 (OUT_ROW then holds indices into
                           out4), else QX_OUT_DIRECT (OUT_ROW holds the rows) */
    uint32_t out4[4];   /* the output rows (byte offsets) */
} qx_vhead;
#define QX_OUT_DIRECT 0xFFu
#define QX_DELTA_ROWS 128  /* output delta rows a value-head phase may use (per group, in HBM) */

typedef struct {        /* a value head column's v or z: relu(F[row] + c x0) (F from the FORMS phase) */
    uint32_t row;       /* shared-memory byte offset of the form's row (the zero row if none) */
    uint16_t pad;
    uint16_t live;      /* 0: the column has no form (reads 0) */
    float c;
} qx_colform;

/* A tensor-core form phase (QX_PH_MMA): F[form][machine] = sum_k W[form][k] X[row_k][machine]
 * as tcgen05 MMAs of M = 128 forms (a form block) x N = 32 machines x K = 16 source rows (a K
 * block), bf16 operands, fp32 accumulators in tensor memory.  ROWS[kr0 .. kr0 + 16 n_kb) are the
 * source rows (byte offsets; padding: the zero row), ROWS[dst0 .. dst0 + 128 n_fb) the form
 * blocks' destination rows (QX_NONE32: no form).  Tiles MMA_TILES[t0 .. t1) in issue order. */
#define QX_MMA_MAX_KB 16 /* K blocks a phase stages (1 KB of bf16 each, in the stream rings) */
#define QX_MMA_MAX_FB 8  /* form blocks a phase accumulates (32 tensor-memory columns each) */
typedef struct {
    uint32_t n_kb, kr0, n_fb, dst0, t0, t1, pad0, pad1;
} qx_mma_phase;
typedef struct {   /* one MMA: A = TILEDATA tile `data` ([128][16] bf16, row = form), B = K block kb */
    uint32_t data, fb, kb, acc; /* acc 0: the form block's first tile (starts the accumulator) */
} qx_mma_tile;

typedef struct {
    uint64_t magic;
    uint32_t version, D;
    uint32_t n_slots, n_scratch;   /* X rows, scratch rows (smem rows of 33 floats each) */
    uint32_t nw;                   /* warps per CTA the warp ranges were balanced for */
    uint32_t n_head_levels;
    uint32_t one_row;              /* byte offset of the constant-one dim's row */
    uint32_t n_ksel_slots;         /* key-head slots one KSEL phase may fill */
    uint32_t qhot_max;
    uint32_t n_fam, n_pay, n_feat, n_emb_rows, n_families;
    uint32_t vocab;
    uint32_t n_born0;              /* PAIRS[0 : n_born0] = (row, dim) of the dims set by an
                                      embedding (ONE and the token features) */
    uint32_t cluster;              /* CTAs (a thread-block cluster) that share one group of 32
                                      machines; stream ranges exist for nw * cluster warps */
    uint32_t flags;                /* QX_PLAN_FLAG_* */
    uint32_t group;                /* machines one CTA runs: 32 (a lane per machine), or 16, 8 or 4
                                      for few machines per GPU: a warp then runs 32 / group stream
                                      records side by side (lines of 32 / group quads), residual
                                      rows are group + 1 floats; no cluster, no tensor cores */
    uint32_t table_bytes;          /* shared memory after the stream rings for plan tables the
                                      token loop reads (0 for groups of 32) */
    /* sections: byte offset from the blob start, element count */
    uint64_t off[48];
    uint64_t cnt[48];
} qx_plan_header;

enum { /* section ids of qx_plan_header.off / cnt */
    QX_S_RUN_PROG = 0,   /* qx_phase: the run-mode program of one token */
    QX_S_STEP_PROG,      /* qx_phase: the step-mode program */
    QX_S_ROWS,           /* uint32: row lists (byte offsets) */
    QX_S_PAIRS,          /* uint32 pairs (row, dim) / (dst, src) */
    QX_S_STREAM,         /* uint4 quads: form, FFN node and key-head records */
    QX_S_VHSUM_ROWS,     /* uint32: rows (byte offsets) that VHSUM phases add output deltas into */
    QX_S_WARP_PTR,       /* uint32: per phase, nw + 1 quad offsets into STREAM */
    QX_S_STAGES,         /* qx_stage */
    QX_S_VHEADS,         /* qx_vhead */
    QX_S_VFORM,          /* qx_colform [vheads][128] */
    QX_S_ZFORM,          /* qx_colform [vheads][128] */
    QX_S_OUT_ROW,        /* uint32 [vheads][128] byte offsets (~0u: no output) */
    QX_S_OUT_W,          /* float  [vheads][128] */
    QX_S_HL_V,           /* uint32 [head levels]: value heads of each head sublayer */
    QX_S_HL_NE,          /* uint32 [head levels]: lag-history rows of each head sublayer */
    QX_S_FAM_ROW,        /* uint32 [n_fam]: rows of the family-id code bits */
    QX_S_PAY_ROW,        /* uint32 [n_pay]: rows of the payload code bits */
    QX_S_FEAT_ROW,       /* uint32 [n_feat]: rows of ONE and the token features */
    QX_S_FAM_IDS,        /* int32 [n_families]: first token of each family */
    QX_S_FAM_SIZE,       /* int32 [n_families] */
    QX_S_FAM_ROW0,       /* int32 [n_families]: first table row (small families), -1 big */
    QX_S_EMB_BASE,       /* float [n_families][n_feat] */
    QX_S_EMB_BITS,       /* float [n_families][n_pay][n_feat] */
    QX_S_EMB_TABLE,      /* float [n_emb_rows][n_feat] */
    QX_S_TABLES,         /* uint32 [99][2]: snapshot table -> (head level, first value head) */
    QX_S_REG_COLS,       /* int32 [32][8] */
    QX_S_FAM_TOUCH_PTR,  /* uint32 [n_families + 1]: offsets into FAM_TOUCH */
    QX_S_FAM_TOUCH,      /* uint32: per family, the features its payload-built embeddings touch */
    QX_S_MMA_PHASES,     /* qx_mma_phase */
    QX_S_MMA_TILES,      /* qx_mma_tile */
    QX_S_TILEDATA,       /* uint16 (bf16): [tiles][128][16] form-block weights */
    QX_S_FEAT_DIM,       /* uint32 [n_feat]: the feature dims (ONE first), FEAT_ROW's order */
    QX_S_CODE_ROW,       /* uint32 [n_code]: rows of the output-code dims (merged readout) */
    QX_S_TEXT_WORDS,     /* uint32 [n_text][5]: each text token's 152 bits (merged) */
    QX_S_TEXT_BASE,      /* float [n_feat]: a text token's features with no bit set */
    QX_S_TEXT_BITS,      /* float [n_text_bits][n_feat]: the features each text bit adds */
    QX_S_PRINTABLE,      /* int32 [n_printable]: the text token of each Q payload */
    QX_S_TEXT_TOUCH,     /* uint32: the features a text token can make nonzero */
    QX_S_MERGED_INFO,    /* uint32 [8]: Q family id, n_text, n_printable, n_text_touch, n_code,
                            n_text_bits, 0, 0 */
    QX_S_COUNT
};
#define QX_PLAN_FLAG_MMA 1u    /* the programs use QX_PH_MMA phases (the kernel holds tensor memory) */
#define QX_PLAN_FLAG_MERGED 2u /* merged readout: the next token from the signs of the code dims,
                                  a Q code naming the text token PRINTABLE[payload] */
#define QX_PLAN_FLAG_DIRECT_OUT 4u /* value-head outputs add straight into the residual rows
                                      (plans of one CTA a group): OUT_ROW and out4 name residual
                                      rows, the programs have no QX_PH_VHSUM phase */
#define QX_FEAT_DEFERRED 0x80000000u /* FEAT_ROW: the feature goes to x[machine][low bits] and is
                                        loaded where it is first used (a LOADX phase) */
#define QX_TEXT_TOKEN (1 << 24) /* a text token in the machine's stream: QX_TEXT_TOKEN | qid */

#define QX_PLAN_VERSION 18
#define QX_RING_QUADS 32   /* quads per half of a warp's stream ring in shared memory */

/* ---- machine images (the traced machine's state, ref.Machine, ref.py:386-414) --------------- */

typedef struct {
    const uint32_t *rom;    /* host: instruction words from 0x40000 (raw; pre-decoded on device) */
    uint32_t rom_words;     /* <= 65536 */
    const uint8_t *drom;    /* host: read-only data bytes from 0x20000, or NULL */
    uint32_t drom_bytes;    /* <= 131072 */
    const uint32_t *ram;    /* host: 8192 RAM words */
    uint32_t x[32];         /* registers (x0 ignored) */
    uint32_t anchor, n;     /* PC = 0x40000 + 4 (anchor + n) */
    const uint8_t *bn;      /* host: the digit file [8][128], or NULL (all zero) */
} qx_machine;

typedef struct {
    uint32_t x[32];
    uint32_t anchor, n;
    uint32_t ram[8192];
} qx_state;

/* ---- entry points -------------------------------------------------------------------------- */

/* Executor2.__init__ (tritonexec.py:176-244): validate the plan, allocate the device buffers for
 * `batch` machines on `device` (weights, residual x [batch][D], lag histories, head states S
 * [batch][V][128][128] per head sublayer, zeroed), copy the plan. */
QX_API qx_status qx_create(const void *plan /*host*/, size_t plan_bytes, int32_t batch, int32_t device,
                    qx_t **out);

/* Releases every device buffer of the executor. */
QX_API qx_status qx_destroy(qx_t *ex);

/* Device pointers of the executor's state buffers (stable for its lifetime), so that a binding
 * can expose them as tensors mutated in place (Executor2.steps[i]["S"], ["hist"], .y).  kind:
 * 0 = x [batch][D]; 1 = S of head sublayer i; 2 = lag history of head sublayer i
 * [3][rows][batch_pad] (lag 1..3, machine fastest); 3 = per-machine error words uint32 [batch];
 * 4 = token hashes uint64 [batch]; 5 = tokens generated int64 [batch]; 6 = index (1-based) of
 * the first HALT token generated, int64 [batch], -1 if none; 7 = head-state bytes read or written
 * by the token kernel so far (uint64 [1], 512 per row transfer: the roofline's touched rows);
 * 8 = the machines' table image slots (int32 [batch], after qx_set_table_images). */
QX_API qx_status qx_buffer(qx_t *ex, int32_t kind, int32_t i, void **dev_ptr, size_t *bytes);

/* Executor2.reset (tritonexec.py:260-263): zero the lag histories of rows [row0, row0 + n). */
QX_API qx_status qx_reset(qx_t *ex, int32_t row0, int32_t n, void *stream);

/* core.snapshot + Executor2.load_init (core.py:1218-1270, tritonexec.py:246-258): build the
 * head states of machines [row0, row0 + n) from host machine images, on the device.  The row's
 * states are replaced entirely (rows the snapshot does not set become 0). */
QX_API qx_status qx_load_machines(qx_t *ex, int32_t row0, int32_t n, const qx_machine *images /*host*/,
                           void *stream);

/* Share the read-only ROM / DROM tables between machines that run the same firmware (the
 * snapshot's byte tables, core.py:1236-1246, byte_rows 1194-1212: 96 of the 191 value heads, 6.3 MB
 * of a machine's 12.5 MB).  The head sublayers that hold only those tables are reallocated as
 * `slots` copies, one per distinct firmware image (ROM words and DROM bytes); later
 * qx_load_machines calls give each machine the slot of its image, writing a slot's rows once, when
 * its image first arrives, and fail with QX_ERR_INVALID_ARG once more than `slots` distinct
 * images have arrived (slots are not reclaimed; calling this again starts over, and the machines
 * must then be loaded again).  qx_buffer(1, i) of such a sublayer is then [slots][V][128][128];
 * qx_buffer(8, 0) is the machines' slots (int32 [batch]).  Synchronises the device.  No
 * counterpart in the reference (each ExecRow holds its own copy). */
QX_API qx_status qx_set_table_images(qx_t *ex, int32_t slots);

/* Executor2.step (tritonexec.py:272-289): one token for every machine.  x (dev, [batch][D],
 * the embeddings in) is updated in place to the residual after every node. */
QX_API qx_status qx_step(qx_t *ex, float *x /*dev*/, void *stream);

/* FreeRun.run (fastexec.py:298-340): n_tokens steps, each decoding the output code into the
 * next token and its embedding, all on the device, starting from the executor's x buffer (the
 * embedding of each machine's next input).  Generated token ids go to tokens (dev,
 * [n_tokens][batch] int32, or NULL); every machine's token hash and counters are updated. */
QX_API qx_status qx_run(qx_t *ex, int32_t n_tokens, int32_t *tokens /*dev*/, void *stream);

/* Sets x row r to the embedding of token tok[r] for rows [row0, row0 + n) (FreeRun.load's first
 * token, fastexec.py:292-296), and clears those rows' hashes and counters. */
QX_API qx_status qx_set_tokens(qx_t *ex, int32_t row0, int32_t n, const int32_t *tok /*host*/,
                        void *stream);

/* The inverse of qx_load_machines for one row: registers, PC anchor / n, RAM words. */
QX_API qx_status qx_readback(qx_t *ex, int32_t row, qx_state *out /*host*/, void *stream);

/* Per-machine 64-bit checksums of (x1..x31, anchor, n, RAM) computed on the device into out
 * (dev, [batch] uint64).  The FNV-1a 64 of those 8,225 words, little-endian. */
QX_API qx_status qx_checksums(qx_t *ex, uint64_t *out /*dev*/, void *stream);

/* OR of every machine's error word (dev -> host copy; synchronises the stream). */
QX_API qx_status qx_errors(qx_t *ex, uint32_t *any /*host*/, void *stream);

/* Facts of the executor's launch shape: QX_INFO_CLUSTER, the CTAs (a thread-block cluster) that
 * share one group of 32 machines; QX_INFO_MAX_CLUSTERS, how many such clusters the device holds at
 * once; QX_INFO_CTAS, the CTAs of one token-kernel launch; QX_INFO_SMEM, shared memory per CTA.
 * No counterpart in the reference (its Executor2 has no launch-shape queries). */
enum { QX_INFO_CLUSTER = 0, QX_INFO_MAX_CLUSTERS = 1, QX_INFO_CTAS = 2, QX_INFO_SMEM = 3 };
QX_API qx_status qx_info(qx_t *ex, int32_t what, int64_t *out /*host*/);

/* How many clusters of `cluster` CTAs (1..8) of the token kernel, with the plan's shared memory
 * per CTA, the device holds at once (cudaOccupancyMaxActiveClusters); lets a caller choose the
 * cluster size for a batch before compiling the plan for it.  No counterpart in the reference. */
QX_API qx_status qx_cluster_capacity(const void *plan, size_t plan_bytes, int32_t device, int32_t cluster,
                                     int32_t *max_clusters /*host*/);

/* The text of the last error on this thread ("" if none). */
QX_API const char *qx_last_error(void);

/* ---- the gated delta-rule decode step (standalone microbenchmark path) ------------------- */

/* For every (b, h) of BH heads: S <- alpha S; kv = S^T k; S <- S + k (x) beta (v - kv);
 * o = S^T q; sums over the key index in order, each product rounded before it is added.  Keys
 * with a single nonzero take a row path that touches only that row (plus the whole matrix when
 * alpha != 1); other keys update the whole matrix.  All dev, fp32: S [BH][128][128], q/k/v/o
 * [BH][128], alpha/beta [BH].  work: dev scratch of qx_gdn_work_bytes(BH) bytes, laid out as
 * uint32 [count, error word, head indices...]; after the step the error word (bytes 4..7) is 0,
 * or QX_ERR_DEVICE_FLAG when a bounded wait of the full-matrix path gave up, in which case the
 * states of that step are undefined.  The first call on a device sets the full-matrix kernel's
 * shared-memory limit there (once per device). */
QX_API size_t qx_gdn_work_bytes(int64_t BH);
QX_API qx_status qx_gdn_step(int64_t BH, float *S, const float *q, const float *k, const float *v,
                      const float *alpha, const float *beta, float *o, void *work, void *stream);

/* qx_gdn_step for callers that must not allocate device memory: hosts whose own allocator has
 * been handed the whole device heap, and latency-bound loops in which a cudaMalloc, which can
 * synchronise the device, is not allowed.  No counterpart in the reference.
 *
 * Same step, same arguments and results as qx_gdn_step, without `work`: the scratch is a
 * fixed array inside this library (QX_GDN_NOALLOC_MAX_BH heads, 256 KB + 8 B per device, kept
 * until the process exits), so the call allocates nothing.  BH above QX_GDN_NOALLOC_MAX_BH is
 * rejected with QX_ERR_INVALID_ARG (use qx_gdn_step with a caller buffer).  The first call on a
 * device sets that device up (looks up the array's address, which can load this library's
 * kernels onto the device, and sets the step kernel's shared-memory limit): make that first
 * call before any stream capture.  Every call on a device shares the one array and clears its
 * count and error word on the stream first, so calls whose kernels can overlap on the GPU
 * (different streams without ordering between them) race; calls on one stream, or otherwise
 * ordered, do not.  err (dev, optional): receives the step's error word (0, or
 * QX_ERR_DEVICE_FLAG when a bounded wait of the full-matrix path gave up). */
#define QX_GDN_NOALLOC_MAX_BH 65536
QX_API qx_status qx_gdn_step_noalloc(int64_t BH, float *S, const float *q, const float *k, const float *v,
                                     const float *alpha, const float *beta, float *o, uint32_t *err,
                                     void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QX_H */
