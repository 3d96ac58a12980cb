/*
 * qx_oracle.c -- CPU ORACLE (test infrastructure only; never the product path).
 *
 * Plain-C restatement of the reference algorithms that the CUDA engine must reproduce bit for
 * bit.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load this library, and only
 * as the checker / the timed CPU baseline.  Reference files are cited by their path inside the
 * reference project; ERV = experimental/riscv.
 *
 *   qxo_step            Executor2.step: one token through every sublayer, fp32
 *                       (ERV/chipformer/rv/tritonexec.py:47-170, 272-289)
 *   qxo_decode          FreeRun._step: output code -> token id -> next embedding
 *                       (ERV/chipformer/rv/fastexec.py:298-307)
 *   qxo_machine_*       the traced machine ref.Machine (ERV/chipformer/rv/ref.py:386-605) with
 *                       decode / alu / div_parts / digit ops (ref.py:102-243, 555-598) and the
 *                       token spec (ERV/chipformer/rv/spec.py:58-149)
 *   qxo_rom_word        the pre-decoded ROM word (ref.py:335-380)
 *   qxo_snapshot        core.snapshot + Executor2.load_init: machine -> head state rows
 *                       (ERV/chipformer/rv/core.py:1177-1270, tritonexec.py:246-258)
 *   qxo_readback        the inverse of qxo_snapshot (registers, PC, RAM words)
 *   qxo_gdn_step        one gated delta-rule decode step with a fixed sequential fp32 order
 *                       (the recurrence of transformers' torch_recurrent_gated_delta_rule,
 *                       models/qwen3_5/modeling_qwen3_5.py, without the query scale)
 *
 * Parity pins: tests/golden/ holds vectors produced by the reference itself (make_golden.py).
 * Build with -ffp-contract=off: every product and sum below is rounded separately.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HD 128
#define M32 0xFFFFFFFFu

/* ======================================================================================== */
/* graph (the arrays of qwenputer_b200/graphfile.GraphData)                                  */
/* ======================================================================================== */

typedef struct {
    const int64_t *ptr;
    const int32_t *idx;
    const float *w;
} qxo_forms;

typedef struct {
    int32_t D;
    int32_t n_levels;
    const int32_t *levels;
    const int8_t *level_kind;
    int32_t n_ffn;
    const int32_t *ffn_level, *ffn_out;
    const int64_t *ffn_uptr;
    const float *unit_coef;
    qxo_forms unit_a, unit_b;
    int32_t n_heads;
    const int32_t *head_level, *head_qhot, *head_q, *head_k; /* head_q/k: [H][HD] */
    qxo_forms q_forms, k_forms;
    int32_t n_vh;
    const int32_t *vh_head, *vh_v, *vh_z, *vh_nrows; /* vh_v/z: [VH][HD] */
    const uint8_t *vh_has_beta;
    qxo_forms v_forms, z_forms, vh_a, vh_beta;
    const int64_t *vh_out_ptr;
    const int32_t *out_col, *out_dim;
    const float *out_w;
} qxo_graph;

/* x: [D] (lag 0), hist: [3][D] (lags 1..3): tritonexec.py:74-79 _lag_load */
static inline float lag_load(const float *x, const float *hist, int32_t D, int32_t i) {
    return i < D ? x[i] : hist[i - D];
}

static float form_dot(const qxo_forms *f, int64_t r, const float *x, const float *hist, int32_t D) {
    float acc = 0.0f;
    for (int64_t j = f->ptr[r]; j < f->ptr[r + 1]; j++) acc += f->w[j] * lag_load(x, hist, D, f->idx[j]);
    return acc;
}

static inline float relu(float v) { return v > 0.0f ? v : 0.0f; }

/* One sublayer of FFN units for one machine (tritonexec.py:47-71 + the apply of 151-170). */
static void ffn_level(const qxo_graph *g, int32_t level, float *x, float *y) {
    int32_t D = g->D;
    memset(y, 0, sizeof(float) * D);
    for (int32_t n = 0; n < g->n_ffn; n++) {
        if (g->ffn_level[n] != level) continue;
        for (int64_t u = g->ffn_uptr[n]; u < g->ffn_uptr[n + 1]; u++) {
            float av = form_dot(&g->unit_a, u, x, NULL, D);
            float bv = form_dot(&g->unit_b, u, x, NULL, D);
            float val = g->unit_coef[u] * av * relu(bv);
            y[g->ffn_out[n]] += val;
        }
    }
    for (int32_t d = 0; d < D; d++) x[d] += y[d];
}

/* One head sublayer for one machine (tritonexec.py:105-148 per value head, then the apply with
 * the lag-history shift, 151-170).  S: [V][HD][HD] of this machine, hist: [3][D]. */
static void head_level(const qxo_graph *g, int32_t level, float *x, float *hist, float *S, float *y) {
    int32_t D = g->D;
    memset(y, 0, sizeof(float) * D);
    int32_t j = 0; /* value-head index within the level */
    float k[HD], q[HD], v[HD], z[HD], o[HD];
    for (int32_t h = 0; h < g->n_heads; h++) {
        if (g->head_level[h] != level) continue;
        for (int32_t c = 0; c < HD; c++) {
            int32_t fk = g->head_k[h * HD + c], fq = g->head_q[h * HD + c];
            k[c] = fk < 0 ? 0.0f : relu(form_dot(&g->k_forms, fk, x, hist, D));
            q[c] = fq < 0 ? 0.0f : relu(form_dot(&g->q_forms, fq, x, hist, D));
        }
        /* argmax: the first maximal channel */
        float kmax = k[0];
        int32_t krow = 0;
        for (int32_t c = 1; c < HD; c++)
            if (k[c] > kmax) { kmax = k[c]; krow = c; }
        for (int32_t vh = 0; vh < g->n_vh; vh++) {
            if (g->vh_head[vh] != h) continue;
            float *Sb = S + (int64_t)j * HD * HD;
            for (int32_t c = 0; c < HD; c++) {
                int32_t fv = g->vh_v[vh * HD + c], fz = g->vh_z[vh * HD + c];
                v[c] = fv < 0 ? 0.0f : relu(form_dot(&g->v_forms, fv, x, hist, D));
                z[c] = fz < 0 ? 0.0f : relu(form_dot(&g->z_forms, fz, x, NULL, D));
            }
            float bv = form_dot(&g->vh_beta, vh, x, NULL, D) + (g->vh_has_beta[vh] ? 0.0f : 1.0f);
            int32_t nr = g->vh_nrows[vh];
            if (nr > 0) {
                float av = form_dot(&g->vh_a, vh, x, NULL, D);
                float fac = av == 0.0f ? 1.0f : (av == 110.0f ? 0.5f : 0.0f);
                if (fac != 1.0f)
                    for (int32_t r = 0; r < nr; r++)
                        for (int32_t c = 0; c < HD; c++) Sb[r * HD + c] = Sb[r * HD + c] * fac;
            }
            if (kmax > 0.0f && bv == 1.0f)
                for (int32_t c = 0; c < HD; c++) Sb[krow * HD + c] = v[c];
            /* the read: at most QHOT rows (the query's argmax, repeatedly) */
            float qq[HD];
            memcpy(qq, q, sizeof(qq));
            for (int32_t c = 0; c < HD; c++) o[c] = 0.0f;
            for (int32_t it = 0; it < g->head_qhot[h]; it++) {
                float qm = qq[0];
                int32_t qi = 0;
                for (int32_t c = 1; c < HD; c++)
                    if (qq[c] > qm) { qm = qq[c]; qi = c; }
                if (qm > 0.0f)
                    for (int32_t c = 0; c < HD; c++) o[c] += Sb[qi * HD + c];
                qq[qi] = 0.0f;
            }
            float ref = o[0] * o[0] + o[1] * o[1];
            float norm = sqrtf(ref / 128.0f); /* IEEE sqrt: correctly rounded */
            for (int64_t e = g->vh_out_ptr[vh]; e < g->vh_out_ptr[vh + 1]; e++) {
                int32_t c = g->out_col[e];
                float w = g->out_w[e];
                if (w == 0.0f) continue;
                float out = ref > 0.0f ? o[c] / norm : 0.0f;
                y[g->out_dim[e]] += out * z[c] * w;
            }
            j++;
        }
    }
    /* apply: lag history moves on, the input x becoming lag 1; then x += y */
    memcpy(hist + 2 * D, hist + D, sizeof(float) * D);
    memcpy(hist + D, hist, sizeof(float) * D);
    memcpy(hist, x, sizeof(float) * D);
    for (int32_t d = 0; d < D; d++) x[d] += y[d];
}

typedef struct {
    const qxo_graph *g;
    int32_t B, lo, hi;
    float *x;
    float **hist; /* per head level: [B][3][D] */
    float **S;    /* per head level: [B][V][HD][HD] */
    const int32_t *V;
} step_job;

static void *step_worker(void *arg) {
    step_job *jb = (step_job *)arg;
    const qxo_graph *g = jb->g;
    int32_t D = g->D;
    float *y = (float *)malloc(sizeof(float) * D);
    for (int32_t b = jb->lo; b < jb->hi; b++) {
        float *x = jb->x + (int64_t)b * D;
        int32_t hl = 0;
        for (int32_t l = 0; l < g->n_levels; l++) {
            if (g->level_kind[l] == 0) {
                ffn_level(g, g->levels[l], x, y);
            } else {
                head_level(g, g->levels[l], x, jb->hist[hl] + (int64_t)b * 3 * D,
                           jb->S[hl] + (int64_t)b * jb->V[hl] * HD * HD, y);
                hl++;
            }
        }
    }
    free(y);
    return NULL;
}

/* One token for B machines, x [B][D] in place. V[i]: value heads of the i-th head level. */
int qxo_step(const qxo_graph *g, int32_t B, float *x, float **hist, float **S, const int32_t *V,
             int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > B) nthreads = B;
    pthread_t th[256];
    step_job jobs[256];
    if (nthreads > 256) nthreads = 256;
    for (int32_t t = 0; t < nthreads; t++) {
        jobs[t] = (step_job){g, B, (int32_t)((int64_t)B * t / nthreads),
                             (int32_t)((int64_t)B * (t + 1) / nthreads), x, hist, S, V};
        if (nthreads == 1) step_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, step_worker, &jobs[t]);
    }
    if (nthreads > 1)
        for (int32_t t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    return 0;
}

/* ======================================================================================== */
/* FreeRun decode (fastexec.py:298-307)                                                      */
/* ======================================================================================== */

typedef struct {
    int32_t nf, npay, F, rows, nfam;
    const int32_t *fam_dims, *pay_dims, *feat_dims;
    const int64_t *fam_ids, *fam_row0;
    const uint8_t *fam_small;
    const float *base, *bits, *table; /* [nf][F], [nf][npay][F], [rows][F] */
} qxo_decoder;

/* out: x after a step [B][D]; writes tok [B] and the next embedding xn [B][D]. Returns the
 * number of rows whose code names no valid token (decode_code == -1, core.py:1273-1284). */
int32_t qxo_decode(const qxo_decoder *e, int32_t B, int32_t D, const float *out, int64_t *tok,
                   float *xn, const int64_t *fam_size) {
    int32_t bad = 0;
    for (int32_t b = 0; b < B; b++) {
        const float *o = out + (int64_t)b * D;
        float fam = 0.0f, pay[32];
        for (int32_t i = 0; i < e->nfam; i++) fam += rintf(o[e->fam_dims[i]]) * ldexpf(1.0f, i);
        float psum = 0.0f;
        for (int32_t i = 0; i < e->npay; i++) {
            pay[i] = rintf(o[e->pay_dims[i]]);
            psum += pay[i] * ldexpf(1.0f, i);
        }
        int64_t fraw = (int64_t)fam;
        int64_t fid = fraw < 0 ? 0 : (fraw > e->nf - 1 ? e->nf - 1 : fraw);
        int64_t p = (int64_t)psum;
        if (fraw != fid || p < 0 || p >= fam_size[fid]) bad++;
        tok[b] = e->fam_ids[fid] + p;
        float *x = xn + (int64_t)b * D;
        memset(x, 0, sizeof(float) * D);
        if (e->fam_small[fid]) {
            int64_t row = e->fam_row0[fid] + p;
            row = row < 0 ? 0 : (row > e->rows - 1 ? e->rows - 1 : row);
            for (int32_t f = 0; f < e->F; f++) x[e->feat_dims[f]] = e->table[row * e->F + f];
        } else {
            for (int32_t f = 0; f < e->F; f++) {
                float acc = 0.0f;
                for (int32_t i = 0; i < e->npay; i++) acc += pay[i] * e->bits[((int64_t)fid * e->npay + i) * e->F + f];
                x[e->feat_dims[f]] = e->base[fid * e->F + f] + acc;
            }
        }
    }
    return bad;
}

/* ======================================================================================== */
/* the RV32 token spec (spec.py:58-149)                                                      */
/* ======================================================================================== */

enum { F_V, F_F0, F_F1, F_F2, F_J, F_R, F_BYTE, F_FLT, F_HEX, F_QS, F_QD, F_BD, N_FAM };
static const int32_t FAM_SIZE[N_FAM] = {1 << 15, 1 << 15, 1 << 15, 4, 1 << 16, 1 << 16,
                                         512, 8, 16, 16, 128, 256};
enum { C_NT, C_ST0, C_ST1, C_SS0, C_SS1, C_HALT, C_GO, C_SC, N_CTRL };

static int32_t fam_base(int32_t f) {
    int32_t b = 0;
    for (int32_t i = 0; i < f; i++) b += FAM_SIZE[i];
    return b;
}
static int32_t tokf(int32_t f, int32_t p) { return fam_base(f) + p; }
static int32_t tokc(int32_t c) { return fam_base(N_FAM) + c; }

int32_t qxo_tok_family(int32_t f, int32_t p) { return f < N_FAM ? tokf(f, p) : tokc(f - N_FAM); }
int32_t qxo_vocab(void) { return fam_base(N_FAM) + N_CTRL; }

#define ROM_BASE 0x40000u
#define ROM_WORDS (1u << 16)
#define DROM_BASE 0x20000u
#define DROM_WORDS (1u << 15)
#define RAM_WORDS (1u << 13)
#define SP_INIT (4u * RAM_WORDS)
#define N_MAX 63
#define MISA 0x40001100u

enum { FAULT_ILLEGAL, FAULT_EBREAK, FAULT_MIS_LOAD, FAULT_MIS_STORE, FAULT_LOAD_RANGE,
       FAULT_STORE_RANGE, FAULT_BAD_JUMP, FAULT_ECALL };

typedef struct {
    int32_t *buf;
    int64_t n, cap;
} tokbuf;

static void put(tokbuf *t, int32_t v) {
    if (t->n < t->cap) t->buf[t->n] = v;
    t->n++;
}

static void value_record(tokbuf *t, uint32_t v) {
    int64_t s = (v >> 31) ? (int64_t)v - 4294967296LL : (int64_t)v;
    uint32_t c0 = v & 0x7FFF, c1 = v >> 15 & 0x7FFF, c2 = v >> 30;
    if (s >= -(1LL << 14) && s < (1LL << 14)) put(t, tokf(F_F0, c0));
    else if (s >= -(1LL << 29) && s < (1LL << 29)) { put(t, tokf(F_V, c0)); put(t, tokf(F_F1, c1)); }
    else { put(t, tokf(F_V, c0)); put(t, tokf(F_V, c1)); put(t, tokf(F_F2, c2)); }
}

/* ======================================================================================== */
/* decode / alu (ref.py:55-243)                                                              */
/* ======================================================================================== */

/* ops 0..52 and 64..69 are the ROM uop numbers (ref.py:55-68); CSR ops follow */
enum {
    ILLEGAL, LUI, AUIPC, MISA_OP, ADDI, SLTI, SLTIU, XORI, ORI, ANDI, SLLI, SRLI, SRAI, ADD, SUB,
    SLL, SLT, SLTU, XOR, SRL, SRA, OR, AND, LB, LH, LW, LBU, LHU, SB, SH, SW, BEQ, BNE, BLT, BGE,
    BLTU, BGEU, JAL, JALR, ECALL, EBREAK, FENCE, MUL, MULH, MULHSU, MULHU, DIV, DIVU, REM, REMU,
    SH1ADD, SH2ADD, SH3ADD,
    BMAC = 64, BMSB, BLD, BGET, BPRD, BSCAN,
    CSRRW = 100, CSRRS, CSRRC, CSRRWI, CSRRSI, CSRRCI
};

typedef struct {
    int32_t op, rd, rs1, rs2;
    int64_t imm;
    int32_t dd;
} inst;

static int64_t sx(uint64_t v, int bits) {
    v &= (bits == 64) ? ~0ULL : ((1ULL << bits) - 1);
    return (v >> (bits - 1)) & 1 ? (int64_t)v - (int64_t)(1ULL << bits) : (int64_t)v;
}

static inst decode(uint32_t w) {
    uint32_t opc = w & 0x7F, rd = w >> 7 & 31, f3 = w >> 12 & 7, rs1 = w >> 15 & 31,
             rs2 = w >> 20 & 31, f7 = w >> 25;
    int64_t i_imm = sx(w >> 20, 12);
    int64_t s_imm = sx((w >> 25) << 5 | (w >> 7 & 31), 12);
    int64_t b_imm = sx((w >> 31 & 1) << 12 | (w >> 7 & 1) << 11 | (w >> 25 & 63) << 5 | (w >> 8 & 15) << 1, 13);
    int64_t j_imm = sx((w >> 31 & 1) << 20 | (w >> 12 & 0xFF) << 12 | (w >> 20 & 1) << 11 | (w >> 21 & 0x3FF) << 1, 21);
    inst r = {ILLEGAL, 0, 0, 0, 0, 0};
    if (opc == 0x37) { r.op = LUI; r.rd = rd; r.imm = sx(w & 0xFFFFF000u, 32); return r; }
    if (opc == 0x17) { r.op = AUIPC; r.rd = rd; r.imm = sx(w & 0xFFFFF000u, 32); return r; }
    if (opc == 0x6F) { r.op = JAL; r.rd = rd; r.imm = j_imm; return r; }
    if (opc == 0x67 && f3 == 0) { r.op = JALR; r.rd = rd; r.rs1 = rs1; r.imm = i_imm; return r; }
    if (opc == 0x63 && f3 != 2 && f3 != 3) {
        static const int32_t B[8] = {BEQ, BNE, 0, 0, BLT, BGE, BLTU, BGEU};
        r.op = B[f3]; r.rs1 = rs1; r.rs2 = rs2; r.imm = b_imm; return r;
    }
    if (opc == 0x03 && (f3 == 0 || f3 == 1 || f3 == 2 || f3 == 4 || f3 == 5)) {
        static const int32_t L[6] = {LB, LH, LW, 0, LBU, LHU};
        r.op = L[f3]; r.rd = rd; r.rs1 = rs1; r.imm = i_imm; return r;
    }
    if (opc == 0x23 && f3 <= 2) {
        static const int32_t St[3] = {SB, SH, SW};
        r.op = St[f3]; r.rs1 = rs1; r.rs2 = rs2; r.imm = s_imm; return r;
    }
    if (opc == 0x13) {
        if (f3 == 1 && f7 == 0) { r.op = SLLI; r.rd = rd; r.rs1 = rs1; r.imm = rs2; return r; }
        if (f3 == 5 && (f7 == 0 || f7 == 0x20)) { r.op = f7 ? SRAI : SRLI; r.rd = rd; r.rs1 = rs1; r.imm = rs2; return r; }
        if (f3 != 1 && f3 != 5) {
            static const int32_t I[8] = {ADDI, 0, SLTI, SLTIU, XORI, 0, ORI, ANDI};
            r.op = I[f3]; r.rd = rd; r.rs1 = rs1; r.imm = i_imm; return r;
        }
    }
    if (opc == 0x33) {
        if (f7 == 0) {
            static const int32_t R[8] = {ADD, SLL, SLT, SLTU, XOR, SRL, OR, AND};
            r.op = R[f3]; r.rd = rd; r.rs1 = rs1; r.rs2 = rs2; return r;
        }
        if (f7 == 0x20 && (f3 == 0 || f3 == 5)) { r.op = f3 == 0 ? SUB : SRA; r.rd = rd; r.rs1 = rs1; r.rs2 = rs2; return r; }
        if (f7 == 1) {
            static const int32_t Mo[8] = {MUL, MULH, MULHSU, MULHU, DIV, DIVU, REM, REMU};
            r.op = Mo[f3]; r.rd = rd; r.rs1 = rs1; r.rs2 = rs2; return r;
        }
        if (f7 == 0x10 && (f3 == 2 || f3 == 4 || f3 == 6)) {
            r.op = f3 == 2 ? SH1ADD : (f3 == 4 ? SH2ADD : SH3ADD); r.rd = rd; r.rs1 = rs1; r.rs2 = rs2; return r;
        }
    }
    if (opc == 0x0B && f3 < 5 && f7 == 0) {
        static const int32_t Cu[5] = {BMAC, BMSB, BLD, BGET, BSCAN};
        r.op = Cu[f3]; r.rd = rd; r.rs1 = rs1; r.rs2 = rs2; return r;
    }
    if (opc == 0x2B && f3 == 0) { r.op = BPRD; r.imm = w >> 20 & 0x7F; r.dd = rd & 7; return r; }
    if (w == 0x00000073u) { r.op = ECALL; return r; }
    if (opc == 0x73 && (f3 == 1 || f3 == 2 || f3 == 3 || f3 == 5 || f3 == 6 || f3 == 7)) {
        static const int32_t Cs[8] = {0, CSRRW, CSRRS, CSRRC, 0, CSRRWI, CSRRSI, CSRRCI};
        r.op = Cs[f3]; r.rd = rd; r.rs1 = rs1; r.imm = w >> 20; return r;
    }
    if (w == 0x00100073u) { r.op = EBREAK; return r; }
    if (opc == 0x0F) { r.op = FENCE; return r; }
    return r;
}

static uint32_t alu(int32_t op, uint32_t a, uint32_t b) {
    int64_t sa = sx(a, 32), sb = sx(b, 32);
    uint64_t r = 0;
    switch (op) {
    case ADD: case ADDI: r = (uint64_t)a + b; break;
    case SUB: r = (uint64_t)a - b; break;
    case SLL: case SLLI: r = (uint64_t)a << (b & 31); break;
    case SRL: case SRLI: r = a >> (b & 31); break;
    case SRA: case SRAI: r = (uint64_t)(sa >> (b & 31)); break;
    case SLT: case SLTI: r = sa < sb; break;
    case SLTU: case SLTIU: r = a < b; break;
    case XOR: case XORI: r = a ^ b; break;
    case OR: case ORI: r = a | b; break;
    case AND: case ANDI: r = a & b; break;
    case MUL: r = (uint64_t)a * b; break;
    case MULH: r = (uint64_t)((sa * sb) >> 32); break;
    case MULHSU: r = (uint64_t)((sa * (int64_t)b) >> 32); break;
    case MULHU: r = ((uint64_t)a * b) >> 32; break;
    case DIV: r = sb == 0 ? M32 : ((sa == -(1LL << 31) && sb == -1) ? (uint64_t)sa : (uint64_t)(sa / sb)); break;
    case DIVU: r = b == 0 ? M32 : a / b; break;
    case REM: r = sb == 0 ? (uint64_t)sa : ((sa == -(1LL << 31) && sb == -1) ? 0 : (uint64_t)(sa % sb)); break;
    case REMU: r = b == 0 ? a : a % b; break;
    case SH1ADD: r = ((uint64_t)a << 1) + b; break;
    case SH2ADD: r = ((uint64_t)a << 2) + b; break;
    case SH3ADD: r = ((uint64_t)a << 3) + b; break;
    default: r = 0;
    }
    return (uint32_t)(r & M32);
}

static int taken(int32_t op, uint32_t a, uint32_t b) {
    int64_t sa = sx(a, 32), sb = sx(b, 32);
    switch (op) {
    case BEQ: return a == b;
    case BNE: return a != b;
    case BLT: return sa < sb;
    case BGE: return sa >= sb;
    case BLTU: return a < b;
    default: return a >= b; /* BGEU */
    }
}

static int32_t nibbles_used(uint32_t v) {
    int32_t n = 0;
    for (int i = 0; i < 8; i++) n += (v >> (4 * i)) != 0;
    return n;
}

/* ref.py:212-222 */
static int32_t div_start(int32_t op, uint32_t a, uint32_t b) {
    int sb = (op == DIV || op == REM) && (b >> 31);
    int32_t da = nibbles_used(a), db = nibbles_used(sb ? (~b & M32) : b);
    if (b == 0) return 0;
    int32_t k = 7 - da + db;
    if (k < 0) k = 0;
    return k > 8 ? 8 : k;
}

static int64_t is_in_rom(uint32_t t) { return t % 4 == 0 && t >= ROM_BASE && t < ROM_BASE + 4 * ROM_WORDS; }

/* ======================================================================================== */
/* the pre-decoded ROM word (ref.py:335-380)                                                 */
/* ======================================================================================== */

static uint32_t pack(int32_t uop, uint32_t rd, uint32_t rs1, uint32_t rs2, uint32_t spare) {
    uint32_t b0 = (uint32_t)uop | (spare & 1) << 7;
    uint32_t b1 = rd << 3 | (spare >> 1 & 7);
    uint32_t b2 = rs1 << 3 | (spare >> 4 & 7);
    uint32_t b3 = rs2 << 3 | (spare >> 7 & 7);
    return b0 | b1 << 8 | b2 << 16 | b3 << 24;
}

static int64_t csr_read(inst in, int *ok) {
    int pure = (in.op == CSRRS || in.op == CSRRC || in.op == CSRRSI || in.op == CSRRCI) && in.rs1 == 0;
    *ok = 0;
    if (!pure) return 0;
    switch (in.imm) {
    case 0xC00: case 0xC01: case 0xC02: case 0xC80: case 0xC81: case 0xC82: case 0xF14: *ok = 1; return 0;
    case 0x301: *ok = 1; return MISA;
    default: return 0;
    }
}

uint32_t qxo_rom_word(uint32_t w, uint32_t pc) {
    inst in = decode(w);
    int32_t op = in.op;
    int64_t imm = in.imm;
    if (op >= CSRRW) {
        int ok;
        int64_t v = csr_read(in, &ok);
        if (!ok) return pack(ILLEGAL, 0, 0, 0, 0);
        return v ? pack(MISA_OP, in.rd, 0, 0, 0) : pack(LUI, in.rd, 0, 0, 0);
    }
    if (op == LUI || op == AUIPC) {
        uint32_t up = (uint32_t)(((op == LUI ? imm : (int64_t)pc + imm) >> 12) & 0xFFFFF);
        return pack(op, in.rd, up & 31, up >> 5 & 31, up >> 10);
    }
    if ((op >= ADDI && op <= SRAI) || (op >= LB && op <= LHU) || op == JALR) {
        uint32_t i = (uint32_t)(imm & 0xFFF);
        return pack(op, in.rd, in.rs1, i & 31, i >> 5);
    }
    if (op >= SB && op <= SW) {
        uint32_t i = (uint32_t)(imm & 0xFFF);
        return pack(op, in.rs2, in.rs1, i & 31, i >> 5);
    }
    if (op >= BEQ && op <= BGEU) {
        uint32_t t = (uint32_t)(((int64_t)pc + imm) & M32);
        uint32_t off = (uint32_t)((imm >> 2) & 0x7FF);
        uint32_t bad = !is_in_rom(t);
        return pack(op, off & 31, in.rs1, in.rs2, off >> 5 | bad << 6);
    }
    if (op == JAL) {
        uint32_t t = (uint32_t)(((int64_t)pc + imm) & M32);
        uint32_t wi = ((t - ROM_BASE) >> 2) & 0xFFFF;
        uint32_t bad = !is_in_rom(t);
        return pack(op, in.rd, wi & 31, wi >> 5 & 31, wi >> 10 | bad << 6);
    }
    if (op == ECALL) return pack(op, 0, 17, 10, 0);
    if (op >= BMAC && op <= BSCAN) {
        if (op == BPRD) return pack(op, 0, 0, (uint32_t)(imm & 31), (uint32_t)(imm >> 5) | (uint32_t)in.dd << 7);
        return pack(op, in.rd, in.rs1, in.rs2, 0);
    }
    if (op == EBREAK || op == FENCE || op == ILLEGAL) return pack(op, 0, 0, 0, 0);
    return pack(op, in.rd, in.rs1, in.rs2, 0);
}

/* ======================================================================================== */
/* the traced machine (ref.py:386-605)                                                       */
/* ======================================================================================== */

typedef struct {
    uint32_t rom[ROM_WORDS];   /* instruction words from ROM_BASE */
    uint32_t ram[RAM_WORDS];   /* words from RAM_BASE */
    uint8_t drom[4 * DROM_WORDS];
    uint32_t drom_len;         /* bytes of DROM content (the rest reads as 0) */
    uint32_t x[32];
    uint32_t anchor, n;
    int32_t halted, fault_cause;
    uint32_t fault_pc;
    int64_t steps, exit_code;
    uint8_t bn[8][128];
    uint8_t out[4096];
    int32_t n_out;
} qxo_machine;

int64_t qxo_machine_size(void) { return (int64_t)sizeof(qxo_machine); }

/* Machine.from_program (ref.py:401-414): text at ROM_BASE, data bytes at data_base. */
void qxo_machine_init(qxo_machine *m, const uint32_t *text, int32_t n_text, const uint8_t *data,
                      int32_t n_data, uint32_t data_base, const uint8_t *rodata, int32_t n_rodata,
                      uint32_t entry) {
    memset(m, 0, sizeof(*m));
    for (int32_t i = 0; i < n_text && i < (int32_t)ROM_WORDS; i++) m->rom[i] = text[i];
    for (int32_t i = 0; i < n_data; i++) {
        uint32_t a = data_base + (uint32_t)i;
        if (a < 4 * RAM_WORDS) m->ram[a >> 2] |= (uint32_t)data[i] << (8 * (a & 3));
    }
    for (int32_t i = 0; i < n_rodata && i < (int32_t)(4 * DROM_WORDS); i++) m->drom[i] = rodata[i];
    m->drom_len = (uint32_t)n_rodata;
    m->x[2] = SP_INIT;
    m->anchor = (entry - ROM_BASE) >> 2;
    m->fault_cause = -1;
    m->exit_code = -1;
}

typedef struct {
    uint32_t x[32];
    uint32_t anchor, n;
    uint32_t ram[RAM_WORDS];
} qxo_state;

void qxo_machine_state(const qxo_machine *m, qxo_state *st);

static void fault(qxo_machine *m, tokbuf *t, int32_t cause, uint32_t pc) {
    m->halted = 1;
    m->fault_cause = cause;
    m->fault_pc = pc;
    put(t, tokf(F_FLT, cause));
    for (int i = 0; i < 8; i++) put(t, tokf(F_HEX, pc >> (4 * (7 - i)) & 15));
    put(t, tokc(C_HALT));
}

static void commit_rd(qxo_machine *m, tokbuf *t, inst in, uint32_t v) {
    m->n++;
    if (in.rd) { m->x[in.rd] = v; value_record(t, v); }
    else put(t, tokc(C_NT));
}

static uint8_t ram_byte(qxo_machine *m, uint32_t ea) {
    ea &= 0x7FFF;
    return m->ram[ea >> 2] >> (8 * (ea & 3)) & 0xFF;
}

static void digit_op(qxo_machine *m, tokbuf *t, inst in, uint32_t a, uint32_t b) {
    int32_t op = in.op;
    m->n++;
    if (op == BPRD) {
        int32_t c = 48 + m->bn[in.dd][in.imm];
        if (m->n_out < 4096) m->out[m->n_out++] = (uint8_t)c;
        put(t, tokf(F_BYTE, c));
        return;
    }
    if (op == BSCAN) {
        uint32_t n = 0;
        while (n < 63) { uint8_t ch = ram_byte(m, a + n); if (ch < 48 || ch > 57) break; n++; }
        for (uint32_t i = 0; i < n; i++) put(t, tokc(C_SC));
        if (in.rd) { m->x[in.rd] = n; value_record(t, n); }
        else put(t, tokc(C_NT));
        return;
    }
    uint32_t dd = b & 7, ds = b >> 3 & 7, ovw = b >> 6 & 1, n = b >> 7 & 63, off = b >> 13 & 127;
    uint32_t mm = b >> 20 & 15;
    if (mm > 9) mm = 9;
    if (op == BGET) {
        uint32_t v = m->bn[dd][off];
        if (in.rd) { m->x[in.rd] = v; value_record(t, v); }
        else put(t, tokc(C_NT));
        return;
    }
    int32_t c = 0;
    for (uint32_t i = 0; i < n; i++) {
        uint32_t r = i + off;
        int32_t d = r < 128 ? m->bn[dd][r] : 0, v;
        if (op == BLD) { v = ram_byte(m, a - 1 - i) & 15; if (v > 9) v = 9; c = 0; }
        else if (op == BMAC) {
            v = (ovw ? 0 : d) + m->bn[ds][i] * (int32_t)mm + c;
            c = v / 10; v = v % 10;
        } else {
            v = d - m->bn[ds][i] * (int32_t)mm - c;
            int32_t r10 = ((v % 10) + 10) % 10; /* Python's v % 10 */
            c = (r10 - v) / 10;
            v = r10;
        }
        if (r < 128) m->bn[dd][r] = (uint8_t)v;
        put(t, tokf(F_BD, v | c << 4));
    }
    if (in.rd) { m->x[in.rd] = (uint32_t)c; value_record(t, (uint32_t)c); }
    else put(t, tokc(C_NT));
}

static void record(qxo_machine *m, tokbuf *t) {
    if (m->n == N_MAX) {
        uint32_t w = m->anchor + m->n;
        m->anchor = w;
        m->n = 0;
        put(t, tokf(F_R, w));
        return;
    }
    uint32_t pc = ROM_BASE + 4 * (m->anchor + m->n);
    uint32_t word = m->rom[((pc - ROM_BASE) >> 2) & (ROM_WORDS - 1)];
    inst in = decode(word);
    int32_t op = in.op;
    uint32_t a = m->x[in.rs1], b = m->x[in.rs2];
    m->steps++;
    if (op == LUI || op == AUIPC || op >= CSRRW) {
        int ok = 1;
        int64_t v = op == LUI ? in.imm : (op == AUIPC ? (int64_t)pc + in.imm : csr_read(in, &ok));
        if (!ok) { fault(m, t, FAULT_ILLEGAL, pc); return; }
        commit_rd(m, t, in, (uint32_t)(v & M32));
        return;
    }
    if (op == JAL || op == JALR || ((op >= BEQ && op <= BGEU) && taken(op, a, b))) {
        uint32_t target = op == JALR ? (uint32_t)(((int64_t)a + in.imm) & M32 & ~1u)
                                     : (uint32_t)(((int64_t)pc + in.imm) & M32);
        if (!is_in_rom(target)) { fault(m, t, FAULT_BAD_JUMP, pc); return; }
        if ((op == JAL || op == JALR) && in.rd) m->x[in.rd] = (pc + 4) & M32;
        m->anchor = (target - ROM_BASE) >> 2;
        m->n = 0;
        put(t, tokf(F_J, m->anchor));
        return;
    }
    if (op >= BEQ && op <= BGEU) { m->n++; put(t, tokc(C_NT)); return; }
    if (op >= LB && op <= LHU) {
        uint32_t ea = (uint32_t)(((int64_t)a + in.imm) & M32);
        uint32_t n = (op == LB || op == LBU) ? 1 : ((op == LH || op == LHU) ? 2 : 4);
        if (ea % n) { fault(m, t, FAULT_MIS_LOAD, pc); return; }
        uint32_t word2;
        if (ea < 4 * RAM_WORDS) word2 = m->ram[ea >> 2];
        else if (ea >= DROM_BASE && ea < DROM_BASE + 4 * DROM_WORDS) {
            uint32_t o = (ea - DROM_BASE) & ~3u;
            word2 = 0;
            for (int i = 0; i < 4; i++) word2 |= (uint32_t)(o + i < m->drom_len ? m->drom[o + i] : 0) << (8 * i);
        } else { fault(m, t, FAULT_LOAD_RANGE, pc); return; }
        uint32_t wv = (uint32_t)((word2 >> (8 * (ea & 3))) & ((1ULL << (8 * n)) - 1));
        uint32_t v = (op == LB || op == LH) ? (uint32_t)(sx(wv, 8 * n) & M32) : wv;
        commit_rd(m, t, in, v);
        return;
    }
    if (op >= SB && op <= SW) {
        uint32_t ea = (uint32_t)(((int64_t)a + in.imm) & M32);
        uint32_t n = op == SB ? 1 : (op == SH ? 2 : 4);
        if (ea % n) { fault(m, t, FAULT_MIS_STORE, pc); return; }
        if (ea >= 4 * RAM_WORDS) { fault(m, t, FAULT_STORE_RANGE, pc); return; }
        uint32_t i = ea >> 2, w4 = i >> 4 & 1;
        m->n++;
        if (op == SW) { m->ram[i] = b; put(t, tokc(w4 ? C_ST1 : C_ST0)); return; }
        uint32_t sh = 8 * (ea & 3);
        uint32_t mask = (uint32_t)((1ULL << (8 * n)) - 1);
        uint32_t mv = (m->ram[i] & ~(mask << sh) & M32) | (b & mask) << sh;
        m->ram[i] = mv;
        put(t, tokf(F_V, mv & 0x7FFF));
        put(t, tokf(F_V, mv >> 15 & 0x7FFF));
        put(t, tokf(F_V, mv >> 30));
        put(t, tokc(w4 ? C_SS1 : C_SS0));
        return;
    }
    if (op == ECALL) {
        uint32_t call = m->x[17], arg = m->x[10];
        if (call == 1) {
            /* ref.py:522 reads `b & 0x1FF < 256`, which Python parses as b & (0x1FF < 256) */
            if ((arg & 1) && m->n_out < 4096) m->out[m->n_out++] = arg & 0xFF;
            m->n++;
            put(t, tokf(F_BYTE, arg & 0x1FF));
            return;
        }
        if (call == 93) { m->halted = 1; m->exit_code = arg; m->n++; put(t, tokc(C_HALT)); return; }
        fault(m, t, FAULT_ECALL, pc);
        return;
    }
    if (op == EBREAK) { fault(m, t, FAULT_EBREAK, pc); return; }
    if (op == FENCE) { m->n++; put(t, tokc(C_NT)); return; }
    if (op == ILLEGAL) { fault(m, t, FAULT_ILLEGAL, pc); return; }
    if (op >= BMAC && op <= BSCAN) { digit_op(m, t, in, a, b); return; }
    if (op >= DIV && op <= REMU) {
        m->n++;
        if (!in.rd) { put(t, tokc(C_NT)); return; }
        int sgn = op == DIV || op == REM;
        int sa = sgn && (a >> 31), sb = sgn && (b >> 31);
        uint32_t ua = sa ? (uint32_t)(-(int64_t)a) : a, ub = sb ? (uint32_t)(-(int64_t)b) : b;
        uint32_t q = ub ? ua / ub : M32;
        int32_t k0 = div_start(op, a, b);
        uint32_t qs = (sa != sb && b) ? (uint32_t)(-(int64_t)q) : q;
        uint32_t res = (op == DIV || op == DIVU) ? qs : (uint32_t)(((uint64_t)a - (uint64_t)qs * b) & M32);
        m->x[in.rd] = res;
        put(t, tokf(F_QS, k0));
        for (int32_t k = k0; k < 8; k++) put(t, tokf(F_QD, k << 4 | (q >> (4 * (7 - k)) & 15)));
        value_record(t, res);
        return;
    }
    if (op >= ADDI && op <= SRAI) { commit_rd(m, t, in, alu(op, a, (uint32_t)(in.imm & M32))); return; }
    commit_rd(m, t, in, alu(op, a, b));
}

/* Machine.run (ref.py:600-605): GO, then records while not halted and fewer than max_tokens
 * tokens so far. Writes at most cap tokens; returns the trace length. */
int64_t qxo_machine_run(qxo_machine *m, int64_t max_tokens, int32_t *toks, int64_t cap) {
    tokbuf t = {toks, 0, cap};
    put(&t, tokc(C_GO));
    while (!m->halted && t.n < max_tokens) record(m, &t);
    return t.n;
}

/* The free-running comparison of n predicted tokens: toks[0..n] = GO and the first n tokens the
 * executor must predict (a machine that halts earlier gives a shorter trace: the return value
 * is the trace length, at most n + 1), and st = the machine state after the last record whose
 * final token is among the n inputs the executor has consumed (toks[0..n-1]).  Two passes over
 * copies of m: the first finds the record boundaries, the second stops at the last one. */
int64_t qxo_trace_and_state(const qxo_machine *m0, int64_t n, int32_t *toks, qxo_state *st) {
    qxo_machine *m = (qxo_machine *)malloc(sizeof(qxo_machine));
    memcpy(m, m0, sizeof(*m));
    tokbuf t = {toks, 0, n + 1};
    put(&t, tokc(C_GO));
    int64_t complete = 0; /* records whose final token index <= n - 1 */
    while (!m->halted && t.n < n + 1) {
        record(m, &t);
        if (t.n <= n) complete++;
    }
    int64_t len = t.n < n + 1 ? t.n : n + 1;
    memcpy(m, m0, sizeof(*m));
    int32_t scratch[256];
    for (int64_t r = 0; r < complete; r++) {
        tokbuf u = {scratch, 0, 256};
        record(m, &u);
    }
    qxo_machine_state(m, st);
    free(m);
    return len;
}

/* One record (after a snapshot); returns its token count. */
int64_t qxo_machine_record(qxo_machine *m, int32_t *toks, int64_t cap) {
    tokbuf t = {toks, 0, cap};
    record(m, &t);
    return t.n;
}

/* ref.div_record (ref.py:240-243) of DIV (0), DIVU (1), REM (2), REMU (3) through the machine's
 * own DIV path: returns the record length. */
int64_t qxo_div_record(int32_t op, uint32_t a, uint32_t b, int32_t *toks, int64_t cap) {
    static const int32_t OPS[4] = {DIV, DIVU, REM, REMU};
    qxo_machine *m = (qxo_machine *)calloc(1, sizeof(qxo_machine));
    m->x[10] = a;
    m->x[11] = b;
    static const uint32_t F3[4] = {4, 5, 6, 7};
    m->rom[0] = 1u << 25 | 11u << 20 | 10u << 15 | F3[op] << 12 | 12u << 7 | 0x33; /* op a2, a0, a1 */
    (void)OPS;
    tokbuf t = {toks, 0, cap};
    record(m, &t);
    free(m);
    return t.n;
}

/* ======================================================================================== */
/* snapshot / readback (core.py:1177-1270)                                                   */
/* ======================================================================================== */

#define A_REF 16777216.0f
#define A_BIT 128.0f

typedef struct {
    int32_t sub, vh0;      /* head sublayer (index among head sublayers), first value head */
} qxo_tpos;

typedef struct {
    qxo_tpos pc, count, j, vcnt, regs[3], quo[4], rom[32], drom[16], bn1[4], bn2[4], ram[32];
    int32_t reg_cols[32][8];
} qxo_tables;

static float *row_of(float **S, const int32_t *V, qxo_tpos p, int32_t x, int32_t r) {
    return S[p.sub] + (((int64_t)(p.vh0 + x)) * HD + r) * HD;
}

static void ballast(float *row) { row[0] = A_REF; row[1] = A_REF; }

/* byte_rows (core.py:1194-1212): the row pair layout of a 32-bit word table */
static void byte_table(float **S, const int32_t *V, const qxo_tpos *pos, int32_t n_heads,
                       const uint32_t *words, int64_t n_words) {
    int64_t per = n_words / n_heads;
    for (int32_t h = 0; h < n_heads; h++)
        for (int32_t x = 0; x < 2; x++) {
            for (int32_t r = 0; r < 128; r++) ballast(row_of(S, V, pos[h], x, r));
            for (int64_t wl = 0; wl < per / 2; wl++) {
                uint32_t wv = words[h * per + x * (per / 2) + wl];
                if (!wv) continue;
                int64_t pp = wl >> 4, half = wl >> 3 & 1, k = wl & 7;
                float *row = row_of(S, V, pos[h], x, (int32_t)(pp + 64 * half));
                for (int b = 0; b < 4; b++) row[2 + 32 * half + 4 * k + b] = (float)(wv >> (8 * b) & 0xFF);
            }
        }
}

/* Fill the head states of one machine from its traced state (as at a record's start). S[i]
 * points at this machine's [V_i][HD][HD] block of the i-th head sublayer, which must be zero. */
void qxo_snapshot(const qxo_tables *tb, const qxo_machine *m, float **S, const int32_t *V) {
    float *r = row_of(S, V, tb->pc, 0, 0);
    ballast(r);
    for (int i = 0; i < 16; i++) r[2 + i] = (m->anchor >> i & 1) ? A_BIT : 0.0f;
    const qxo_tpos *ctr[3] = {&tb->count, &tb->j, &tb->vcnt};
    for (int c = 0; c < 3; c++) {
        uint32_t k = c == 0 ? m->n : 0;
        row_of(S, V, *ctr[c], 0, 0)[2] = ldexpf(A_BIT, -(int)k);
        ballast(row_of(S, V, *ctr[c], 0, 1));
    }
    for (int p = 0; p < 3; p++)
        for (int reg = 1; reg < 32; reg++) {
            float *row = row_of(S, V, tb->regs[p], 0, reg);
            ballast(row);
            for (int i = 0; i < 32; i++)
                if (m->x[reg] >> i & 1) row[tb->reg_cols[i][0]] = A_BIT;
        }
    for (int h = 0; h < 4; h++)
        for (int x = 0; x < 2; x++) ballast(row_of(S, V, tb->quo[h], x, 0));
    static uint32_t rom_pd[ROM_WORDS]; /* not re-entrant: the oracle is single-threaded here */
    for (uint32_t i = 0; i < ROM_WORDS; i++) rom_pd[i] = m->rom[i] ? qxo_rom_word(m->rom[i], ROM_BASE + 4 * i) : 0;
    byte_table(S, V, tb->rom, 32, rom_pd, ROM_WORDS);
    static uint32_t drom_w[DROM_WORDS];
    for (uint32_t i = 0; i < DROM_WORDS; i++) {
        uint32_t w = 0;
        for (int b = 0; b < 4; b++) w |= (uint32_t)(4 * i + b < m->drom_len ? m->drom[4 * i + b] : 0) << (8 * b);
        drom_w[i] = w;
    }
    byte_table(S, V, tb->drom, 16, drom_w, DROM_WORDS);
    for (int port = 0; port < 2; port++)
        for (int h = 0; h < 4; h++)
            for (int x = 0; x < 2; x++)
                for (int rr = 0; rr < 128; rr++) {
                    float *row = row_of(S, V, port ? tb->bn2[h] : tb->bn1[h], x, rr);
                    ballast(row);
                    uint8_t dg = m->bn[2 * h + x][rr];
                    for (int b = 0; b < 4; b++) row[2 + b] = (dg >> b & 1) ? A_BIT : 0.0f;
                }
    for (uint32_t wi = 0; wi < RAM_WORDS; wi++) {
        if (!m->ram[wi]) continue;
        uint32_t h = (wi & 15) | (wi >> 12) << 4;
        float *row = row_of(S, V, tb->ram[h], wi >> 4 & 1, wi >> 5 & 127);
        ballast(row);
        for (int i = 0; i < 32; i++) row[2 + i] = (m->ram[wi] >> i & 1) ? A_BIT : 0.0f;
    }
}


/* Registers from the rs1 port (a bit is set when any of its source columns is), PC anchor and n
 * from the pc / count heads, RAM words from block A + block B of their row (core.py:820-852). */
void qxo_readback(const qxo_tables *tb, float **S, const int32_t *V, qxo_state *st) {
    memset(st, 0, sizeof(*st));
    for (int reg = 1; reg < 32; reg++) {
        const float *row = row_of(S, V, tb->regs[0], 0, reg);
        uint32_t v = 0;
        for (int i = 0; i < 32; i++)
            for (int c = 0; c < 8 && tb->reg_cols[i][c] >= 0; c++)
                if (row[tb->reg_cols[i][c]] != 0.0f) { v |= 1u << i; break; }
        st->x[reg] = v;
    }
    const float *pc = row_of(S, V, tb->pc, 0, 0);
    for (int i = 0; i < 16; i++)
        if (pc[2 + i] != 0.0f) st->anchor |= 1u << i;
    float c2 = row_of(S, V, tb->count, 0, 0)[2];
    st->n = c2 > 0.0f ? (uint32_t)lrintf(log2f(A_BIT / c2)) : 0xFFFFFFFFu;
    for (uint32_t wi = 0; wi < RAM_WORDS; wi++) {
        uint32_t h = (wi & 15) | (wi >> 12) << 4;
        const float *row = row_of(S, V, tb->ram[h], wi >> 4 & 1, wi >> 5 & 127);
        uint32_t v = 0;
        for (int i = 0; i < 32; i++)
            if (row[2 + i] + row[34 + i] != 0.0f) v |= 1u << i;
        st->ram[wi] = v;
    }
}

/* FNV-1a 64 over 32-bit words (little-endian bytes) */
uint64_t qxo_fnv1a(const uint32_t *w, int64_t n, uint64_t h) {
    for (int64_t i = 0; i < n; i++)
        for (int b = 0; b < 4; b++) {
            h ^= (w[i] >> (8 * b)) & 0xFF;
            h *= 0x100000001b3ULL;
        }
    return h;
}

/* The machine-state checksum: x1..x31, anchor, n, the 8,192 RAM words, in that order. */
uint64_t qxo_state_checksum(const qxo_state *st) {
    uint64_t h = 0xcbf29ce484222325ULL;
    h = qxo_fnv1a(st->x + 1, 31, h);
    h = qxo_fnv1a(&st->anchor, 1, h);
    h = qxo_fnv1a(&st->n, 1, h);
    return qxo_fnv1a(st->ram, RAM_WORDS, h);
}

void qxo_machine_state(const qxo_machine *m, qxo_state *st) {
    memcpy(st->x, m->x, sizeof(st->x));
    st->x[0] = 0;
    st->anchor = m->anchor;
    st->n = m->n;
    memcpy(st->ram, m->ram, sizeof(st->ram));
}

/* ======================================================================================== */
/* gated delta-rule decode step                                                              */
/* ======================================================================================== */

/* For every (b, h): S <- alpha S; kv = S^T k; delta = beta (v - kv); S <- S + k (x) delta;
 * o = S^T q.  Sums run over the key index i = 0..127 in order, each product rounded before it
 * is added (no fused multiply-add).  S: [BH][dk][dv]; q, k: [BH][dk]; v, o: [BH][dv]. */
void qxo_gdn_step(int64_t BH, int32_t dk, int32_t dv, float *S, const float *q, const float *k,
                  const float *v, const float *alpha, const float *beta, float *o) {
    float *kv = (float *)malloc(sizeof(float) * dv);
    for (int64_t bh = 0; bh < BH; bh++) {
        float *s = S + bh * dk * dv;
        const float *kk = k + bh * dk, *qq = q + bh * dk, *vv = v + bh * dv;
        float a = alpha[bh], be = beta[bh];
        for (int64_t i = 0; i < (int64_t)dk * dv; i++) s[i] = s[i] * a;
        for (int j = 0; j < dv; j++) {
            float acc = 0.0f;
            for (int i = 0; i < dk; i++) acc = acc + s[i * dv + j] * kk[i];
            kv[j] = acc;
        }
        for (int j = 0; j < dv; j++) kv[j] = (vv[j] - kv[j]) * be; /* delta */
        for (int i = 0; i < dk; i++)
            for (int j = 0; j < dv; j++) s[i * dv + j] = s[i * dv + j] + kk[i] * kv[j];
        for (int j = 0; j < dv; j++) {
            float acc = 0.0f;
            for (int i = 0; i < dk; i++) acc = acc + s[i * dv + j] * qq[i];
            o[bh * dv + j] = acc;
        }
    }
    free(kv);
}
