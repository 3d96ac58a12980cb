// qx_exec.cu -- the persistent per-token kernel of the executor.
//
// One CTA owns 32 machines (one per lane) and runs the plan's phase program for every token:
// the residual stream of its machines stays in shared memory as rows of 33 floats (lanes walk
// machines: conflict-free), the head states S stay in HBM and only the rows a key writes or a
// query reads are touched.  A phase ends with __syncthreads(); no grid-wide synchronisation is
// ever needed because machines never exchange data.
//
// Semantics follow the reference executor (ERV = experimental/riscv):
//   FFN units    coef * a * relu(b) into the node's dim          ERV/chipformer/rv/tritonexec.py:47-71
//   heads        q/k/v/z relu projections over the lagged input,
//                decay (a: 0 -> 1, 110 -> 1/2, else 0) of the first nrows rows, the one-row
//                write at the key's argmax when beta == 1, the read of at most QHOT query
//                rows, out = o / sqrt_rn(ref / 128), y += out * z * w  tritonexec.py:105-148
//   apply        the lag history moves on after a head sublayer     tritonexec.py:151-170
//   decode       output code -> token -> next embedding             ERV/chipformer/rv/fastexec.py:298-307
#include <cuda_runtime.h>

#include "qx_exec.cuh"

namespace {

__device__ __forceinline__ float relu(float v) { return v > 0.0f ? v : 0.0f; }

__device__ __forceinline__ float sm_row(const float *sm, uint32_t row, int lane) {
    return row == QX_NONE ? 0.0f : sm[row * QX_RP + lane];
}

// sum of w * sm[row][lane] over packed entries (row | bf16 weight << 16), 4 per uint4
__device__ __forceinline__ float form_sum(const float *sm, const uint32_t *nnz, uint32_t nnz0,
                                          uint32_t nnz4, int lane) {
    const uint4 *q = reinterpret_cast<const uint4 *>(nnz + nnz0);
    float acc0 = 0.0f, acc1 = 0.0f;
    uint32_t k = 0;
    for (; k + 1 < nnz4; k += 2) {
        uint4 e = __ldg(q + k), f = __ldg(q + k + 1);
        acc0 = fmaf(__uint_as_float(e.x & 0xFFFF0000u), sm[(e.x & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(e.y & 0xFFFF0000u), sm[(e.y & 0xFFFFu) * QX_RP + lane], acc1);
        acc0 = fmaf(__uint_as_float(e.z & 0xFFFF0000u), sm[(e.z & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(e.w & 0xFFFF0000u), sm[(e.w & 0xFFFFu) * QX_RP + lane], acc1);
        acc0 = fmaf(__uint_as_float(f.x & 0xFFFF0000u), sm[(f.x & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(f.y & 0xFFFF0000u), sm[(f.y & 0xFFFFu) * QX_RP + lane], acc1);
        acc0 = fmaf(__uint_as_float(f.z & 0xFFFF0000u), sm[(f.z & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(f.w & 0xFFFF0000u), sm[(f.w & 0xFFFFu) * QX_RP + lane], acc1);
    }
    if (k < nnz4) {
        uint4 e = __ldg(q + k);
        acc0 = fmaf(__uint_as_float(e.x & 0xFFFF0000u), sm[(e.x & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(e.y & 0xFFFF0000u), sm[(e.y & 0xFFFFu) * QX_RP + lane], acc1);
        acc0 = fmaf(__uint_as_float(e.z & 0xFFFF0000u), sm[(e.z & 0xFFFFu) * QX_RP + lane], acc0);
        acc1 = fmaf(__uint_as_float(e.w & 0xFFFF0000u), sm[(e.w & 0xFFFFu) * QX_RP + lane], acc1);
    }
    return acc0 + acc1;
}

// argmax over 128 channel values held 4 per lane (channel = lane + 32 i): the first maximum
__device__ __forceinline__ void warp_argmax(float v, int idx, float &bv, int &bi) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        int oi = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
        if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    bv = v;
    bi = idx;
}

__device__ __forceinline__ void lane_best(const float c[4], int lane, float &v, int &idx) {
    v = c[0];
    idx = lane;
#pragma unroll
    for (int i = 1; i < 4; i++)
        if (c[i] > v) { v = c[i]; idx = lane + 32 * i; }
}

__device__ __forceinline__ uint64_t fnv_word(uint64_t h, uint32_t w) {
#pragma unroll
    for (int b = 0; b < 4; b++) {
        h ^= (w >> (8 * b)) & 0xFFu;
        h *= 0x100000001b3ULL;
    }
    return h;
}

}  // namespace

template <int RUN>
__global__ void __launch_bounds__(QX_NT, 1)
    qx_token_kernel(const __grid_constant__ QxDev d, int32_t n_tokens, int32_t *tokens) {
    extern __shared__ __align__(16) float sm[];
    int *ksel = reinterpret_cast<int *>(sm + (size_t)d.smem_rows * QX_RP);  // [slots][32]
    int *qsel = ksel + d.ksel_slots * 32;                                    // [slots][qhot][32]
    int *dec_i = qsel + d.ksel_slots * d.qhot_max * 32;                      // [2][32]
    float *dec_pay = reinterpret_cast<float *>(dec_i + 64);                  // [16][32]
    unsigned int *touched = reinterpret_cast<unsigned int *>(dec_pay + 16 * 32);  // state rows
    if (threadIdx.x == 0) *touched = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int m = blockIdx.x * 32 + lane;  // this lane's machine
    const bool act = m < d.B;
    const int mbase = blockIdx.x * 32;

    // run mode: the embedding of each machine's next input comes from x
    uint64_t hash = 0;
    int64_t count = 0, halt_at = -1;
    if (RUN) {
        for (int i = warp; i < d.n_born0; i += QX_NW) {
            uint2 p = d.pairs[i];
            sm[p.x * QX_RP + lane] = act ? d.x[(size_t)m * d.D + p.y] : 0.0f;
        }
        if (warp == 0 && act) {
            hash = d.hash[m];
            count = d.count[m];
            halt_at = d.halt_at[m];
        }
        __syncthreads();
    }
    const qx_phase *prog = RUN ? d.run_prog : d.step_prog;
    for (int32_t t = 0; t < n_tokens; t++) {
        for (int pc = 0;; pc++) {
            const qx_phase ph = prog[pc];
            if (ph.kind == QX_PH_END) break;
            switch (ph.kind) {
            case QX_PH_ZERO:
                for (uint32_t i = warp; i < ph.b; i += QX_NW) sm[d.rows[ph.a + i] * QX_RP + lane] = 0.0f;
                break;
            case QX_PH_LOADX:
                for (uint32_t i = warp; i < ph.b; i += QX_NW) {
                    uint2 p = d.pairs[ph.a + i];
                    sm[p.x * QX_RP + lane] = act ? d.x[(size_t)m * d.D + p.y] : 0.0f;
                }
                break;
            case QX_PH_WRITEOUT:
                if (act)
                    for (uint32_t i = warp; i < ph.b; i += QX_NW) {
                        uint2 p = d.pairs[ph.a + i];
                        d.x[(size_t)m * d.D + p.y] = sm[p.x * QX_RP + lane];
                    }
                break;
            case QX_PH_APPLY:
                for (uint32_t i = warp; i < ph.b; i += QX_NW) {
                    uint2 p = d.pairs[ph.a + i];
                    sm[p.x * QX_RP + lane] += sm[p.y * QX_RP + lane];
                }
                break;
            case QX_PH_STAGE: {
                // stage lags 1..3 of this head sublayer's history into scratch rows, then move
                // the history on: lag 1 <- the input x, lag k <- lag k-1
                float *H = d.hist[ph.c];
                const size_t ne = d.NE[ph.c], bp = d.Bpad;
                for (uint32_t i = warp; i < ph.b; i += QX_NW) {
                    const qx_stage s = d.stages[ph.a + i];
                    float *h = H + (size_t)s.e * bp + m;
                    float h0 = h[0];
                    float h1 = s.ml >= 2 ? h[ne * bp] : 0.0f;
                    float h2 = s.ml >= 3 ? h[2 * ne * bp] : 0.0f;
                    if (s.stage[0] != QX_NONE) sm[s.stage[0] * QX_RP + lane] = h0;
                    if (s.stage[1] != QX_NONE) sm[s.stage[1] * QX_RP + lane] = h1;
                    if (s.stage[2] != QX_NONE) sm[s.stage[2] * QX_RP + lane] = h2;
                    h[0] = sm[s.x_row * QX_RP + lane];
                    if (s.ml >= 2) h[ne * bp] = h0;
                    if (s.ml >= 3) h[2 * ne * bp] = h1;
                }
                break;
            }
            case QX_PH_FORMS: {
                const uint32_t f1 = d.warp_ptr[ph.c + warp + 1];
                for (uint32_t f = d.warp_ptr[ph.c + warp]; f < f1; f++) {
                    const qx_form fm = d.forms[f];
                    sm[fm.dst * QX_RP + lane] = form_sum(sm, d.nnz, fm.nnz0, fm.nnz4, lane);
                }
                break;
            }
            case QX_PH_UNITS: {
                const float x0 = sm[d.one_row * QX_RP + lane];
                const uint32_t n1 = d.warp_ptr[ph.c + warp + 1];
                for (uint32_t n = d.warp_ptr[ph.c + warp]; n < n1; n++) {
                    const qx_node nd = d.nodes[n];
                    float acc = 0.0f;
                    for (uint32_t u = nd.u0; u < nd.u0 + nd.nu; u++) {
                        const qx_unit un = d.units[u];
                        float av = sm_row(sm, un.a, lane) + un.ca * x0;
                        float bv = sm_row(sm, un.b, lane) + un.cb * x0;
                        acc += __fmul_rn(__fmul_rn(un.coef, av), relu(bv));
                    }
                    atomicAdd(&sm[nd.out * QX_RP + lane], acc);
                }
                break;
            }
            case QX_PH_KSEL: {
                // per (key head, machine): lanes walk the 128 channels
                const uint32_t n = ph.b - ph.a;
                for (uint32_t task = warp; task < n * 32; task += QX_NW) {
                    const qx_khead kh = d.kheads[ph.a + task / 32];
                    const int mm = task % 32;
                    const float x0 = sm[d.one_row * QX_RP + mm];
                    float kc[4], qc[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int c = lane + 32 * i;
                        uint16_t kr = d.kq_row[kh.chan + c], qr = d.kq_row[kh.chan + 128 + c];
                        kc[i] = relu(sm_row(sm, kr, mm) + d.kq_c[kh.chan + c] * x0);
                        qc[i] = relu(sm_row(sm, qr, mm) + d.kq_c[kh.chan + 128 + c] * x0);
                    }
                    float bv;
                    int bi, lv;
                    float lvv;
                    lane_best(kc, lane, lvv, lv);
                    warp_argmax(lvv, lv, bv, bi);
                    int npos = 0;
#pragma unroll
                    for (int i = 0; i < 4; i++) npos += __popc(__ballot_sync(0xFFFFFFFFu, kc[i] > 0.0f));
                    const int gm = mbase + mm;
                    if (lane == 0) {
                        ksel[kh.slot * 32 + mm] = bv > 0.0f ? bi : -1;
                        if (npos > 1 && gm < d.B) atomicOr(&d.err[gm], QX_E_KEY);
                    }
                    int qpos = 0;
#pragma unroll
                    for (int i = 0; i < 4; i++) qpos += __popc(__ballot_sync(0xFFFFFFFFu, qc[i] > 0.0f));
                    for (int j = 0; j < d.qhot_max; j++) {
                        int sel = -1;
                        if (j < kh.qhot) {
                            lane_best(qc, lane, lvv, lv);
                            warp_argmax(lvv, lv, bv, bi);
                            sel = bv > 0.0f ? bi : -1;
                            if ((bi & 31) == lane) qc[bi >> 5] = 0.0f;
                        }
                        if (lane == 0) qsel[(kh.slot * d.qhot_max + j) * 32 + mm] = sel;
                    }
                    if (lane == 0 && qpos > kh.qhot && gm < d.B) atomicOr(&d.err[gm], QX_E_QUERY);
                }
                break;
            }
            case QX_PH_VH: {
                // per (value head, machine): lanes own 4 columns each
                const uint32_t n = ph.b - ph.a;
                for (uint32_t task = warp; task < n * 32; task += QX_NW) {
                    const int mm = task % 32, gm = mbase + mm;
                    if (gm >= d.B) continue;
                    const qx_vhead vh = d.vheads[ph.a + task / 32];
                    const float x0 = sm[d.one_row * QX_RP + mm];
                    float *Sb = d.S[vh.hl] + ((size_t)gm * d.V[vh.hl] + vh.vh) * (QX_HD * QX_HD) + lane * 4;
                    unsigned int rows = 0;  // 512-byte row transfers of this task
                    if (vh.nrows > 0) {
                        float av = sm_row(sm, vh.a_row, mm) + vh.ca * x0;
                        float fac = av == 0.0f ? 1.0f : (av == 110.0f ? 0.5f : 0.0f);
                        if (fac != 1.0f) rows += 2 * vh.nrows;
                        if (fac != 1.0f)
                            for (int r = 0; r < vh.nrows; r++) {
                                float4 *p = reinterpret_cast<float4 *>(Sb + r * QX_HD);
                                float4 s = *p;
                                s.x = __fmul_rn(s.x, fac); s.y = __fmul_rn(s.y, fac);
                                s.z = __fmul_rn(s.z, fac); s.w = __fmul_rn(s.w, fac);
                                *p = s;
                            }
                    }
                    const float bv = (sm_row(sm, vh.b_row, mm) + vh.cb * x0) + vh.bconst;
                    const int krow = ksel[vh.slot * 32 + mm];
                    if (krow >= 0 && bv == 1.0f) {
                        float v[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const qx_colform cf = d.vform[vh.col + lane * 4 + i];
                            v[i] = cf.live ? relu(form_sum(sm, d.nnz, cf.nnz0, cf.nnz4, mm) + cf.c * x0) : 0.0f;
                        }
                        *reinterpret_cast<float4 *>(Sb + krow * QX_HD) = make_float4(v[0], v[1], v[2], v[3]);
                        rows++;
                    }
                    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
                    bool any = false;
                    for (int j = 0; j < d.qhot_max; j++) {
                        const int qi = qsel[(vh.slot * d.qhot_max + j) * 32 + mm];
                        if (qi >= 0) {
                            float4 s = *reinterpret_cast<const float4 *>(Sb + qi * QX_HD);
                            o.x = __fadd_rn(o.x, s.x); o.y = __fadd_rn(o.y, s.y);
                            o.z = __fadd_rn(o.z, s.z); o.w = __fadd_rn(o.w, s.w);
                            any = true;
                            rows++;
                        }
                    }
                    if (lane == 0 && rows) atomicAdd(touched, rows);
                    if (!any) continue;
                    float ref = __fadd_rn(__fmul_rn(o.x, o.x), __fmul_rn(o.y, o.y));
                    ref = __shfl_sync(0xFFFFFFFFu, ref, 0);
                    const float norm = __fsqrt_rn(__fdiv_rn(ref, 128.0f));
                    const float oc[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int c = lane * 4 + i;
                        const uint16_t orow = d.out_row[vh.col + c];
                        if (orow == QX_NONE) continue;
                        const qx_colform zf = d.zform[vh.col + c];
                        const float z = zf.live ? relu(form_sum(sm, d.nnz, zf.nnz0, zf.nnz4, mm) + zf.c * x0) : 0.0f;
                        const float out = ref > 0.0f ? __fdiv_rn(oc[i], norm) : 0.0f;
                        atomicAdd(&sm[orow * QX_RP + mm], __fmul_rn(__fmul_rn(out, z), d.out_w[vh.col + c]));
                    }
                }
                break;
            }
            case QX_PH_DECODE: {
                if (warp == 0) {
                    float fam = 0.0f, psum = 0.0f;
                    for (int i = 0; i < d.n_fam; i++)
                        fam = __fadd_rn(fam, __fmul_rn(rintf(sm[d.fam_row[i] * QX_RP + lane]), ldexpf(1.0f, i)));
                    for (int i = 0; i < d.n_pay; i++) {
                        const float p = rintf(sm[d.pay_row[i] * QX_RP + lane]);
                        dec_pay[i * 32 + lane] = p;
                        psum = __fadd_rn(psum, __fmul_rn(p, ldexpf(1.0f, i)));
                    }
                    const long long fraw = (long long)fam;
                    const int fid = fraw < 0 ? 0 : (fraw > d.n_families - 1 ? d.n_families - 1 : (int)fraw);
                    const long long p = (long long)psum;
                    const long long tok = (long long)d.fam_ids[fid] + p;
                    dec_i[lane] = fid;
                    dec_i[32 + lane] = (int)p;
                    if (act) {
                        if (fraw != fid || p < 0 || p >= d.fam_size[fid]) atomicOr(&d.err[m], QX_E_CODE);
                        if (tokens) tokens[(size_t)t * d.B + m] = (int32_t)tok;
                        hash = fnv_word(hash, (uint32_t)tok);
                        count++;
                        if (halt_at < 0 && tok == d.halt_tok) halt_at = count;
                    }
                }
                __syncthreads();
                // next embedding (FreeRun: table row for small families, base + payload bits)
                for (int mm = warp; mm < 32; mm += QX_NW) {
                    const int fid = dec_i[mm], p = dec_i[32 + mm];
                    const int row0 = d.fam_row0[fid];
                    if (row0 >= 0) {
                        int r = row0 + p;
                        r = r < 0 ? 0 : (r > d.n_emb_rows - 1 ? d.n_emb_rows - 1 : r);
                        for (int f = lane; f < d.n_feat; f += 32)
                            sm[d.feat_row[f] * QX_RP + mm] = __ldg(d.emb_table + (size_t)r * d.n_feat + f);
                    } else {
                        const float *bits = d.emb_bits + (size_t)fid * d.n_pay * d.n_feat;
                        for (int f = lane; f < d.n_feat; f += 32) {
                            float acc = 0.0f;
                            for (int i = 0; i < d.n_pay; i++)
                                acc = __fadd_rn(acc, __fmul_rn(dec_pay[i * 32 + mm], __ldg(bits + (size_t)i * d.n_feat + f)));
                            sm[d.feat_row[f] * QX_RP + mm] = __fadd_rn(__ldg(d.emb_base + (size_t)fid * d.n_feat + f), acc);
                        }
                    }
                }
                break;
            }
            default:
                break;
            }
            __syncthreads();
        }
    }
    if (threadIdx.x == 0 && d.state_bytes) atomicAdd(d.state_bytes, 512ull * *touched);
    if (RUN) {
        for (int i = warp; i < d.n_born0; i += QX_NW) {
            uint2 p = d.pairs[i];
            if (act) d.x[(size_t)m * d.D + p.y] = sm[p.x * QX_RP + lane];
        }
        if (warp == 0 && act) {
            d.hash[m] = hash;
            d.count[m] = count;
            d.halt_at[m] = halt_at;
        }
    }
}

template __global__ void qx_token_kernel<0>(const __grid_constant__ QxDev, int32_t, int32_t *);
template __global__ void qx_token_kernel<1>(const __grid_constant__ QxDev, int32_t, int32_t *);

// Sets rows [row0, row0 + n) of x to the embeddings of the given tokens (FreeRun.load).
__global__ void qx_embed_kernel(const __grid_constant__ QxDev d, int32_t row0, int32_t n, const int32_t *tok) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const int m = row0 + r;
    const int t = tok[r];
    float *x = d.x + (size_t)m * d.D;
    for (int i = threadIdx.x; i < d.D; i += blockDim.x) x[i] = 0.0f;
    __syncthreads();
    int fid = 0;
    for (int f = 0; f < d.n_families; f++)
        if (t >= d.fam_ids[f] && t < d.fam_ids[f] + d.fam_size[f]) fid = f;
    const int p = t - d.fam_ids[fid];
    const int row0f = d.fam_row0[fid];
    for (int f = threadIdx.x; f < d.n_feat; f += blockDim.x) {
        const int dim = d.pairs[f].y;  // PAIRS[0 : n_feat] are (row, dim) of the feature dims
        float v;
        if (row0f >= 0) {
            v = d.emb_table[(size_t)(row0f + p) * d.n_feat + f];
        } else {
            float acc = 0.0f;
            for (int i = 0; i < d.n_pay; i++)
                acc = __fadd_rn(acc, __fmul_rn((float)((p >> i) & 1), d.emb_bits[((size_t)fid * d.n_pay + i) * d.n_feat + f]));
            v = __fadd_rn(d.emb_base[(size_t)fid * d.n_feat + f], acc);
        }
        x[dim] = v;
    }
    if (threadIdx.x == 0) {
        d.hash[m] = 0xcbf29ce484222325ULL;
        d.count[m] = 0;
        d.halt_at[m] = -1;
        d.err[m] = 0;
    }
}
