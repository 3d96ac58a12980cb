// qx_exec.cu -- the persistent per-token kernel of the executor.
//
// One CTA owns 32 machines (one per lane) and runs the plan's phase program for every token:
// the residual stream of its machines stays in shared memory as rows of 33 floats (lanes walk
// machines: conflict-free), the head states S stay in HBM and only the rows a key writes or a
// query reads are touched.  A phase ends with __syncthreads(); no grid-wide synchronisation is
// ever needed because machines never exchange data.
//
// The plan's form / unit / key-head records reach each warp as a stream of 16-byte quads that
// the warp copies from L2 into its own two-half ring in shared memory with cp.async, one half
// ahead of the half it reads; all 32 lanes then read each quad with one broadcast load.
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

__device__ __forceinline__ uint64_t fnv_word(uint64_t h, uint32_t w) {
#pragma unroll
    for (int b = 0; b < 4; b++) {
        h ^= (w >> (8 * b)) & 0xFFu;
        h *= 0x100000001b3ULL;
    }
    return h;
}

// ---- the machine group's cluster: every CTA keeps a full copy of the group's rows ----------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// the address of a shared-memory location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void *p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(a)
                 : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
    return a;
}
// a row value every copy must see: stored in each CTA of the cluster
__device__ __forceinline__ void put_all(float *p, float v, int C) {
    if (C == 1) {
        *p = v;
        return;
    }
    for (int r = 0; r < C; r++)
        asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(peer_addr(p, r)), "f"(v) : "memory");
}
__device__ __forceinline__ void put_all(uint32_t *p, uint32_t v, int C) {
    if (C == 1) {
        *p = v;
        return;
    }
    for (int r = 0; r < C; r++)
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_addr(p, r)), "r"(v) : "memory");
}
// atomic maximum of a selection word in copy `r` of the cluster (the local copy when C == 1);
// returns the word it replaced
__device__ __forceinline__ uint32_t max_at(uint32_t *p, uint32_t v, int C, uint32_t r) {
    if (C == 1) return atomicMax(p, v);
    uint32_t old;
    asm volatile("atom.relaxed.cluster.shared::cluster.max.u32 %0, [%1], %2;" : "=r"(old) : "r"(peer_addr(p, r)), "r"(v)
                 : "memory");
    return old;
}
// A key-select slot word: 0 for no channel, else a positive channel's value bits above bit 7 and
// 127 - channel in bits 0..6, so that a larger word is a larger value, or the same value
// (to 7 bits less) at a lower channel: the order of the reference's first-maximum selection,
// in which parts of one record merge by atomic maxima.
__device__ __forceinline__ uint32_t kq_word(float v, int ch) {
    return max(__float_as_uint(v) & ~0x7Fu, 0x80u) | (uint32_t)(127 - ch);
}
__device__ __forceinline__ int kq_channel(uint32_t w) { return w ? 127 - (int)(w & 0x7Fu) : -1; }
// a part's positive channel into slot levels p[0], p[stride], ... (qhot of them) of every copy:
// each level keeps the larger word and passes the smaller one down, so after every part of the
// record the levels hold its qhot largest words (a lock-free tournament); returns true when a
// positive word fell off the last level of copy 0 (more positive channels than the levels hold)
__device__ __forceinline__ bool kq_insert(uint32_t *p, int stride, int levels, uint32_t w, int C) {
    bool over = false;
    for (int r = 0; r < C; r++) {
        uint32_t x = w;
        for (int l = 0; l < levels && x; l++) x = min(x, max_at(p + l * stride, x, C, (uint32_t)r));
        if (r == 0) over = x != 0;
    }
    return over;
}
// a contribution to a row that several records sum into, added in each CTA of the cluster
__device__ __forceinline__ void add_all(float *p, float v, int C) {
    if (C == 1) {
        // one shared-window float reduction per contribution
        asm volatile("red.shared.add.f32 [%0], %1;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "f"(v)
                     : "memory");
        return;
    }
    for (int r = 0; r < C; r++)
        asm volatile("red.relaxed.cluster.shared::cluster.add.f32 [%0], %1;" ::"r"(peer_addr(p, r)), "f"(v) : "memory");
}
// the end of a phase: every warp of the CTA, or of the whole cluster (whose writes into this
// CTA's rows are then visible here)
__device__ __forceinline__ void phase_sync(int C) {
    if (C == 1) {
        __syncthreads();
    } else {
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- tensor cores (tcgen05): the linear forms of a tensor-core phase ----------------------------
// D[form][machine] (fp32, tensor memory: lane = form of the block, column = machine) +=
// A[form][k] (bf16 weights, tensor memory: lane = form, 8 columns of two k each) x B[machine][k]
// (bf16 source rows staged in shared memory, K-major, no swizzle: core matrices of 8 machines x
// 16 bytes, the two 8-row halves of K 128 B apart, machine groups of 8 rows 256 B apart).
// Tensor-memory columns: [0, 256) accumulators (32 per form block), [256, 384) A tiles (8 each).
#define QX_TMEM_COLS 512
#define QX_TMEM_A0 256
__device__ __forceinline__ uint32_t su32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (uint64_t)(128u >> 4) << 16 | (uint64_t)(256u >> 4) << 32 |
           (uint64_t)1 << 46;  // descriptor version of sm_100; base offset 0, no swizzle
}
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, N = 32, M = 128
constexpr uint32_t kMmaIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((32u >> 3) << 17) | ((128u >> 4) << 24);
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t acc) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d), "r"(a), "l"(bdesc),
                 "r"(kMmaIdesc), "r"(acc)
                 : "memory");
}
// bounded wait (about 2^31 SM cycles, ~1 s) for the completion of phase `par` of a shared-memory
// mbarrier (false: gave up)
__device__ __forceinline__ bool mbar_wait(const uint64_t *bar, uint32_t par) {
    uint32_t done = 0;
    const long long t0 = clock64();
    while (!done) {
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done)
                     : "r"(su32(bar)), "r"(par)
                     : "memory");
        if (!done && clock64() - t0 > (1ll << 31)) return false;
    }
    return true;
}

// A warp's view of its range [begin, end) of the plan stream, read through a ring of QX_NCHUNK
// chunks of QX_CHUNK lines of R quads (R = 32 / group: the record slots of a bundled plan, 1 for a
// 32-machine group): while the warp reads one chunk, the next QX_NCHUNK - 1 are in flight.
// `left` and the pieces count lines.
#define QX_CHUNK 32
#define QX_NCHUNK 2
static_assert(QX_CHUNK * QX_NCHUNK == 2 * QX_RING_QUADS, "a warp's ring holds 2 * QX_RING_QUADS lines");
template <int R>
struct Stream {
    static constexpr uint32_t CQ = QX_CHUNK * R;  // quads per chunk
    const uint4 *g;
    uint4 *ring;        // this warp's QX_NCHUNK * CQ quads
    const uint4 *rp;    // next line to read (in the ring)
    uint32_t begin, end, chunk;
    int left, lane;     // lines left in the current chunk

    __device__ __forceinline__ void issue(uint32_t c) {
#pragma unroll
        for (int k = 0; k < R; k++) {
            const uint32_t q = begin + c * CQ + k * 32 + lane;
            if (q < end) cp_async16(ring + (c % QX_NCHUNK) * CQ + k * 32 + lane, g + q);
        }
        cp_commit();
    }
    __device__ __forceinline__ void settle() {
        rp = ring + (chunk % QX_NCHUNK) * CQ;
        const uint32_t rest = end - (begin + chunk * CQ);
        left = rest < CQ ? (int)(rest / R) : QX_CHUNK;
    }
    // begin reading: the first QX_NCHUNK chunks in flight, wait for the first
    __device__ __forceinline__ void start(const uint4 *g_, uint4 *ring_, uint32_t b, uint32_t e, int l) {
        g = g_; ring = ring_; begin = b; end = e; lane = l; chunk = 0;
#pragma unroll
        for (int c = 0; c < QX_NCHUNK; c++) issue(c);
        cp_wait<QX_NCHUNK - 1>();
        __syncwarp();
        settle();
    }
    // the next chunk: once every lane is done with the current one, refill its slot
    // QX_NCHUNK chunks ahead
    __device__ __forceinline__ void advance() {
        chunk++;
        __syncwarp();
        issue(chunk + QX_NCHUNK - 1);
        cp_wait<QX_NCHUNK - 1>();
        __syncwarp();
        settle();
    }
    __device__ __forceinline__ bool more() const { return left > 0 || begin + (chunk + 1) * CQ < end; }
    // past a piece of n body lines
    __device__ __forceinline__ void skip(uint32_t n) {
        rp += R * (1 + n);
        left -= 1 + (int)n;
    }
    __device__ __forceinline__ void finish() {
        cp_wait<0>();
        __syncwarp();
    }
};


// One tensor-core form phase (QX_PH_MMA): a function of its own (not inlined), so that its
// registers (a round's tile rows in flight) do not add to the pressure of the CUDA-core phases.
__device__ __noinline__ void mma_forms_phase(const QxDev &d, uint32_t pi, int32_t t, float *sm, char *rings,
                                             const uint32_t *tslot, const uint64_t *mbar, int warp, int lane,
                                             bool act, int m) {
    float *sml = sm + lane;
    const qx_mma_phase mp = d.mma_phases[pi];
    char *const stage = rings;  // K block j: 1 KB at j * 1024
    // a wait for the tensor cores that gave up in an earlier phase (the CTA's machines carry
    // QX_E_BUSY): no further tensor-core work in this launch
    volatile uint32_t *dead = const_cast<uint32_t *>(tslot) + 1;
    if (*dead) return;
    const uint32_t tmem = *tslot;
    // the mbarrier's phase parity: its commits so far (pad0: this token's before this
    // phase; pad1: a token's, in total)
    uint32_t mma_par = (mp.pad0 + (uint32_t)t * mp.pad1) & 1u;
    uint32_t inexact = 0;
    bool tc_busy = false;
    // 1. stage the source rows as bf16 (exact: the circuit's values are bf16 numbers,
    //    checked here), warp w the K blocks w, w + 16, ...; lane = machine = B row
    for (uint32_t j = warp; j < mp.n_kb; j += QX_NW) {
        const uint4 *ro = reinterpret_cast<const uint4 *>(d.rows + mp.kr0 + 16 * j);
        uint32_t pk[8];
#pragma unroll
        for (int q4 = 0; q4 < 4; q4++) {
            const uint4 o = __ldg(ro + q4);
            const uint32_t a0 = __float_as_uint(QX_AT(sml, o.x)), a1 = __float_as_uint(QX_AT(sml, o.y)),
                           a2 = __float_as_uint(QX_AT(sml, o.z)), a3 = __float_as_uint(QX_AT(sml, o.w));
            inexact |= (a0 | a1 | a2 | a3) & 0xFFFFu;
            pk[2 * q4] = (a0 >> 16) | (a1 & 0xFFFF0000u);
            pk[2 * q4 + 1] = (a2 >> 16) | (a3 & 0xFFFF0000u);
        }
        char *dst = stage + j * 1024 + (lane >> 3) * 256 + (lane & 7) * 16;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4 *>(dst + 128) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    if (inexact && act) atomicOr(&d.err[m], QX_E_INEXACT);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the MMAs
    // 2. the tiles in rounds of up to 16 A slots: team warp / 4 loads tiles team,
    //    team + 4, ... of the round (lane quarter warp % 4 = tile rows 32q .. 32q + 31),
    //    one thread issues the round's MMAs and commits them to the mbarrier
    const int team = warp >> 2, q = warp & 3;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    for (uint32_t r0 = mp.t0; r0 < mp.t1; r0 += 16) {
        const uint32_t nt = min(16u, mp.t1 - r0);
        uint4 a[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t t = team + 4 * i;
            if (t < nt) {
                const uint4 *src = d.tiledata + (size_t)__ldg(&d.mma_tiles[r0 + t].data) * 256 + (q * 32 + lane) * 2;
                a[i][0] = __ldg(src);
                a[i][1] = __ldg(src + 1);
            }
        }
        if (r0 > mp.t0) {  // the previous round's MMAs have read their A slots
            tc_busy = !mbar_wait(mbar, mma_par);
            mma_par ^= 1;
            tc_after();
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t t = team + 4 * i;
            if (t < nt)
                asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(
                                 tq + QX_TMEM_A0 + 8 * t),
                             "r"(a[i][0].x), "r"(a[i][0].y), "r"(a[i][0].z), "r"(a[i][0].w), "r"(a[i][1].x),
                             "r"(a[i][1].y), "r"(a[i][1].z), "r"(a[i][1].w)
                             : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_before();
        tc_busy = __syncthreads_or(tc_busy);  // (one decision for the whole CTA)
        tc_after();
        if (tc_busy) break;
        if (threadIdx.x == 0) {
            for (uint32_t t = 0; t < nt; t++) {
                const qx_mma_tile tl = d.mma_tiles[r0 + t];
                mma_ts(tmem + 32 * tl.fb, tmem + QX_TMEM_A0 + 8 * t, umma_desc_kmajor(su32(stage + tl.kb * 1024)),
                       tl.acc);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             su32(mbar))
                         : "memory");
        }
    }
    if (!tc_busy) tc_busy = !mbar_wait(mbar, mma_par);  // the phase's accumulators are complete
    tc_busy = __syncthreads_or(tc_busy);
    tc_after();
    if (tc_busy) {
        *dead = 1u;
        if (act) atomicOr(&d.err[m], QX_E_BUSY);
        return;
    }
    // 3. team t reads form blocks t, t + 4, ...: its lane quarter holds forms 32q ..
    //    32q + 31 of the block, 32 machines each, stored into their rows
    for (uint32_t fb = team; fb < mp.n_fb; fb += 4) {
        const uint32_t dst = __ldg(d.rows + mp.dst0 + fb * 128 + q * 32 + lane);
        float *row = reinterpret_cast<float *>(reinterpret_cast<char *>(sm) + (dst != QX_NONE32 ? dst : 0));
#pragma unroll
        for (int h = 0; h < 2; h++) {  // machines 16h .. 16h + 15
            uint32_t v[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
                "%12, %13, %14, %15}, [%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                  "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
                  "=r"(v[14]), "=r"(v[15])
                : "r"(tq + 32 * fb + 16 * h)
                : "memory");
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (dst != QX_NONE32) {
#pragma unroll
                for (int n = 0; n < 16; n++) row[16 * h + n] = __uint_as_float(v[n]);
            }
        }
    }
    tc_before();  // these reads precede the next phase's MMAs (across its barrier)
}
}  // namespace

// R: record slots a warp runs side by side (1: a group of 32 machines, one a lane; 2, 4, 8: a
// group of M = 32 / R machines, lane = slot * M + machine, the stream in lines of R quads)
template <int RUN, int QH, int TC, int R>
__global__ void __launch_bounds__(QX_NT, 1)
    qx_token_kernel(const __grid_constant__ QxDev d, int32_t n_tokens, int32_t *tokens) {
    constexpr int M = 32 / R;   // machines of the CTA's group
    constexpr int RP = M + 1;   // floats per residual row
    static_assert(R == 1 || !TC, "tensor-core phases need a group of 32 machines");
    extern __shared__ __align__(16) float sm[];
    // key-select slot words (kq_word): [slots][32] keys, then [slots][qhot][32] query levels
    // (machine-indexed; a group of M < 32 uses the first M of each 32)
    uint32_t *ksel = reinterpret_cast<uint32_t *>(sm + (size_t)(d.smem_rows + 1) * RP);
    uint32_t *qsel = ksel + d.ksel_slots * 32;
    const int nsel = d.ksel_slots * 32 * (1 + d.qhot_max);
    int *dec_i = reinterpret_cast<int *>(qsel + d.ksel_slots * d.qhot_max * 32);  // [2][32]
    float *dec_pay = reinterpret_cast<float *>(dec_i + 64);                  // [16][32]
    unsigned int *touched = reinterpret_cast<unsigned int *>(dec_pay + 16 * 32);  // state rows
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // this lane's record slot and machine (R == 1: slot 0, machine = lane)
    const int way = lane / M, ml = lane % M;
    // a group of 32 machines runs on C CTAs; stream ranges are per warp of the group (gw of nwv),
    // interleaved over the CTAs (the plan hands its largest records to the lowest warps)
    const int C = d.cluster;
    const int crank = C > 1 ? (int)cluster_rank() : 0;
    const int gw = warp * C + crank, nwv = C * QX_NW;
    uint4 *ring = reinterpret_cast<uint4 *>(reinterpret_cast<char *>(sm) + qx_ring_offset(d)) +
                  warp * QX_NCHUNK * QX_CHUNK * R;
    float *sml = sm + ml;  // this lane's machine column: the row at byte offset o is QX_AT(sml, o)
    unsigned int *wcount = touched + 1;  // [2] value-head worklist lengths, used in turn
    int vpar = 0;                        // which of the two the next VH phase appends to
    // value-head phases reuse the stream rings for their worklist; their outputs are summed in
    // the group's delta rows in global memory (two buffers used in turn: the one a VHSUM phase
    // read is cleared by the next serving phase, dprev rows of it)
    char *rings = reinterpret_cast<char *>(sm) + qx_ring_offset(d);
    float *const D0 = d.vdelta + (size_t)(blockIdx.x / d.cluster) * (2 * QX_DELTA_ROWS * 32);
    int dpar = 0;
    uint32_t dprev = 0;
    if (threadIdx.x < RP) sm[(size_t)d.smem_rows * RP + threadIdx.x] = 0.0f;  // the zero row
    for (int i = threadIdx.x; i < nsel; i += QX_NT) ksel[i] = 0u;  // (cleared again by each VHRUN)
    if (threadIdx.x == 0) { touched[0] = 0; touched[1] = 0; touched[2] = 0; touched[13] = 0; }
    // tensor-core phases: the CTA's tensor memory (warp 0 allocates it; a CTA per SM) and the
    // mbarrier its MMA commits arrive on, in the counter block
    uint64_t *mbar = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(touched + 4) + 7) & ~(uintptr_t)7);
    uint32_t *tslot = touched + 12;
    if (TC) {
        if (warp == 0) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tslot)),
                         "r"(QX_TMEM_COLS)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        if (threadIdx.x == 0) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(mbar)) : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        tc_before();
    }
    const int grp = blockIdx.x / C;
    const int m = grp * M + ml;  // this lane's machine
    const bool act = m < d.B;
    const bool lact = lane < M && act;  // this lane is its machine's decode lane (warp 0)
    const int mbase = grp * M;

    // run mode: the embedding of each machine's next input comes from x
    uint64_t hash = 0;
    int64_t count = 0, halt_at = -1;
    if (RUN) {
        for (int i = warp * R + way; i < d.n_born0; i += QX_NW * R) {
            uint2 p = d.pairs[i];
            QX_AT(sml, p.x) = act ? d.x[(size_t)m * d.D + p.y] : 0.0f;
        }
        if (warp == 0 && lact) {
            hash = d.hash[m];
            count = d.count[m];
            halt_at = d.halt_at[m];
        }
    }
    // the plan tables the token loop reads: copied into the shared-memory table area where the
    // executor placed them (bundled plans), else read from global memory
    const qx_phase *prog = RUN ? d.run_prog : d.step_prog;
    const uint32_t *warp_ptr = d.warp_ptr, *rows_t = d.rows, *vhsum_t = d.vhsum_rows;
    const qx_vhead *vheads_t = d.vheads;
    const qx_stage *stages_t = d.stages;
    if (R > 1 && d.table_bytes) {
        const void *src[6] = {prog, warp_ptr, vheads_t, rows_t, vhsum_t, stages_t};
        const void *dst[6];
        char *area = rings + qx_ring_bytes(d);
#pragma unroll
        for (int t = 0; t < 6; t++) {
            dst[t] = src[t];
            if (d.tab_off[t] == QX_NONE32) continue;
            uint32_t *to = reinterpret_cast<uint32_t *>(area + d.tab_off[t]);
            const uint32_t *from = static_cast<const uint32_t *>(src[t]);
            const uint32_t nw = t == QX_TAB_PROG ? (RUN ? d.n_run_prog : d.n_step_prog) * 4 : d.tab_words[t];
            for (uint32_t i = threadIdx.x; i < nw; i += QX_NT) to[i] = __ldg(from + i);
            dst[t] = to;
        }
        prog = static_cast<const qx_phase *>(dst[QX_TAB_PROG]);
        warp_ptr = static_cast<const uint32_t *>(dst[QX_TAB_WARP_PTR]);
        vheads_t = static_cast<const qx_vhead *>(dst[QX_TAB_VHEADS]);
        rows_t = static_cast<const uint32_t *>(dst[QX_TAB_ROWS]);
        vhsum_t = static_cast<const uint32_t *>(dst[QX_TAB_VHSUM]);
        stages_t = static_cast<const qx_stage *>(dst[QX_TAB_STAGES]);
    }
    phase_sync(C);  // (with C > 1, also: every CTA of the cluster runs before rows are shared)
    if (TC) tc_after();
    for (int32_t t = 0; t < n_tokens; t++) {
        for (int pc = 0;; pc++) {
            const qx_phase ph = prog[pc];
            const uint32_t kind = ph.kind & 0xFFu;
            if (kind == QX_PH_END) break;
#ifdef QX_PHASE_CLOCKS
            const long long pclk0 = clock64();  // (thread 0: the phase up to its barrier's release)
#endif
            switch (kind) {
            case QX_PH_ZERO:
                for (uint32_t i = warp * R + way; i < ph.b; i += QX_NW * R) QX_AT(sml, rows_t[ph.a + i]) = 0.0f;
                break;
            case QX_PH_LOADX:
                for (uint32_t i = warp * R + way; i < ph.b; i += QX_NW * R) {
                    uint2 p = d.pairs[ph.a + i];
                    QX_AT(sml, p.x) = act ? d.x[(size_t)m * d.D + p.y] : 0.0f;
                }
                break;
            case QX_PH_WRITEOUT:
                if (act)
                    for (uint32_t i = gw * R + way; i < ph.b; i += nwv * R) {
                        uint2 p = d.pairs[ph.a + i];
                        d.x[(size_t)m * d.D + p.y] = QX_AT(sml, p.x);
                    }
                break;
            case QX_PH_APPLY:
                for (uint32_t i = warp * R + way; i < ph.b; i += QX_NW * R) {
                    uint2 p = d.pairs[ph.a + i];
                    QX_AT(sml, p.x) += QX_AT(sml, p.y);
                }
                break;
            case QX_PH_STAGE: {
                // stage lags 1..3 of this head sublayer's history into scratch rows, then move
                // the history on: lag 1 <- the input x, lag k <- lag k-1
                float *H = d.hist[ph.c];
                const size_t ne = d.NE[ph.c], bp = d.Bpad;
                for (uint32_t i = gw * R + way; i < ph.b; i += nwv * R) {
                    const qx_stage s = stages_t[ph.a + i];
                    float *h = H + (size_t)s.e * bp + m;
                    float h0 = h[0];
                    float h1 = s.ml >= 2 ? h[ne * bp] : 0.0f;
                    float h2 = s.ml >= 3 ? h[2 * ne * bp] : 0.0f;
                    if (s.stage[0] != QX_NONE32) put_all(&QX_AT(sml, s.stage[0]), h0, C);
                    if (s.stage[1] != QX_NONE32) put_all(&QX_AT(sml, s.stage[1]), h1, C);
                    if (s.stage[2] != QX_NONE32) put_all(&QX_AT(sml, s.stage[2]), h2, C);
                    h[0] = QX_AT(sml, s.x_row);
                    if (s.ml >= 2) h[ne * bp] = h0;
                    if (s.ml >= 3) h[2 * ne * bp] = h1;
                }
                break;
            }
            case QX_PH_FORMS: {
                // two forms a record: pieces [dst A, dst B, 0, n | flags] + n quads [row, w of A,
                // row, w of B]: F = sum w * X[row], two independent sums a lane (a bundled plan:
                // lines of R quads, this lane's record is quad `way` of each line)
                const uint32_t b0 = warp_ptr[ph.c + gw], b1 = warp_ptr[ph.c + gw + 1];
                if (b0 == b1) break;
                Stream<R> st;
                st.start(d.stream, ring, b0, b1, lane);
                float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
                while (true) {
                    if (st.left == 0) {
                        if (!st.more()) break;
                        st.advance();
                    }
                    const uint4 h = st.rp[way];
                    const uint32_t n = h.w & 0xFFFFFFu, fl = h.w >> 24;
                    if (fl & QX_R_SKIP) {
                        st.left = 0;
                        continue;
                    }
                    const uint4 *q = st.rp + R + way;
                    if (fl & QX_R_FIRST) a0 = a1 = a2 = a3 = 0.0f;  // a0, a2: form A; a1, a3: B
                    uint32_t j = 0;
#pragma unroll 2
                    for (; j + 2 <= n; j += 2) {
                        const uint4 e0 = q[j * R], e1 = q[(j + 1) * R];
                        const float v0 = QX_AT(sml, e0.x), v1 = QX_AT(sml, e0.z), v2 = QX_AT(sml, e1.x),
                                    v3 = QX_AT(sml, e1.z);
                        a0 = fmaf(__uint_as_float(e0.y), v0, a0);
                        a1 = fmaf(__uint_as_float(e0.w), v1, a1);
                        a2 = fmaf(__uint_as_float(e1.y), v2, a2);
                        a3 = fmaf(__uint_as_float(e1.w), v3, a3);
                    }
                    if (j < n) {
                        const uint4 e = q[j * R];
                        a0 = fmaf(__uint_as_float(e.y), QX_AT(sml, e.x), a0);
                        a1 = fmaf(__uint_as_float(e.w), QX_AT(sml, e.z), a1);
                    }
                    if (fl & QX_R_LAST) {
                        float sa = a0 + a2, sb = a1 + a3;
                        if (R > 1 && (fl & QX_R_SPLIT)) {
                            // one pair over every slot (the whole warp takes this branch): the
                            // slots' partial sums meet across the lanes of each machine
#pragma unroll
                            for (int off = M; off < 32; off <<= 1) {
                                sa += __shfl_xor_sync(0xFFFFFFFFu, sa, off);
                                sb += __shfl_xor_sync(0xFFFFFFFFu, sb, off);
                            }
                        }
                        if (!(fl & QX_R_NOP) && (!(fl & QX_R_SPLIT) || way == 0)) {
                            put_all(&QX_AT(sml, h.x), sa, C);
                            put_all(&QX_AT(sml, h.y), sb, C);
                        }
                    }
                    st.skip(n);
                }
                st.finish();
                break;
            }
            case QX_PH_MMA:
                // linear forms on the tensor cores; every CTA of a cluster computes all of them
                if (TC) mma_forms_phase(d, ph.a, t, sm, rings, tslot, mbar, warp, lane, act, m);
                break;
            case QX_PH_UNITS: {
                // pieces [out, n_const, 0, n | flags] + n_const quads [F[b] row, k, cb, 0]
                // (k relu(F[b] + cb)) + two quads per unit with an a form, [F[a] row, F[b] row,
                // coef, ca] [cb, ...] (coef (F[a] + ca) relu(F[b] + cb)); ONE is 1 on every
                // machine (no sublayer writes it), so its constant terms enter as plain constants
                // (a bundle's records share n and n_const piece by piece)
                const uint32_t b0 = warp_ptr[ph.c + gw], b1 = warp_ptr[ph.c + gw + 1];
                if (b0 == b1) break;
                Stream<R> st;
                st.start(d.stream, ring, b0, b1, lane);
                float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f, acc3 = 0.0f;
                while (true) {
                    if (st.left == 0) {
                        if (!st.more()) break;
                        st.advance();
                    }
                    const uint4 h = st.rp[way];
                    const uint32_t n = h.w & 0xFFFFFFu, fl = h.w >> 24;
                    if (fl & QX_R_SKIP) {
                        st.left = 0;
                        continue;
                    }
                    const uint4 *q = st.rp + R + way;
                    if (fl & QX_R_FIRST) acc0 = acc1 = acc2 = acc3 = 0.0f;
                    const uint32_t nc = h.y;
                    uint32_t j = 0;
#pragma unroll 2
                    for (; j + 2 <= nc; j += 2) {
                        const uint4 u0 = q[j * R], u1 = q[(j + 1) * R];
                        const float f0 = QX_AT(sml, u0.x), f1 = QX_AT(sml, u1.x);
                        acc0 = fmaf(__uint_as_float(u0.y), relu(f0 + __uint_as_float(u0.z)), acc0);
                        acc1 = fmaf(__uint_as_float(u1.y), relu(f1 + __uint_as_float(u1.z)), acc1);
                    }
                    if (j < nc) {
                        const uint4 u0 = q[j * R];
                        acc2 = fmaf(__uint_as_float(u0.y), relu(QX_AT(sml, u0.x) + __uint_as_float(u0.z)), acc2);
                        j++;
                    }
                    for (; j < n; j += 2) {
                        const uint4 u = q[j * R], u2 = q[(j + 1) * R];
                        const float av = QX_AT(sml, u.x) + __uint_as_float(u.w);
                        const float bv = QX_AT(sml, u.y) + __uint_as_float(u2.x);
                        acc1 += __fmul_rn(__fmul_rn(__uint_as_float(u.z), av), relu(bv));
                    }
                    if ((fl & (QX_R_LAST | QX_R_NOP)) == QX_R_LAST) {
                        const float tot = (acc0 + acc1) + (acc2 + acc3);
                        if (fl & QX_R_STORE)
                            put_all(&QX_AT(sml, h.x), QX_AT(sml, h.x) + tot, C);  // the row's only record
                        else
                            add_all(&QX_AT(sml, h.x), tot, C);  // records into one row meet
                    }
                    st.skip(n);
                }
                st.finish();
                break;
            }
            case QX_PH_KSEL: {
                // per key head, lanes walk machines: pieces [slot | qhot << 16 | first channel
                // << 24, common row, lag-ONE row, n | flags] + n channels [row, c0, c1, has
                // common]: the key's first maximal channel (a write when positive), then
                // (R_QUERY) the query's top-qhot positive channels.  A record split into parts
                // (R_MERGE) merges each part's selection into the slot words by atomic maxima
                // (the slots start at 0: cleared by the value-head serving phase before)
                // (a bundle holds keys only or queries only)
                const uint32_t b0 = warp_ptr[ph.c + gw], b1 = warp_ptr[ph.c + gw + 1];
                if (b0 == b1) break;
                Stream<R> st;
                st.start(d.stream, ring, b0, b1, lane);
                float bk = 0.0f, qb[QH];
                int ik = -1, npos = 0, qi[QH], base = 0;
                while (true) {
                    if (st.left == 0) {
                        if (!st.more()) break;
                        st.advance();
                    }
                    const uint4 h = st.rp[way];
                    const uint32_t n = h.w & 0xFFFFFFu, fl = h.w >> 24;
                    if (fl & QX_R_SKIP) {
                        st.left = 0;
                        continue;
                    }
                    const uint4 *q = st.rp + R + way;
                    const float com = QX_AT(sml, h.y), x1 = QX_AT(sml, h.z);
                    const uint32_t slot = h.x & 0xFFFFu, qhot = (h.x >> 16) & 0xFFu;
                    if (fl & QX_R_FIRST) {
                        bk = 0.0f;
                        ik = -1;
                        npos = 0;
                        base = (int)(h.x >> 24);
#pragma unroll
                        for (int k = 0; k < QH; k++) {
                            qb[k] = 0.0f;
                            qi[k] = -1;
                        }
                    }
                    if (!(fl & QX_R_QUERY)) {
                        for (uint32_t j = 0; j < n; j++) {
                            const uint4 c = q[j * R];
                            const float v = relu(fmaf(__uint_as_float(c.z), x1,
                                                      __uint_as_float(c.y) + fmaf(__uint_as_float(c.w), com, QX_AT(sml, c.x))));
                            npos += v > 0.0f;
                            if (v > bk) {
                                bk = v;
                                ik = base + (int)j;
                            }
                        }
                    } else {
                        for (uint32_t j = 0; j < n; j++) {
                            const uint4 c = q[j * R];
                            float v = relu(fmaf(__uint_as_float(c.z), x1,
                                                __uint_as_float(c.y) + fmaf(__uint_as_float(c.w), com, QX_AT(sml, c.x))));
                            int vi = base + (int)j;
                            npos += v > 0.0f;
                            // insertion into the descending top list: a value displaces only a
                            // strictly smaller one, so ties keep the lower channel first
#pragma unroll
                            for (int k = 0; k < QH; k++) {
                                if (k < (int)qhot && v > qb[k]) {
                                    const float tv = qb[k];
                                    const int ti = qi[k];
                                    qb[k] = v;
                                    qi[k] = vi;
                                    v = tv;
                                    vi = ti;
                                }
                            }
                        }
                    }
                    base += (int)n;
                    if ((fl & (QX_R_LAST | QX_R_NOP)) == QX_R_LAST) {
                        if (!(fl & QX_R_QUERY)) {
                            uint32_t *kp = &ksel[slot * 32 + ml];
                            const uint32_t w = ik >= 0 ? kq_word(bk, ik) : 0u;
                            bool err = npos > 1;
                            // merged: a positive channel of another part shows as a word that
                            // falls off the slot's one level (more than one positive channel)
                            if (!(fl & QX_R_MERGE)) put_all(kp, w, C);
                            else if (w) err |= kq_insert(kp, 0, 1, w, C);
                            if (err && act) atomicOr(&d.err[m], QX_E_KEY);
                        } else {
                            uint32_t *qp = &qsel[slot * d.qhot_max * 32 + ml];
                            bool err = npos > (int)qhot;
                            if (!(fl & QX_R_MERGE)) {
#pragma unroll
                                for (int k = 0; k < 4; k++)
                                    if (k < d.qhot_max)
                                        put_all(qp + k * 32, k < QH && qi[k < QH ? k : 0] >= 0 ? kq_word(qb[k < QH ? k : 0], qi[k < QH ? k : 0]) : 0u, C);
                            } else {
#pragma unroll
                                for (int k = 0; k < QH; k++)
                                    if (qi[k] >= 0) err |= kq_insert(qp, 32, (int)qhot, kq_word(qb[k], qi[k]), C);
                            }
                            if (err && act) atomicOr(&d.err[m], QX_E_QUERY);
                        }
                    }
                    st.skip(n);
                }
                st.finish();
                break;
            }
            case QX_PH_VH: {
                // per value head, lanes walk machines: list every machine whose decay, write or
                // read touches a state row (record: value head, machine, decay factor, write row,
                // query rows) in the CTA's worklist, which lives in the idle stream rings
                // (R record slots: R value heads a warp at a time, each over its M machines)
                const uint32_t n = ph.b - ph.a;
                uint2 *wl = reinterpret_cast<uint2 *>(rings);
                for (uint32_t i0 = gw * R; i0 < n; i0 += nwv * R) {
                    const uint32_t i = i0 + way;
                    const bool vin = R == 1 || i < n;
                    const qx_vhead vh = vheads_t[ph.a + (vin ? i : i0)];
                    const float x0 = QX_AT(sml, d.one_row);
                    uint32_t fcode = 0;  // decay factor: 0 -> 1, 1 -> 1/2, 2 -> 0
                    if (vh.nrows > 0) {
                        const float av = fmaf(vh.ca, x0, QX_AT(sml, vh.a_row));
                        fcode = av == 0.0f ? 0u : (av == 110.0f ? 1u : 2u);
                    }
                    const float bv = fmaf(vh.cb, x0, QX_AT(sml, vh.b_row)) + vh.bconst;
                    const int kr = kq_channel(ksel[vh.slot * 32 + ml]);
                    const int wrow = (kr >= 0 && bv == 1.0f) ? kr : -1;
                    uint32_t qpack = 0;
                    bool anyq = false;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int qj = j < d.qhot_max ? kq_channel(qsel[(vh.slot * d.qhot_max + j) * 32 + ml]) : -1;
                        qpack |= (uint32_t)(qj + 1) << (8 * j);
                        anyq |= qj >= 0;
                    }
                    const bool need = act && vin && (fcode != 0 || wrow >= 0 || anyq);
                    const unsigned mask = __ballot_sync(0xFFFFFFFFu, need);
                    if (!mask) continue;
                    // the value head's records, padded to a multiple of four (pad records: bit 31)
                    // so that every batch of four the serving warps take shares one value head
                    const unsigned gm = R == 1 ? mask : (mask >> (way * M)) & ((1u << (M & 31)) - 1u);
                    const unsigned nrec = __popc(gm), npad = ((nrec + 3u) & ~3u) - nrec;
                    unsigned base = 0;
                    if (ml == 0 && gm) base = atomicAdd(wcount + vpar, nrec + npad);
                    base = __shfl_sync(0xFFFFFFFFu, base, way * M);
                    if (need) {
                        const unsigned pos = base + __popc(gm & ((1u << ml) - 1u));
                        wl[pos] = make_uint2(i | (uint32_t)ml << 8 | fcode << 13 | (uint32_t)(wrow + 1) << 16, qpack);
                    }
                    if (gm && (unsigned)ml < npad) wl[base + nrec + ml] = make_uint2(i | 1u << 31, 0u);
                }
                break;
            }
            case QX_PH_VHRUN: {
                // the listed row work, four records (one value head, four machines) a warp at a
                // time with lanes over columns (4 each).  Every state-row load of the batch (the
                // decayed rows, the query rows) and every column descriptor is issued before any
                // result is needed; reads then take the decayed or written value from registers:
                // the read of row r sees v if r is the write row, old * f if r < nrows, else old
                // (decay, then write, then read, as the reference orders them).
                // the other length was last read by the previous serve phase, a barrier ago
                const uint32_t cnt = wcount[vpar];
                const uint2 *wl = reinterpret_cast<const uint2 *>(rings);
                float *const Dp = D0 + dpar * (QX_DELTA_ROWS * 32);  // this phase's output deltas
                {
                    float *const Dq = D0 + (dpar ^ 1) * (QX_DELTA_ROWS * 32);  // read by the last VHSUM
                    for (uint32_t j = gw; j < dprev; j += nwv) Dq[j * 32 + lane] = 0.0f;
                }
                if (threadIdx.x == 0) wcount[vpar ^ 1] = 0;
                vpar ^= 1;
                // the key-select slots were read by the VH phase before: cleared for the next
                // KSEL phase (a barrier away), whose merged parts take atomic maxima into them
                for (int i = threadIdx.x; i < nsel; i += QX_NT) ksel[i] = 0u;
                for (uint32_t r0 = warp * 4; r0 < cnt; r0 += QX_NW * 4) {
                    uint2 rec[4];
#pragma unroll
                    for (int b = 0; b < 4; b++) rec[b] = wl[r0 + b];
                    const qx_vhead vh = vheads_t[ph.a + (rec[0].x & 0xFFu)];
                    const size_t mstride = (size_t)d.V[vh.hl] * (QX_HD * QX_HD);
                    const float *S0 = d.S[vh.hl] + (size_t)vh.vh * (QX_HD * QX_HD) + lane * 4;
                    int mmv[4], wr[4], qr[4][QH];
                    float f[4];
                    bool valid[4], anyw = false, anyq = false;
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        valid[b] = !(rec[b].x >> 31);
                        mmv[b] = (rec[b].x >> 8) & 31;
                        const uint32_t fc = (rec[b].x >> 13) & 3u;
                        f[b] = fc == 0 ? 1.0f : (fc == 1 ? 0.5f : 0.0f);
                        wr[b] = valid[b] ? (int)((rec[b].x >> 16) & 0xFFu) - 1 : -1;
                        anyw |= wr[b] >= 0;
#pragma unroll
                        for (int j = 0; j < QH; j++) {
                            qr[b][j] = valid[b] ? (int)((rec[b].y >> (8 * j)) & 0xFFu) - 1 : -1;
                            anyq |= qr[b][j] >= 0;
                        }
                    }
                    // loads: query rows (old values), then the column descriptors
                    float4 qv[4][QH];
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        const float *Sb = S0 + qx_copy(d, vh.hl, mbase + mmv[b]) * mstride;
#pragma unroll
                        for (int j = 0; j < QH; j++)
                            qv[b][j] = qr[b][j] >= 0 ? *reinterpret_cast<const float4 *>(Sb + qr[b][j] * QX_HD)
                                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    qx_colform vf[4], zf[4];
                    uint32_t orow[4];
                    float ow[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t c = vh.col + lane * 4 + k;
                        if (anyw) vf[k] = d.vform[c];
                        if (anyq) {
                            zf[k] = d.zform[c];
                            orow[k] = d.out_row[c];
                            ow[k] = d.out_w[c];
                        }
                    }
                    unsigned int rows = 0;  // 512-byte row transfers
                    // per record: decay, write, then the read of its query rows as decayed and
                    // written (o), and its normaliser; the four records' chains are independent
                    float4 o[4];
                    float norm[4], inv[4];
                    bool any[4], pw2[4];
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        o[b] = make_float4(0.f, 0.f, 0.f, 0.f);
                        any[b] = false;
                        if (!valid[b]) continue;
                        float *Sb = const_cast<float *>(S0) + qx_copy(d, vh.hl, mbase + mmv[b]) * mstride;
                        const float *smm = sm + mmv[b];
                        const float x0m = QX_ATC(smm, d.one_row);
                        // decay of the first nrows rows (rare: a read-modify-write of its own)
                        if (f[b] != 1.0f) {
                            rows += 2 * vh.nrows;
                            for (int r = 0; r < vh.nrows; r++) {
                                float4 *p = reinterpret_cast<float4 *>(Sb + r * QX_HD);
                                float4 sv = *p;
                                sv.x = __fmul_rn(sv.x, f[b]); sv.y = __fmul_rn(sv.y, f[b]);
                                sv.z = __fmul_rn(sv.z, f[b]); sv.w = __fmul_rn(sv.w, f[b]);
                                *p = sv;
                            }
                        }
                        float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (wr[b] >= 0) {
                            float v[4];
#pragma unroll
                            for (int k = 0; k < 4; k++)
                                v[k] = vf[k].live ? relu(fmaf(vf[k].c, x0m, QX_ATC(smm, vf[k].row))) : 0.0f;
                            wv = make_float4(v[0], v[1], v[2], v[3]);
                            *reinterpret_cast<float4 *>(Sb + wr[b] * QX_HD) = wv;
                            rows++;
                        }
                        // the read: sum of the query rows as decayed and written
#pragma unroll
                        for (int j = 0; j < QH; j++) {
                            if (qr[b][j] < 0) continue;
                            float4 sv = qv[b][j];
                            if (qr[b][j] == wr[b]) {
                                sv = wv;
                            } else if (qr[b][j] < (int)vh.nrows && f[b] != 1.0f) {
                                sv.x = __fmul_rn(sv.x, f[b]); sv.y = __fmul_rn(sv.y, f[b]);
                                sv.z = __fmul_rn(sv.z, f[b]); sv.w = __fmul_rn(sv.w, f[b]);
                            }
                            o[b].x = __fadd_rn(o[b].x, sv.x); o[b].y = __fadd_rn(o[b].y, sv.y);
                            o[b].z = __fadd_rn(o[b].z, sv.z); o[b].w = __fadd_rn(o[b].w, sv.w);
                            any[b] = true;
                            rows++;
                        }
                    }
                    // ref = o0^2 + o1^2 of each read (columns 0 and 1: lane 0), norm = sqrt(ref / 128);
                    // when norm is a power of two (the usual read: the markers give ref = 128 * 4^e),
                    // multiplying by its exact reciprocal rounds the same as the division
#pragma unroll
                    for (int b = 0; b < 4; b++) {
                        float ref = __fadd_rn(__fmul_rn(o[b].x, o[b].x), __fmul_rn(o[b].y, o[b].y));
                        ref = __shfl_sync(0xFFFFFFFFu, ref, 0);  // (uniform: the batch's records are)
                        any[b] = any[b] && ref > 0.0f;  // a zero read adds nothing
                        norm[b] = __fsqrt_rn(__fdiv_rn(ref, 128.0f));
                        const uint32_t nb = __float_as_uint(norm[b]);
                        pw2[b] = (nb & 0x7FFFFFu) == 0u && nb >= 0x01000000u && nb < 0x7E800000u;
                        inv[b] = pw2[b] ? __uint_as_float(0x7F000000u - nb) : 0.0f;
                    }
                    if (vh.nout != QX_OUT_DIRECT) {
                        // at most 4 output rows: per (record, row) the sum over the warp's columns,
                        // reduced-and-scattered over the lanes (16 sums in 16 shuffles: lane L
                        // ends with sum (L >> 1), record (L >> 3), row (L >> 1) & 3), one L2 add each
                        float pv[16];
#pragma unroll
                        for (int i = 0; i < 16; i++) pv[i] = 0.0f;
#pragma unroll
                        for (int b = 0; b < 4; b++) {
                            if (!any[b]) continue;
                            const float *smm = sm + mmv[b];
                            const float x0m = QX_ATC(smm, d.one_row);
                            const float oc[4] = {o[b].x, o[b].y, o[b].z, o[b].w};
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                if (orow[k] == QX_NONE32) continue;
                                const float z = zf[k].live ? relu(fmaf(zf[k].c, x0m, QX_ATC(smm, zf[k].row))) : 0.0f;
                                const float out = pw2[b] ? oc[k] * inv[b] : __fdiv_rn(oc[k], norm[b]);
                                const float val = __fmul_rn(__fmul_rn(out, z), ow[k]);
#pragma unroll
                                for (int r = 0; r < 4; r++) pv[4 * b + r] += orow[k] == (uint32_t)r ? val : 0.0f;
                            }
                        }
#pragma unroll
                        for (int half = 8, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
                            // keep half of the sums (the upper half where this lane's bit is set),
                            // add the partner's copy of the same half
                            const bool up = lane & bit;
#pragma unroll
                            for (int i = 0; i < half; i++) {
                                const float give = up ? pv[i] : pv[half + i];
                                const float keep = up ? pv[half + i] : pv[i];
                                pv[i] = keep + __shfl_xor_sync(0xFFFFFFFFu, give, bit);
                            }
                        }
                        pv[0] += __shfl_xor_sync(0xFFFFFFFFu, pv[0], 1);
                        const int sb = lane >> 3, sr = (lane >> 1) & 3;
                        if (!(lane & 1) && (uint32_t)sr < vh.nout) {
                            bool hit = false;
                            int mm = 0;
#pragma unroll
                            for (int b = 0; b < 4; b++)
                                if (b == sb) { hit = any[b]; mm = mmv[b]; }
                            const uint32_t orw = sr == 0 ? vh.out4[0] : sr == 1 ? vh.out4[1] : sr == 2 ? vh.out4[2] : vh.out4[3];
                            if (hit) {
                                if (d.direct_out) add_all(&QX_AT(sm + mm, orw), pv[0], 1);  // the residual row
                                else atomicAdd(Dp + (orw >> 2) + mm, pv[0]);  // an L2 reduction
                            }
                        }
                    } else {
#pragma unroll
                        for (int b = 0; b < 4; b++) {
                            if (!any[b]) continue;
                            const float *smm = sm + mmv[b];
                            const float x0m = QX_ATC(smm, d.one_row);
                            const float oc[4] = {o[b].x, o[b].y, o[b].z, o[b].w};
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                if (orow[k] == QX_NONE32) continue;
                                const float z = zf[k].live ? relu(fmaf(zf[k].c, x0m, QX_ATC(smm, zf[k].row))) : 0.0f;
                                const float out = pw2[b] ? oc[k] * inv[b] : __fdiv_rn(oc[k], norm[b]);
                                const float val = __fmul_rn(__fmul_rn(out, z), ow[k]);
                                if (d.direct_out) add_all(&QX_AT(sm + mmv[b], orow[k]), val, 1);
                                else atomicAdd(Dp + (orow[k] >> 2) + mmv[b], val);
                            }
                        }
                    }
                    if (lane == 0) atomicAdd(touched, rows);
                }
                break;
            }
            case QX_PH_VHSUM: {
                // the phase's output deltas into this copy's rows (L2 reads: the adds bypassed L1)
                const float *Dp = D0 + dpar * (QX_DELTA_ROWS * 32);
                for (uint32_t j = warp * R + way; j < ph.b; j += QX_NW * R)
                    QX_AT(sml, vhsum_t[ph.a + j]) += __ldcg(Dp + j * 32 + ml);
                dprev = ph.b;
                dpar ^= 1;
                break;
            }
            case QX_PH_DECODE: {
                // the next token of every machine (warp 0, lanes = machines), then its embedding
                // (FreeRun._step, fastexec.py:298-307; merged readout: core.py:1287-1304)
                if (warp == 0) {
                    int kind = 0, fid = 0, pay = 0;  // kind 0: chip token, 1: text token, 2: none
                    long long tok = -1;
                    bool bad = false;
                    if (!d.merged) {
                        float fam = 0.0f, psum = 0.0f;
                        for (int i = 0; i < d.n_fam; i++)
                            fam = __fadd_rn(fam, __fmul_rn(rintf(QX_AT(sml, d.fam_row[i])), ldexpf(1.0f, i)));
                        for (int i = 0; i < d.n_pay; i++) {
                            const float pv = rintf(QX_AT(sml, d.pay_row[i]));
                            dec_pay[i * 32 + lane] = pv;
                            psum = __fadd_rn(psum, __fmul_rn(pv, ldexpf(1.0f, i)));
                        }
                        const long long fraw = (long long)fam;
                        fid = fraw < 0 ? 0 : (fraw > d.n_families - 1 ? d.n_families - 1 : (int)fraw);
                        const long long p = (long long)psum;
                        pay = (int)p;
                        tok = (long long)d.fam_ids[fid] + p;
                        bad = fraw != fid || p < 0 || p >= d.fam_size[fid];
                    } else {
                        // merged: a code dim > 0 is a 1 bit; all zero: the circuit predicts nothing
                        const int nfam = d.n_code - 16;
                        uint32_t fb = 0, pb = 0;
                        bool anyc = false;
                        for (int i = 0; i < d.n_code; i++) {
                            const float v = QX_AT(sml, d.code_row[i]);
                            anyc |= v != 0.0f;
                            if (v > 0.0f) {
                                if (i < nfam) fb |= 1u << i;
                                else pb |= 1u << (i - nfam);
                            }
                        }
                        for (int i = 0; i < 16; i++) dec_pay[i * 32 + lane] = (float)(pb >> i & 1u);
                        pay = (int)pb;
                        if (!anyc) {
                            kind = 2;
                        } else if ((int)fb == d.q_fid) {
                            if ((int)pb < d.n_printable) {
                                kind = 1;
                                pay = d.printable[pb];  // the text token's qid
                                tok = QX_TEXT_TOKEN + (long long)pay;
                            } else {
                                kind = 2;
                                bad = true;
                            }
                        } else if ((int)fb < d.n_families && (int)pb < d.fam_size[fb]) {
                            fid = (int)fb;
                            tok = (long long)d.fam_ids[fid] + pb;
                        } else {
                            kind = 2;
                            bad = true;
                        }
                    }
                    dec_i[lane] = fid | kind << 24;
                    dec_i[32 + lane] = pay;
                    if (lact) {
                        if (crank == 0) {
                            if (bad) atomicOr(&d.err[m], QX_E_CODE);
                            if (tokens) tokens[(size_t)t * d.B + m] = (int32_t)tok;
                        }
                        hash = fnv_word(hash, (uint32_t)tok);
                        count++;
                        if (halt_at < 0 && tok == d.halt_tok) halt_at = count;
                    }
                }
                __syncthreads();
                // next embedding (FreeRun: table row for small families, base + payload bits;
                // a text token: its base + the rows of their bits; no token: the bare text base).
                // A group of fewer machines than warps shares each machine's features between
                // K = 16 / M warps: first every feature that is not a table row's is zeroed, then
                // (after a barrier) the touched ones are written; warp k of a machine takes
                // features k * 32 + lane, stepping 32 K.  Larger groups: a warp a machine.
                if constexpr (M < QX_NW) {
                    constexpr int K = QX_NW / M;
                    const int mfirst = warp % M, kk = warp / M;
                    for (int mm = mfirst; mm < M; mm += QX_NW) {
                        const int fid = dec_i[mm] & 0xFFFFFF, kind = dec_i[mm] >> 24;
                        if (kind == 0 && d.fam_row0[fid] >= 0) continue;  // a table row: written below
                        float *smw = sm + mm;
                        float *xm = d.x + (size_t)(mbase + mm) * d.D;
                        const bool mact = mbase + mm < d.B;
                        for (int f = kk * 32 + lane; f < d.n_feat; f += 32 * K) {
                            const uint32_t fr = d.feat_row[f];
                            if (!(fr & QX_FEAT_DEFERRED)) QX_AT(smw, fr) = 0.0f;
                            else if (mact) xm[fr & ~QX_FEAT_DEFERRED] = 0.0f;
                        }
                    }
                    __syncthreads();
                    for (int mm = mfirst; mm < M; mm += QX_NW) {
                        const int fid = dec_i[mm] & 0xFFFFFF, kind = dec_i[mm] >> 24, p = dec_i[32 + mm];
                        float *smw = sm + mm;
                        float *xm = d.x + (size_t)(mbase + mm) * d.D;
                        const bool mact = mbase + mm < d.B;
                        // a feature's value into its row, or (deferred) into x where its sublayer loads it
                        auto put = [&](int f, float v) {
                            const uint32_t fr = d.feat_row[f];
                            if (!(fr & QX_FEAT_DEFERRED)) QX_AT(smw, fr) = v;
                            else if (mact) xm[fr & ~QX_FEAT_DEFERRED] = v;
                        };
                        if (kind != 0) {
                            const uint32_t *w = d.text_words + (size_t)(kind == 1 ? p : 0) * 5;
                            uint32_t wv[5];
#pragma unroll
                            for (int k = 0; k < 5; k++) wv[k] = kind == 1 ? __ldg(w + k) : 0u;
                            for (int tt = kk * 32 + lane; tt < d.n_text_touch; tt += 32 * K) {
                                const int f = (int)d.text_touch[tt];
                                float acc = __ldg(d.text_base + f);
#pragma unroll 1
                                for (int k = 0; k < 5; k++) {
                                    uint32_t bits = wv[k];
                                    while (bits) {
                                        const int j = 32 * k + __ffs(bits) - 1;
                                        bits &= bits - 1;
                                        acc = __fadd_rn(acc, __ldg(d.text_bits + (size_t)j * d.n_feat + f));
                                    }
                                }
                                put(f, acc);
                            }
                            continue;
                        }
                        const int row0 = d.fam_row0[fid];
                        if (row0 >= 0) {
                            int r = row0 + p;
                            r = r < 0 ? 0 : (r > d.n_emb_rows - 1 ? d.n_emb_rows - 1 : r);
                            for (int f = kk * 32 + lane; f < d.n_feat; f += 32 * K)
                                put(f, __ldg(d.emb_table + (size_t)r * d.n_feat + f));
                        } else {
                            // the family's touched features: base + the payload bits' rows (four
                            // partial sums: exact values, any order)
                            const int npay = d.merged ? 16 : d.n_pay;  // (a merged graph reads no payload dims)
                            const float *bits = d.emb_bits + (size_t)fid * npay * d.n_feat;
                            const uint32_t t1 = d.fam_touch_ptr[fid + 1];
                            for (uint32_t tt = d.fam_touch_ptr[fid] + kk * 32 + lane; tt < t1; tt += 32 * K) {
                                const int f = (int)d.fam_touch[tt];
                                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                int i = 0;
                                for (; i + 4 <= npay; i += 4) {
                                    float w[4];
#pragma unroll
                                    for (int u = 0; u < 4; u++) w[u] = __ldg(bits + (size_t)(i + u) * d.n_feat + f);
#pragma unroll
                                    for (int u = 0; u < 4; u++) acc[u] = __fadd_rn(acc[u], __fmul_rn(dec_pay[(i + u) * 32 + mm], w[u]));
                                }
                                for (; i < npay; i++)
                                    acc[0] = __fadd_rn(acc[0], __fmul_rn(dec_pay[i * 32 + mm], __ldg(bits + (size_t)i * d.n_feat + f)));
                                const float tot = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
                                put(f, __fadd_rn(__ldg(d.emb_base + (size_t)fid * d.n_feat + f), tot));
                            }
                        }
                    }
                } else {
                    for (int mm = warp; mm < M; mm += QX_NW) {
                        const int fid = dec_i[mm] & 0xFFFFFF, kind = dec_i[mm] >> 24, p = dec_i[32 + mm];
                        float *smw = sm + mm;
                        float *xm = d.x + (size_t)(mbase + mm) * d.D;
                        const bool mact = mbase + mm < d.B;
                        // a feature's value into its row, or (deferred) into x where its sublayer loads it
                        auto put = [&](int f, float v) {
                            const uint32_t fr = d.feat_row[f];
                            if (!(fr & QX_FEAT_DEFERRED)) QX_AT(smw, fr) = v;
                            else if (mact) xm[fr & ~QX_FEAT_DEFERRED] = v;
                        };
                        if (kind != 0) {
                            const uint32_t *w = d.text_words + (size_t)(kind == 1 ? p : 0) * 5;
                            uint32_t wv[5];
#pragma unroll
                            for (int k = 0; k < 5; k++) wv[k] = kind == 1 ? __ldg(w + k) : 0u;
                            for (int f = lane; f < d.n_feat; f += 32) put(f, 0.0f);
                            __syncwarp();
                            for (int tt = lane; tt < d.n_text_touch; tt += 32) {
                                const int f = (int)d.text_touch[tt];
                                float acc = __ldg(d.text_base + f);
#pragma unroll 1
                                for (int k = 0; k < 5; k++) {
                                    uint32_t bits = wv[k];
                                    while (bits) {
                                        const int j = 32 * k + __ffs(bits) - 1;
                                        bits &= bits - 1;
                                        acc = __fadd_rn(acc, __ldg(d.text_bits + (size_t)j * d.n_feat + f));
                                    }
                                }
                                put(f, acc);
                            }
                            continue;
                        }
                        const int row0 = d.fam_row0[fid];
                        if (row0 >= 0) {
                            int r = row0 + p;
                            r = r < 0 ? 0 : (r > d.n_emb_rows - 1 ? d.n_emb_rows - 1 : r);
                            for (int f = lane; f < d.n_feat; f += 32) put(f, __ldg(d.emb_table + (size_t)r * d.n_feat + f));
                        } else {
                            // every feature 0, then the family's touched ones: base + the payload
                            // bits' rows (four partial sums: exact values, any order)
                            const int npay = d.merged ? 16 : d.n_pay;  // (a merged graph reads no payload dims)
                            const float *bits = d.emb_bits + (size_t)fid * npay * d.n_feat;
                            for (int f = lane; f < d.n_feat; f += 32) put(f, 0.0f);
                            __syncwarp();
                            const uint32_t t1 = d.fam_touch_ptr[fid + 1];
                            for (uint32_t tt = d.fam_touch_ptr[fid] + lane; tt < t1; tt += 32) {
                                const int f = (int)d.fam_touch[tt];
                                float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                                int i = 0;
                                for (; i + 4 <= npay; i += 4) {
                                    float w[4];
#pragma unroll
                                    for (int u = 0; u < 4; u++) w[u] = __ldg(bits + (size_t)(i + u) * d.n_feat + f);
#pragma unroll
                                    for (int u = 0; u < 4; u++) acc[u] = __fadd_rn(acc[u], __fmul_rn(dec_pay[(i + u) * 32 + mm], w[u]));
                                }
                                for (; i < npay; i++)
                                    acc[0] = __fadd_rn(acc[0], __fmul_rn(dec_pay[i * 32 + mm], __ldg(bits + (size_t)i * d.n_feat + f)));
                                const float tot = __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
                                put(f, __fadd_rn(__ldg(d.emb_base + (size_t)fid * d.n_feat + f), tot));
                            }
                        }
                    }
                }
                break;
            }
            default:
                break;
            }
            if (!(ph.kind & QX_PH_NOSYNC)) phase_sync(C);
#ifdef QX_PHASE_CLOCKS
            if (threadIdx.x == 0 && d.phase_clk && pc < 256) {
                atomicAdd(&d.phase_clk[2 * pc], (unsigned long long)(clock64() - pclk0));
                atomicAdd(&d.phase_clk[2 * pc + 1], 1ull);
            }
#endif
        }
    }
    if (threadIdx.x == 0 && d.state_bytes) atomicAdd(d.state_bytes, 512ull * *touched);
    if (TC) {
        // (the last phase ended with a barrier after tc_before)  After a wait that gave up, the
        // issuing thread first waits, bounded again, for every MMA it issued: a fresh commit on a
        // second mbarrier tracks them all
        if (threadIdx.x == 0 && tslot[1]) {
            uint64_t *bar2 = mbar + 1;
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(bar2)) : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar2))
                         : "memory");
            mbar_wait(bar2, 0);
        }
        tc_before();
        __syncthreads();
        if (warp == 0) {
            tc_after();
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tslot), "r"(QX_TMEM_COLS)
                         : "memory");
        }
    }
    if (RUN && crank == 0) {
        for (int i = warp * R + way; i < d.n_born0; i += QX_NW * R) {
            uint2 p = d.pairs[i];
            if (act) d.x[(size_t)m * d.D + p.y] = QX_AT(sml, p.x);
        }
        if (warp == 0 && lact) {
            d.hash[m] = hash;
            d.count[m] = count;
            d.halt_at[m] = halt_at;
        }
    }
    // the delta rows the last VHSUM read are cleared for the next launch (every copy has read
    // them: the last phase ended with a barrier)
    {
        float *const Dq = D0 + (dpar ^ 1) * (QX_DELTA_ROWS * 32);
        for (uint32_t j = gw; j < dprev; j += nwv) Dq[j * 32 + lane] = 0.0f;
    }
    if (C > 1) phase_sync(C);  // no CTA leaves while a peer may still address its rows
}

// QH: query rows a value head reads, at most (2 when the plan's heads read at most 2, else 4);
// TC: the plan has tensor-core form phases (the CTA holds tensor memory); a plan without them
// runs an instantiation that contains no tensor-core code at all; R: record slots a warp (groups
// of 32 / R machines a CTA)
#define QX_TOKEN_INST(RUN, QH, TC, R) \
    template __global__ void qx_token_kernel<RUN, QH, TC, R>(const __grid_constant__ QxDev, int32_t, int32_t *);
#define QX_TOKEN_INST_QH(QH, TC, R) QX_TOKEN_INST(0, QH, TC, R) QX_TOKEN_INST(1, QH, TC, R)
QX_TOKEN_INST_QH(2, 0, 1)
QX_TOKEN_INST_QH(4, 0, 1)
QX_TOKEN_INST_QH(2, 1, 1)
QX_TOKEN_INST_QH(4, 1, 1)
QX_TOKEN_INST_QH(2, 0, 2)
QX_TOKEN_INST_QH(4, 0, 2)
QX_TOKEN_INST_QH(2, 0, 4)
QX_TOKEN_INST_QH(4, 0, 4)
QX_TOKEN_INST_QH(2, 0, 8)
QX_TOKEN_INST_QH(4, 0, 8)

// Sets rows [row0, row0 + n) of x to the embeddings of the given tokens (FreeRun.load): chip
// tokens through the family tables, text tokens (merged graphs) through their bits.
__global__ void qx_embed_kernel(const __grid_constant__ QxDev d, int32_t row0, int32_t n, const int32_t *tok) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const int m = row0 + r;
    const int t = tok[r];
    float *x = d.x + (size_t)m * d.D;
    for (int i = threadIdx.x; i < d.D; i += blockDim.x) x[i] = 0.0f;
    __syncthreads();
    const bool bad = t >= QX_TEXT_TOKEN && (!d.merged || t - QX_TEXT_TOKEN >= d.n_text);  // no such text token
    if (t >= QX_TEXT_TOKEN) {
        const int q = t - QX_TEXT_TOKEN;
        if (!bad) {
            const uint32_t *w = d.text_words + (size_t)q * 5;
            for (int f = threadIdx.x; f < d.n_feat; f += blockDim.x) {
                float acc = d.text_base[f];
                for (int j = 0; j < d.n_text_bits; j++)
                    if (w[j >> 5] >> (j & 31) & 1u) acc = __fadd_rn(acc, d.text_bits[(size_t)j * d.n_feat + f]);
                x[d.feat_dim[f]] = acc;
            }
        }
    } else {
        int fid = 0;
        for (int f = 0; f < d.n_families; f++)
            if (t >= d.fam_ids[f] && t < d.fam_ids[f] + d.fam_size[f]) fid = f;
        const int p = t - d.fam_ids[fid];
        const int row0f = d.fam_row0[fid];
        const int npay = d.merged ? 16 : d.n_pay;
        for (int f = threadIdx.x; f < d.n_feat; f += blockDim.x) {
            float v;
            if (row0f >= 0) {
                v = d.emb_table[(size_t)(row0f + p) * d.n_feat + f];
            } else {
                float acc = 0.0f;
                for (int i = 0; i < npay; i++)
                    acc = __fadd_rn(acc, __fmul_rn((float)((p >> i) & 1), d.emb_bits[((size_t)fid * npay + i) * d.n_feat + f]));
                v = __fadd_rn(d.emb_base[(size_t)fid * d.n_feat + f], acc);
            }
            x[d.feat_dim[f]] = v;
        }
    }
    if (threadIdx.x == 0) {
        d.hash[m] = 0xcbf29ce484222325ULL;
        d.count[m] = 0;
        d.halt_at[m] = -1;
        d.err[m] = bad ? QX_E_CODE : 0u;
    }
}
