// qx_gdn.cu -- one gated delta-rule decode step over BH independent heads (dk = dv = 128).
//
//   S <- alpha S;  kv = S^T k;  delta = beta (v - kv);  S <- S + k (x) delta;  o = S^T q
//
// (the recurrence of transformers' torch_recurrent_gated_delta_rule,
// models/qwen3_5/modeling_qwen3_5.py, without its query scale; the circuit's one-hot case is
// ERV/chipformer/q35/ir.py:470-495).  Sums over the key index run i = 0..127 in order with every
// product rounded before it is added, so results do not depend on the path taken:
//
//   row path     alpha == 1, a key with at most one nonzero, a query with at most one nonzero:
//                one warp reads the key's row and the query's row (512 B each), rewrites the
//                key's row; every other row is unchanged (x + 0 * delta == x);
//   matrix path  everything else: one CTA streams the 64 KB state through shared memory with
//                TMA bulk copies (cp.async.bulk), scales it, forms kv column by column, applies
//                the rank-1 update and the read, and writes the state back.  alpha == 0 skips
//                the load (0 * S == 0).
//
// The row path runs first and queues the matrix-path heads in `work` (a count, an error word,
// then head indices); the matrix kernel drains that queue.  Waits on the TMA barrier are bounded:
// on timeout the CTA records QX_ERR_DEVICE_FLAG in the error word (work[1]), waits (bounded
// again) for its copy in flight and returns; the states of a flagged step are undefined.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "qx.h"

#define GDN_D 128
#define GDN_MAT (GDN_D * GDN_D)

namespace {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// position of the single nonzero among 128 values held 4 per lane (-1: none, -2: several)
__device__ __forceinline__ int single_nonzero(float4 a, int lane, float &val) {
    const float c[4] = {a.x, a.y, a.z, a.w};
    int cnt = 0, pos = -1;
    float v = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (c[i] != 0.0f) { cnt++; pos = lane * 4 + i; v = c[i]; }
    const int tot = __reduce_add_sync(0xFFFFFFFFu, cnt);
    if (tot == 0) { val = 0.0f; return -1; }
    if (tot > 1) return -2;
    const unsigned who = __ballot_sync(0xFFFFFFFFu, cnt == 1);
    const int src = __ffs(who) - 1;
    val = __shfl_sync(0xFFFFFFFFu, v, src);
    return __shfl_sync(0xFFFFFFFFu, pos, src);
}

}  // namespace

__global__ void __launch_bounds__(256) qx_gdn_rows_kernel(int64_t BH, float *__restrict__ S,
                                                          const float *__restrict__ q, const float *__restrict__ k,
                                                          const float *__restrict__ v, const float *__restrict__ alpha,
                                                          const float *__restrict__ beta, float *__restrict__ o,
                                                          uint32_t *work) {
    const int lane = threadIdx.x & 31;
    // the matrix kernel may be scheduled now: it waits (griddepcontrol.wait) for this grid's
    // completion before it reads the queue, but its CTAs are resident and set up by then
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int64_t bh = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (bh >= BH) return;
    const float4 kk = reinterpret_cast<const float4 *>(k + bh * GDN_D)[lane];
    const float4 qq = reinterpret_cast<const float4 *>(q + bh * GDN_D)[lane];
    const float a = alpha[bh];
    float kr, qv;
    const int r = single_nonzero(kk, lane, kr);
    const int rq = single_nonzero(qq, lane, qv);
    if (a != 1.0f || r == -2 || rq == -2) {
        if (lane == 0) work[2 + atomicAdd(&work[0], 1u)] = (uint32_t)bh;
        return;
    }
    float *Sb = S + bh * GDN_MAT;
    float4 row = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r >= 0) {
        const float4 vv = reinterpret_cast<const float4 *>(v + bh * GDN_D)[lane];
        const float b = beta[bh];
        float4 *pr = reinterpret_cast<float4 *>(Sb + (size_t)r * GDN_D) + lane;
        row = *pr;
        // kv_j = S[r][j] k_r; delta_j = (v_j - kv_j) beta; S[r][j] += k_r delta_j
        row.x = __fadd_rn(row.x, __fmul_rn(kr, __fmul_rn(__fsub_rn(vv.x, __fmul_rn(row.x, kr)), b)));
        row.y = __fadd_rn(row.y, __fmul_rn(kr, __fmul_rn(__fsub_rn(vv.y, __fmul_rn(row.y, kr)), b)));
        row.z = __fadd_rn(row.z, __fmul_rn(kr, __fmul_rn(__fsub_rn(vv.z, __fmul_rn(row.z, kr)), b)));
        row.w = __fadd_rn(row.w, __fmul_rn(kr, __fmul_rn(__fsub_rn(vv.w, __fmul_rn(row.w, kr)), b)));
        *pr = row;
    }
    float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rq >= 0) {
        const float4 sq = rq == r ? row : reinterpret_cast<const float4 *>(Sb + (size_t)rq * GDN_D)[lane];
        out = make_float4(__fmul_rn(sq.x, qv), __fmul_rn(sq.y, qv), __fmul_rn(sq.z, qv), __fmul_rn(sq.w, qv));
    }
    reinterpret_cast<float4 *>(o + bh * GDN_D)[lane] = out;
}

// One CTA (128 threads: thread j owns column j) per queued head; the state goes through 64 KB
// of shared memory via TMA bulk copies.
__global__ void __launch_bounds__(128) qx_gdn_matrix_kernel(float *__restrict__ S, const float *__restrict__ q,
                                                            const float *__restrict__ k, const float *__restrict__ v,
                                                            const float *__restrict__ alpha,
                                                            const float *__restrict__ beta, float *__restrict__ o,
                                                            uint32_t *work) {
    extern __shared__ __align__(128) float sS[];  // [128][128]
    __shared__ float sk[GDN_D], sq[GDN_D];
    __shared__ __align__(8) uint64_t bar;
    const int j = threadIdx.x;
    if (j == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the row kernel (launched before this one, which may start early) has finished and its
    // queue is visible after this
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t n = *reinterpret_cast<volatile uint32_t *>(&work[0]);
    __syncthreads();
    uint32_t phase = 0;
    for (uint32_t it = blockIdx.x; it < n; it += gridDim.x) {
        const int64_t bh = work[2 + it];
        float *Sb = S + bh * GDN_MAT;
        const float a = alpha[bh], b = beta[bh];
        sk[j] = k[bh * GDN_D + j];
        sq[j] = q[bh * GDN_D + j];
        const float vj = v[bh * GDN_D + j];
        if (a != 0.0f) {
            if (j == 0) {
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&bar)),
                             "r"(GDN_MAT * 4)
                             : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        smem_addr(sS)),
                    "l"(Sb), "r"(GDN_MAT * 4), "r"(smem_addr(&bar))
                    : "memory");
            }
            // bounded wait on the barrier phase
            uint32_t done = 0;
            for (uint32_t spin = 0; spin < (1u << 24) && !done; spin++) {
                asm volatile(
                    "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                    : "=r"(done)
                    : "r"(smem_addr(&bar)), "r"(phase)
                    : "memory");
            }
            phase ^= 1;
            if (!__syncthreads_and(done)) {
                // the copy may still be landing in this CTA's shared memory: give it a second
                // bounded wait before the CTA leaves (a flagged step leaves S undefined)
                if (j == 0) {
                    atomicOr(&work[1], QX_ERR_DEVICE_FLAG);
                    for (uint32_t spin = 0; spin < (1u << 24) && !done; spin++) {
                        asm volatile(
                            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, "
                            "0, p; }"
                            : "=r"(done)
                            : "r"(smem_addr(&bar)), "r"(phase ^ 1)
                            : "memory");
                    }
                }
                __syncthreads();
                return;
            }
        } else {
            __syncthreads();
            for (int i = 0; i < GDN_D; i++) sS[i * GDN_D + j] = 0.0f;  // 0 * S (no load needed)
        }
        // two passes over the column: alpha * S is recomputed (the same rounding) instead of
        // being written back first
        float kv = 0.0f;
#pragma unroll 8
        for (int i = 0; i < GDN_D; i++) kv = __fadd_rn(kv, __fmul_rn(__fmul_rn(sS[i * GDN_D + j], a), sk[i]));
        const float delta = __fmul_rn(__fsub_rn(vj, kv), b);
        float oj = 0.0f;
#pragma unroll 8
        for (int i = 0; i < GDN_D; i++) {
            const float s2 = __fadd_rn(__fmul_rn(sS[i * GDN_D + j], a), __fmul_rn(sk[i], delta));
            sS[i * GDN_D + j] = s2;
            oj = __fadd_rn(oj, __fmul_rn(s2, sq[i]));
        }
        o[bh * GDN_D + j] = oj;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (j == 0) {
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(Sb), "r"(smem_addr(sS)),
                         "r"(GDN_MAT * 4)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        }
        __syncthreads();
    }
    if (j == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

cudaError_t qx_gdn_launch(int64_t BH, float *S, const float *q, const float *k, const float *v, const float *alpha,
                          const float *beta, float *o, uint32_t *work, cudaStream_t st) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaMemsetAsync(work, 0, 8, st);
    if (e != cudaSuccess) return e;
    const int per = 8;  // warps per CTA in the row kernel
    qx_gdn_rows_kernel<<<(unsigned)((BH + per - 1) / per), per * 32, 0, st>>>(BH, S, q, k, v, alpha, beta, o, work);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // programmatic dependent launch: the matrix kernel's CTAs start while the row kernel drains
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms * 3));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = GDN_MAT * 4;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, qx_gdn_matrix_kernel, S, q, k, v, alpha, beta, o, work);
}

cudaError_t qx_gdn_prepare() {
    return cudaFuncSetAttribute(qx_gdn_matrix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_MAT * 4);
}

#define QX_GDN_MAX_DEVICES 64

// qx_gdn_prepare on the current device, once per device (the attribute belongs to the device,
// not to the calling thread); later calls only read a flag.
cudaError_t qx_gdn_prepare_current() {
    static std::mutex mu;
    static bool done[QX_GDN_MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= QX_GDN_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        e = qx_gdn_prepare();
        if (e != cudaSuccess) return e;
        done[dev] = true;
    }
    return cudaSuccess;
}

// ---- scratch for the allocation-free entry point (qx_gdn_step_noalloc) ------------------------
// The queue of the step (count, error word, head indices) for up to QX_GDN_NOALLOC_MAX_BH heads,
// as a fixed array of this library's device image: 256 KB + 8 B on every device that loads the
// library, held until the process exits.  Every call on a device shares it; the launch clears the
// count and the error word, and the row kernel writes each index before the matrix kernel reads it.
static __device__ __align__(256) uint32_t g_gdn_scratch[2 + QX_GDN_NOALLOC_MAX_BH];

// The array's address on the current device.  The first request on a device, with that device
// current, looks the address up (which can load this library's kernels onto the device) and sets
// the matrix kernel's shared-memory limit there; later requests only read the cached address.
cudaError_t qx_gdn_noalloc_scratch(uint32_t **out) {
    static std::mutex mu;
    static uint32_t *addr[QX_GDN_MAX_DEVICES] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= QX_GDN_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gdn_scratch);
        if (e != cudaSuccess) return e;
        e = qx_gdn_prepare_current();
        if (e != cudaSuccess) return e;
        addr[dev] = static_cast<uint32_t *>(p);
    }
    *out = addr[dev];
    return cudaSuccess;
}
