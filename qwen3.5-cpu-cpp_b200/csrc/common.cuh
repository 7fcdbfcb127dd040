// Shared device helpers for the sm_100a kernels: mbarriers, 1-D bulk TMA copies,
// programmatic-dependent-launch control, bounded waits and the device error flag.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace qwc {

// Error codes a kernel can post in the device error word it is given (first one wins).
// A bounded wait that expires posts its code and the kernel returns early instead of
// hanging the GPU; the host reads the word after each synchronised call.
enum DevError : int {
    DEV_OK = 0,
    DEV_GEMV_FULL_TIMEOUT = 1,    // consumer waited too long for a weight stage
    DEV_GEMV_EMPTY_TIMEOUT = 2,   // producer waited too long for a free stage
    DEV_GEMV_DRAIN_TIMEOUT = 3,   // bulk copies still in flight at exit
    DEV_BAD_TOKEN = 4,            // token id out of range at the embedding
    DEV_BAD_POS = 5,              // position beyond the KV cache
    DEV_PREFILL_TIMEOUT = 6,
    DEV_STEP_BARRIER_TIMEOUT = 7, // a persistent-step CTA waited too long for the grid
    DEV_TC_PRODUCER_TIMEOUT = 8,  // tensor-core GEMM: TMA producer waited for a free stage
    DEV_TC_MMA_TIMEOUT = 9,       // tensor-core GEMM: MMA issuer waited for operands
    DEV_TC_EPI_TIMEOUT = 10,      // tensor-core GEMM: epilogue waited for an accumulator
    DEV_TC_DRAIN_TIMEOUT = 11,    // tensor-core GEMM: in-flight copies / MMAs at exit
    DEV_TP_BARRIER_TIMEOUT = 12,  // peer-memory all-reduce: a rank did not reach a barrier
};

__device__ __forceinline__ void post_error(int* flag, int code) {
    if (flag) atomicCAS(flag, 0, code);
}

// Wall-clock limit of every spin wait (ns). Far above any legitimate wait (a stage
// lands within microseconds), far below a watchdog.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- PDL
// griddepcontrol.wait: wait until the preceding grid(s) completed and their memory is
// visible. A no-op when the kernel was not launched as a programmatic dependent.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// griddepcontrol.launch_dependents: allow the next kernel in the stream to launch.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on phase `parity`; returns false (and posts `err`) when the limit expires.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* flag, int err) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            post_error(flag, err);
            return false;
        }
    }
}

// ---------------------------------------------------------------- bulk TMA (1-D)
// cp.async.bulk global -> shared, completion counted on `bar` in bytes. src, dst and
// bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// As bulk_g2s, with an L2 cache-policy hint (e.g. evict-first for streamed weights).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
        "[%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// L2 policy: lines brought in under it are the first candidates for eviction.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Hint: pull [src, src+bytes) into L2 (no completion to wait on).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- math helpers
// bf16 -> fp32 is exact: the bf16 bits are the top half of the fp32 bits.
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Same formulas as the reference's inline helpers (include/forward_pass.h:21-24), with
// CUDA's expf / log1pf.
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

}  // namespace qwc

namespace qwc {
// Loads n floats (n % 4 == 0, 16-byte aligned) with up to kMaxV float4 per thread issued
// before any is used, so the whole vector costs one memory round trip instead of one per
// loop iteration. Returns false (nothing loaded) if n exceeds 4*kMaxV*nthreads.
template <int kMaxV>
__device__ __forceinline__ bool load_vec4(const float* __restrict__ src, int n, int t, int nthreads,
                                          float4 (&r)[kMaxV]) {
    const int n4 = n >> 2;
    if (n4 > kMaxV * nthreads) return false;
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int k = 0; k < kMaxV; ++k) {
        const int i = t + k * nthreads;
        r[k] = i < n4 ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return true;
}
}  // namespace qwc
