// Decode GEMV family: bf16 weights streamed from HBM straight into registers, fp32 dot
// products on CUDA cores, fused prologues/epilogues (see kernels.h).
//
// Work split. The rows of W are cut into gridDim balanced contiguous ranges (one CTA per
// SM), and each CTA range into 8 balanced contiguous warp ranges. A warp walks its rows
// as one flat stream of "groups": 32 lanes x 16 bytes = 256 consecutive elements of a
// row. Loads are 128-bit, non-coherent, L1-bypassing, issued in batches of kU groups per
// lane into two register buffers used in ping-pong, so every warp keeps up to 2*kU x 512 B
// in flight; two CTAs per SM.
//
// Programmatic dependent launch: the weights do not depend on the previous kernel, so
// before griddepcontrol.wait each warp (a) asks L2 to prefetch the start of its row
// block and (b) issues its first register batch. Only x (the activation) waits.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>

namespace qwc {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kU = 8;                       // groups per batch per lane
constexpr uint32_t kPrefetchPiece = 8192;   // bytes per L2 prefetch request
constexpr uint32_t kPrefetchCap = 32768;    // bytes prefetched per warp before the wait

size_t gemv_smem_bytes(const GemvParams& p) { return ((size_t)p.x_len * 4 + 15) / 16 * 16; }

// 128-bit streaming load: read-only path, no L1 allocation, 256-byte L2 fetch granule.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// dot of 8 bf16 weights (one uint4) with 8 fp32 x values
__device__ __forceinline__ float dot8(uint4 w, const float* x, float acc) {
    const float4 x0 = *reinterpret_cast<const float4*>(x);
    const float4 x1 = *reinterpret_cast<const float4*>(x + 4);
    acc = fmaf(bf16lo(w.x), x0.x, acc);
    acc = fmaf(bf16hi(w.x), x0.y, acc);
    acc = fmaf(bf16lo(w.y), x0.z, acc);
    acc = fmaf(bf16hi(w.y), x0.w, acc);
    acc = fmaf(bf16lo(w.z), x1.x, acc);
    acc = fmaf(bf16hi(w.z), x1.y, acc);
    acc = fmaf(bf16lo(w.w), x1.z, acc);
    acc = fmaf(bf16hi(w.w), x1.w, acc);
    return acc;
}

// Block-wide sum in double, identical result in every thread.
__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w];
    return s;
}

// Cursor over a warp's group stream: group -> (row, q), q = group index inside the row.
struct Cursor {
    int row, q;
    __device__ __forceinline__ void next(int gpr) {
        if (++q == gpr) { q = 0; ++row; }
    }
};

template <int PRO, int EPI>
__global__ void __launch_bounds__(kThreads, 2) k_gemv(const GemvParams p) {
    extern __shared__ __align__(16) float xs[];
    __shared__ double red_d[kWarps];
    __shared__ float rv[kWarps];
    __shared__ int ri[kWarps];
    __shared__ int s_last;

    const int in = p.in_dim, xlen = p.x_len;
    const int cpr = in >> 3;             // 16-byte chunks per row
    const int gpr = (cpr + 31) >> 5;     // groups per row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int r0 = (int)((long long)p.rows * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)p.rows * (blockIdx.x + 1) / gridDim.x);
    const int nr = r1 - r0;
    const int a = r0 + (int)((long long)nr * warp / kWarps);
    const int b = r0 + (int)((long long)nr * (warp + 1) / kWarps);
    const long long G = (long long)(b - a) * gpr;
    const uint16_t* W = p.W;

    // ---- before the dependency wait: L2 prefetch + first register batch of weights
    if (b > a) {
        const uint8_t* base = reinterpret_cast<const uint8_t*>(W + (size_t)a * in);
        const size_t bytes = (size_t)(b - a) * in * 2;
        const uint32_t cap = kPrefetchCap, piece = kPrefetchPiece;
        const uint32_t lim = bytes < (size_t)cap ? (uint32_t)bytes : cap;
        for (uint32_t off = lane * piece; off < lim; off += 32 * piece)
            bulk_prefetch_l2(base + off, min(piece, lim - off));
    }
    uint4 cur[kU], nxt[kU];
    Cursor lc{a, 0};  // load cursor
    auto load_batch = [&](long long g0, uint4* dst) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int c = lc.q * 32 + lane;
            if (g0 + u < G && c < cpr) dst[u] = ld_stream(W + (size_t)lc.row * in + (size_t)c * 8);
            else dst[u] = make_uint4(0u, 0u, 0u, 0u);
            if (g0 + u < G) lc.next(gpr);
        }
    };
    load_batch(0, cur);

    pdl_wait();
    // ---- prologue: build x in shared memory
    if constexpr (PRO == PRO_PLAIN) {
        for (int i = tid; i < xlen; i += kThreads) xs[i] = p.x[i];
        __syncthreads();
    } else if constexpr (PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM) {
        if constexpr (PRO == PRO_EMBED_RMSNORM) {
            int tok = p.tokens[*p.pos];
            if (tok < 0 || tok >= p.vocab) {
                if (tid == 0) post_error(p.dev_err, DEV_BAD_TOKEN);
                tok = 0;
            }
            const uint16_t* row = p.embed + (size_t)tok * xlen;
            for (int i = tid; i < xlen; i += kThreads) {
                const float v = __uint_as_float((uint32_t)row[i] << 16);
                xs[i] = v;
                if (blockIdx.x == 0) p.hidden_out[i] = v;
            }
        } else {
            for (int i = tid; i < xlen; i += kThreads) xs[i] = p.x[i];
        }
        double ss = 0.0;
        for (int i = tid; i < xlen; i += kThreads) ss += (double)xs[i] * xs[i];
        ss = block_sum_d(ss, red_d);  // also orders the xs stores above
        const float inv = 1.0f / sqrtf((float)(ss / xlen) + p.eps);
        for (int i = tid; i < xlen; i += kThreads) xs[i] = xs[i] * inv * p.norm_w[i];
        __syncthreads();
    } else if constexpr (PRO == PRO_GATED_NORM) {
        // one warp per head of gn_dim values: w * (o * inv_head) * silu(z)
        const int D = p.gn_dim, nh = xlen / D;
        for (int h = warp; h < nh; h += kWarps) {
            const float* o = p.x + (size_t)h * D;
            double ss = 0.0;
            for (int i = lane; i < D; i += 32) ss += (double)o[i] * o[i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float inv = 1.0f / sqrtf((float)(ss / D) + p.eps);
            for (int i = lane; i < D; i += 32)
                xs[(size_t)h * D + i] = p.norm_w[i] * (o[i] * inv) * silu_f(p.z[(size_t)h * D + i]);
        }
        __syncthreads();
    }
    pdl_launch_dependents();

    // ---- main stream: two register buffers in ping-pong, no copies between them, so
    // one batch stays in flight while the other is consumed
    float acc = 0.f, acc_u = 0.f;
    float best = -INFINITY;
    int best_idx = 0x7fffffff;
    Cursor cc{a, 0};  // compute cursor
    auto consume = [&](long long g0, const uint4* buf) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            if (g0 + u < G) {
                const int c = cc.q * 32 + lane;
                if (c < cpr) {
                    const int col = c * 8;
                    if (EPI == EPI_SWIGLU && col >= xlen) acc_u = dot8(buf[u], xs + (col - xlen), acc_u);
                    else acc = dot8(buf[u], xs + col, acc);
                }
                if (cc.q == gpr - 1) {
                    const float s = warp_sum(acc);
                    float su = 0.f;
                    if constexpr (EPI == EPI_SWIGLU) su = warp_sum(acc_u);
                    if (lane == 0) {
                        const int row = cc.row;
                        if constexpr (EPI == EPI_STORE) {
                            p.y[row] = s;
                        } else if constexpr (EPI == EPI_RESIDUAL) {
                            p.y[row] = p.y[row] + s;
                        } else if constexpr (EPI == EPI_SWIGLU) {
                            p.y[row] = silu_f(s) * su;
                        } else {
                            p.y[row] = s;
                            if (s > best) { best = s; best_idx = row; }
                        }
                    }
                    acc = 0.f;
                    acc_u = 0.f;
                }
                cc.next(gpr);
            }
        }
    };
    for (long long g0 = 0; g0 < G; g0 += 2 * kU) {
        if (g0 + kU < G) load_batch(g0 + kU, nxt);
        consume(g0, cur);
        if (g0 + 2 * kU < G) load_batch(g0 + 2 * kU, cur);
        if (g0 + kU < G) consume(g0 + kU, nxt);
    }

    if constexpr (EPI == EPI_ARGMAX) {
        // CTA argmax: larger value wins, equal values -> lower index (strict '>' scan).
        if (lane == 0) { rv[warp] = best; ri[warp] = best_idx; }
        __syncthreads();
        if (tid == 0) {
            float bv = rv[0];
            int bi = ri[0];
            for (int w = 1; w < kWarps; ++w)
                if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
            p.am_val[blockIdx.x] = bv;
            p.am_idx[blockIdx.x] = bi;
            __threadfence();
            const unsigned t = atomicAdd(p.am_counter, 1u);
            s_last = (t == gridDim.x - 1) ? 1 : 0;
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = tid; c < (int)gridDim.x; c += kThreads) {
                const float v = __ldcg(&p.am_val[c]);
                const int i = __ldcg(&p.am_idx[c]);
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            __syncthreads();
            if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
            __syncthreads();
            if (tid == 0) {
                bv = rv[0];
                bi = ri[0];
                for (int w = 1; w < kWarps; ++w)
                    if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
                if (bi == 0x7fffffff) bi = 0;  // all logits NaN: the reference scan keeps id 0
                if (p.argmax_out) *p.argmax_out = bi;
                if (p.pos_inout) {
                    const int pos = *p.pos_inout;
                    if (p.tokens_out && pos + 1 < p.max_ctx && pos + 1 >= *p.n_prompt) p.tokens_out[pos + 1] = bi;
                    *p.pos_inout = pos + 1;
                }
                *p.am_counter = 0u;
            }
        }
    }
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// One CTA per SM by default: a GEMV CTA holds half of an SM's registers, so the CTA of
// the next kernel (programmatic dependent launch) fits beside it and prefetches its own
// weights while this one streams. The lm_head, last of the step, uses two per SM.
int gemv_grid(int rows, int per_sm) {
    static int override_per_sm = -1;
    if (override_per_sm < 0) {
        const char* e = std::getenv("QWC_GEMV_CTAS_PER_SM");  // tuning knob, 0 = default
        override_per_sm = e ? std::atoi(e) : 0;
    }
    if (override_per_sm > 0) per_sm = override_per_sm;
    return std::max(1, std::min(rows, per_sm * num_sms()));
}

template <int PRO, int EPI>
static cudaError_t launch_one(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = gemv_smem_bytes(p);
    auto kern = k_gemv<PRO, EPI>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

cudaError_t launch_gemv(int pro, int epi, GemvParams p, int grid, cudaStream_t s, bool pdl) {
    if (p.in_dim <= 0 || p.in_dim % 8 != 0 || p.rows <= 0 || p.x_len <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.W) & 15) != 0) return cudaErrorInvalidValue;
    if (epi == EPI_SWIGLU ? (p.in_dim != 2 * p.x_len || p.x_len % 8) : (p.in_dim != p.x_len))
        return cudaErrorInvalidValue;
    if (gemv_smem_bytes(p) > 96 * 1024) return cudaErrorInvalidValue;
#define QWC_GEMV_CASE(PR, EP) \
    if (pro == PR && epi == EP) return launch_one<PR, EP>(p, grid, s, pdl);
    QWC_GEMV_CASE(PRO_PLAIN, EPI_STORE)
    QWC_GEMV_CASE(PRO_PLAIN, EPI_RESIDUAL)
    QWC_GEMV_CASE(PRO_RMSNORM, EPI_STORE)
    QWC_GEMV_CASE(PRO_EMBED_RMSNORM, EPI_STORE)
    QWC_GEMV_CASE(PRO_GATED_NORM, EPI_RESIDUAL)
    QWC_GEMV_CASE(PRO_RMSNORM, EPI_SWIGLU)
    QWC_GEMV_CASE(PRO_RMSNORM, EPI_ARGMAX)
#undef QWC_GEMV_CASE
    return cudaErrorInvalidValue;
}

}  // namespace qwc
