// Decode GEMV family: bf16 weight streaming by 1-D bulk TMA into a shared-memory ring,
// fp32 dot products on CUDA cores, fused prologues/epilogues (see kernels.h).
//
// Work split. The rows of W are cut into gridDim contiguous, balanced ranges (one CTA
// per SM). Inside a CTA, consumer warp w owns rows r0+w, r0+w+8, ...; each row is
// staged in segments of up to 1024 elements (2 KB). Every consumer warp has its own
// `slots_per_warp` ring slots (a full/empty mbarrier pair each); one producer warp
// issues the bulk copies round-robin over the warps. The first ring fill (up to 96 KB
// per CTA) is issued BEFORE griddepcontrol.wait, so under programmatic dependent
// launch the weights of this kernel stream in while the previous kernel finishes.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace qwc {

constexpr int kCW = 8;                    // consumer warps
constexpr int kThreads = (kCW + 1) * 32;  // + 1 producer warp
constexpr int kSeg = 1024;                // elements per staged segment
constexpr int kMaxSlots = 6;

struct SmemPlan {
    size_t ring, xs, bars, red, total;
};

static __host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static __host__ __device__ inline SmemPlan plan_smem(int x_len, int slots) {
    SmemPlan s;
    s.ring = 0;
    size_t ring_bytes = (size_t)kCW * slots * kSeg * 2;
    s.xs = ring_bytes;
    s.bars = align_up(s.xs + (size_t)x_len * 4, 16);
    s.red = s.bars + (size_t)2 * kCW * slots * 8;
    s.total = align_up(s.red + 64 * 4, 128);
    return s;
}

size_t gemv_smem_bytes(const GemvParams& p) { return plan_smem(p.x_len, p.slots_per_warp).total; }

// Consumer-warp named barrier (the producer warp does not take part).
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory");
}

// dot of 8 bf16 weights (one uint4) with 8 fp32 x values
__device__ __forceinline__ float dot8(uint4 w, const float* x, float acc) {
    acc = fmaf(bf16lo(w.x), x[0], acc);
    acc = fmaf(bf16hi(w.x), x[1], acc);
    acc = fmaf(bf16lo(w.y), x[2], acc);
    acc = fmaf(bf16hi(w.y), x[3], acc);
    acc = fmaf(bf16lo(w.z), x[4], acc);
    acc = fmaf(bf16hi(w.z), x[5], acc);
    acc = fmaf(bf16lo(w.w), x[6], acc);
    acc = fmaf(bf16hi(w.w), x[7], acc);
    return acc;
}

// Block-wide (consumer warps) sum in double, identical result in every thread.
__device__ __forceinline__ double consumers_sum_d(double v, double* red_d) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red_d[warp] = v;
    consumers_sync();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kCW; ++w) s += red_d[w];
    consumers_sync();
    return s;
}

template <int PRO, int EPI, bool XREG>
__global__ void __launch_bounds__(kThreads, 2) k_gemv(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int SL = p.slots_per_warp;
    const SmemPlan plan = plan_smem(p.x_len, SL);
    uint16_t* ring = reinterpret_cast<uint16_t*>(smem);
    float* xs = reinterpret_cast<float*>(smem + plan.xs);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.bars);
    uint64_t* empty = full + kCW * SL;
    double* red_d = reinterpret_cast<double*>(smem + plan.red);

    const int in = p.in_dim, xlen = p.x_len;
    const int seg_len = in < kSeg ? in : kSeg;
    const int nseg = (in + seg_len - 1) / seg_len;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = (int)((long long)p.rows * blockIdx.x / gridDim.x);
    const int r1 = (int)((long long)p.rows * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kCW * SL; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // ------------------------------------------------------------ producer warp
    if (warp == kCW) {
        if (lane == 0) {
            const int max_rows_w = (r1 - r0 + kCW - 1) / kCW;
            const int max_items = max_rows_w * nseg;
            int issued[kCW * kMaxSlots];
            for (int i = 0; i < kCW * SL; ++i) issued[i] = 0;
            bool ok = true, waited = false;
            for (int k = 0; k < max_items && ok; ++k) {
                if (k == SL && !waited) {
                    pdl_wait();
                    pdl_launch_dependents();
                    waited = true;
                }
                const int j = k / nseg, s = k - j * nseg;
                for (int w = 0; w < kCW; ++w) {
                    const int row = r0 + w + kCW * j;
                    if (row >= r1) break;
                    const int slot = w * SL + (k % SL);
                    if (k >= SL &&
                        !mbar_wait_bounded(&empty[slot], ((k / SL) - 1) & 1, p.dev_err, DEV_GEMV_EMPTY_TIMEOUT)) {
                        ok = false;
                        break;
                    }
                    const int c0 = s * seg_len;
                    const int len = min(seg_len, in - c0);
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)len * 2);
                    bulk_g2s(ring + (size_t)slot * kSeg, p.W + (size_t)row * in + c0, (uint32_t)len * 2,
                             &full[slot]);
                    issued[slot]++;
                }
            }
            if (!waited) {
                pdl_wait();
                pdl_launch_dependents();
            }
            // Drain: every issued copy must have landed before this CTA may exit. One
            // overall time window; after it expires the remaining slots are not awaited.
            bool drained = true;
            for (int i = 0; i < kCW * SL && drained; ++i)
                if (issued[i] > 0)
                    drained = mbar_wait_bounded(&full[i], (issued[i] - 1) & 1, p.dev_err, DEV_GEMV_DRAIN_TIMEOUT);
        }
        return;
    }

    // ------------------------------------------------------------ consumer warps
    pdl_wait();
    const int tid = threadIdx.x;  // 0 .. kCW*32-1
    constexpr int NT = kCW * 32;
    if constexpr (PRO == PRO_PLAIN) {
        for (int i = tid; i < xlen; i += NT) xs[i] = p.x[i];
        consumers_sync();
    } else if constexpr (PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM) {
        const float* src = p.x;
        if constexpr (PRO == PRO_EMBED_RMSNORM) {
            int tok = p.tokens[*p.pos];
            if (tok < 0 || tok >= p.vocab) {
                if (tid == 0) post_error(p.dev_err, DEV_BAD_TOKEN);
                tok = 0;
            }
            const uint16_t* row = p.embed + (size_t)tok * xlen;
            for (int i = tid; i < xlen; i += NT) {
                float v = __uint_as_float((uint32_t)row[i] << 16);
                xs[i] = v;
                if (blockIdx.x == 0) p.hidden_out[i] = v;
            }
            consumers_sync();
        } else {
            for (int i = tid; i < xlen; i += NT) xs[i] = src[i];
            consumers_sync();
        }
        double ss = 0.0;
        for (int i = tid; i < xlen; i += NT) ss += (double)xs[i] * xs[i];
        ss = consumers_sum_d(ss, red_d);
        const float inv = 1.0f / sqrtf((float)(ss / xlen) + p.eps);
        for (int i = tid; i < xlen; i += NT) xs[i] = xs[i] * inv * p.norm_w[i];
        consumers_sync();
    } else if constexpr (PRO == PRO_GATED_NORM) {
        // one warp per head of gn_dim values: w * (o * inv_head) * silu(z)
        const int D = p.gn_dim, nh = xlen / D;
        for (int h = warp; h < nh; h += kCW) {
            const float* o = p.x + (size_t)h * D;
            double ss = 0.0;
            for (int i = lane; i < D; i += 32) ss += (double)o[i] * o[i];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float inv = 1.0f / sqrtf((float)(ss / D) + p.eps);
            for (int i = lane; i < D; i += 32) {
                const float zz = p.z[(size_t)h * D + i];
                xs[(size_t)h * D + i] = p.norm_w[i] * (o[i] * inv) * silu_f(zz);
            }
        }
        consumers_sync();
    }
    pdl_launch_dependents();

    // x chunks of this lane in registers when one 1024-element segment spans all of x
    float xr[XREG ? 4 : 1][8];
    if constexpr (XREG) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 8; ++e) xr[c][e] = xs[(lane + 32 * c) * 8 + e];
    }

    float best = -INFINITY;
    int best_idx = 0x7fffffff;
    bool ok = true;
    int k = 0;  // item counter of this warp
    for (int row = r0 + warp; row < r1 && ok; row += kCW) {
        float acc = 0.f, acc_u = 0.f;
        for (int s = 0; s < nseg; ++s, ++k) {
            const int slot = warp * SL + (k % SL);
            if (!mbar_wait_bounded(&full[slot], (k / SL) & 1, p.dev_err, DEV_GEMV_FULL_TIMEOUT)) {
                ok = false;
                break;
            }
            const uint4* wv = reinterpret_cast<const uint4*>(ring + (size_t)slot * kSeg);
            const int c0 = s * seg_len;
            const int nch = min(seg_len, in - c0) / 8;
            if constexpr (XREG) {
                float a = 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int ch = lane + 32 * c;
                    if (ch < nch) a = dot8(wv[ch], xr[c], a);
                }
                if (EPI == EPI_SWIGLU && c0 >= xlen) acc_u += a; else acc += a;
            } else {
                for (int ch = lane; ch < nch; ch += 32) {
                    const int col = c0 + ch * 8;
                    if (EPI == EPI_SWIGLU && col >= xlen) {
                        acc_u = dot8(wv[ch], xs + (col - xlen), acc_u);
                    } else {
                        acc = dot8(wv[ch], xs + col, acc);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (!ok) break;
        acc = warp_sum(acc);
        if constexpr (EPI == EPI_SWIGLU) acc_u = warp_sum(acc_u);
        if (lane == 0) {
            if constexpr (EPI == EPI_STORE) {
                p.y[row] = acc;
            } else if constexpr (EPI == EPI_RESIDUAL) {
                p.y[row] = p.y[row] + acc;
            } else if constexpr (EPI == EPI_SWIGLU) {
                p.y[row] = silu_f(acc) * acc_u;
            } else {
                p.y[row] = acc;
                if (acc > best) { best = acc; best_idx = row; }
            }
        }
    }

    if constexpr (EPI == EPI_ARGMAX) {
        // CTA argmax: larger value wins, equal values -> lower index (strict '>' scan).
        float* rv = reinterpret_cast<float*>(red_d);
        int* ri = reinterpret_cast<int*>(rv + kCW);
        if (lane == 0) { rv[warp] = best; ri[warp] = best_idx; }
        consumers_sync();
        __shared__ int s_last;
        if (tid == 0) {
            float bv = rv[0];
            int bi = ri[0];
            for (int w = 1; w < kCW; ++w)
                if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
            p.am_val[blockIdx.x] = bv;
            p.am_idx[blockIdx.x] = bi;
            __threadfence();
            const unsigned t = atomicAdd(p.am_counter, 1u);
            s_last = (t == gridDim.x - 1) ? 1 : 0;
        }
        consumers_sync();
        if (s_last) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = tid; c < (int)gridDim.x; c += NT) {
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
            if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
            consumers_sync();
            if (tid == 0) {
                bv = rv[0];
                bi = ri[0];
                for (int w = 1; w < kCW; ++w)
                    if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
                if (bi == 0x7fffffff) bi = 0;  // all logits NaN: the reference scan keeps id 0
                if (p.argmax_out) *p.argmax_out = bi;
                if (p.pos_inout) {
                    const int pos = *p.pos_inout;
                    if (p.tokens_out && pos + 1 < p.max_ctx && pos + 1 >= *p.n_prompt)
                        p.tokens_out[pos + 1] = bi;
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

int gemv_grid(int rows) { return std::max(1, std::min(rows, num_sms())); }

template <int PRO, int EPI, bool XREG>
static cudaError_t launch_one(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    const size_t smem = gemv_smem_bytes(p);
    auto kern = k_gemv<PRO, EPI, XREG>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 120 * 1024);
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

template <int PRO, int EPI>
static cudaError_t launch_x(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    const int seg_len = p.in_dim < kSeg ? p.in_dim : kSeg;
    const bool xreg = (p.x_len == kSeg) && (seg_len == kSeg);
    return xreg ? launch_one<PRO, EPI, true>(p, grid, s, pdl) : launch_one<PRO, EPI, false>(p, grid, s, pdl);
}

cudaError_t launch_gemv(int pro, int epi, GemvParams p, int grid, cudaStream_t s, bool pdl) {
    if (p.in_dim <= 0 || p.in_dim % 8 != 0 || p.rows <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(p.W) & 15) != 0) return cudaErrorInvalidValue;
    // ring depth: keep the CTA under ~112 KB so two GEMV CTAs fit one SM (PDL overlap)
    const size_t xs_bytes = (size_t)p.x_len * 4;
    int slots = (int)((112 * 1024 - 1024 - (long)xs_bytes) / (kCW * kSeg * 2));
    p.slots_per_warp = std::max(2, std::min(kMaxSlots, slots));
    if (gemv_smem_bytes(p) > 120 * 1024) return cudaErrorInvalidValue;
#define QWC_GEMV_CASE(PR, EP) \
    if (pro == PR && epi == EP) return launch_x<PR, EP>(p, grid, s, pdl);
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
