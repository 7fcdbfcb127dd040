// Decode gated GQA attention (QwenModel::attn_step, src/qwen_model.cpp:118-150):
//   q_h = rope(rmsnorm(q_raw_h) * (1+q_norm)), k = rope(rmsnorm(k_raw) * (1+k_norm))
//   K[pos] = k, V[pos] = v_raw                          (cache append)
//   o_h = softmax(q_h K^T / sqrt(HD)) V over positions 0..pos, then o_h *= sigmoid(gate_h)
//
// Grid (NKV, nsplit): CTA (kv, sp) takes a contiguous range of positions for the GRP
// query heads of kv head `kv` (flash-decode: online softmax over 64-position tiles).
// The number of active splits follows the live context length (read from the device
// position, so one captured graph serves every step). The CTA whose range holds the
// new position computes and stores K/V[pos] itself and is the only reader of that row.
// The last CTA of a kv head (atomic ticket) merges the partial (max, sum, acc) triples
// and applies the sigmoid gate.
//
// RoPE angle: pos * inv_freq[i] in double, cos/sin in double, rounded to float, with
// inv_freq = theta^(-2i/rot) tabulated on the host in double (forward_pass.cpp:102-112).
#include "common.cuh"
#include "kernels.h"

namespace qwc {

constexpr int kHD = 256;
constexpr int kTile = 64;
constexpr int kAttnThreads = 256;

__device__ __forceinline__ void load8(const void* base, int kv_bf16, size_t off, float* o) {
    if (kv_bf16) {
        const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + off);
        o[0] = bf16lo(w.x); o[1] = bf16hi(w.x); o[2] = bf16lo(w.y); o[3] = bf16hi(w.y);
        o[4] = bf16lo(w.z); o[5] = bf16hi(w.z); o[6] = bf16lo(w.w); o[7] = bf16hi(w.w);
    } else {
        const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
        const float4 a = f[0], b = f[1];
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
}
__device__ __forceinline__ float load1(const void* base, int kv_bf16, size_t off) {
    if (kv_bf16) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(base)[off] << 16);
    return reinterpret_cast<const float*>(base)[off];
}
// fp32 -> bf16 round-to-nearest-even (finite inputs)
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// sum over the 256 threads in double, same value in all threads
__device__ __forceinline__ double block256_sum_d(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w];
    return s;
}

// rmsnorm(x)*(1+w) then partial rotate_half RoPE, one vector of kHD in shared memory.
// Thread d handles element d.
__device__ __forceinline__ void norm_rope(float* v, const float* w1, float eps, int rot,
                                          const double* inv_freq, int pos, double* red) {
    const int d = threadIdx.x;
    const float x = v[d];
    const double ss = block256_sum_d((double)x * x, red);
    const float inv = 1.0f / sqrtf((float)(ss / kHD) + eps);
    v[d] = x * inv * w1[d];
    __syncthreads();
    const int half = rot / 2;
    if (d < half) {
        const double ang = (double)pos * inv_freq[d];
        const float c = (float)cos(ang), s = (float)sin(ang);
        const float x1 = v[d], x2 = v[d + half];
        v[d] = x1 * c - x2 * s;
        v[d + half] = x2 * c + x1 * s;
    }
    __syncthreads();
}

template <int GRP>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeParams p) {
    __shared__ float qs[GRP][kHD];
    __shared__ float sc[GRP][kTile];
    __shared__ float s_m[GRP], s_scale[GRP], s_l[GRP];
    __shared__ double red_d[8];
    __shared__ float kn[kHD];
    __shared__ int s_last;

    const int kv = blockIdx.x, sp = blockIdx.y;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int NQ = p.NQ, NKV = p.NKV;
    const int HD2 = 2 * kHD;

    pdl_wait();
    pdl_launch_dependents();

    const bool decode = p.proj != nullptr;
    const int pos = decode ? *p.pos_ptr : p.n_ctx_val - 1;
    const int n_ctx = pos + 1;
    // active splits: at least 64 positions each
    int n_act = (n_ctx + kTile - 1) / kTile;
    if (n_act > p.nsplit) n_act = p.nsplit;
    if (sp >= n_act) return;
    const int chunk = (n_ctx + n_act - 1) / n_act;
    const int j0 = sp * chunk;
    const int j1 = min(n_ctx, j0 + chunk);

    // ---- query heads of this group: norm + rope (decode) or given
    for (int g = 0; g < GRP; ++g) {
        const int h = kv * GRP + g;
        if (decode) {
            qs[g][t] = p.proj[(size_t)h * HD2 + t];
            __syncthreads();
            norm_rope(qs[g], p.qn1, p.eps, p.rot, p.inv_freq, pos, red_d);
        } else {
            qs[g][t] = p.q_in[(size_t)h * kHD + t];
        }
    }
    // ---- the CTA owning the new position appends K/V[pos]
    const size_t cache_head = (size_t)kv * p.max_ctx * kHD;
    if (decode && pos >= j0 && pos < j1) {
        const float* kraw = p.proj + (size_t)NQ * HD2 + (size_t)kv * kHD;
        const float* vraw = p.proj + (size_t)NQ * HD2 + (size_t)NKV * kHD + (size_t)kv * kHD;
        kn[t] = kraw[t];
        __syncthreads();
        norm_rope(kn, p.kn1, p.eps, p.rot, p.inv_freq, pos, red_d);
        const size_t off = cache_head + (size_t)pos * kHD + t;
        if (p.kv_bf16) {
            reinterpret_cast<uint16_t*>(p.k_cache)[off] = f2bf(kn[t]);
            reinterpret_cast<uint16_t*>(p.v_cache)[off] = f2bf(vraw[t]);
        } else {
            reinterpret_cast<float*>(p.k_cache)[off] = kn[t];
            reinterpret_cast<float*>(p.v_cache)[off] = vraw[t];
        }
    }
    __syncthreads();

    // q chunk of this lane in registers: dims lane*8 .. lane*8+7
    float qr[GRP][8];
#pragma unroll
    for (int g = 0; g < GRP; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) qr[g][e] = qs[g][lane * 8 + e];

    float acc[GRP];
#pragma unroll
    for (int g = 0; g < GRP; ++g) acc[g] = 0.f;
    if (t < GRP) { s_m[t] = -INFINITY; s_l[t] = 0.f; }
    const float scale = 1.0f / sqrtf((float)kHD);

    for (int tj = j0; tj < j1; tj += kTile) {
        const int nt = min(kTile, j1 - tj);
        // scores: warp w takes positions w, w+8, ...
        for (int jj = warp; jj < nt; jj += 8) {
            float kk[8];
            load8(p.k_cache, p.kv_bf16, cache_head + (size_t)(tj + jj) * kHD + lane * 8, kk);
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) d = fmaf(qr[g][e], kk[e], d);
                d = warp_sum(d);
                if (lane == 0) sc[g][jj] = d * scale;
            }
        }
        __syncthreads();
        // per head: tile max, probabilities, tile sum (one warp per head)
        for (int g = warp; g < GRP; g += 8) {
            const float a0 = lane < nt ? sc[g][lane] : -INFINITY;
            const float a1 = lane + 32 < nt ? sc[g][lane + 32] : -INFINITY;
            const float mt = warp_max(fmaxf(a0, a1));
            const float m_old = s_m[g];
            const float m_new = fmaxf(m_old, mt);
            const float e0 = lane < nt ? expf(a0 - m_new) : 0.f;
            const float e1 = lane + 32 < nt ? expf(a1 - m_new) : 0.f;
            sc[g][lane] = e0;
            sc[g][lane + 32] = e1;
            const float ls = warp_sum(e0 + e1);
            if (lane == 0) {
                const float f = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
                s_scale[g] = f;
                s_l[g] = s_l[g] * f + ls;
                s_m[g] = m_new;
            }
        }
        __syncthreads();
        // PV: thread t owns dim t
#pragma unroll
        for (int g = 0; g < GRP; ++g) acc[g] *= s_scale[g];
        for (int jj = 0; jj < nt; ++jj) {
            const float v = load1(p.v_cache, p.kv_bf16, cache_head + (size_t)(tj + jj) * kHD + t);
#pragma unroll
            for (int g = 0; g < GRP; ++g) acc[g] = fmaf(sc[g][jj], v, acc[g]);
        }
        __syncthreads();
    }

    // ---- single split: finish here; otherwise publish partials, last CTA merges
    auto gate_of = [&](int h) -> float {
        return decode ? p.proj[(size_t)h * HD2 + kHD + t] : p.gate_in[(size_t)h * kHD + t];
    };
    if (n_act == 1) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            const int h = kv * GRP + g;
            p.out[(size_t)h * kHD + t] = (acc[g] / s_l[g]) * sigmoid_f(gate_of(h));
        }
        return;
    }
    const size_t pbase = ((size_t)kv * p.nsplit + sp) * GRP;
#pragma unroll
    for (int g = 0; g < GRP; ++g) p.part_o[(pbase + g) * kHD + t] = acc[g];
    if (t < GRP) {
        p.part_ml[(pbase + t) * 2 + 0] = s_m[t];
        p.part_ml[(pbase + t) * 2 + 1] = s_l[t];
    }
    __threadfence();
    __syncthreads();
    if (t == 0) {
        const unsigned tk = atomicAdd(&p.counters[kv], 1u);
        s_last = (tk == (unsigned)n_act - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        float M = -INFINITY;
        for (int s2 = 0; s2 < n_act; ++s2)
            M = fmaxf(M, __ldcg(&p.part_ml[(((size_t)kv * p.nsplit + s2) * GRP + g) * 2]));
        float L = 0.f, o = 0.f;
        for (int s2 = 0; s2 < n_act; ++s2) {
            const size_t b = ((size_t)kv * p.nsplit + s2) * GRP + g;
            const float m = __ldcg(&p.part_ml[b * 2]);
            const float f = (m == -INFINITY) ? 0.f : expf(m - M);
            L += __ldcg(&p.part_ml[b * 2 + 1]) * f;
            o += __ldcg(&p.part_o[b * kHD + t]) * f;
        }
        const int h = kv * GRP + g;
        p.out[(size_t)h * kHD + t] = (o / L) * sigmoid_f(gate_of(h));
    }
    if (t == 0) p.counters[kv] = 0u;
}

int attn_nsplit_for(int max_ctx) {
    // enough splits to cover the SMs at long context, each >= 64 positions
    int want = (max_ctx + kTile - 1) / kTile;
    int cap = 2 * num_sms();
    return want < 1 ? 1 : (want > cap ? cap : want);
}

cudaError_t launch_attn_decode(const AttnDecodeParams& p, cudaStream_t s, bool pdl) {
    if (p.NKV <= 0 || p.NQ % p.NKV != 0 || p.rot > kHD || p.rot % 2 != 0) return cudaErrorInvalidValue;
    const int grp = p.NQ / p.NKV;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.NKV, p.nsplit);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (grp) {
        case 1: return cudaLaunchKernelEx(&cfg, k_attn_decode<1>, p);
        case 2: return cudaLaunchKernelEx(&cfg, k_attn_decode<2>, p);
        case 4: return cudaLaunchKernelEx(&cfg, k_attn_decode<4>, p);
        case 8: return cudaLaunchKernelEx(&cfg, k_attn_decode<8>, p);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qwc
