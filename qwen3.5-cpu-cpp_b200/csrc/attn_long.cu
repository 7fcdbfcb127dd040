// Gated GQA attention decode over a long cache (the kernel-level op, qwc_attention_decode,
// at contexts of 2048 positions and more): softmax(q K^T / sqrt(HD)) V over positions
// 0..n_ctx-1, times sigmoid(gate) (attn_step, src/qwen_model.cpp:134-150).
//
// Split-K over positions: CTA (kv head, split) owns a contiguous position range for the
// GRP query heads of its kv head; 8 warps take blocks of 32 positions in turn. Per block:
//   scores  lane = position: the lane's K row (512 B for bf16, read-only path) against the
//           GRP query rows broadcast from shared memory -- per-lane dot products, no
//           shuffles; the query is pre-scaled by log2(e) / sqrt(HD), so the softmax runs in
//           the log2 domain (exp2);
//   softmax one max and one sum reduction per head per block (not per position);
//   values  lane = 8 dims: the block's V rows (coalesced) times the lanes' weights,
//           broadcast by shuffle.
// Warps merge through shared memory; each split writes (max, sum, acc) partials, and a
// second small kernel combines the splits for every (q head, 32 dims) with the sigmoid gate.
#include "common.cuh"
#include "kernels.h"

namespace qwc {
namespace {

constexpr int kLHD = 256, kLWarps = 8, kLThreads = kLWarps * 32, kLBlock = 32;

__device__ __forceinline__ void bf8(const uint4 w, float* o) {
    o[0] = bf16lo(w.x); o[1] = bf16hi(w.x); o[2] = bf16lo(w.y); o[3] = bf16hi(w.y);
    o[4] = bf16lo(w.z); o[5] = bf16hi(w.z); o[6] = bf16lo(w.w); o[7] = bf16hi(w.w);
}
// 8 consecutive cache values at element offset `off` (bf16 or fp32 cache), read-only path
__device__ __forceinline__ void load8nc(const void* base, int kv_bf16, size_t off, float* o) {
    if (kv_bf16) {
        bf8(__ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + off)), o);
    } else {
        const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
        const float4 a = __ldg(f), b = __ldg(f + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    }
}

// two CTAs per SM (16 warps to hide load latency) where the accumulators allow it
template <int GRP>
__global__ void __launch_bounds__(kLThreads, GRP <= 4 ? 2 : 1) k_attn_long(const AttnDecodeParams p) {
    __shared__ __align__(16) float qs[GRP][kLHD];
    __shared__ __align__(16) float wacc[kLWarps][kLHD];
    __shared__ float wm[kLWarps][GRP], wl[kLWarps][GRP];
    const int kv = blockIdx.x, sp = blockIdx.y, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int n_ctx = p.n_ctx_val;
    const int chunk = ((n_ctx + p.nsplit - 1) / p.nsplit + kLBlock - 1) / kLBlock * kLBlock;
    const int j0 = sp * chunk, j1 = min(n_ctx, j0 + chunk);
    const float qscale = 1.4426950408889634f / sqrtf((float)kLHD);  // log2(e) / sqrt(HD)
#pragma unroll
    for (int g = 0; g < GRP; ++g) qs[g][t] = p.q_in[(size_t)(kv * GRP + g) * kLHD + t] * qscale;
    __syncthreads();

    const size_t head = (size_t)kv * p.max_ctx;
    float m[GRP], l[GRP], acc[GRP][8];
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    }
    for (int b = j0 + warp * kLBlock; b < j1; b += kLWarps * kLBlock) {
        // ---- scores: lane = position b + lane
        const int j = b + lane;
        const bool valid = j < j1;
        const size_t krow = (head + (size_t)(valid ? j : b)) * kLHD;
        float s[GRP];
#pragma unroll
        for (int g = 0; g < GRP; ++g) s[g] = 0.f;
#pragma unroll 1
        for (int c0 = 0; c0 < kLHD; c0 += 64) {  // 64 dims per round: 8 loads in flight
            float kx[8][8];
#pragma unroll
            for (int u = 0; u < 8; ++u) load8nc(p.k_cache, p.kv_bf16, krow + c0 + u * 8, kx[u]);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int g = 0; g < GRP; ++g) {
                    const float4 qa = *reinterpret_cast<const float4*>(&qs[g][c0 + u * 8]);
                    const float4 qb = *reinterpret_cast<const float4*>(&qs[g][c0 + u * 8 + 4]);
                    s[g] = fmaf(qa.x, kx[u][0], s[g]); s[g] = fmaf(qa.y, kx[u][1], s[g]);
                    s[g] = fmaf(qa.z, kx[u][2], s[g]); s[g] = fmaf(qa.w, kx[u][3], s[g]);
                    s[g] = fmaf(qb.x, kx[u][4], s[g]); s[g] = fmaf(qb.y, kx[u][5], s[g]);
                    s[g] = fmaf(qb.z, kx[u][6], s[g]); s[g] = fmaf(qb.w, kx[u][7], s[g]);
                }
            }
        }
        // ---- online softmax, once per block and head
        float pw[GRP];
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            const float sc = valid ? s[g] : -INFINITY;
            const float mn = fmaxf(m[g], warp_max(sc));
            const float corr = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - mn);
            pw[g] = valid ? exp2f(sc - mn) : 0.f;
            l[g] = l[g] * corr + warp_sum(pw[g]);
            m[g] = mn;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] *= corr;
        }
        // ---- values: lane = dims 8 lane .. 8 lane + 7, the block's rows in groups of 8
        const int nb = min(kLBlock, j1 - b);
#pragma unroll 1
        for (int r0 = 0; r0 < kLBlock; r0 += 8) {
            float vx[8][8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (r0 + u < nb) load8nc(p.v_cache, p.kv_bf16, (head + (size_t)(b + r0 + u)) * kLHD + lane * 8, vx[u]);
                else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) vx[u][e] = 0.f;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int g = 0; g < GRP; ++g) {
                    const float pr = __shfl_sync(0xffffffffu, pw[g], r0 + u);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pr, vx[u][e], acc[g][e]);
                }
            }
        }
    }
    // ---- merge the warps: per head M = max m_w, L = sum l_w 2^(m_w - M), o = sum acc_w 2^(m_w - M)
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
    }
    const size_t pbase = ((size_t)kv * p.nsplit + sp) * GRP;
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[warp][lane * 8 + e] = acc[g][e];
        __syncthreads();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kLWarps; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int w = 0; w < kLWarps; ++w) {
            const float f = (wm[w][g] == -INFINITY) ? 0.f : exp2f(wm[w][g] - M);
            L += wl[w][g] * f;
            o += wacc[w][t] * f;
        }
        if (p.nsplit == 1) {
            const int h = kv * GRP + g;
            p.out[(size_t)h * kLHD + t] = (o / L) * sigmoid_f(p.gate_in[(size_t)h * kLHD + t]);
        } else {
            p.part_o[(pbase + g) * kLHD + t] = o;
            if (t == 0) {
                p.part_ml[(pbase + g) * 2 + 0] = M;
                p.part_ml[(pbase + g) * 2 + 1] = L;
            }
        }
        __syncthreads();
    }
}

// CTA = (q head, 32 dims); its 8 warps take every 8th split, then sum through shared memory.
__global__ void __launch_bounds__(256) k_attn_long_combine(const AttnDecodeParams p) {
    __shared__ float2 ml[1024];
    __shared__ float red_o[8][32];
    __shared__ float red_l[8];
    const int h = blockIdx.x, grp = p.NQ / p.NKV, kv = h / grp, g = h % grp;
    const int t = threadIdx.x, sg = t >> 5, dl = t & 31, d = blockIdx.y * 32 + dl;
    const int ns = p.nsplit;
    for (int s = t; s < ns; s += 256)
        ml[s] = reinterpret_cast<const float2*>(p.part_ml)[((size_t)kv * ns + s) * grp + g];
    __syncthreads();
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, ml[s].x);
    float o = 0.f, L = 0.f;
#pragma unroll 4
    for (int s = sg; s < ns; s += 8) {
        const float f = (ml[s].x == -INFINITY) ? 0.f : exp2f(ml[s].x - M);
        o += __ldcg(&p.part_o[(((size_t)kv * ns + s) * grp + g) * kLHD + d]) * f;
        L += ml[s].y * f;
    }
    red_o[sg][dl] = o;
    if (dl == 0) red_l[sg] = L;
    __syncthreads();
    if (sg == 0) {
        float os = 0.f, ls = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
            os += red_o[w][dl];
            ls += red_l[w];
        }
        p.out[(size_t)h * kLHD + d] = (os / ls) * sigmoid_f(p.gate_in[(size_t)h * kLHD + d]);
    }
}

}  // namespace

int attn_long_nsplit(int n_ctx, int nkv, int grp) {
    int want = (n_ctx + kLWarps * kLBlock - 1) / (kLWarps * kLBlock);
    int cap = (grp <= 4 ? 2 : 1) * num_sms() / (nkv > 0 ? nkv : 1);
    if (cap > 1024) cap = 1024;
    return want < 1 ? 1 : (want > cap ? cap : want);
}

cudaError_t launch_attn_long(const AttnDecodeParams& p, cudaStream_t s) {
    if (p.proj || p.NKV <= 0 || p.NQ % p.NKV || p.nsplit < 1 || p.nsplit > 1024) return cudaErrorInvalidValue;
    const int grp = p.NQ / p.NKV;
    dim3 grid(p.NKV, p.nsplit);
    switch (grp) {
        case 1: k_attn_long<1><<<grid, kLThreads, 0, s>>>(p); break;
        case 2: k_attn_long<2><<<grid, kLThreads, 0, s>>>(p); break;
        case 4: k_attn_long<4><<<grid, kLThreads, 0, s>>>(p); break;
        case 8: k_attn_long<8><<<grid, kLThreads, 0, s>>>(p); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || p.nsplit == 1) return e;
    k_attn_long_combine<<<dim3(p.NQ, kLHD / 32), 256, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace qwc
