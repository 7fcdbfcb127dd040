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

// Online softmax of one block of up to 32 positions (one max / sum reduction per head):
// the lanes' weights pw, the running max / sum updated and the accumulators rescaled.
template <int GRP>
__device__ __forceinline__ void block_softmax(bool valid, const float (&s)[GRP], float (&m)[GRP], float (&l)[GRP],
                                              float (&acc)[GRP][8], float (&pw)[GRP]) {
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
}
// 8 V rows (bf16 or fp32 values vx[u][dims of this lane]) times the weights of positions
// r0 + u, broadcast from their lanes
template <int GRP>
__device__ __forceinline__ void pv8(const float (&vx)[8][8], int r0, const float (&pw)[GRP], float (&acc)[GRP][8]) {
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
// Softmax of a block, then its V rows (lane = 8 dims) straight from global memory.
template <int GRP>
__device__ __forceinline__ void block_softmax_pv(const AttnDecodeParams& p, size_t head, int b, int j1, int lane,
                                                 bool valid, const float (&s)[GRP], float (&m)[GRP], float (&l)[GRP],
                                                 float (&acc)[GRP][8]) {
    float pw[GRP];
    block_softmax<GRP>(valid, s, m, l, acc, pw);
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
        pv8<GRP>(vx, r0, pw, acc);
    }
}

// Merge of the CTA's warps (per head M = max m_w, L = sum l_w 2^(m_w - M), o = sum acc_w
// 2^(m_w - M)) and the split's partial (or, with one split, the gated output).
template <int GRP>
__device__ __forceinline__ void merge_store(const AttnDecodeParams& p, int kv, int sp, const float (&m)[GRP],
                                            const float (&l)[GRP], const float (&acc)[GRP][8], float (*wacc)[kLHD],
                                            float (*wm)[GRP], float (*wl)[GRP]) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
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

// position range of split sp
__device__ __forceinline__ void split_range(const AttnDecodeParams& p, int sp, int& j0, int& j1) {
    const int n_ctx = p.n_ctx_val;
    const int chunk = ((n_ctx + p.nsplit - 1) / p.nsplit + kLBlock - 1) / kLBlock * kLBlock;
    j0 = sp * chunk;
    j1 = min(n_ctx, j0 + chunk);
}

// fp32 caches: the lane's K row straight from global memory, 8 loads per 64 dims.
// Two CTAs per SM (16 warps to hide load latency) where the accumulators allow it.
template <int GRP>
__global__ void __launch_bounds__(kLThreads, GRP <= 4 ? 2 : 1) k_attn_long(const AttnDecodeParams p) {
    __shared__ __align__(16) float qs[GRP][kLHD];
    __shared__ __align__(16) float wacc[kLWarps][kLHD];
    __shared__ float wm[kLWarps][GRP], wl[kLWarps][GRP];
    const int kv = blockIdx.x, sp = blockIdx.y, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    int j0, j1;
    split_range(p, sp, j0, j1);
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
        block_softmax_pv<GRP>(p, head, b, j1, lane, valid, s, m, l, acc);
    }
    merge_store<GRP>(p, kv, sp, m, l, acc, wacc, wm, wl);
}

// bf16 caches: K and V arrive through a per-warp ring of four 4 KB slots copied by
// cp.async, three slots ahead of the one being consumed, so the bytes in flight no longer
// depend on registers (one CTA per SM, no register cap). Per block of 32 positions the ring
// carries 4 K slices (32 rows x 64 dims; each 16-byte piece q of row r at piece q ^ (r % 8)
// of its 128-byte slot, so the lane-per-row reads hit distinct banks), then 4 V slices
// (8 whole rows each, read with lane = 8 dims).
constexpr int kStSlices = 4;
constexpr int kStSlice = kLBlock * 128;  // bytes
constexpr size_t kStSmem = (size_t)kLWarps * kStSlices * kStSlice;
__device__ __forceinline__ void cp16z(uint32_t dst, const void* src, bool pred) {
    const int nb = pred ? 16 : 0;  // 0: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(nb) : "memory");
}
template <int GRP>
__global__ void __launch_bounds__(kLThreads, 1) k_attn_long_st(const AttnDecodeParams p) {
    __shared__ __align__(16) float qs[GRP][kLHD];
    __shared__ __align__(16) float wacc[kLWarps][kLHD];
    __shared__ float wm[kLWarps][GRP], wl[kLWarps][GRP];
    extern __shared__ __align__(128) uint8_t ring_all[];
    const int kv = blockIdx.x, sp = blockIdx.y, t = threadIdx.x, warp = t >> 5, lane = t & 31;
    int j0, j1;
    split_range(p, sp, j0, j1);
    const float qscale = 1.4426950408889634f / sqrtf((float)kLHD);
#pragma unroll
    for (int g = 0; g < GRP; ++g) qs[g][t] = p.q_in[(size_t)(kv * GRP + g) * kLHD + t] * qscale;
    __syncthreads();

    const size_t head = (size_t)kv * p.max_ctx;
    const uint16_t* kc = reinterpret_cast<const uint16_t*>(p.k_cache);
    uint8_t* ring = ring_all + (size_t)warp * kStSlices * kStSlice;
    const uint32_t ring_s = smem_u32(ring);
    const int bw = j0 + warp * kLBlock;  // this warp's first block
    const int nblk = bw < j1 ? (j1 - bw + kLWarps * kLBlock - 1) / (kLWarps * kLBlock) : 0;
    const uint16_t* vc = reinterpret_cast<const uint16_t*>(p.v_cache);
    const int nsl = nblk * 8;  // per block 4 K slices of 64 dims, then 4 V slices of 8 rows
    // K slice (i % 8 < 4): lane -> row u * 4 + lane / 8, piece lane % 8 (a warp copies 4
    // whole 128-byte row pieces at a time); V slice: row 8 (i % 4) + u, piece lane (a warp
    // copies one whole 512-byte row at a time)
    auto issue = [&](int i) {
        if (i < nsl) {
            const int b = bw + (i >> 3) * kLWarps * kLBlock, part = i & 3;
            const uint32_t dst0 = ring_s + (uint32_t)((i % kStSlices) * kStSlice);
            if ((i & 4) == 0) {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int r = u * 4 + (lane >> 3), q = lane & 7;
                    const bool ok = b + r < j1;
                    const uint16_t* src = kc + (head + (size_t)(ok ? b + r : b)) * kLHD + part * 64 + q * 8;
                    cp16z(dst0 + (uint32_t)(r * 128 + ((q ^ (r & 7)) << 4)), src, ok);
                }
            } else {
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int r = part * 8 + u;
                    const bool ok = b + r < j1;
                    const uint16_t* src = vc + (head + (size_t)(ok ? b + r : b)) * kLHD + lane * 8;
                    cp16z(dst0 + (uint32_t)(u * 512 + lane * 16), src, ok);
                }
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    for (int i = 0; i < kStSlices - 1; ++i) issue(i);

    float m[GRP], l[GRP], acc[GRP][8];
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    }
    float s[GRP], pw[GRP];
#pragma unroll 1
    for (int i = 0; i < nsl; ++i) {
        issue(i + kStSlices - 1);
        asm volatile("cp.async.wait_group %0;" ::"n"(kStSlices - 1) : "memory");  // slot i has landed (this lane's part)
        __syncwarp();                                         // ... and every lane's
        const uint8_t* slot = ring + (i % kStSlices) * kStSlice;
        if (i & 4) {
            // values: rows 8 (i % 4) .. of the block, lane = dims 8 lane ..
            float vx[8][8];
#pragma unroll
            for (int u = 0; u < 8; ++u) bf8(*reinterpret_cast<const uint4*>(slot + u * 512 + lane * 16), vx[u]);
            pv8<GRP>(vx, (i & 3) * 8, pw, acc);
            __syncwarp();  // every lane is done with the slot before the next issue refills it
            continue;
        }
        const int d0 = (i & 3) * 64;
        if ((i & 3) == 0) {
#pragma unroll
            for (int g = 0; g < GRP; ++g) s[g] = 0.f;
        }
        const uint8_t* row = slot + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float kx[8];
            bf8(*reinterpret_cast<const uint4*>(row + ((q ^ (lane & 7)) << 4)), kx);
#pragma unroll
            for (int g = 0; g < GRP; ++g) {
                const float4 qa = *reinterpret_cast<const float4*>(&qs[g][d0 + q * 8]);
                const float4 qb = *reinterpret_cast<const float4*>(&qs[g][d0 + q * 8 + 4]);
                s[g] = fmaf(qa.x, kx[0], s[g]); s[g] = fmaf(qa.y, kx[1], s[g]);
                s[g] = fmaf(qa.z, kx[2], s[g]); s[g] = fmaf(qa.w, kx[3], s[g]);
                s[g] = fmaf(qb.x, kx[4], s[g]); s[g] = fmaf(qb.y, kx[5], s[g]);
                s[g] = fmaf(qb.z, kx[6], s[g]); s[g] = fmaf(qb.w, kx[7], s[g]);
            }
        }
        __syncwarp();  // every lane is done with the slot before the next issue refills it
        if ((i & 3) == 3) block_softmax<GRP>(bw + (i >> 3) * kLWarps * kLBlock + lane < j1, s, m, l, acc, pw);
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    merge_store<GRP>(p, kv, sp, m, l, acc, wacc, wm, wl);
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

int attn_long_nsplit(int n_ctx, int nkv, int grp, int kv_bf16) {
    int want = (n_ctx + kLWarps * kLBlock - 1) / (kLWarps * kLBlock);
    // one split per resident CTA: two per SM for the fp32-cache kernel with GQA groups up
    // to 4, one for the staged bf16 kernel
    int cap = (!kv_bf16 && grp <= 4 ? 2 : 1) * num_sms() / (nkv > 0 ? nkv : 1);
    if (cap > 1024) cap = 1024;
    return want < 1 ? 1 : (want > cap ? cap : want);
}

cudaError_t launch_attn_long(const AttnDecodeParams& p, cudaStream_t s) {
    if (p.proj || p.NKV <= 0 || p.NQ % p.NKV || p.nsplit < 1 || p.nsplit > 1024) return cudaErrorInvalidValue;
    const int grp = p.NQ / p.NKV;
    dim3 grid(p.NKV, p.nsplit);
    auto go = [&](auto direct, auto staged) -> cudaError_t {
        if (!p.kv_bf16) {
            direct<<<grid, kLThreads, 0, s>>>(p);
            return cudaGetLastError();
        }
        cudaError_t e2 = cudaFuncSetAttribute(staged, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStSmem);
        if (e2 != cudaSuccess) return e2;
        staged<<<grid, kLThreads, kStSmem, s>>>(p);
        return cudaGetLastError();
    };
    cudaError_t e;
    switch (grp) {
        case 1: e = go(k_attn_long<1>, k_attn_long_st<1>); break;
        case 2: e = go(k_attn_long<2>, k_attn_long_st<2>); break;
        case 4: e = go(k_attn_long<4>, k_attn_long_st<4>); break;
        case 8: e = go(k_attn_long<8>, k_attn_long_st<8>); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || p.nsplit == 1) return e;
    k_attn_long_combine<<<dim3(p.NQ, kLHD / 32), 256, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace qwc
