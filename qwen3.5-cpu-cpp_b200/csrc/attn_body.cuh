// Device body of the decode gated GQA attention, shared by the standalone kernel
// (attn_decode.cu) and the persistent decode-step kernel (decode_step.cu).
//
// Decode gated GQA attention (QwenModel::attn_step, src/qwen_model.cpp:118-150):
//   q_h = rope(rmsnorm(q_raw_h) * (1+q_norm)), k = rope(rmsnorm(k_raw) * (1+k_norm))
//   K[pos] = k, V[pos] = v_raw                          (cache append)
//   o_h = softmax(q_h K^T / sqrt(HD)) V over positions 0..pos, then o_h *= sigmoid(gate_h)
//
// Grid (NKV, nsplit): CTA (kv, sp) takes a contiguous range of positions for the GRP
// query heads of kv head `kv`. The number of active splits follows the live context
// length (read from the device position, so one captured graph serves every step).
// Inside a CTA each warp owns every 8th position and keeps its own online softmax
// (running max, sum and a 256-wide accumulator per head, 8 dims per lane); the K and V
// rows of the next positions are in flight while the current ones are consumed. Warps are merged through shared
// memory, CTAs by the last CTA of each kv head (atomic ticket), which also applies the
// sigmoid gate.
//
// Prologue: one warp per head normalises and rotates q (and, in the CTA that owns the
// new position, k, which it appends to the cache with v). The kernel is latency-bound at
// decode context lengths, so every independent load is issued as early as possible:
// position + raw projections together, then the first K/V rows together with the RoPE
// row. RoPE: rotate_half pairs (i, i+rot/2); (cos, sin) of pos * theta^(-2i/rot) come from
// a per-position table that the host fills in double precision exactly as apply_rope does
// (forward_pass.cpp:102-112).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace qwc {

constexpr int kHD = 256;
constexpr int kWarpsA = 8;
constexpr int kAttnThreads = kWarpsA * 32;
constexpr int kMinChunk = 32;  // positions per split at least

// Barrier over the kAttnThreads threads that run an item (named barrier 2), so that a
// larger CTA can run the item on its first kAttnThreads threads only.
__device__ __forceinline__ void attn_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }
static_assert(kAttnThreads == 256, "attn_sync counts 256 threads");

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
// fp32 -> bf16 round-to-nearest-even (finite inputs)
__device__ __forceinline__ uint16_t f2bf(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// One warp: x[8] (dims lane*8..lane*8+7 of a 256-vector) <- rope(rmsnorm(x) * w1).
// Requires rot % 16 == 0 so that rotation partners are whole lanes apart. cs_row holds
// (cos, sin) of pair i at cs_row[2i], cs_row[2i+1] for the current position.
__device__ __forceinline__ void warp_norm_rope(float* x, const float* w1, float eps, int rot,
                                               const float* cs_row) {
    const int lane = threadIdx.x & 31;
    const int half = rot / 2, dl = half / 8;  // partner lane distance
    const int d0 = lane * 8;
    const bool lo = d0 < half, hi = d0 >= half && d0 < rot;
    // this lane's 8 (cos, sin) pairs: i = d0.. (lo) or d0-half.. (hi), 64 contiguous bytes
    float4 c4[4];
    if (lo || hi) {
        const float4* src = reinterpret_cast<const float4*>(cs_row + 2 * (lo ? d0 : d0 - half));
#pragma unroll
        for (int i = 0; i < 4; ++i) c4[i] = src[i];
    }
    float w[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = w1[d0 + e];
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += (double)x[e] * x[e];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf((float)(ss / kHD) + eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = x[e] * inv * w[e];
    float partner[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float up = __shfl_down_sync(0xffffffffu, x[e], dl);  // x[d + half] for lo lanes
        const float dn = __shfl_up_sync(0xffffffffu, x[e], dl);    // x[d - half] for hi lanes
        partner[e] = lo ? up : dn;
    }
    if (lo || hi) {
        const float* cf = reinterpret_cast<const float*>(c4);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float c = cf[2 * e], s = cf[2 * e + 1];
            // lo: x1 = x[d], x2 = x[d+half] -> x1*c - x2*s ; hi: x2 = x[d], x1 = x[d-half] -> x2*c + x1*s
            x[e] = lo ? (x[e] * c - partner[e] * s) : (x[e] * c + partner[e] * s);
        }
    }
}

// One (kv head, split) item on 256 threads (one CTA). The split count follows the live
// context length, so an item whose split is beyond it returns at once (uniformly). Each
// warp works on groups of DEPTH positions with two register buffers: the next group's
// K/V rows are loaded while the current group is consumed (DEPTH 1 in the decode step,
// where contexts are short and registers are shared with the GEMV phases; 2 for the
// standalone kernel).
template <int GRP, int DEPTH = 1>
__device__ __forceinline__ void attn_decode_item(const AttnDecodeParams& p, int kv, int sp,
                                                 long long* marks = nullptr) {
    auto mark = [&](int k) {
        if (marks && threadIdx.x == 0) marks[k] = (long long)globaltimer_ns();
    };
    __shared__ __align__(16) float qs[GRP][kHD];
    __shared__ __align__(16) float kvn[2][kHD];  // k (normed, roped) and v of the new position
    __shared__ __align__(16) float wacc[kWarpsA][kHD];
    __shared__ float wm[kWarpsA][GRP], wl[kWarpsA][GRP];
    __shared__ int s_last;

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int NQ = p.NQ, NKV = p.NKV;
    const int HD2 = 2 * kHD;
    const bool decode = p.proj != nullptr;
    const int nroles = decode ? GRP + 2 : GRP;  // q heads, then k and v of the new position

    // ---- round trip 1: the position and this warp's raw inputs, issued together
    auto raw_ptr = [&](int hh) -> const float* {
        if (!decode) return p.q_in + (size_t)(kv * GRP + hh) * kHD;
        if (hh < GRP) return p.proj + (size_t)(kv * GRP + hh) * HD2;
        if (hh == GRP) return p.proj + (size_t)NQ * HD2 + (size_t)kv * kHD;
        return p.proj + (size_t)NQ * HD2 + (size_t)NKV * kHD + (size_t)kv * kHD;
    };
    float x[8];
    if (warp < nroles) {
        const float4* src = reinterpret_cast<const float4*>(raw_ptr(warp) + lane * 8);
        const float4 a = src[0], b = src[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    const int pos = decode ? *p.pos_ptr : p.n_ctx_val - 1;

    const int n_ctx = pos + 1;
    int n_act = (n_ctx + p.min_chunk - 1) / p.min_chunk;
    if (n_act > p.nsplit) n_act = p.nsplit;
    if (sp >= n_act) return;
    const int chunk = (n_ctx + n_act - 1) / n_act;
    const int j0 = sp * chunk;
    const int j1 = min(n_ctx, j0 + chunk);
    const size_t cache_head = (size_t)kv * p.max_ctx * kHD;
    const bool owner = decode && pos >= j0 && pos < j1;

    // ---- round trip 2: this warp's first DEPTH K/V rows (the new row comes from smem)
    float kr[DEPTH][8], vr[DEPTH][8], kr2[DEPTH][8], vr2[DEPTH][8];
    auto fetch = [&](int j, float* kk, float* vv) {
        if (j < j1 && !(decode && j == pos)) {
            load8(p.k_cache, p.kv_bf16, cache_head + (size_t)j * kHD + lane * 8, kk);
            load8(p.v_cache, p.kv_bf16, cache_head + (size_t)j * kHD + lane * 8, vv);
        }
    };
    int j = j0 + warp;
#pragma unroll
    for (int d = 0; d < DEPTH; ++d) fetch(j + d * kWarpsA, kr[d], vr[d]);

    // ---- prologue roles: q heads (norm + rope), and in the owner CTA k (norm + rope) / v
    const float* cs_row = decode ? p.rope_cs + (size_t)pos * p.rot : nullptr;
    for (int hh = warp; hh < nroles; hh += kWarpsA) {
        if (hh != warp) {
            const float4* src = reinterpret_cast<const float4*>(raw_ptr(hh) + lane * 8);
            const float4 a = src[0], b = src[1];
            x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        }
        if (hh < GRP) {
            if (decode) warp_norm_rope(x, p.qn1, p.eps, p.rot, cs_row);
#pragma unroll
            for (int e = 0; e < 8; ++e) qs[hh][lane * 8 + e] = x[e];
        } else if (owner) {
            const int which = hh - GRP;  // 0: k, 1: v
            if (which == 0) warp_norm_rope(x, p.kn1, p.eps, p.rot, cs_row);
            void* cache = which == 0 ? p.k_cache : p.v_cache;
            const size_t off = cache_head + (size_t)pos * kHD + lane * 8;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                kvn[which][lane * 8 + e] = x[e];
                if (p.kv_bf16) reinterpret_cast<uint16_t*>(cache)[off + e] = f2bf(x[e]);
                else reinterpret_cast<float*>(cache)[off + e] = x[e];
            }
        }
    }
    attn_sync();
    mark(0);

    float qr[GRP][8];
#pragma unroll
    for (int g = 0; g < GRP; ++g)
#pragma unroll
        for (int e = 0; e < 8; ++e) qr[g][e] = qs[g][lane * 8 + e];
    float m[GRP], l[GRP], acc[GRP][8];
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    }
    const float scale = 1.0f / sqrtf((float)kHD);

    // position jj with K row kk and V row vv (the new position reads k/v from smem; with
    // a bf16 cache its values are rounded like the stored row)
    auto consume = [&](int jj, float* kk, float* vv) {
        if (jj >= j1) return;
        if (decode && jj == pos) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float kx = kvn[0][lane * 8 + e], vx = kvn[1][lane * 8 + e];
                if (p.kv_bf16) {
                    kx = __uint_as_float((uint32_t)f2bf(kx) << 16);
                    vx = __uint_as_float((uint32_t)f2bf(vx) << 16);
                }
                kk[e] = kx;
                vv[e] = vx;
            }
        }
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) d = fmaf(qr[g][e], kk[e], d);
            const float sc = warp_sum(d) * scale;
            const float mn = fmaxf(m[g], sc);
            const float corr = (m[g] == -INFINITY) ? 0.f : expf(m[g] - mn);
            const float pe = expf(sc - mn);
            l[g] = l[g] * corr + pe;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] = fmaf(pe, vv[e], acc[g][e] * corr);
            m[g] = mn;
        }
    };
    // groups of DEPTH positions: the next group's loads are issued before the current
    // group is consumed (two static register buffers, alternating)
    constexpr int G = DEPTH * kWarpsA;
    while (j < j1) {
#pragma unroll
        for (int d = 0; d < DEPTH; ++d) fetch(j + G + d * kWarpsA, kr2[d], vr2[d]);
#pragma unroll
        for (int d = 0; d < DEPTH; ++d) consume(j + d * kWarpsA, kr[d], vr[d]);
        j += G;
        if (j >= j1) break;
#pragma unroll
        for (int d = 0; d < DEPTH; ++d) fetch(j + G + d * kWarpsA, kr[d], vr[d]);
#pragma unroll
        for (int d = 0; d < DEPTH; ++d) consume(j + d * kWarpsA, kr2[d], vr2[d]);
        j += G;
    }
    mark(1);
    // ---- merge the warps: per head, M = max m_w, L = sum l_w e^(m_w-M), o = sum acc_w e^(m_w-M)
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
    }
    float cm[GRP], cl[GRP], co[GRP];  // this CTA's (max, sum, acc[t]) per head, thread t = dim
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
#pragma unroll
        for (int e = 0; e < 8; ++e) wacc[warp][lane * 8 + e] = acc[g][e];
        attn_sync();
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarpsA; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, o = 0.f;
#pragma unroll
        for (int w = 0; w < kWarpsA; ++w) {
            const float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
            L += wl[w][g] * f;
            o += wacc[w][t] * f;
        }
        cm[g] = M;
        cl[g] = L;
        co[g] = o;
        attn_sync();
    }

    mark(2);
    auto gate_of = [&](int h) -> float {
        return decode ? p.proj[(size_t)h * HD2 + kHD + t] : p.gate_in[(size_t)h * kHD + t];
    };
    if (n_act == 1 && !p.defer_combine) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            const int h = kv * GRP + g;
            p.out[(size_t)h * kHD + t] = (co[g] / cl[g]) * sigmoid_f(gate_of(h));
        }
        return;
    }
    const size_t pbase = ((size_t)kv * p.nsplit + sp) * GRP;
#pragma unroll
    for (int g = 0; g < GRP; ++g) p.part_o[(pbase + g) * kHD + t] = co[g];
    if (t == 0) {
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
            p.part_ml[(pbase + g) * 2 + 0] = cm[g];
            p.part_ml[(pbase + g) * 2 + 1] = cl[g];
        }
    }
    if (p.defer_combine) return;  // the next phase combines (after its grid barrier)
    // publish: every thread's partial is ordered before thread 0's release fence by the
    // CTA barrier; the CTA that takes the last ticket fences again before reading
    attn_sync();
    if (t == 0) {
        __threadfence();
        const unsigned tk = atomicAdd(&p.counters[kv], 1u);
        s_last = (tk == (unsigned)n_act - 1) ? 1 : 0;
        if (s_last) __threadfence();
    }
    attn_sync();
    if (!s_last) return;
    float gate[GRP];
#pragma unroll
    for (int g = 0; g < GRP; ++g) gate[g] = gate_of(kv * GRP + g);
    // all (max, sum) pairs of this kv head staged in shared memory with one parallel load
    // (wacc is free again after the warp merge)
    const int npairs = n_act * GRP;
    const size_t pair0 = (size_t)kv * p.nsplit * GRP;
    float2* ml_s = reinterpret_cast<float2*>(&wacc[0][0]);
    const bool staged = npairs <= kWarpsA * kHD / 2;
    if (staged) {
        for (int i = t; i < npairs; i += kAttnThreads) ml_s[i] = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + pair0 + i);
        attn_sync();
    }
    auto ml_of = [&](int s2, int g) -> float2 {
        return staged ? ml_s[s2 * GRP + g] : __ldcg(reinterpret_cast<const float2*>(p.part_ml) + pair0 + (size_t)s2 * GRP + g);
    };
    // every head's partials are loaded together (GRP x 8 in flight); per head the sums run
    // over the splits in order
    float M[GRP], L[GRP], o[GRP];
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        M[g] = -INFINITY;
        for (int s2 = 0; s2 < n_act; ++s2) M[g] = fmaxf(M[g], ml_of(s2, g).x);
        L[g] = 0.f;
        o[g] = 0.f;
    }
    for (int s0 = 0; s0 < n_act; s0 += 8) {
        float po[GRP][8];
#pragma unroll
        for (int g = 0; g < GRP; ++g)
#pragma unroll
            for (int u = 0; u < 8; ++u)
                po[g][u] = s0 + u < n_act ? __ldcg(&p.part_o[((pair0 + (size_t)(s0 + u) * GRP + g)) * kHD + t]) : 0.f;
#pragma unroll
        for (int g = 0; g < GRP; ++g) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                if (s0 + u < n_act) {
                    const float2 ml = ml_of(s0 + u, g);
                    const float f = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M[g]);
                    L[g] += ml.y * f;
                    o[g] += po[g][u] * f;
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < GRP; ++g) {
        const int h = kv * GRP + g;
        p.out[(size_t)h * kHD + t] = (o[g] / L[g]) * sigmoid_f(gate[g]);
    }
    if (t == 0) p.counters[kv] = 0u;
    mark(3);
}

}  // namespace qwc
