// Device body of the decode Gated DeltaNet mixer core, shared by the standalone kernel
// (gdn_decode.cu) and the persistent decode-step kernel (decode_step.cu).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace qwc {

__device__ __forceinline__ void bar_sync_128() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

constexpr int kDK = 128, kDV = 128, kVS = 16;

// Sum of v[0..15] over the 32 lanes, scattered: returns sum of index idx(lane) where
// idx = bits (lane>>4, lane>>3, lane>>2, lane>>1); lanes l and l^1 hold the same value.
// 8+4+2+1+1 = 16 shuffles instead of 16 full butterflies of 5.
__device__ __forceinline__ float reduce_scatter16(const float (&v)[kVS], int lane) {
    float w8[8], w4[4], w2[2];
    const bool b4 = (lane >> 4) & 1, b3 = (lane >> 3) & 1, b2 = (lane >> 2) & 1, b1 = (lane >> 1) & 1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float send = b4 ? v[i] : v[i + 8], keep = b4 ? v[i + 8] : v[i];
        w8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float send = b3 ? w8[i] : w8[i + 4], keep = b3 ? w8[i + 4] : w8[i];
        w4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float send = b2 ? w4[i] : w4[i + 2], keep = b2 ? w4[i + 2] : w4[i];
        w2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const float send = b1 ? w2[0] : w2[1], keep = b1 ? w2[1] : w2[0];
    float w1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return w1 + __shfl_xor_sync(0xffffffffu, w1, 1);
}
__device__ __forceinline__ int scatter_index(int lane) {
    return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// One (value head, 16-column slice) item on 128 threads (t = 0..127). `wait` runs between
// the prologue (state slice + conv weights: nothing the preceding work writes) and the
// rest; barriers inside are named barrier 1 over these 128 threads only.
template <class WaitFn>
__device__ __forceinline__ void gdn_decode_item(const GdnDecodeParams& p, int vh, int vs, int t, WaitFn wait) {
    __shared__ double red_d[4][2];
    __shared__ float red16[4][kVS];
    __shared__ float s_v[kVS];
    __shared__ float s_d[kVS];

    const int warp = t >> 5, lane = t & 31;
    const int KH = p.KH, VH = p.VH, rep = VH / KH, kh = vh / rep;
    const int KD = KH * kDK;

    // ---- prologue: state slice and conv weights (independent of the previous kernel)
    float S[kVS];
    float* Srow = p.state + ((size_t)vh * kDK + t) * kDV + vs * kVS;
    {
        const float4* s4 = reinterpret_cast<const float4*>(Srow);
#pragma unroll
        for (int i = 0; i < kVS / 4; ++i) {
            const float4 v = s4[i];
            S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
        }
    }
    const int cq = kh * kDK + t, ck = KD + kh * kDK + t;
    const int cv = 2 * KD + vh * kDV + vs * kVS + t;  // used by t < 16
    const float4* cw4 = reinterpret_cast<const float4*>(p.conv_w);
    const float4 wq = cw4[cq], wk = cw4[ck];
    const float4 wv = t < kVS ? cw4[cv] : make_float4(0.f, 0.f, 0.f, 0.f);
    const float nA = p.neg_exp_A[vh], dtb = p.dt_bias[vh];

    wait();

    // ---- every input of this token, loaded together
    const int pos = p.pos_ptr ? *p.pos_ptr : p.pos_val;
    float4* ring = reinterpret_cast<float4*>(p.conv_ring);
    const float xq = p.mixed[cq], xk = p.mixed[ck];
    const float4 stq = ring[cq], stk = ring[ck];
    float xv = 0.f;
    float4 stv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < kVS) { xv = p.mixed[cv]; stv = ring[cv]; }
    const float av = p.a[vh], bv = p.b[vh];

    const int cur = pos & 3, m1 = (pos + 3) & 3, m2 = (pos + 2) & 3, m3 = (pos + 1) & 3;
    // causal conv over x[t-3], x[t-2], x[t-1], x[t] in the reference's order, then SiLU
    auto slot = [](float4 st, int i) -> float {
        return i == 0 ? st.x : (i == 1 ? st.y : (i == 2 ? st.z : st.w));
    };
    auto conv = [&](float x, float4 st, float4 w) -> float {
        float acc = 0.f;
        acc += w.x * slot(st, m3);
        acc += w.y * slot(st, m2);
        acc += w.z * slot(st, m1);
        acc += w.w * x;
        return silu_f(acc);
    };
    float q = conv(xq, stq, wq);
    float k = conv(xk, stk, wk);
    if (vs == 0 && vh % rep == 0) {  // one CTA stores the new q/k inputs of this head
        reinterpret_cast<float*>(&ring[cq])[cur] = xq;
        reinterpret_cast<float*>(&ring[ck])[cur] = xk;
    }
    if (t < kVS) {
        s_v[t] = conv(xv, stv, wv);
        reinterpret_cast<float*>(&ring[cv])[cur] = xv;
    }

    // l2norm of q and k over DK (sums in double), then q *= 1/sqrt(DK)
    double sq = (double)q * q, sk = (double)k * k;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    if (lane == 0) { red_d[warp][0] = sq; red_d[warp][1] = sk; }
    bar_sync_128();
    sq = (red_d[0][0] + red_d[1][0]) + (red_d[2][0] + red_d[3][0]);
    sk = (red_d[0][1] + red_d[1][1]) + (red_d[2][1] + red_d[3][1]);
    q = q * (1.0f / sqrtf((float)sq + 1e-6f));
    q = q * (1.0f / sqrtf((float)kDK));
    k = k * (1.0f / sqrtf((float)sk + 1e-6f));

    const float g = nA * softplus_f(av + dtb);
    const float decay = expf(g), beta = sigmoid_f(bv);

    // S *= decay; km = S^T k
    float part[kVS];
#pragma unroll
    for (int j = 0; j < kVS; ++j) {
        S[j] *= decay;
        part[j] = S[j] * k;
    }
    const int sidx = scatter_index(lane);
    float r = reduce_scatter16(part, lane);
    if ((lane & 1) == 0) red16[warp][sidx] = r;
    bar_sync_128();
    if (t < kVS) {
        const float km = (red16[0][t] + red16[1][t]) + (red16[2][t] + red16[3][t]);
        s_d[t] = (s_v[t] - km) * beta;
    }
    bar_sync_128();
    // S += k (x) d; o = S^T q
#pragma unroll
    for (int j = 0; j < kVS; ++j) {
        S[j] += k * s_d[j];
        part[j] = S[j] * q;
    }
    r = reduce_scatter16(part, lane);
    if ((lane & 1) == 0) red16[warp][sidx] = r;
    {
        float4* s4 = reinterpret_cast<float4*>(Srow);
#pragma unroll
        for (int i = 0; i < kVS / 4; ++i) s4[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    }
    bar_sync_128();
    if (t < kVS)
        p.out[(size_t)vh * kDV + vs * kVS + t] = (red16[0][t] + red16[1][t]) + (red16[2][t] + red16[3][t]);
}

}  // namespace qwc
