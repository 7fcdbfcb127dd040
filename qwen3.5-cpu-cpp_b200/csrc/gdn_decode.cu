// Decode Gated DeltaNet mixer core, one token (QwenModel::gdn_step,
// src/qwen_model.cpp:173-207):
//   conv:  c = silu(w0*x[t-3] + w1*x[t-2] + w2*x[t-1] + w3*x[t]) per channel
//   prep:  q,k l2-normalised (eps 1e-6), q *= 1/sqrt(DK)
//   gates: g = -exp(A_log) * softplus(a + dt_bias), decay = exp(g), beta = sigmoid(b)
//   delta: S *= decay; km = S^T k; d = (v - km) * beta; S += k (x) d; o = S^T q
//
// Grid (VH, DV/16): CTA (vh, vs) owns the 16 state columns [vs*16, vs*16+16) of value
// head vh. Columns of S are independent given k and q, so the 128x16 fp32 slice
// (8 KB) lives in registers: thread t holds row k=t. The slice is loaded before
// griddepcontrol.wait (it was last written by this layer one token ago), overlapping
// the tail of the in-projection GEMV.
//
// Conv state is a ring of K=4 slots per channel addressed by pos % 4 instead of the
// reference's shifted window of K-1: the slot written at pos is the one holding
// x[pos-4], which nobody reads any more, so the eight CTAs that share a q/k channel can
// read the three previous inputs without racing the single CTA that stores the new one.
#include "common.cuh"
#include "kernels.h"

namespace qwc {

constexpr int kDK = 128, kDV = 128, kVS = 16;

// block (128 threads) sum in double; identical in all threads
__device__ __forceinline__ double block128_sum_d(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return (red[0] + red[1]) + (red[2] + red[3]);
}

__global__ void __launch_bounds__(128) k_gdn_decode(const GdnDecodeParams p) {
    __shared__ double red_d[4];
    __shared__ float red16[4][kVS];
    __shared__ float s_v[kVS];
    __shared__ float s_km[kVS];

    const int vh = blockIdx.x, vs = blockIdx.y;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int KH = p.KH, VH = p.VH, rep = VH / KH, kh = vh / rep;
    const int KD = KH * kDK;

    // ---- prologue: state slice, conv weights (independent of the previous kernel)
    float S[kVS];
    float* Srow = p.state + ((size_t)vh * kDK + t) * kDV + vs * kVS;
    {
        const float4* s4 = reinterpret_cast<const float4*>(Srow);
#pragma unroll
        for (int i = 0; i < kVS / 4; ++i) {
            float4 v = s4[i];
            S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
        }
    }
    const int cq = kh * kDK + t, ck = KD + kh * kDK + t;
    const float4 wq = reinterpret_cast<const float4*>(p.conv_w)[cq];
    const float4 wk = reinterpret_cast<const float4*>(p.conv_w)[ck];
    const int cv = 2 * KD + vh * kDV + vs * kVS + t;  // valid for t < 16
    float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < kVS) wv = reinterpret_cast<const float4*>(p.conv_w)[cv];
    const float nA = p.neg_exp_A[vh], dtb = p.dt_bias[vh];

    pdl_wait();
    pdl_launch_dependents();

    const int pos = p.pos_ptr ? *p.pos_ptr : p.pos_val;
    const int cur = pos & 3, m1 = (pos + 3) & 3, m2 = (pos + 2) & 3, m3 = (pos + 1) & 3;
    float4* ring = reinterpret_cast<float4*>(p.conv_ring);

    auto conv = [&](int ch, float4 w, bool store) -> float {
        const float x = p.mixed[ch];
        const float4 st = ring[ch];
        const float sv[4] = {st.x, st.y, st.z, st.w};
        float acc = 0.f;
        acc += w.x * sv[m3];
        acc += w.y * sv[m2];
        acc += w.z * sv[m1];
        acc += w.w * x;
        if (store) reinterpret_cast<float*>(&ring[ch])[cur] = x;
        return silu_f(acc);
    };
    const bool owner_qk = (vs == 0) && (vh % rep == 0);
    float q = conv(cq, wq, owner_qk);
    float k = conv(ck, wk, owner_qk);
    if (t < kVS) s_v[t] = conv(cv, wv, true);

    // l2norm q and k over DK (sum in double), then q *= 1/sqrt(DK)
    const double sq = block128_sum_d((double)q * q, red_d);
    const double sk = block128_sum_d((double)k * k, red_d);
    q = q * (1.0f / sqrtf((float)sq + 1e-6f));
    q = q * (1.0f / sqrtf((float)kDK));
    k = k * (1.0f / sqrtf((float)sk + 1e-6f));

    const float g = nA * softplus_f(p.a[vh] + dtb);
    const float decay = expf(g), beta = sigmoid_f(p.b[vh]);

    // S *= decay; km = S^T k
    float part[kVS];
#pragma unroll
    for (int j = 0; j < kVS; ++j) {
        S[j] *= decay;
        part[j] = S[j] * k;
    }
#pragma unroll
    for (int j = 0; j < kVS; ++j) part[j] = warp_sum(part[j]);
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j < kVS; ++j) red16[warp][j] = part[j];
    }
    __syncthreads();
    if (t < kVS) {
        const float km = (red16[0][t] + red16[1][t]) + (red16[2][t] + red16[3][t]);
        s_km[t] = (s_v[t] - km) * beta;
    }
    __syncthreads();
    // S += k (x) d; o = S^T q
#pragma unroll
    for (int j = 0; j < kVS; ++j) {
        S[j] += k * s_km[j];
        part[j] = S[j] * q;
    }
#pragma unroll
    for (int j = 0; j < kVS; ++j) part[j] = warp_sum(part[j]);
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j < kVS; ++j) red16[warp][j] = part[j];
    }
    {
        float4* s4 = reinterpret_cast<float4*>(Srow);
#pragma unroll
        for (int i = 0; i < kVS / 4; ++i) s4[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
    }
    __syncthreads();
    if (t < kVS)
        p.out[(size_t)vh * kDV + vs * kVS + t] = (red16[0][t] + red16[1][t]) + (red16[2][t] + red16[3][t]);
}

cudaError_t launch_gdn_decode(const GdnDecodeParams& p, cudaStream_t s, bool pdl) {
    if (p.KH <= 0 || p.VH <= 0 || p.VH % p.KH != 0) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.VH, kDV / kVS);
    cfg.blockDim = dim3(128);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gdn_decode, p);
}

}  // namespace qwc
