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
#include "gdn_body.cuh"

namespace qwc {

__global__ void __launch_bounds__(128) k_gdn_decode(const GdnDecodeParams p) {
    gdn_decode_item(p, blockIdx.x, blockIdx.y, threadIdx.x, [] {
        pdl_wait();
        pdl_launch_dependents();
    });
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
