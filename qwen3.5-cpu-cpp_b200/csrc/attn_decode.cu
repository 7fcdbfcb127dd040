// Standalone split-K attention decode kernel (body in attn_body.cuh).
#include "attn_body.cuh"

namespace qwc {

template <int GRP>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnDecodeParams p) {
    pdl_wait();
    pdl_launch_dependents();
    attn_decode_item<GRP, 2>(p, blockIdx.x, blockIdx.y);
}

int attn_nsplit_for(int max_ctx, int nkv) {
    // splits of >= kMinChunk positions, at most one CTA per SM over all kv heads: more
    // splits shorten each CTA's loop but lengthen the serial combine of the partials
    int want = (max_ctx + kMinChunk - 1) / kMinChunk;
    int cap = num_sms() / (nkv > 0 ? nkv : 1);
    return want < 1 ? 1 : (want > cap ? cap : want);
}

cudaError_t launch_attn_decode(const AttnDecodeParams& p, cudaStream_t s, bool pdl) {
    if (p.NKV <= 0 || p.NQ % p.NKV != 0) return cudaErrorInvalidValue;
    if (p.proj && (p.rot > kHD || p.rot % 16 != 0)) return cudaErrorInvalidValue;
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
