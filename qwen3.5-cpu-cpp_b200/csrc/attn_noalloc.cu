// qwc_attention_decode_noalloc: attention decode for callers that must not allocate
// device memory while they run (a plugin whose host application owns all device memory
// through its own pool; a latency-critical loop that cannot afford cudaMalloc's implicit
// synchronisation). The split-K workspace that qwc_attention_decode grows with cudaMalloc
// lives here in one fixed array in device global memory instead.
#include <cstdio>
#include <mutex>

#include "kernels.h"

#include <algorithm>
#include "qwen_cuda.h"

namespace {

// 4 MiB per GPU that loads the library, held until the process exits. Layout:
// [0, 256) split counters (NKV <= 64), then part_ml, then part_o (256-byte aligned).
constexpr size_t kScratchBytes = 4u << 20;
constexpr int kMaxDevices = 64;
constexpr int kMaxKvHeads = 64;
constexpr int kHeadDim = 256;

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kScratchBytes];

// Device address of g_attn_noalloc_scratch per device. In host code the symbol name is
// only a host-side stand-in, so the address is looked up once per device with that
// device current, and passed to the kernel as a plain pointer.
void* g_scratch_dev[kMaxDevices] = {};
std::mutex g_setup_mu;

size_t round256(size_t v) { return (v + 255) & ~(size_t)255; }

int scratch_for_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        qwc::set_api_error("qwc_attention_decode_noalloc: no usable current device");
        return QWC_E_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_dev[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            char msg[256];
            std::snprintf(msg, sizeof msg, "qwc_attention_decode_noalloc: cudaGetSymbolAddress failed: %s",
                          cudaGetErrorString(e));
            qwc::set_api_error(msg);
            return QWC_E_CUDA;
        }
        g_scratch_dev[dev] = p;
    }
    *out = g_scratch_dev[dev];
    return QWC_OK;
}

}  // namespace

extern "C" int qwc_attention_decode_noalloc(const float* q, const float* gate, const void* k_cache,
                                            const void* v_cache, int kv_dtype, int NQ, int NKV, int max_ctx,
                                            int n_ctx, float* out, void* stream) {
    if (!q || !gate || !k_cache || !v_cache || !out || NKV <= 0 || NQ <= 0 || NQ % NKV || n_ctx <= 0 ||
        n_ctx > max_ctx || (kv_dtype != QWC_DTYPE_F32 && kv_dtype != QWC_DTYPE_BF16)) {
        qwc::set_api_error("qwc_attention_decode_noalloc: invalid argument");
        return QWC_E_INVALID;
    }
    // this entry keeps its own split rule (positions / 32, at most 2 per SM), in which its
    // documented workspace limit is stated; the result matches qwc_attention_decode to
    // rounding (the partials are grouped differently)
    const int nsplit = std::max(1, std::min((n_ctx + 31) / 32, 2 * qwc::num_sms()));
    const size_t rows = (size_t)NQ * nsplit;  // NKV * nsplit * GRP partial rows
    const size_t off_ml = 256;
    const size_t off_o = round256(off_ml + rows * 2 * sizeof(float));
    const size_t need = off_o + rows * kHeadDim * sizeof(float);
    if (NKV > kMaxKvHeads || need > kScratchBytes) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "qwc_attention_decode_noalloc: workspace of %zu bytes (NQ=%d, NKV=%d, %d splits) "
                      "exceeds the %zu-byte static scratch (or NKV > %d)",
                      need, NQ, NKV, nsplit, kScratchBytes, kMaxKvHeads);
        qwc::set_api_error(msg);
        return QWC_E_INVALID;
    }
    void* base = nullptr;
    int rc = scratch_for_current_device(&base);
    if (rc != QWC_OK) return rc;
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the array keeps the previous call's contents: the split counters must start at 0
    if (cudaMemsetAsync(b, 0, (size_t)NKV * sizeof(unsigned), s) != cudaSuccess) {
        qwc::set_api_error("qwc_attention_decode_noalloc: clearing the split counters failed");
        return QWC_E_CUDA;
    }
    qwc::AttnDecodeParams p;
    p.q_in = q;
    p.gate_in = gate;
    p.k_cache = const_cast<void*>(k_cache);
    p.v_cache = const_cast<void*>(v_cache);
    p.kv_bf16 = kv_dtype == QWC_DTYPE_BF16;
    p.max_ctx = max_ctx;
    p.n_ctx_val = n_ctx;
    p.NQ = NQ;
    p.NKV = NKV;
    p.nsplit = nsplit;
    p.out = out;
    p.counters = reinterpret_cast<unsigned*>(b);
    p.part_ml = reinterpret_cast<float*>(b + off_ml);
    p.part_o = reinterpret_cast<float*>(b + off_o);
    cudaError_t e = qwc::launch_attn_decode(p, s, false);
    if (e != cudaSuccess) {
        char msg[256];
        std::snprintf(msg, sizeof msg, "qwc_attention_decode_noalloc: %s", cudaGetErrorString(e));
        qwc::set_api_error(msg);
        return QWC_E_CUDA;
    }
    return QWC_OK;
}
