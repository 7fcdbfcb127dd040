// libqwen_cuda engine: the C ABI of include/qwen_cuda.h.
//
// Lifetime (QwenModel::QwenModel, src/qwen_model.cpp:12-96): every weight is resolved
// by name once, re-laid out for the decode kernels and uploaded into ONE device weight
// arena; the GDN recurrent state, the GDN conv state, the KV cache and the scratch
// arena are each one cudaMalloc sized by the memory equation; the decode step is
// captured once as a CUDA graph. qwc_step / qwc_generate_greedy then only replay the
// graph (zero allocation per token), with token id, position and the greedy argmax
// kept on the device.
#include "qwen_cuda.h"
#include "common.cuh"
#include "kernels.h"

#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <thread>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

using namespace qwc;

namespace {

thread_local std::string g_last_error;

__device__ int g_kernel_api_error;  // error word of the kernel-level entry points

struct Layer {
    int is_attn = 0, idx = 0;
    const float* in_ln1 = nullptr;   // 1 + input_layernorm.weight
    const float* post_ln1 = nullptr; // 1 + post_attention_layernorm.weight
    const uint16_t* w_in = nullptr;  // GDN: [qkv ; z ; b ; a] x H   attn: [q ; k ; v] x H
    int in_rows = 0;
    const uint16_t* w_out = nullptr; // GDN out_proj [H][VD]   attn o_proj [H][NQ*HD]
    int out_in = 0;
    const uint16_t* w_gu = nullptr;  // [I][2H], row i = [gate_i | up_i]
    const uint16_t* w_down = nullptr;// [H][I]
    // GDN
    const float* conv_w = nullptr;   // [C][4]
    const float* neg_exp_A = nullptr;// [VH]
    const float* dt_bias = nullptr;  // [VH]
    const float* gn_w = nullptr;     // [DV]
    // attention
    const float* qn1 = nullptr;      // 1 + q_norm
    const float* kn1 = nullptr;      // 1 + k_norm
};

// Where the mutable state of one sequence lives (the handle's decode state, or a
// temporary one for the stateless forward pass).
struct StateView {
    float* gdn_state = nullptr;  // [n_gdn][VH][DK][DV]
    float* conv_ring = nullptr;  // [n_gdn][C][4]
    void* kv = nullptr;          // [n_attn][2][NKV][max_ctx][HD]
    int max_ctx = 0;
};

}  // namespace

struct qwc_handle {
    int device = 0;
    cudaStream_t stream = nullptr;
    qwc_config cfg{};
    int max_ctx = 0, kv_dtype = QWC_DTYPE_F32, kv_bytes = 4;
    int H = 0, I = 0, V = 0, L = 0, NQ = 0, NKV = 0, HD = 0, ROT = 0;
    int KH = 0, VH = 0, DK = 0, DV = 0, KD = 0, VD = 0, C = 0, KER = 0;
    int n_gdn = 0, n_attn = 0, nsplit = 1, step_min_chunk = 8;
    float eps = 1e-6f;

    // arenas
    uint8_t* w_arena = nullptr;
    size_t w_bytes = 0;
    StateView st;
    size_t gdn_bytes = 0, conv_bytes = 0, kvc_bytes = 0;
    uint8_t* scratch = nullptr;
    size_t scratch_bytes = 0;

    std::vector<Layer> layers;
    const uint16_t* embed = nullptr;
    const uint16_t* head = nullptr;
    const float* final_ln1 = nullptr;
    const float* rope_cs = nullptr;  // [max_ctx][rot/2][2] RoPE cos/sin per position

    // scratch views
    float *hidden = nullptr, *proj = nullptr, *mix = nullptr, *ffn_h = nullptr, *logits = nullptr;
    float *am_val = nullptr, *part_o = nullptr, *part_ml = nullptr;
    int *am_idx = nullptr, *tokens = nullptr, *pos = nullptr, *n_prompt = nullptr, *argmax = nullptr;
    int* tp_vote = nullptr;  // tensor parallelism: the status vote of qwc_tp_gather_state
    int* dev_err = nullptr;
    unsigned *am_counter = nullptr, *attn_counters = nullptr;

    int* h_pin = nullptr;  // pinned host ints for small transfers
    struct Stager* stager = nullptr;  // weight upload staging (creation only)

    // persistent decode-step kernel (step_grid == 0: per-kernel path)
    StepParams step;
    StepPhase* step_phases = nullptr;  // device array
    int step_grid = 0;
    std::vector<int> step_kinds;  // QWC_K_* of each phase
    std::vector<StepPhase> step_host;  // host copy of the phases (algorithmic bytes)
    unsigned long long* step_bar = nullptr;
    unsigned* step_done = nullptr;

    // batched forward pass (prefill): weight tensor maps (built on first use) and a
    // workspace for chunks of up to pf_cap tokens
    bool pf_maps_ready = false;
    std::vector<CUtensorMap> pf_map_in, pf_map_out, pf_map_gu, pf_map_down;
    CUtensorMap pf_map_head{};
    uint8_t* pf_ws = nullptr;
    int pf_cap = 0;
    long pf_ldp = 0, pf_lda = 0, pf_ldb = 0;
    int* pf_ids = nullptr;
    float *pf_hid = nullptr, *pf_proj = nullptr, *pf_o = nullptr, *pf_qn = nullptr, *pf_kn = nullptr,
          *pf_vc = nullptr, *pf_glog = nullptr, *pf_beta = nullptr, *pf_qbuf = nullptr, *pf_logits = nullptr;
    float *pf_u = nullptr, *pf_w = nullptr, *pf_kd = nullptr, *pf_gc = nullptr;
    // GDN bf16-pair operands of the tensor-core output kernel: Gamma Q, P, S^T and E^T
    uint16_t *pf_qg = nullptr, *pf_p = nullptr, *pf_st = nullptr, *pf_et = nullptr;
    uint16_t *pf_xa = nullptr, *pf_xb = nullptr;
    uint16_t* pf_vsplit = nullptr;  // [NKV][chunk][512] V of the chunk as bf16 pairs
    // tensor-core attention: per attention layer K [NKV][ctx][512] and V^T [NKV][512][ctx]
    // as bf16 pairs, for the positions of one batched pass
    uint16_t* pf_kvs = nullptr;
    size_t pf_kvs_bytes = 0;
    float* pf_fa_part = nullptr;  // key-split partials of the prefill attention (O, then m / l)
    size_t pf_fa_part_bytes = 0;

    // tensor parallelism: this handle holds `shard` of a tp_world-rank group; the working
    // sizes above (KH, VH, KD, VD, C, NQ, NKV, I) are the shard's, g_* the whole model's
    int tp_rank = 0, tp_world = 1;
    qwc_tp_shard shard{};
    int gKH = 0, gVH = 0, gKD = 0, gVD = 0, gC = 0, gNQ = 0, gNKV = 0, gI = 0;
    ncclComm_t nccl = nullptr;       // non-blocking communicator (calls are settled, waits bounded)
    int tp_timeout_ms = 300000;      // bound on every wait for the group (env QWC_TP_TIMEOUT_MS)
    bool nccl_aborted = false;       // the communicator was aborted: the handle refuses work
    // peer-memory all-reduce of the residual stream (tp_p2p.cu); off after a failed setup
    // vote or with QWC_TP_ALLREDUCE=nccl, in which case NCCL's all-reduce is used
    P2pGroup* p2p = nullptr;
    bool p2p_off = false;
    int p2p_gen = 0;
    unsigned long long p2p_epoch = 0;
    uint64_t tp_group = 0;           // hash of the group's NCCL id: names the exchange sockets
    // QWC_PF_TIMING=1: per batched pass, the device time of the whole pass and of its
    // parts by category (event pairs from a pool reused across passes) on stderr
    bool pf_timing = false;
    std::vector<cudaEvent_t> pf_ev;  // [0] [1]: the pass; then one pair per timed part
    size_t pf_ev_used = 0;
    std::vector<int> pf_pair_cat;    // category of each pair

    cudaGraphExec_t graph = nullptr;
    bool use_graph = true, use_pdl = true;
    int pos_host = 0;
    qwc_budget budget{};
    std::string err;
};

// ------------------------------------------------------------------ error helpers
static int nccl_settle(qwc_handle* h, ncclResult_t r, const char* what);  // group failures, below
static int fail(qwc_handle* h, int code, const std::string& msg) {
    if (h) h->err = msg;
    g_last_error = msg;
    return code;
}
#define CU(call)                                                                         \
    do {                                                                                 \
        cudaError_t e_ = (call);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return fail(h, QWC_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

static int check_device_error(qwc_handle* h) {
    int v = 0;
    CU(cudaMemcpyAsync(&h->h_pin[8], h->dev_err, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    CU(cudaStreamSynchronize(h->stream));
    v = h->h_pin[8];
    if (v != 0) {
        cudaMemsetAsync(h->dev_err, 0, sizeof(int), h->stream);
        return fail(h, QWC_E_DEVICE, "device kernel reported error code " + std::to_string(v));
    }
    return QWC_OK;
}

// ------------------------------------------------------------------ config / budget
extern "C" void qwc_default_config(qwc_config* c) {
    // ModelConfig defaults (include/model_config.h:11-63)
    std::memset(c, 0, sizeof(*c));
    c->hidden_size = 1024;
    c->n_layers_total = 24;
    c->n_layers_gdn = 18;
    c->n_layers_attn = 6;
    c->gdn_k_heads = 16;
    c->gdn_v_heads = 16;
    c->gdn_k_head_dim = 128;
    c->gdn_v_head_dim = 128;
    c->gdn_conv_kernel = 4;
    c->attn_q_heads = 8;
    c->attn_kv_heads = 2;
    c->attn_head_dim = 256;
    c->ffn_intermediate = 3584;
    c->vocab_size = 248320;
    c->native_max_context = 262144;
    c->rms_norm_eps = 1e-6f;
    c->tie_word_embeddings = 1;
    c->rope_theta = 10000000.0;
    c->partial_rotary_factor = 0.25f;
    c->attn_interval = 4;
    c->n_params = 800000000LL;
}

static size_t conv_state_bytes_eq(const qwc_config* c) {
    // gdn_conv_state_bytes (include/memory_budget.h:23-28)
    size_t kd = (size_t)c->gdn_k_heads * c->gdn_k_head_dim, vd = (size_t)c->gdn_v_heads * c->gdn_v_head_dim;
    return (size_t)c->n_layers_gdn * (kd * 2 + vd) * (c->gdn_conv_kernel - 1) * sizeof(float);
}

extern "C" int qwc_compute_budget(const qwc_config* c, int bpw, int max_context, int kvb,
                                  int max_vision_tiles, int vit_dim, qwc_budget* out) {
    if (!c || !out) return fail(nullptr, QWC_E_INVALID, "qwc_compute_budget: null argument");
    // compute_budget (src/memory_budget.cpp:30-54) and its two estimators (:4-28)
    out->weight_bytes = (uint64_t)c->n_params * (uint64_t)bpw;
    out->gdn_state_bytes = (uint64_t)c->n_layers_gdn * c->gdn_v_heads * c->gdn_k_head_dim *
                           c->gdn_v_head_dim * sizeof(float);
    out->gdn_conv_bytes = conv_state_bytes_eq(c);
    out->kv_cache_bytes = (uint64_t)c->n_layers_attn * (uint64_t)max_context * 2 * c->attn_kv_heads *
                          c->attn_head_dim * kvb;
    size_t ffn = (size_t)c->ffn_intermediate * sizeof(float) * 2;
    size_t attn = (size_t)(c->attn_q_heads * c->attn_head_dim + 2 * c->attn_kv_heads * c->attn_head_dim) *
                  sizeof(float);
    size_t gdn = (size_t)(3 * c->gdn_v_heads * c->gdn_v_head_dim) * sizeof(float);
    size_t act = ffn;
    if (attn > act) act = attn;
    if (gdn > act) act = gdn;
    out->activation_bytes = act;
    const size_t ppt = 256;
    out->vision_scratch_bytes = (uint64_t)max_vision_tiles * ppt * vit_dim * sizeof(float) +
                                (uint64_t)ppt * vit_dim * sizeof(float) * 2;
    return QWC_OK;
}

extern "C" int64_t qwc_solve_max_context(const qwc_config* c, uint64_t ram, uint64_t wb, uint64_t gb,
                                         uint64_t ab, uint64_t vb, uint64_t margin, int kvb) {
    // solve_max_context (src/memory_budget.cpp:56-81)
    uint64_t fixed = wb + gb + ab + vb + margin;
    if (fixed >= ram) return -1;
    uint64_t per_tok = (uint64_t)c->n_layers_attn * 2 * c->attn_kv_heads * c->attn_head_dim * kvb;
    if (per_tok == 0) return -1;
    int64_t ctx = (int64_t)((ram - fixed) / per_tok);
    return ctx < c->native_max_context ? ctx : c->native_max_context;
}

namespace qwc {
void set_api_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace qwc

extern "C" const char* qwc_last_error(const qwc_handle* h) {
    return h ? h->err.c_str() : g_last_error.c_str();
}

// ------------------------------------------------------------------ weight upload
namespace {

struct HostTensor {
    const qwc_tensor* t;
    int64_t numel;
};

struct Builder {
    qwc_handle* h;
    std::unordered_map<std::string, HostTensor> by_name;
    std::string missing;

    const qwc_tensor* find(const std::string& n) {
        auto it = by_name.find(n);
        return it == by_name.end() ? nullptr : it->second.t;
    }
    const qwc_tensor* need(const std::string& n) {
        const qwc_tensor* t = find(n);
        if (!t && missing.empty()) missing = n;
        return t;
    }
};

int64_t numel_of(const qwc_tensor* t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
    return t->ndim ? n : 0;
}

float elem_f32(const qwc_tensor* t, int64_t i) {
    if (t->dtype == QWC_DTYPE_F32) return static_cast<const float*>(t->data)[i];
    uint32_t u = (uint32_t)static_cast<const uint16_t*>(t->data)[i] << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// A bump allocator over the weight arena: first pass measures, second pass places.
struct Arena {
    uint8_t* base = nullptr;
    size_t off = 0;
    void* take(size_t bytes) {
        off = (off + 255) & ~(size_t)255;
        void* p = base ? base + off : nullptr;
        off += bytes;
        return p;
    }
};

}  // namespace

// Weight upload through pinned staging: the checkpoint stays in the caller's (memory-
// mapped) host buffers; each piece is packed into one of two pinned buffers and copied to
// the device asynchronously, so the host packs piece k+1 while the DMA engine moves piece
// k. No full-file host copy is made, and no pageable copy is synchronous.
struct Stager {
    static constexpr size_t kCap = 32u << 20;  // bytes per pinned buffer
    cudaStream_t s = nullptr;
    uint8_t* pin[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int cur = 0;
    bool ok = false;
    explicit Stager(cudaStream_t stream) : s(stream) {
        ok = cudaHostAlloc(&pin[0], kCap, cudaHostAllocDefault) == cudaSuccess &&
             cudaHostAlloc(&pin[1], kCap, cudaHostAllocDefault) == cudaSuccess &&
             cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming) == cudaSuccess &&
             cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming) == cudaSuccess;
    }
    ~Stager() {
        if (s) cudaStreamSynchronize(s);
        for (int i = 0; i < 2; ++i) {
            if (pin[i]) cudaFreeHost(pin[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
    }
    // rows x width bytes from src (row pitch spitch) to dst (row pitch dpitch), in batches
    // of whole rows that fit one buffer (a row wider than a buffer is split into columns)
    cudaError_t copy2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t rows) {
        if (width > kCap) {
            for (size_t c0 = 0; c0 < width; c0 += kCap) {
                const size_t w = std::min(kCap, width - c0);
                cudaError_t e = copy2d(static_cast<uint8_t*>(dst) + c0, dpitch, static_cast<const uint8_t*>(src) + c0,
                                       spitch, w, rows);
                if (e != cudaSuccess) return e;
            }
            return cudaSuccess;
        }
        const size_t per = kCap / width;
        for (size_t r0 = 0; r0 < rows; r0 += per) {
            const size_t n = std::min(per, rows - r0);
            cudaError_t e = cudaEventSynchronize(done[cur]);  // this buffer's previous DMA is over
            if (e != cudaSuccess) return e;
            const uint8_t* sp = static_cast<const uint8_t*>(src) + r0 * spitch;
            if (spitch == width) {
                std::memcpy(pin[cur], sp, n * width);
            } else {
                for (size_t r = 0; r < n; ++r) std::memcpy(pin[cur] + r * width, sp + r * spitch, width);
            }
            e = cudaMemcpy2DAsync(static_cast<uint8_t*>(dst) + r0 * dpitch, dpitch, pin[cur], width, width, n,
                                  cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return e;
            if ((e = cudaEventRecord(done[cur], s)) != cudaSuccess) return e;
            cur ^= 1;
        }
        return cudaSuccess;
    }
};

static int h2d(qwc_handle* h, void* dst, size_t dpitch, const void* src, size_t spitch, size_t width, size_t rows) {
    cudaError_t e = h->stager ? h->stager->copy2d(dst, dpitch, src, spitch, width, rows)
                              : cudaMemcpy2D(dst, dpitch, src, spitch, width, rows, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return fail(h, QWC_E_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
    return QWC_OK;
}

static int upload_f32(qwc_handle* h, float* dst, const std::vector<float>& v) {
    return h2d(h, dst, v.size() * sizeof(float), v.data(), v.size() * sizeof(float), v.size() * sizeof(float), 1);
}

// Copies a BF16 matrix [rows][cols] into dst with destination row pitch `dpitch` elements.
static int upload_mat(qwc_handle* h, uint16_t* dst, size_t dpitch, const qwc_tensor* t, int64_t rows,
                      int64_t cols) {
    if (t->dtype != QWC_DTYPE_BF16)
        return fail(h, QWC_E_SHAPE, std::string("matrix ") + t->name + " must be BF16");
    if (numel_of(t) != rows * cols)
        return fail(h, QWC_E_SHAPE, std::string("tensor ") + t->name + " has an unexpected shape");
    return h2d(h, dst, dpitch * 2, t->data, cols * 2, cols * 2, rows);
}

// Rows [row0, row0+nrows) of a BF16 matrix [total_rows][cols] into dst (row pitch dpitch).
static int upload_rows(qwc_handle* h, uint16_t* dst, size_t dpitch, const qwc_tensor* t, int64_t total_rows,
                       int64_t cols, int64_t row0, int64_t nrows) {
    if (t->dtype != QWC_DTYPE_BF16)
        return fail(h, QWC_E_SHAPE, std::string("matrix ") + t->name + " must be BF16");
    if (numel_of(t) != total_rows * cols)
        return fail(h, QWC_E_SHAPE, std::string("tensor ") + t->name + " has an unexpected shape");
    const uint16_t* src = static_cast<const uint16_t*>(t->data) + row0 * cols;
    return h2d(h, dst, dpitch * 2, src, cols * 2, cols * 2, nrows);
}

// Columns [col0, col0+ncols) of a BF16 matrix [rows][total_cols] into a dense [rows][ncols].
static int upload_cols(qwc_handle* h, uint16_t* dst, const qwc_tensor* t, int64_t rows, int64_t total_cols,
                       int64_t col0, int64_t ncols) {
    if (t->dtype != QWC_DTYPE_BF16)
        return fail(h, QWC_E_SHAPE, std::string("matrix ") + t->name + " must be BF16");
    if (numel_of(t) != rows * total_cols)
        return fail(h, QWC_E_SHAPE, std::string("tensor ") + t->name + " has an unexpected shape");
    const uint16_t* src = static_cast<const uint16_t*>(t->data) + col0;
    return h2d(h, dst, ncols * 2, src, total_cols * 2, ncols * 2, rows);
}

static int vec_f32(qwc_handle* h, const qwc_tensor* t, int64_t n, std::vector<float>& out, float add = 0.f) {
    if (numel_of(t) != n) return fail(h, QWC_E_SHAPE, std::string("tensor ") + t->name + " has an unexpected size");
    out.resize(n);
    for (int64_t i = 0; i < n; ++i) out[i] = add == 0.f ? elem_f32(t, i) : (add + elem_f32(t, i));
    return QWC_OK;
}

// Resolve, lay out and upload all weights. With arena.base == nullptr only measures.
static int place_weights(qwc_handle* h, Builder& b, Arena& a) {
    const bool doit = a.base != nullptr;
    const int H = h->H, I = h->I;
    const std::string LM = "model.language_model.";
    int ai = 0, gi = 0;
    h->layers.assign(h->L, Layer());
    std::vector<float> tmp;
    for (int L = 0; L < h->L; ++L) {
        Layer& lw = h->layers[L];
        const std::string P = LM + "layers." + std::to_string(L) + ".";
        const qwc_tensor* iln = b.need(P + "input_layernorm.weight");
        const qwc_tensor* pln = b.need(P + "post_attention_layernorm.weight");
        const qwc_tensor* gp = b.need(P + "mlp.gate_proj.weight");
        const qwc_tensor* up = b.need(P + "mlp.up_proj.weight");
        const qwc_tensor* dp = b.need(P + "mlp.down_proj.weight");
        lw.in_ln1 = (const float*)a.take((size_t)H * 4);
        lw.post_ln1 = (const float*)a.take((size_t)H * 4);
        lw.w_gu = (const uint16_t*)a.take((size_t)I * 2 * H * 2);
        lw.w_down = (const uint16_t*)a.take((size_t)H * I * 2);
        const bool attn = (L + 1) % h->cfg.attn_interval == 0;
        lw.is_attn = attn ? 1 : 0;
        if (attn) {
            lw.idx = ai++;
            const std::string A = P + "self_attn.";
            const qwc_tensor* q = b.need(A + "q_proj.weight");
            const qwc_tensor* k = b.need(A + "k_proj.weight");
            const qwc_tensor* v = b.need(A + "v_proj.weight");
            const qwc_tensor* o = b.need(A + "o_proj.weight");
            const qwc_tensor* qn = b.need(A + "q_norm.weight");
            const qwc_tensor* kn = b.need(A + "k_norm.weight");
            // this shard's q heads [q0, q0+NQ) and the kv heads [kv0, kv0+NKV) they read
            const int qr = 2 * h->NQ * h->HD, kr = h->NKV * h->HD;
            const int64_t q0 = h->shard.q0, kv0 = h->shard.kv0;
            lw.in_rows = qr + 2 * kr;
            lw.w_in = (const uint16_t*)a.take((size_t)lw.in_rows * H * 2);
            lw.out_in = h->NQ * h->HD;
            lw.w_out = (const uint16_t*)a.take((size_t)H * lw.out_in * 2);
            lw.qn1 = (const float*)a.take((size_t)h->HD * 4);
            lw.kn1 = (const float*)a.take((size_t)h->HD * 4);
            if (doit && b.missing.empty()) {
                uint16_t* wi = const_cast<uint16_t*>(lw.w_in);
                int rc;
                const int64_t HD = h->HD;
                if ((rc = upload_rows(h, wi, H, q, 2L * h->gNQ * HD, H, q0 * 2 * HD, qr))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)qr * H, H, k, (int64_t)h->gNKV * HD, H, kv0 * HD, kr))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)(qr + kr) * H, H, v, (int64_t)h->gNKV * HD, H, kv0 * HD, kr))) return rc;
                if ((rc = upload_cols(h, const_cast<uint16_t*>(lw.w_out), o, H, (int64_t)h->gNQ * HD, q0 * HD, lw.out_in))) return rc;
                if ((rc = vec_f32(h, qn, h->HD, tmp, 1.0f)) || (rc = upload_f32(h, const_cast<float*>(lw.qn1), tmp))) return rc;
                if ((rc = vec_f32(h, kn, h->HD, tmp, 1.0f)) || (rc = upload_f32(h, const_cast<float*>(lw.kn1), tmp))) return rc;
            }
        } else {
            lw.idx = gi++;
            const std::string G = P + "linear_attn.";
            const qwc_tensor* qkv = b.need(G + "in_proj_qkv.weight");
            const qwc_tensor* z = b.need(G + "in_proj_z.weight");
            const qwc_tensor* bb = b.need(G + "in_proj_b.weight");
            const qwc_tensor* aa = b.need(G + "in_proj_a.weight");
            const qwc_tensor* cw = b.need(G + "conv1d.weight");
            const qwc_tensor* dt = b.need(G + "dt_bias");
            const qwc_tensor* al = b.need(G + "A_log");
            const qwc_tensor* gn = b.need(G + "norm.weight");
            const qwc_tensor* op = b.need(G + "out_proj.weight");
            lw.in_rows = h->C + h->VD + 2 * h->VH;
            lw.w_in = (const uint16_t*)a.take((size_t)lw.in_rows * H * 2);
            lw.out_in = h->VD;
            lw.w_out = (const uint16_t*)a.take((size_t)H * h->VD * 2);
            lw.conv_w = (const float*)a.take((size_t)h->C * 4 * 4);
            lw.neg_exp_A = (const float*)a.take((size_t)h->VH * 4);
            lw.dt_bias = (const float*)a.take((size_t)h->VH * 4);
            lw.gn_w = (const float*)a.take((size_t)h->DV * 4);
            if (doit && b.missing.empty()) {
                // this shard's k heads [kh0, +KH) and v heads [vh0, +VH): their q, k, v channels,
                // z rows, b / a rows, conv channels and gates, out_proj input columns
                uint16_t* wi = const_cast<uint16_t*>(lw.w_in);
                const int64_t kh0 = h->shard.kh0, vh0 = h->shard.vh0, DK = h->DK, DV = h->DV;
                const int64_t KD = h->KD, VD = h->VD, C = h->C, VHl = h->VH;
                int rc;
                if ((rc = upload_rows(h, wi, H, qkv, h->gC, H, kh0 * DK, KD))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)KD * H, H, qkv, h->gC, H, h->gKD + kh0 * DK, KD))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)2 * KD * H, H, qkv, h->gC, H, 2L * h->gKD + vh0 * DV, VD))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)C * H, H, z, h->gVD, H, vh0 * DV, VD))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)(C + VD) * H, H, bb, h->gVH, H, vh0, VHl))) return rc;
                if ((rc = upload_rows(h, wi + (size_t)(C + VD + VHl) * H, H, aa, h->gVH, H, vh0, VHl))) return rc;
                if ((rc = upload_cols(h, const_cast<uint16_t*>(lw.w_out), op, H, h->gVD, vh0 * DV, VD))) return rc;
                if ((rc = vec_f32(h, cw, (int64_t)h->gC * h->KER, tmp))) return rc;
                {
                    std::vector<float> cl((size_t)C * h->KER);
                    auto take = [&](int64_t dst_ch, int64_t src_ch, int64_t n) {
                        std::memcpy(&cl[(size_t)dst_ch * h->KER], &tmp[(size_t)src_ch * h->KER], (size_t)n * h->KER * 4);
                    };
                    take(0, kh0 * DK, KD);
                    take(KD, h->gKD + kh0 * DK, KD);
                    take(2 * KD, 2L * h->gKD + vh0 * DV, VD);
                    if ((rc = upload_f32(h, const_cast<float*>(lw.conv_w), cl))) return rc;
                }
                // -exp(A_log) with the host expf, as the reference evaluates it
                if ((rc = vec_f32(h, al, h->gVH, tmp))) return rc;
                tmp = std::vector<float>(tmp.begin() + vh0, tmp.begin() + vh0 + VHl);
                for (auto& x : tmp) x = -std::exp(x);
                if ((rc = upload_f32(h, const_cast<float*>(lw.neg_exp_A), tmp))) return rc;
                if ((rc = vec_f32(h, dt, h->gVH, tmp))) return rc;
                tmp = std::vector<float>(tmp.begin() + vh0, tmp.begin() + vh0 + VHl);
                if ((rc = upload_f32(h, const_cast<float*>(lw.dt_bias), tmp))) return rc;
                if ((rc = vec_f32(h, gn, h->DV, tmp)) || (rc = upload_f32(h, const_cast<float*>(lw.gn_w), tmp))) return rc;
            }
        }
        if (doit && b.missing.empty()) {
            int rc;
            if ((rc = vec_f32(h, iln, H, tmp, 1.0f)) || (rc = upload_f32(h, const_cast<float*>(lw.in_ln1), tmp))) return rc;
            if ((rc = vec_f32(h, pln, H, tmp, 1.0f)) || (rc = upload_f32(h, const_cast<float*>(lw.post_ln1), tmp))) return rc;
            // this shard's intermediate rows [i0, i0+I) of gate / up and down_proj columns
            uint16_t* gu = const_cast<uint16_t*>(lw.w_gu);
            const int64_t i0 = h->shard.i0;
            if ((rc = upload_rows(h, gu, 2 * (size_t)H, gp, h->gI, H, i0, I))) return rc;
            if ((rc = upload_rows(h, gu + H, 2 * (size_t)H, up, h->gI, H, i0, I))) return rc;
            if ((rc = upload_cols(h, const_cast<uint16_t*>(lw.w_down), dp, H, h->gI, i0, I))) return rc;
        }
    }
    const qwc_tensor* emb = b.need(LM + "embed_tokens.weight");
    const qwc_tensor* fn = b.need(LM + "norm.weight");
    // dedicated lm_head if present, else the tied embedding (src/qwen_model.cpp:67-69)
    const qwc_tensor* lmh = b.find("lm_head.weight");
    if (!lmh) lmh = b.find(LM + "lm_head.weight");
    h->embed = (const uint16_t*)a.take((size_t)h->V * H * 2);
    h->head = lmh ? (const uint16_t*)a.take((size_t)h->V * H * 2) : h->embed;
    h->final_ln1 = (const float*)a.take((size_t)H * 4);
    h->rope_cs = (const float*)a.take((size_t)h->max_ctx * (h->ROT / 2) * 2 * 4 + 16);
    if (doit && b.missing.empty()) {
        int rc;
        if (emb->ndim != 2 || emb->shape[1] != H || emb->shape[0] < h->V)
            return fail(h, QWC_E_SHAPE, "embed_tokens.weight rows < vocab_size or width != hidden_size");
        if ((rc = upload_mat(h, const_cast<uint16_t*>(h->embed), H, emb, h->V, H) )) {
            // the embedding may hold more rows than vocab_size: upload only vocab_size rows
            if (emb->dtype != QWC_DTYPE_BF16) return rc;
            if ((rc = h2d(h, const_cast<uint16_t*>(h->embed), (size_t)H * 2, emb->data, (size_t)H * 2, (size_t)H * 2,
                          (size_t)h->V)))
                return rc;
        }
        if (lmh) {
            if (lmh->dtype != QWC_DTYPE_BF16 || lmh->ndim != 2 || lmh->shape[1] != H || lmh->shape[0] < h->V)
                return fail(h, QWC_E_SHAPE, "lm_head.weight must be BF16 [>=vocab, hidden]");
            if ((rc = h2d(h, const_cast<uint16_t*>(h->head), (size_t)H * 2, lmh->data, (size_t)H * 2, (size_t)H * 2,
                          (size_t)h->V)))
                return rc;
        }
        if ((rc = vec_f32(h, fn, H, tmp, 1.0f)) || (rc = upload_f32(h, const_cast<float*>(h->final_ln1), tmp))) return rc;
        // RoPE table, exactly as apply_rope evaluates it (src/forward_pass.cpp:102-112):
        // inv_freq and the angle in double, cos/sin in double, rounded to float.
        const int half = h->ROT / 2;
        if (half > 0) {
            std::vector<double> invf(half);
            for (int i = 0; i < half; ++i) invf[i] = std::pow(h->cfg.rope_theta, -(double)(2 * i) / h->ROT);
            std::vector<float> tab((size_t)h->max_ctx * half * 2);
            for (int pp = 0; pp < h->max_ctx; ++pp)
                for (int i = 0; i < half; ++i) {
                    const double ang = (double)pp * invf[i];
                    tab[((size_t)pp * half + i) * 2] = (float)std::cos(ang);
                    tab[((size_t)pp * half + i) * 2 + 1] = (float)std::sin(ang);
                }
            if ((rc = h2d(h, const_cast<float*>(h->rope_cs), tab.size() * 4, tab.data(), tab.size() * 4, tab.size() * 4, 1)))
                return rc;
        }
    }
    if (!b.missing.empty()) return fail(h, QWC_E_MISSING, "[qwen] missing weight: " + b.missing);
    return QWC_OK;
}

// ------------------------------------------------------------------ the decode step
static GemvParams gp_base(qwc_handle* h) {
    GemvParams p;
    p.eps = h->eps;
    p.dev_err = h->dev_err;
    return p;
}

// Optional per-launch timing of an eager step (qwc_profile_step).
struct StepProfile {
    int cap = 0, n = 0;
    std::vector<cudaEvent_t> ev;  // ev[0] before the first launch, ev[i+1] after launch i
    std::vector<int> kind;
    std::vector<int64_t> bytes;
};

// The decode step as a list of phases (one per kernel of the per-kernel path, one per
// grid-barrier phase of the persistent kernel), with the profiling kind of each.
static void make_phases(qwc_handle* h, const StateView& sv, int attn_nsplit, std::vector<StepPhase>& out,
                        std::vector<int>& kinds, bool defer_attn = false, int min_chunk = 32) {
    const int H = h->H;
    out.clear();
    kinds.clear();
    const size_t kv_layer = (size_t)2 * h->NKV * sv.max_ctx * h->HD * h->kv_bytes;
    auto gemv = [&](int pro, int epi, const GemvParams& g, int kind) {
        StepPhase ph;
        ph.type = PH_GEMV;
        ph.pro = pro;
        ph.epi = epi;
        ph.g = g;
        out.push_back(ph);
        kinds.push_back(kind);
    };
    for (int L = 0; L < h->L; ++L) {
        const Layer& lw = h->layers[L];
        // mixer input projection with the input RMSNorm (and the embedding at layer 0)
        GemvParams p = gp_base(h);
        p.W = lw.w_in;
        p.rows = lw.in_rows;
        p.in_dim = H;
        p.x_len = H;
        p.x = h->hidden;
        p.norm_w = lw.in_ln1;
        p.y = h->proj;
        int pro = PRO_RMSNORM;
        if (L == 0) {
            pro = PRO_EMBED_RMSNORM;
            p.embed = h->embed;
            p.tokens = h->tokens;
            p.pos = h->pos;
            p.vocab = h->V;
            p.hidden_out = h->hidden;
        }
        gemv(pro, EPI_STORE, p, QWC_K_MIX_IN);
        if (lw.is_attn) {
            StepPhase ph;
            ph.type = PH_ATTN;
            AttnDecodeParams& a = ph.a;
            a.proj = h->proj;
            a.qn1 = lw.qn1;
            a.kn1 = lw.kn1;
            a.rope_cs = h->rope_cs;
            uint8_t* kvl = static_cast<uint8_t*>(sv.kv) + kv_layer * lw.idx;
            a.k_cache = kvl;
            a.v_cache = kvl + kv_layer / 2;
            a.kv_bf16 = h->kv_dtype == QWC_DTYPE_BF16;
            a.max_ctx = sv.max_ctx;
            a.pos_ptr = h->pos;
            a.part_o = h->part_o;
            a.part_ml = h->part_ml;
            a.counters = h->attn_counters;
            a.out = h->mix;
            a.NQ = h->NQ;
            a.NKV = h->NKV;
            a.rot = h->ROT;
            a.nsplit = attn_nsplit;
            a.min_chunk = min_chunk;
            a.eps = h->eps;
            a.defer_combine = defer_attn ? 1 : 0;
            out.push_back(ph);
            kinds.push_back(QWC_K_ATTN);
            GemvParams o = gp_base(h);
            o.W = lw.w_out;
            o.rows = H;
            o.in_dim = lw.out_in;
            o.x_len = lw.out_in;
            o.x = h->mix;
            o.y = h->hidden;
            int opro = PRO_PLAIN;
            if (defer_attn) {  // o_proj combines the attention partials in its prologue
                opro = PRO_ATTN_COMBINE;
                o.x = h->proj;  // the gates
                o.part_o = h->part_o;
                o.part_ml = h->part_ml;
                o.pos = h->pos;
                o.nsplit = attn_nsplit;
                o.min_chunk = min_chunk;
                o.nq = h->NQ;
                o.nkv = h->NKV;
            }
            gemv(opro, EPI_RESIDUAL, o, QWC_K_MIX_OUT);
        } else {
            StepPhase ph;
            ph.type = PH_GDN;
            GdnDecodeParams& g = ph.d;
            g.mixed = h->proj;
            g.b = h->proj + h->C + h->VD;
            g.a = h->proj + h->C + h->VD + h->VH;
            g.conv_w = lw.conv_w;
            g.neg_exp_A = lw.neg_exp_A;
            g.dt_bias = lw.dt_bias;
            g.conv_ring = sv.conv_ring + (size_t)lw.idx * h->C * 4;
            g.state = sv.gdn_state + (size_t)lw.idx * h->VH * h->DK * h->DV;
            g.out = h->mix;
            g.pos_ptr = h->pos;
            g.KH = h->KH;
            g.VH = h->VH;
            out.push_back(ph);
            kinds.push_back(QWC_K_GDN);
            GemvParams o = gp_base(h);
            o.W = lw.w_out;
            o.rows = H;
            o.in_dim = h->VD;
            o.x_len = h->VD;
            o.x = h->mix;
            o.z = h->proj + h->C;
            o.norm_w = lw.gn_w;
            o.gn_dim = h->DV;
            o.y = h->hidden;
            gemv(PRO_GATED_NORM, EPI_RESIDUAL, o, QWC_K_MIX_OUT);
        }
        // FFN: post-attention RMSNorm + gate/up + SwiGLU, then down + residual
        GemvParams f = gp_base(h);
        f.W = lw.w_gu;
        f.rows = h->I;
        f.in_dim = 2 * H;
        f.x_len = H;
        f.x = h->hidden;
        f.norm_w = lw.post_ln1;
        f.y = h->ffn_h;
        gemv(PRO_RMSNORM, EPI_SWIGLU, f, QWC_K_GATE_UP);
        GemvParams d = gp_base(h);
        d.W = lw.w_down;
        d.rows = H;
        d.in_dim = h->I;
        d.x_len = h->I;
        d.x = h->ffn_h;
        d.y = h->hidden;
        gemv(PRO_PLAIN, EPI_RESIDUAL, d, QWC_K_DOWN);
    }
    GemvParams o = gp_base(h);
    o.W = h->head;
    o.rows = h->V;
    o.in_dim = H;
    o.x_len = H;
    o.x = h->hidden;
    o.norm_w = h->final_ln1;
    o.y = h->logits;
    o.am_val = h->am_val;
    o.am_idx = h->am_idx;
    o.am_counter = h->am_counter;
    o.argmax_out = h->argmax;
    o.tokens_out = h->tokens;
    o.n_prompt = h->n_prompt;
    o.pos_inout = h->pos;
    o.max_ctx = sv.max_ctx;
    gemv(PRO_RMSNORM, EPI_ARGMAX, o, QWC_K_LM_HEAD);
}

// Algorithmic HBM bytes of one phase at position `pos` (for qwc_profile_step).
static int64_t phase_bytes(const qwc_handle* h, const StepPhase& ph, int pos) {
    if (ph.type == PH_GEMV) {
        const GemvParams& g = ph.g;
        return (int64_t)g.rows * g.in_dim * 2 + (int64_t)g.x_len * 8 +
               (int64_t)g.rows * (ph.epi == EPI_RESIDUAL ? 8 : 4);
    }
    if (ph.type == PH_GDN)
        return (int64_t)h->VH * h->DK * h->DV * 8 + (int64_t)h->C * (16 + 4 + 16 + 4) + (int64_t)h->VD * 4;
    return (int64_t)(pos + 1) * h->NKV * h->HD * h->kv_bytes * 2 + (int64_t)(2 * h->NQ * h->HD + 2 * h->NKV * h->HD) * 4 +
           (int64_t)h->NQ * h->HD * 4;
}

// Enqueue one decode step as separate kernels (embedding -> layers -> lm_head + argmax).
static int enqueue_step(qwc_handle* h, const StateView& sv, bool pdl, StepProfile* prof = nullptr,
                        int pos_for_bytes = 0) {
    std::vector<StepPhase> phases;
    std::vector<int> kinds;
    make_phases(h, sv, h->nsplit, phases, kinds);
    if (prof) CU(cudaEventRecord(prof->ev[0], h->stream));
    for (size_t i = 0; i < phases.size(); ++i) {
        const StepPhase& ph = phases[i];
        const bool use_pdl = pdl && i > 0;
        if (ph.type == PH_GEMV) {
            const int per_sm = ph.epi == EPI_ARGMAX ? 2 : 1;
            CU(launch_gemv(ph.pro, ph.epi, ph.g, gemv_grid(ph.g.rows, per_sm), h->stream, use_pdl));
        } else if (ph.type == PH_GDN) {
            CU(launch_gdn_decode(ph.d, h->stream, use_pdl));
        } else {
            CU(launch_attn_decode(ph.a, h->stream, use_pdl));
        }
        if (prof) {
            if (prof->n < prof->cap) {
                CU(cudaEventRecord(prof->ev[prof->n + 1], h->stream));
                prof->kind[prof->n] = kinds[i];
                prof->bytes[prof->n] = phase_bytes(h, ph, pos_for_bytes);
            }
            prof->n++;
        }
    }
    return QWC_OK;
}

// One launch of the persistent decode-step kernel.
static int enqueue_persistent(qwc_handle* h) {
    CU(launch_decode_step(h->step, h->NQ / h->NKV, h->step_grid, h->stream));
    return QWC_OK;
}

static int build_graph(qwc_handle* h) {
    if (h->graph) {
        cudaGraphExecDestroy(h->graph);
        h->graph = nullptr;
    }
    if (!h->use_graph) return QWC_OK;
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    int rc = h->step_grid > 0 ? enqueue_persistent(h) : enqueue_step(h, h->st, h->use_pdl);
    cudaError_t e = cudaStreamEndCapture(h->stream, &g);
    if (rc != QWC_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(h, QWC_E_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
    e = cudaGraphInstantiate(&h->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(h, QWC_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
    return QWC_OK;
}

static int run_step(qwc_handle* h) {
    if (h->graph) {
        CU(cudaGraphLaunch(h->graph, h->stream));
        return QWC_OK;
    }
    return h->step_grid > 0 ? enqueue_persistent(h) : enqueue_step(h, h->st, h->use_pdl);
}

// Choose the persistent decode-step kernel when the shapes allow it (every GEMV input
// length a multiple of 256, one co-resident CTA per SM) unless QWC_DECODE=kernels.
static int setup_persistent(qwc_handle* h) {
    h->step_grid = 0;
    const char* mode = std::getenv("QWC_DECODE");
    if (mode && std::string(mode) == "kernels") return QWC_OK;
    const int grp = h->NQ / h->NKV;
    if (h->H % 256 || h->I % 256 || h->VD % 256 || (h->NQ * h->HD) % 256 || h->H > 4096) return QWC_OK;
    const int xs_max = std::max({h->H, h->I, h->VD, h->NQ * h->HD});
    const int grid0 = num_sms();
    // attention items are spread one per CTA: at most grid / NKV splits of >= step_min_chunk
    const int nsplit = std::max(1, std::min({h->nsplit, grid0 / h->NKV,
                                             (h->max_ctx + h->step_min_chunk - 1) / h->step_min_chunk}));
    std::vector<StepPhase> phases;
    // the o_proj phase combines the split attention partials when a warp per q head fits
    make_phases(h, h->st, nsplit, phases, h->step_kinds, /*defer_attn=*/h->NQ <= 8, h->step_min_chunk);
    const int np = (int)phases.size();
    // Ring depth: three 4 KB slots per consumer warp (96 KB per SM) measured fastest with
    // the producer warp; deeper rings queue latency-critical loads behind weights.
    int nslot = std::min(step_slots(xs_max, grp, np), 3);
    if (const char* e = std::getenv("QWC_STEP_SLOTS")) nslot = std::max(2, std::min(step_slots(xs_max, grp, np), std::atoi(e)));
    const int grid = decode_step_max_grid(grp, nslot, xs_max, np);
    if (grid <= 0) return QWC_OK;
    CU(cudaMalloc(&h->step_phases, phases.size() * sizeof(StepPhase)));
    CU(cudaMemcpy(h->step_phases, phases.data(), phases.size() * sizeof(StepPhase), cudaMemcpyHostToDevice));
    h->step_host = phases;
    h->step.phases = h->step_phases;
    h->step.nphases = (int)phases.size();
    h->step.bar = h->step_bar;
    h->step.done = h->step_done;
    h->step.dev_err = h->dev_err;
    h->step.nslot = nslot;
    h->step.xs_max = xs_max;
    h->step_grid = grid;
    return QWC_OK;
}

// ------------------------------------------------------------------ create / destroy
static int validate_config(qwc_handle* h, const qwc_config* c) {
    if (c->hidden_size <= 0 || c->hidden_size % 8) return fail(h, QWC_E_SHAPE, "hidden_size must be a positive multiple of 8");
    if (c->gdn_k_head_dim != 128 || c->gdn_v_head_dim != 128)
        return fail(h, QWC_E_SHAPE, "GDN head dims other than 128 are not supported");
    if (c->gdn_conv_kernel != 4) return fail(h, QWC_E_SHAPE, "GDN conv kernel other than 4 is not supported");
    if (c->attn_head_dim != 256) return fail(h, QWC_E_SHAPE, "attention head_dim other than 256 is not supported");
    if (c->attn_kv_heads <= 0 || c->attn_q_heads % c->attn_kv_heads)
        return fail(h, QWC_E_SHAPE, "num_attention_heads must be a multiple of num_key_value_heads");
    const int grp = c->attn_q_heads / c->attn_kv_heads;
    if (grp != 1 && grp != 2 && grp != 4 && grp != 8) return fail(h, QWC_E_SHAPE, "GQA group must be 1, 2, 4 or 8");
    if (c->gdn_k_heads <= 0 || c->gdn_v_heads % c->gdn_k_heads)
        return fail(h, QWC_E_SHAPE, "linear_num_value_heads must be a multiple of linear_num_key_heads");
    if (c->ffn_intermediate <= 0 || c->ffn_intermediate % 8) return fail(h, QWC_E_SHAPE, "intermediate_size must be a multiple of 8");
    if (c->attn_interval <= 0 || c->n_layers_total <= 0) return fail(h, QWC_E_SHAPE, "bad layer layout");
    const int rot = (int)(c->attn_head_dim * c->partial_rotary_factor);
    if (rot < 0 || rot > c->attn_head_dim || rot % 2) return fail(h, QWC_E_SHAPE, "bad partial_rotary_factor");
    if (c->vocab_size <= 0) return fail(h, QWC_E_SHAPE, "bad vocab_size");
    return QWC_OK;
}

extern "C" void qwc_destroy(qwc_handle* h) {
    if (!h) return;
    cudaSetDevice(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    if (h->graph) cudaGraphExecDestroy(h->graph);
    cudaFree(h->w_arena);
    cudaFree(h->st.gdn_state);
    cudaFree(h->st.conv_ring);
    cudaFree(h->st.kv);
    cudaFree(h->scratch);
    cudaFree(h->step_phases);
    for (cudaEvent_t e : h->pf_ev) cudaEventDestroy(e);
    cudaFree(h->pf_ws);
    cudaFree(h->pf_kvs);
    cudaFree(h->pf_fa_part);
    p2p_destroy(h->p2p);
    if (h->nccl) {
        // a communicator whose group is incomplete would block ncclCommDestroy: abort it
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(h->nccl, &st);
        if (st == ncclSuccess) ncclCommDestroy(h->nccl);
        else ncclCommAbort(h->nccl);
    }
    if (h->h_pin) cudaFreeHost(h->h_pin);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h;
}

extern "C" int qwc_tp_shard_of(const qwc_config* c, int rank, int world, qwc_tp_shard* o) {
    if (!c || !o || world < 1 || rank < 0 || rank >= world) return fail(nullptr, QWC_E_INVALID, "qwc_tp_shard_of: invalid argument");
    const int KH = c->gdn_k_heads, VH = c->gdn_v_heads, NQ = c->attn_q_heads, NKV = c->attn_kv_heads;
    const int I = c->ffn_intermediate;
    if (KH <= 0 || VH <= 0 || NKV <= 0 || NQ % NKV || VH % KH)
        return fail(nullptr, QWC_E_SHAPE, "qwc_tp_shard_of: inconsistent head counts");
    if (KH % world || VH % world || NQ % world || I % world || (world > 1 && (I / world) % 64) ||
        !(NKV % world == 0 || world % NKV == 0))
        return fail(nullptr, QWC_E_SHAPE, "the model does not split over " + std::to_string(world) + " ranks");
    o->n_kh = KH / world;
    o->kh0 = rank * o->n_kh;
    o->n_vh = VH / world;
    o->vh0 = rank * o->n_vh;
    o->n_q = NQ / world;
    o->q0 = rank * o->n_q;
    if (world <= NKV) {
        o->n_kv = NKV / world;
        o->kv0 = rank * o->n_kv;
    } else {  // several ranks share (a replica of) one kv head
        o->n_kv = 1;
        o->kv0 = o->q0 / (NQ / NKV);
    }
    o->n_i = I / world;
    o->i0 = rank * o->n_i;
    return QWC_OK;
}

extern "C" int qwc_tp_unique_id(void* out, int bytes) {
    if (!out || bytes < (int)sizeof(ncclUniqueId)) return fail(nullptr, QWC_E_INVALID, "qwc_tp_unique_id: buffer too small");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return fail(nullptr, QWC_E_CUDA, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
    return QWC_OK;
}

static int create_impl(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors, int max_context,
                       int kv_dtype, int device, int rank, int world, const void* unique_id, qwc_handle** out);

extern "C" int qwc_create(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors, int max_context,
                          int kv_dtype, int device, qwc_handle** out) {
    return create_impl(cfg, tensors, n_tensors, max_context, kv_dtype, device, 0, 1, nullptr, out);
}

extern "C" int qwc_create_tp(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors, int max_context,
                             int kv_dtype, int device, int rank, int world, const void* unique_id, qwc_handle** out) {
    if (world > 1 && !unique_id) return fail(nullptr, QWC_E_INVALID, "qwc_create_tp: unique_id is required");
    return create_impl(cfg, tensors, n_tensors, max_context, kv_dtype, device, rank, world, unique_id, out);
}

// The longest context that fits the current device's free memory (max_context <= 0 at
// creation): solve_max_context over the free bytes with the weight arena (as measured
// with a one-position RoPE table), the GDN state and conv ring as fixed costs, a reserve
// for the scratch, the step kernel and the batched pass's workspace, and an effective
// per-element KV size that also carries the per-position RoPE table, token slot and
// batched-pass attention operands.
static int64_t plan_max_context(qwc_handle* h) {
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return -1;
    qwc_config local = h->cfg;
    local.gdn_k_heads = h->KH;
    local.gdn_v_heads = h->VH;
    local.attn_q_heads = h->NQ;
    local.attn_kv_heads = h->NKV;
    local.ffn_intermediate = h->I;
    qwc_budget b{};
    qwc_compute_budget(&local, 2, 1, h->kv_bytes, 4, 1024, &b);
    const uint64_t state = b.gdn_state_bytes + (uint64_t)h->n_gdn * h->C * 4 * sizeof(float);
    const uint64_t per_elem_tokens = (uint64_t)h->n_attn * 2 * h->NKV * h->HD;  // KV elements per position
    if (per_elem_tokens == 0) return h->cfg.native_max_context;
    const uint64_t extra = (uint64_t)h->ROT * 4 + 8 + (uint64_t)8 * h->NKV * h->HD * h->n_attn;
    const int kvb_eff = (int)((per_elem_tokens * h->kv_bytes + extra + per_elem_tokens - 1) / per_elem_tokens);
    const uint64_t reserve = 3ull << 30;  // scratch, step, batched-pass workspace (4096-token chunks)
    const uint64_t margin = 512ull << 20;
    return qwc_solve_max_context(&local, free_b, h->w_bytes, state, reserve, 0, margin, kvb_eff);
}

static int create_impl(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors, int max_context,
                       int kv_dtype, int device, int rank, int world, const void* unique_id, qwc_handle** out) {
    if (!cfg || !out || (!tensors && n_tensors > 0) || world < 1 || rank < 0 || rank >= world)
        return fail(nullptr, QWC_E_INVALID, "qwc_create: invalid argument");
    if (kv_dtype != QWC_DTYPE_F32 && kv_dtype != QWC_DTYPE_BF16)
        return fail(nullptr, QWC_E_INVALID, "qwc_create: kv_dtype must be F32 or BF16");
    *out = nullptr;
    qwc_handle* h = new qwc_handle();
    h->device = device;
    h->cfg = *cfg;
    int rc = validate_config(h, cfg);
    if (rc) { g_last_error = h->err; delete h; return rc; }
    if (cudaSetDevice(device) != cudaSuccess) {
        delete h;
        return fail(nullptr, QWC_E_CUDA, "cudaSetDevice failed");
    }
    const char* ng = std::getenv("QWC_NO_GRAPH");
    h->use_graph = !(ng && ng[0] == '1');
    const char* pt = std::getenv("QWC_PF_TIMING");
    h->pf_timing = pt && pt[0] == '1';
    const char* np = std::getenv("QWC_NO_PDL");
    h->use_pdl = !(np && np[0] == '1');
    h->max_ctx = max_context > 0 ? max_context : 0;  // 0: planned once the weights are measured
    h->kv_dtype = kv_dtype;
    h->kv_bytes = kv_dtype == QWC_DTYPE_BF16 ? 2 : 4;
    h->H = cfg->hidden_size;
    h->I = cfg->ffn_intermediate;
    h->V = cfg->vocab_size;
    h->L = cfg->n_layers_total;
    h->NQ = cfg->attn_q_heads;
    h->NKV = cfg->attn_kv_heads;
    h->HD = cfg->attn_head_dim;
    h->ROT = (int)(h->HD * cfg->partial_rotary_factor);
    h->KH = cfg->gdn_k_heads;
    h->VH = cfg->gdn_v_heads;
    h->DK = cfg->gdn_k_head_dim;
    h->DV = cfg->gdn_v_head_dim;
    h->KD = h->KH * h->DK;
    h->VD = h->VH * h->DV;
    h->C = 2 * h->KD + h->VD;
    h->KER = cfg->gdn_conv_kernel;
    h->eps = cfg->rms_norm_eps;
    h->n_attn = h->L / cfg->attn_interval;
    h->n_gdn = h->L - h->n_attn;
    h->cfg.n_layers_attn = h->n_attn;
    h->cfg.n_layers_gdn = h->n_gdn;
    // tensor-parallel shard: the working sizes become the shard's
    h->tp_rank = rank;
    h->tp_world = world;
    h->gKH = h->KH; h->gVH = h->VH; h->gKD = h->KD; h->gVD = h->VD; h->gC = h->C;
    h->gNQ = h->NQ; h->gNKV = h->NKV; h->gI = h->I;
    rc = qwc_tp_shard_of(&h->cfg, rank, world, &h->shard);
    if (rc) { delete h; return rc; }
    h->KH = h->shard.n_kh;
    h->VH = h->shard.n_vh;
    h->KD = h->KH * h->DK;
    h->VD = h->VH * h->DV;
    h->C = 2 * h->KD + h->VD;
    h->NQ = h->shard.n_q;
    h->NKV = h->shard.n_kv;
    h->I = h->shard.n_i;

    Builder b;
    b.h = h;
    for (int i = 0; i < n_tensors; ++i) {
        if (!tensors[i].name || !tensors[i].data) continue;
        b.by_name[tensors[i].name] = HostTensor{&tensors[i], numel_of(&tensors[i])};
    }
    // pass 1: measure
    Arena meas;
    rc = place_weights(h, b, meas);
    if (rc) { g_last_error = h->err; delete h; return rc; }
    h->w_bytes = meas.off;
    if (h->max_ctx <= 0) {
        // max_context <= 0: the longest context that fits the device's free memory, planned
        // with the memory equation (solve_max_context, src/memory_budget.cpp:56-81)
        int64_t ctx = plan_max_context(h);
        if (ctx < 1) {
            fail(h, QWC_E_OOM, "qwc_create: the model does not fit the free device memory");
            g_last_error = h->err;
            delete h;
            return QWC_E_OOM;
        }
        h->max_ctx = (int)std::min<int64_t>(ctx, 1 << 30);
        max_context = h->max_ctx;
        Arena again;  // the RoPE table grows with the context
        rc = place_weights(h, b, again);
        if (rc) { g_last_error = h->err; delete h; return rc; }
        h->w_bytes = again.off;
    }

    auto bail = [&](int code) { g_last_error = h->err; qwc_destroy(h); return code; };
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess)
        return bail(fail(h, QWC_E_CUDA, "cudaStreamCreate failed"));
    if (cudaMalloc(&h->w_arena, h->w_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "weight arena allocation failed"));
    Arena real;
    real.base = h->w_arena;
    {
        Stager st(h->stream);
        if (st.ok) h->stager = &st;  // else plain synchronous copies
        rc = place_weights(h, b, real);
        h->stager = nullptr;
    }  // every staged copy has completed here
    if (rc) return bail(rc);

    // state arenas, sized by the memory equation (compute_budget with bpw 2) for this shard
    qwc_config local = h->cfg;
    local.gdn_k_heads = h->KH;
    local.gdn_v_heads = h->VH;
    local.attn_q_heads = h->NQ;
    local.attn_kv_heads = h->NKV;
    local.ffn_intermediate = h->I;
    qwc_compute_budget(&local, 2, max_context, h->kv_bytes, 4, 1024, &h->budget);
    h->gdn_bytes = h->budget.gdn_state_bytes;
    h->kvc_bytes = h->budget.kv_cache_bytes;
    // conv state: a ring of K slots per channel (the equation counts K-1)
    h->conv_bytes = (size_t)h->n_gdn * h->C * 4 * sizeof(float);
    h->st.max_ctx = max_context;
    if (h->gdn_bytes && cudaMalloc(&h->st.gdn_state, h->gdn_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "GDN state allocation failed"));
    if (h->conv_bytes && cudaMalloc(&h->st.conv_ring, h->conv_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "conv state allocation failed"));
    if (h->kvc_bytes && cudaMalloc(&h->st.kv, h->kvc_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "KV cache allocation failed"));

    // scratch arena
    h->nsplit = attn_nsplit_for(max_context, h->NKV);
    // the persistent step splits attention into items of >= step_min_chunk positions (one
    // per warp at 8), one (kv head, split) item per CTA: the partials are sized for both
    if (const char* e = std::getenv("QWC_STEP_MIN_CHUNK")) h->step_min_chunk = std::max(1, std::atoi(e));
    h->nsplit = std::max(h->nsplit, std::min((max_context + h->step_min_chunk - 1) / h->step_min_chunk,
                                             std::max(1, num_sms() / h->NKV)));
    const int grp = h->NQ / h->NKV;
    Arena s;
    auto carve = [&](size_t bytes) { return s.take(bytes); };
    const int proj_n = std::max(h->C + h->VD + 2 * h->VH, 2 * h->NQ * h->HD + 2 * h->NKV * h->HD);
    const int nsm = gemv_grid(h->V, 2);  // CTAs of the lm_head GEMV: one argmax partial each
    struct { void** p; size_t bytes; } plan[] = {
        {(void**)&h->hidden, (size_t)h->H * 4},
        {(void**)&h->proj, (size_t)proj_n * 4},
        {(void**)&h->mix, (size_t)std::max(h->VD, h->NQ * h->HD) * 4},
        {(void**)&h->ffn_h, (size_t)h->I * 4},
        {(void**)&h->logits, (size_t)h->V * 4},
        {(void**)&h->am_val, (size_t)nsm * 4},
        {(void**)&h->am_idx, (size_t)nsm * 4},
        {(void**)&h->am_counter, 16},
        {(void**)&h->attn_counters, (size_t)h->NKV * 4},
        {(void**)&h->part_o, (size_t)h->NKV * h->nsplit * grp * h->HD * 4},
        {(void**)&h->part_ml, (size_t)h->NKV * h->nsplit * grp * 2 * 4},
        {(void**)&h->tokens, (size_t)(max_context + 1) * 4},
        {(void**)&h->pos, 16},
        {(void**)&h->n_prompt, 16},
        {(void**)&h->argmax, 16},
        {(void**)&h->dev_err, 16},
        {(void**)&h->tp_vote, 16},
        // grid-barrier counters on their own 4 KB lines, away from the other counters
        {(void**)&h->step_bar, 4096},
        {(void**)&h->step_done, 4096},
    };
    for (auto& e : plan) carve(e.bytes);
    h->scratch_bytes = s.off;
    if (cudaMalloc(&h->scratch, h->scratch_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "scratch allocation failed"));
    s.base = h->scratch;
    s.off = 0;
    for (auto& e : plan) *e.p = carve(e.bytes);
    if (cudaMemset(h->scratch, 0, h->scratch_bytes) != cudaSuccess)
        return bail(fail(h, QWC_E_CUDA, "scratch memset failed"));
    if (cudaMallocHost(&h->h_pin, 64 * sizeof(int)) != cudaSuccess)
        return bail(fail(h, QWC_E_OOM, "pinned host allocation failed"));
    // reconcile the activation arena with the real allocation (qwen_model.cpp:84-87)
    h->budget.activation_bytes = h->scratch_bytes;
    h->budget.vision_scratch_bytes = 0;

    rc = qwc_reset(h);
    if (rc) return bail(rc);
    if (world > 1) {
        if (const char* e = std::getenv("QWC_TP_TIMEOUT_MS")) h->tp_timeout_ms = std::max(1, std::atoi(e));
        ncclUniqueId id;
        std::memcpy(&id, unique_id, sizeof(id));
        uint64_t hsh = 1469598103934665603ull;  // FNV-1a of the id: the same on every rank
        for (size_t i = 0; i < sizeof(id); ++i) hsh = (hsh ^ (uint8_t)id.internal[i]) * 1099511628211ull;
        h->tp_group = hsh;
        ncclConfig_t ncfg = NCCL_CONFIG_INITIALIZER;
        ncfg.blocking = 0;  // every wait for the group is bounded (nccl_settle, stream_wait)
        const ncclResult_t r = ncclCommInitRankConfig(&h->nccl, world, id, rank, &ncfg);
        if (r != ncclSuccess && r != ncclInProgress) {
            h->nccl = nullptr;
            return bail(fail(h, QWC_E_CUDA, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r)));
        }
        if ((rc = nccl_settle(h, r, "ncclCommInitRankConfig"))) return bail(rc);
        *out = h;  // decode state machinery is single-GPU only
        return QWC_OK;
    }
    rc = setup_persistent(h);
    if (rc) return bail(rc);
    rc = build_graph(h);
    if (rc && h->step_grid > 0) {
        // the persistent kernel could not be captured: use the per-kernel path
        std::fprintf(stderr, "[qwc] persistent decode step unavailable (%s); using separate kernels\n",
                     h->err.c_str());
        h->step_grid = 0;
        rc = build_graph(h);
    }
    if (rc) return bail(rc);
    *out = h;
    return QWC_OK;
}

// ------------------------------------------------------------------ decode API
extern "C" int qwc_reset(qwc_handle* h) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_reset: null handle");
    CU(cudaSetDevice(h->device));
    // QwenModel::reset (src/qwen_model.cpp:98-104): zero every cache and the position
    if (h->gdn_bytes) CU(cudaMemsetAsync(h->st.gdn_state, 0, h->gdn_bytes, h->stream));
    if (h->conv_bytes) CU(cudaMemsetAsync(h->st.conv_ring, 0, h->conv_bytes, h->stream));
    if (h->kvc_bytes) CU(cudaMemsetAsync(h->st.kv, 0, h->kvc_bytes, h->stream));
    CU(cudaMemsetAsync(h->pos, 0, sizeof(int), h->stream));
    if (h->step_bar) CU(cudaMemsetAsync(h->step_bar, 0, 16, h->stream));
    if (h->step_done) CU(cudaMemsetAsync(h->step_done, 0, 16, h->stream));
    CU(cudaStreamSynchronize(h->stream));
    h->pos_host = 0;
    return QWC_OK;
}

extern "C" int qwc_position(const qwc_handle* h) { return h ? h->pos_host : -1; }

extern "C" int qwc_max_context(const qwc_handle* h) { return h ? h->max_ctx : -1; }

extern "C" int qwc_step(qwc_handle* h, int token, float* logits_host, int* argmax_out) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_step: null handle");
    if (h->tp_world > 1) return fail(h, QWC_E_INVALID, "qwc_step: decode needs a single-GPU handle");
    if (token < 0 || token >= h->V) return fail(h, QWC_E_INVALID, "qwc_step: token id out of range");
    if (h->pos_host >= h->max_ctx) return fail(h, QWC_E_CONTEXT, "qwc_step: position would exceed max_context");
    CU(cudaSetDevice(h->device));
    // the token goes to tokens[pos]; n_prompt = max_ctx keeps the argmax from writing tokens
    h->h_pin[0] = token;
    h->h_pin[1] = h->max_ctx;
    CU(cudaMemcpyAsync(h->tokens + h->pos_host, &h->h_pin[0], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    CU(cudaMemcpyAsync(h->n_prompt, &h->h_pin[1], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    int rc = run_step(h);
    if (rc) return rc;
    if (logits_host)
        CU(cudaMemcpyAsync(logits_host, h->logits, (size_t)h->V * 4, cudaMemcpyDeviceToHost, h->stream));
    CU(cudaMemcpyAsync(&h->h_pin[2], h->argmax, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    rc = check_device_error(h);  // synchronises
    if (rc) return rc;
    h->pos_host++;
    if (argmax_out) *argmax_out = h->h_pin[2];
    return QWC_OK;
}

extern "C" int qwc_generate_greedy(qwc_handle* h, const int* prompt, int n_prompt, int n_new, int* out_tokens) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_generate_greedy: null handle");
    if (h->tp_world > 1) return fail(h, QWC_E_INVALID, "qwc_generate_greedy: decode needs a single-GPU handle");
    if (n_prompt < 0 || n_new < 0 || (n_prompt > 0 && !prompt) || (n_new > 0 && !out_tokens))
        return fail(h, QWC_E_INVALID, "qwc_generate_greedy: invalid argument");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= h->V) return fail(h, QWC_E_INVALID, "qwc_generate_greedy: token id out of range");
    if ((long)n_prompt + n_new > h->max_ctx)
        return fail(h, QWC_E_CONTEXT, "qwc_generate_greedy: prompt + n_new exceeds max_context");
    int rc = qwc_reset(h);
    if (rc) return rc;
    if (n_prompt == 0) return QWC_OK;  // the reference produces nothing without a prompt
    CU(cudaMemcpyAsync(h->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, h->stream));
    h->h_pin[3] = n_prompt;
    CU(cudaMemcpyAsync(h->n_prompt, &h->h_pin[3], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    for (int i = 0; i < n_prompt + n_new; ++i) {
        rc = run_step(h);
        if (rc) return rc;
    }
    if (n_new > 0)
        CU(cudaMemcpyAsync(out_tokens, h->tokens + n_prompt, (size_t)n_new * 4, cudaMemcpyDeviceToHost, h->stream));
    rc = check_device_error(h);
    if (rc) return rc;
    h->pos_host = n_prompt + n_new;
    return QWC_OK;
}

extern "C" int qwc_get_budget(const qwc_handle* h, qwc_budget* out) {
    if (!h || !out) return fail(nullptr, QWC_E_INVALID, "qwc_get_budget: null argument");
    *out = h->budget;
    return QWC_OK;
}

extern "C" int qwc_get_config(const qwc_handle* h, qwc_config* out) {
    if (!h || !out) return fail(nullptr, QWC_E_INVALID, "qwc_get_config: null argument");
    *out = h->cfg;
    return QWC_OK;
}

// ------------------------------------------------------------------ prefill (stepping)
// First implementation: the prompt goes through the decode step one token at a time,
// exactly as the reference's generate_greedy feeds it (src/qwen_model.cpp:245).
// ------------------------------------------------------------------ batched forward pass
// QwenForward::prefill (src/qwen_forward.cpp:154-206) as whole-chunk GEMMs on the tensor
// cores plus token-parallel kernels (prefill.cu, tc_gemm.cu), continuing from and updating
// a decode state, so the same code serves the stateless forward pass (fresh state) and
// the prefill that seeds decoding.
// Tokens per chunk (bounds the workspace); QWC_PREFILL_CHUNK overrides. A tensor-parallel
// rank uses twice as many: its all-reduces are one per row-parallel projection and chunk,
// and larger messages use NVLink better (2B shape, 131072 tokens, two GPUs: 1319 -> 1287
// ms per pass; on one GPU the larger chunk is 1.5 % slower).
constexpr int kPfChunk = 4096, kPfChunkTp = 8192;
static int pf_chunk(const qwc_handle* h) {
    const char* e = std::getenv("QWC_PREFILL_CHUNK");
    const int v = e ? std::atoi(e) : 0;
    return v > 0 ? v : (h->tp_world > 1 ? kPfChunkTp : kPfChunk);
}
constexpr int kPfLogitRows = 128;  // lm_head rows per GEMM when every position's logits are wanted

static int pf_build_maps(qwc_handle* h) {
    if (h->pf_maps_ready) return QWC_OK;
    const int L = h->L;
    h->pf_map_in.resize(L);
    h->pf_map_out.resize(L);
    h->pf_map_gu.resize(L);
    h->pf_map_down.resize(L);
    for (int l = 0; l < L; ++l) {
        const Layer& lw = h->layers[l];
        if (tc_make_map(&h->pf_map_in[l], lw.w_in, lw.in_rows, h->H, h->H) ||
            tc_make_map(&h->pf_map_out[l], lw.w_out, h->H, lw.out_in, lw.out_in) ||
            // [I][2H] rows [gate_i | up_i] read as [2I][H]: rows alternate gate_i, up_i
            tc_make_map(&h->pf_map_gu[l], lw.w_gu, 2L * h->I, h->H, h->H) ||
            tc_make_map(&h->pf_map_down[l], lw.w_down, h->H, h->I, h->I))
            return fail(h, QWC_E_CUDA, "prefill: tensor map creation failed");
    }
    if (tc_make_map(&h->pf_map_head, h->head, h->V, h->H, h->H))
        return fail(h, QWC_E_CUDA, "prefill: tensor map creation failed");
    h->pf_maps_ready = true;
    return QWC_OK;
}

// Causal attention of the batched pass on the tensor cores (default) or, with
// QWC_PREFILL_ATTN=simt, the fp32 CUDA-core kernel.
static bool pf_attn_tc() {
    const char* e = std::getenv("QWC_PREFILL_ATTN");
    return !(e && std::strcmp(e, "simt") == 0);
}

static int pf_workspace(qwc_handle* h, int cap) {
    if (h->pf_cap >= cap) return QWC_OK;
    cudaFree(h->pf_ws);
    h->pf_ws = nullptr;
    h->pf_cap = 0;
    int ldp = 0;
    for (const Layer& lw : h->layers) ldp = std::max(ldp, lw.in_rows);
    h->pf_ldp = (ldp + 63) / 64 * 64;
    const long ka = std::max({h->H, h->VD, h->NQ * h->HD});
    h->pf_lda = 2 * ka;
    h->pf_ldb = 2L * h->I;
    size_t off = 0;
    auto carve = [&](size_t bytes) {
        const size_t o = off;
        off += (bytes + 255) / 256 * 256;
        return o;
    };
    const size_t c = (size_t)cap;
    const size_t o_ids = carve(c * 4), o_hid = carve(c * h->H * 4), o_proj = carve(c * h->pf_ldp * 4),
                 o_o = carve(c * h->VD * 4), o_qn = carve(c * h->KD * 4), o_kn = carve(c * h->KD * 4),
                 o_vc = carve(c * h->VD * 4), o_dec = carve(c * h->VH * 4), o_beta = carve(c * h->VH * 4),
                 o_qbuf = carve(c * h->NQ * h->HD * 4), o_log = carve((size_t)kPfLogitRows * h->V * 4),
                 o_u = carve(c * h->VD * 4), o_w = carve((c + 63) / 64 * 64 * h->VD * 4), o_qg = carve((c + 63) / 64 * 64 * h->VD * 4),
                 o_kd = carve(c * h->VD * 4), o_p = carve((size_t)h->VH * ((c + 63) / 64) * 2 * 64 * 64 * 2),
                 o_gc = carve((size_t)h->VH * ((c + 63) / 64) * 4),
                 o_xa = carve(c * h->pf_lda * 2), o_xb = carve(c * h->pf_ldb * 2),
                 o_vs = carve(c * h->NKV * 2 * h->HD * 2),
                 o_st = carve((size_t)h->VH * ((c + 63) / 64) * 2 * 128 * 128 * 2),
                 o_et = carve((size_t)h->VH * ((c + 63) / 64) * 2 * 128 * 64 * 2);
    if (cudaMalloc(&h->pf_ws, off) != cudaSuccess) {
        h->pf_ws = nullptr;
        return fail(h, QWC_E_OOM, "prefill workspace allocation failed");
    }
    uint8_t* b = h->pf_ws;
    h->pf_ids = reinterpret_cast<int*>(b + o_ids);
    h->pf_hid = reinterpret_cast<float*>(b + o_hid);
    h->pf_proj = reinterpret_cast<float*>(b + o_proj);
    h->pf_o = reinterpret_cast<float*>(b + o_o);
    h->pf_qn = reinterpret_cast<float*>(b + o_qn);
    h->pf_kn = reinterpret_cast<float*>(b + o_kn);
    h->pf_vc = reinterpret_cast<float*>(b + o_vc);
    h->pf_glog = reinterpret_cast<float*>(b + o_dec);
    h->pf_u = reinterpret_cast<float*>(b + o_u);
    h->pf_w = reinterpret_cast<float*>(b + o_w);
    h->pf_qg = reinterpret_cast<uint16_t*>(b + o_qg);
    h->pf_kd = reinterpret_cast<float*>(b + o_kd);
    h->pf_p = reinterpret_cast<uint16_t*>(b + o_p);
    h->pf_gc = reinterpret_cast<float*>(b + o_gc);
    h->pf_beta = reinterpret_cast<float*>(b + o_beta);
    h->pf_qbuf = reinterpret_cast<float*>(b + o_qbuf);
    h->pf_logits = reinterpret_cast<float*>(b + o_log);
    h->pf_xa = reinterpret_cast<uint16_t*>(b + o_xa);
    h->pf_xb = reinterpret_cast<uint16_t*>(b + o_xb);
    h->pf_vsplit = reinterpret_cast<uint16_t*>(b + o_vs);
    h->pf_st = reinterpret_cast<uint16_t*>(b + o_st);
    h->pf_et = reinterpret_cast<uint16_t*>(b + o_et);
    h->pf_cap = cap;
    return QWC_OK;
}

// ------------------------------------------------------------------ group failures
// The communicator is non-blocking: an NCCL call may return ncclInProgress, and the
// group's state is polled with ncclCommGetAsyncError. Every wait for the group is bounded
// by tp_timeout_ms; when it runs out (a rank died, or never posted its part of a
// collective) the communicator is aborted -- its kernels stop waiting -- and the call
// returns QWC_E_DEVICE. An aborted handle refuses further work.
static double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
static int tp_abort(qwc_handle* h, const std::string& why) {
    if (h->nccl && !h->nccl_aborted) {
        ncclCommAbort(h->nccl);
        h->nccl = nullptr;
        h->nccl_aborted = true;
        // the aborted collectives return; let the rest of the stream drain (bounded)
        const double t0 = now_ms();
        while (cudaStreamQuery(h->stream) == cudaErrorNotReady && now_ms() - t0 < 10000.0)
            std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    return fail(h, QWC_E_DEVICE, why);
}
// An NCCL call's return code: settles ncclInProgress (bounded), aborts on group errors.
static int nccl_settle(qwc_handle* h, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return QWC_OK;
    if (r != ncclInProgress) return tp_abort(h, std::string(what) + ": " + ncclGetErrorString(r));
    const double t0 = now_ms();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclCommGetAsyncError(h->nccl, &st);
        if (st == ncclSuccess) return QWC_OK;
        if (st != ncclInProgress) return tp_abort(h, std::string(what) + ": " + ncclGetErrorString(st));
        if (now_ms() - t0 > h->tp_timeout_ms) return tp_abort(h, std::string(what) + ": timed out");
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
// Waits for the handle's stream: plain for a single-GPU handle; for a tensor-parallel one
// polled together with the group's error state, bounded by tp_timeout_ms.
static int stream_wait(qwc_handle* h, const char* who) {
    if (h->tp_world == 1) {
        CU(cudaStreamSynchronize(h->stream));
        return QWC_OK;
    }
    const double t0 = now_ms();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(h->stream);
        if (q == cudaSuccess) return QWC_OK;
        if (q != cudaErrorNotReady) return fail(h, QWC_E_CUDA, std::string(who) + ": " + cudaGetErrorString(q));
        ncclResult_t st = ncclSuccess;
        if (h->nccl) ncclCommGetAsyncError(h->nccl, &st);
        if (st != ncclSuccess && st != ncclInProgress)
            return tp_abort(h, std::string(who) + ": tensor-parallel group error: " + ncclGetErrorString(st));
        if (now_ms() - t0 > h->tp_timeout_ms)
            return tp_abort(h, std::string(who) + ": the tensor-parallel group did not complete in time (a rank is gone?)");
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// Parts of a batched pass timed under QWC_PF_TIMING.
enum PfCat { PF_CAT_ALLREDUCE, PF_CAT_GDN, PF_CAT_GDN_STATE, PF_CAT_ATTN, PF_CAT_GEMM, PF_NCAT };
static const char* const kPfCatName[PF_NCAT] = {"all-reduce + add", "gdn mixer (all kernels)", "gdn state pass",
                                                "attention", "projections (tc_gemm)"};

// next event of the timing pool (QWC_PF_TIMING)
static cudaEvent_t pf_event(qwc_handle* h) {
    if (h->pf_ev_used == h->pf_ev.size()) {
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        h->pf_ev.push_back(e);
    }
    return h->pf_ev[h->pf_ev_used++];
}
// A timed part: two consecutive events of the pool, recorded by the caller.
struct PfPair {
    cudaEvent_t b = nullptr, e = nullptr;
};
static PfPair pf_pair(qwc_handle* h, int cat) {
    PfPair pr;
    if (!h->pf_timing) return pr;
    pr.b = pf_event(h);
    pr.e = pf_event(h);
    h->pf_pair_cat.push_back(cat);
    return pr;
}
static void pf_rec(qwc_handle* h, cudaEvent_t e) {
    if (e) cudaEventRecord(e, h->stream);
}
// events 0 / 1: the pass; then the pairs, summed by category
static void pf_timing_report(qwc_handle* h, int T) {
    if (!h->pf_timing || h->pf_ev_used < 2) return;
    float total = 0.f, t = 0.f, cat[PF_NCAT] = {};
    int calls[PF_NCAT] = {};
    cudaEventElapsedTime(&total, h->pf_ev[0], h->pf_ev[1]);
    for (size_t k = 0; k < h->pf_pair_cat.size(); ++k) {
        if (cudaEventElapsedTime(&t, h->pf_ev[2 + 2 * k], h->pf_ev[3 + 2 * k]) != cudaSuccess) continue;
        cat[h->pf_pair_cat[k]] += t;
        ++calls[h->pf_pair_cat[k]];
    }
    std::fprintf(stderr, "[qwc] prefill T=%d rank %d/%d: %.3f ms device", T, h->tp_rank, h->tp_world, total);
    for (int c = 0; c < PF_NCAT; ++c)
        if (calls[c]) std::fprintf(stderr, "; %s %.3f ms (%d)", kPfCatName[c], cat[c], calls[c]);
    std::fprintf(stderr, "\n");
}

static int pf_gemm(qwc_handle* h, const CUtensorMap& mw, const uint16_t* xs, long ldxs, int M, int N, int K,
                   TcGemmParams p) {
    CUtensorMap mx;
    if (tc_make_map(&mx, xs, N, 2L * K, ldxs)) return fail(h, QWC_E_CUDA, "prefill: activation tensor map failed");
    p.M = M;
    p.N = N;
    p.K = K;
    p.err = h->dev_err;
    const PfPair pr = pf_pair(h, PF_CAT_GEMM);
    pf_rec(h, pr.b);
    CU(launch_tc_gemm(mw, mx, p, h->stream));
    pf_rec(h, pr.e);
    return QWC_OK;
}

// hidden += W x for a row-parallel projection. One rank: the GEMM's residual epilogue.
// Tensor parallel: each rank's partial sum over its input columns, summed over the ranks
// by an NCCL all-reduce, then added to the (replicated) hidden state.
static int pf_residual_gemm(qwc_handle* h, const CUtensorMap& mw, const uint16_t* xs, long ldxs, int Tc, int K) {
    TcGemmParams g;
    g.ldy = h->H;
    if (h->tp_world == 1) {
        g.epi = TC_RESIDUAL;
        g.y = h->pf_hid;
        return pf_gemm(h, mw, xs, ldxs, h->H, Tc, K, g);
    }
    // Rank 0 adds its partial to the residual in place; every other rank overwrites its
    // replica of the residual with its partial. The in-place all-reduce then leaves
    // residual + sum of partials on every rank, with no separate partial buffer or add.
    g.epi = h->tp_rank == 0 ? TC_RESIDUAL : TC_STORE;
    g.y = h->pf_hid;
    int rc = pf_gemm(h, mw, xs, ldxs, h->H, Tc, K, g);
    if (rc) return rc;
    const PfPair ar = pf_pair(h, PF_CAT_ALLREDUCE);
    pf_rec(h, ar.b);
    if (h->p2p) {
        const unsigned long long wait_ns = (unsigned long long)std::min(h->tp_timeout_ms, 60000) * 1000000ull;
        CU(p2p_allreduce(h->p2p, (size_t)Tc * h->H, h->p2p_epoch, wait_ns, h->dev_err, h->stream));
    } else {
        rc = nccl_settle(h, ncclAllReduce(h->pf_hid, h->pf_hid, (size_t)Tc * h->H, ncclFloat32, ncclSum, h->nccl,
                                          h->stream),
                         "ncclAllReduce");
        if (rc) return rc;
    }
    pf_rec(h, ar.e);
    return QWC_OK;
}

// Collective: the peer-memory all-reduce buffers for `floats` residual values per rank.
// Every rank sets up (or declines: QWC_TP_ALLREDUCE=nccl) and the group votes; unless
// every rank succeeded, all of them stay on NCCL's all-reduce for the handle's lifetime.
static int p2p_ensure(qwc_handle* h, size_t floats) {
    if (h->p2p_off || (h->p2p && p2p_capacity_floats(h->p2p) >= floats)) return QWC_OK;
    int rc = stream_wait(h, "peer-memory setup");  // nothing of this rank in flight
    if (rc) return rc;
    p2p_destroy(h->p2p);  // the peers no longer use it: the last pass ended with a group barrier
    h->p2p = nullptr;
    P2pGroup* g = nullptr;
    const char* e = std::getenv("QWC_TP_ALLREDUCE");
    int mine = (e && std::strcmp(e, "nccl") == 0) ? 0 : 1;
    if (mine) {
        std::string why;
        const int tmo = std::min(h->tp_timeout_ms, 60000);
        if (p2p_setup(&g, h->tp_rank, h->tp_world, h->device, h->tp_group, ++h->p2p_gen, floats * sizeof(float), tmo,
                      why) != 0) {
            std::fprintf(stderr, "[qwc] rank %d: peer-memory all-reduce unavailable (%s); using NCCL\n", h->tp_rank,
                         why.c_str());
            mine = 0;
        }
    }
    h->h_pin[5] = mine;
    CU(cudaMemcpyAsync(h->tp_vote, &h->h_pin[5], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    rc = nccl_settle(h, ncclAllReduce(h->tp_vote, h->tp_vote, 1, ncclInt32, ncclMin, h->nccl, h->stream),
                     "peer-memory setup: vote");
    if (rc) {
        p2p_destroy(g);
        return rc;
    }
    CU(cudaMemcpyAsync(&h->h_pin[5], h->tp_vote, sizeof(int), cudaMemcpyDeviceToHost, h->stream));
    if ((rc = stream_wait(h, "peer-memory setup"))) {
        p2p_destroy(g);
        return rc;
    }
    if (h->h_pin[5] == 1) {
        h->p2p = g;
    } else {
        p2p_destroy(g);
        h->p2p_off = true;
    }
    return QWC_OK;
}

// Forward pass of ids[0..T) at positions p0.. on state sv. Logits: every position's
// rows into logits_host[T][V] (all), only the last position's into logits_host[V]
// (!all), or none (logits_host == nullptr).
static int pf_run(qwc_handle* h, const StateView& sv, const int* ids, int T, int p0, float* logits_host, bool all,
                  float* hidden_host = nullptr) {
    if (h->tp_world > 1 && !h->nccl)
        return fail(h, QWC_E_DEVICE, "the tensor-parallel communicator was aborted after a group failure");
    if (h->H % 64 || h->I % 64 || h->VD % 64 || (h->NQ * h->HD) % 64)
        return fail(h, QWC_E_SHAPE, "batched prefill needs hidden, intermediate, GDN value and attention widths that are multiples of 64");
    int rc = pf_build_maps(h);
    if (rc) return rc;
    const int chunk = pf_chunk(h);
    rc = pf_workspace(h, std::min(T, chunk));
    if (rc) return rc;
    if (h->tp_world > 1) {  // the residual stream lives in the peer-mapped buffer when there is one
        if ((rc = p2p_ensure(h, (size_t)std::min(T, chunk) * h->H))) return rc;
        if (h->p2p) h->pf_hid = p2p_local_data(h->p2p);
    }
    const int H = h->H;
    h->pf_ev_used = 0;
    h->pf_pair_cat.clear();
    if (h->pf_timing) {
        pf_event(h);  // [0] start, [1] end of the pass
        pf_event(h);
        CU(cudaEventRecord(h->pf_ev[0], h->stream));
    }
    const size_t kv_layer = (size_t)2 * h->NKV * sv.max_ctx * h->HD * h->kv_bytes;
    // tensor-core attention operands for positions [0, p0 + T): K and V^T pairs per layer
    const bool attn_tc = pf_attn_tc() && h->HD == 256 && h->n_attn > 0;
    const int ctx_pad = (p0 + T + 63) / 64 * 64;
    const size_t kvs_layer = (size_t)2 * h->NKV * ctx_pad * 2 * h->HD;  // elements
    if (attn_tc && h->pf_kvs_bytes < kvs_layer * 2 * h->n_attn) {
        cudaFree(h->pf_kvs);
        h->pf_kvs = nullptr;
        h->pf_kvs_bytes = 0;
        if (cudaMalloc(&h->pf_kvs, kvs_layer * 2 * h->n_attn) != cudaSuccess) {
            h->pf_kvs = nullptr;
            return fail(h, QWC_E_OOM, "prefill attention operand allocation failed");
        }
        h->pf_kvs_bytes = kvs_layer * 2 * h->n_attn;
        // every entry holds a finite value: positions past the prompt meet zero weights
        CU(cudaMemsetAsync(h->pf_kvs, 0, h->pf_kvs_bytes, h->stream));
    }
    // key-split partials: the most splits any chunk of this pass uses (more for later chunks)
    int fa_splits = 1;
    if (attn_tc)
        for (int c0 = 0; c0 < T; c0 += chunk)
            fa_splits = std::max(fa_splits, pf_fattn_splits(std::min(chunk, T - c0), p0 + c0, h->NQ, h->NKV));
    const size_t fa_rows = (size_t)std::min(T, chunk) * h->NQ;
    const size_t fa_bytes = fa_splits > 1 ? (size_t)fa_splits * fa_rows * (h->HD + 2) * 4 : 0;
    if (fa_bytes > h->pf_fa_part_bytes) {
        cudaFree(h->pf_fa_part);
        h->pf_fa_part = nullptr;
        h->pf_fa_part_bytes = 0;
        if (cudaMalloc(&h->pf_fa_part, fa_bytes) != cudaSuccess) {
            h->pf_fa_part = nullptr;
            return fail(h, QWC_E_OOM, "prefill attention split workspace allocation failed");
        }
        h->pf_fa_part_bytes = fa_bytes;
    }
    for (int c0 = 0; c0 < T; c0 += chunk) {
        const int Tc = std::min(chunk, T - c0), pc = p0 + c0;
        CU(cudaMemcpyAsync(h->pf_ids, ids + c0, (size_t)Tc * 4, cudaMemcpyHostToDevice, h->stream));
        CU(pf_embed(h->pf_ids, Tc, h->embed, H, h->V, h->pf_hid, h->dev_err, h->stream));
        // residual stream [L+1][T][H]: after the embedding and after every layer
        auto save_hidden = [&](int slot) -> int {
            if (hidden_host)
                CU(cudaMemcpyAsync(hidden_host + ((size_t)slot * T + c0) * H, h->pf_hid, (size_t)Tc * H * 4,
                                   cudaMemcpyDeviceToHost, h->stream));
            return QWC_OK;
        };
        if ((rc = save_hidden(0))) return rc;
        for (int l = 0; l < h->L; ++l) {
            const Layer& lw = h->layers[l];
            CU(pf_rmsnorm_split(h->pf_hid, H, Tc, lw.in_ln1, H, h->eps, h->pf_xa, h->pf_lda, h->stream));
            TcGemmParams gi;
            gi.epi = TC_STORE;
            gi.y = h->pf_proj;
            gi.ldy = h->pf_ldp;
            if ((rc = pf_gemm(h, h->pf_map_in[l], h->pf_xa, h->pf_lda, lw.in_rows, Tc, H, gi))) return rc;
            if (lw.is_attn) {
                uint8_t* kvl = static_cast<uint8_t*>(sv.kv) + kv_layer * lw.idx;
                PfAttnArgs a;
                a.proj = h->pf_proj;
                a.ldp = h->pf_ldp;
                a.qn1 = lw.qn1;
                a.kn1 = lw.kn1;
                a.rope_cs = h->rope_cs;
                a.qbuf = h->pf_qbuf;
                a.k_cache = kvl;
                a.v_cache = kvl + kv_layer / 2;
                a.kv_bf16 = h->kv_dtype == QWC_DTYPE_BF16;
                a.max_ctx = sv.max_ctx;
                a.p0 = pc;
                a.T = Tc;
                a.NQ = h->NQ;
                a.NKV = h->NKV;
                a.rot = h->ROT;
                a.eps = h->eps;
                a.xs = h->pf_xa;
                a.ldxs = h->pf_lda;
                if (attn_tc) {
                    a.part_o = h->pf_fa_part;
                    a.part_ml = h->pf_fa_part ? h->pf_fa_part + (size_t)fa_splits * fa_rows * h->HD : nullptr;
                    a.part_splits = fa_splits;
                    a.ksplit = h->pf_kvs + kvs_layer * lw.idx;
                    a.vt = a.ksplit + kvs_layer / 2;
                    a.vsplit = h->pf_vsplit;
                    a.ctx_pad = ctx_pad;
                    a.err = h->dev_err;
                }
                const PfPair pa = pf_pair(h, PF_CAT_ATTN);
                pf_rec(h, pa.b);
                CU(pf_attention(a, h->stream));
                pf_rec(h, pa.e);
            } else {
                PfGdnArgs g;
                g.proj = h->pf_proj;
                g.ldp = h->pf_ldp;
                g.b_in = h->pf_proj + h->C + h->VD;
                g.a_in = h->pf_proj + h->C + h->VD + h->VH;
                g.ldab = h->pf_ldp;
                g.conv_w = lw.conv_w;
                g.ring = sv.conv_ring + (size_t)lw.idx * h->C * 4;
                g.neg_exp_A = lw.neg_exp_A;
                g.dt_bias = lw.dt_bias;
                g.qn = h->pf_qn;
                g.kn = h->pf_kn;
                g.vc = h->pf_vc;
                g.glog = h->pf_glog;
                g.U = h->pf_u;
                g.W = h->pf_w;
                g.QG = h->pf_qg;
                g.KD = h->pf_kd;
                g.P = h->pf_p;
                g.gC = h->pf_gc;
                g.ST = h->pf_st;
                g.ET = h->pf_et;
                g.err = h->dev_err;
                g.beta = h->pf_beta;
                g.state = sv.gdn_state + (size_t)lw.idx * h->VH * h->DK * h->DV;
                g.out = h->pf_o;
                g.T = Tc;
                g.p0 = pc;
                g.KH = h->KH;
                g.VH = h->VH;
                g.C = h->C;
                g.VD = h->VD;
                const PfPair pg = pf_pair(h, PF_CAT_GDN), ps = pf_pair(h, PF_CAT_GDN_STATE);
                g.ev_state0 = ps.b;
                g.ev_state1 = ps.e;
                pf_rec(h, pg.b);
                CU(pf_gdn(g, h->stream));
                CU(pf_gated_norm_split(h->pf_o, h->VD, h->pf_proj + h->C, h->pf_ldp, lw.gn_w, Tc, h->VH, h->eps,
                                       h->pf_xa, h->pf_lda, h->stream));
                pf_rec(h, pg.e);
            }
            if ((rc = pf_residual_gemm(h, h->pf_map_out[l], h->pf_xa, h->pf_lda, Tc, lw.out_in))) return rc;
            // FFN: post-attention norm, gate/up + SwiGLU (written as hi/lo for down), down + residual
            CU(pf_rmsnorm_split(h->pf_hid, H, Tc, lw.post_ln1, H, h->eps, h->pf_xa, h->pf_lda, h->stream));
            TcGemmParams gu;
            gu.epi = TC_SWIGLU_SPLIT;
            gu.ys = h->pf_xb;
            gu.ldys = h->pf_ldb;
            gu.split_k = h->I;
            if ((rc = pf_gemm(h, h->pf_map_gu[l], h->pf_xa, h->pf_lda, 2 * h->I, Tc, H, gu))) return rc;
            if ((rc = pf_residual_gemm(h, h->pf_map_down[l], h->pf_xb, h->pf_ldb, Tc, h->I))) return rc;
            if ((rc = save_hidden(l + 1))) return rc;
        }
        // final norm + lm_head for the rows whose logits are wanted
        if (!logits_host) continue;
        const bool last_chunk = c0 + Tc == T;
        if (!all && !last_chunk) continue;
        const int r0 = all ? 0 : Tc - 1, nrows = all ? Tc : 1;
        for (int g0 = 0; g0 < nrows; g0 += kPfLogitRows) {
            const int gn = std::min(kPfLogitRows, nrows - g0);
            CU(pf_rmsnorm_split(h->pf_hid + (size_t)(r0 + g0) * H, H, gn, h->final_ln1, H, h->eps, h->pf_xa,
                                h->pf_lda, h->stream));
            TcGemmParams gl;
            gl.epi = TC_STORE;
            gl.y = h->pf_logits;
            gl.ldy = h->V;
            if ((rc = pf_gemm(h, h->pf_map_head, h->pf_xa, h->pf_lda, h->V, gn, H, gl))) return rc;
            float* dst = logits_host + (all ? (size_t)(c0 + g0) * h->V : 0);
            CU(cudaMemcpyAsync(dst, h->pf_logits, (size_t)gn * h->V * 4, cudaMemcpyDeviceToHost, h->stream));
        }
    }
    if (h->pf_timing) CU(cudaEventRecord(h->pf_ev[1], h->stream));
    if ((rc = stream_wait(h, "prefill"))) return rc;
    pf_timing_report(h, T);
    rc = check_device_error(h);
    if (rc && h->p2p && h->h_pin[8] == DEV_TP_BARRIER_TIMEOUT) {
        // a peer-memory barrier may have run out: the group's epochs no longer agree
        p2p_destroy(h->p2p);
        h->p2p = nullptr;
        h->p2p_off = true;
        return tp_abort(h, h->err + " (tensor-parallel pass)");
    }
    return rc;
}

extern "C" int qwc_prefill(qwc_handle* h, const int* ids, int T, float* logits_out, int last_only) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_prefill: null handle");
    if (T <= 0 || !ids) return fail(h, QWC_E_INVALID, "qwc_prefill: empty prompt");
    if (T > h->max_ctx) return fail(h, QWC_E_CONTEXT, "qwc_prefill: T exceeds max_context");
    for (int i = 0; i < T; ++i)
        if (ids[i] < 0 || ids[i] >= h->V) return fail(h, QWC_E_INVALID, "qwc_prefill: token id out of range");
    int rc = qwc_reset(h);
    if (rc) return rc;
    // the batched pass fills the KV cache, GDN state and conv ring for positions 0..T-1;
    // decoding continues at position T
    CU(cudaMemcpyAsync(h->tokens, ids, (size_t)T * 4, cudaMemcpyHostToDevice, h->stream));
    rc = pf_run(h, h->st, ids, T, 0, logits_out, last_only == 0);
    if (rc) return rc;
    h->h_pin[4] = T;
    CU(cudaMemcpyAsync(h->pos, &h->h_pin[4], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    CU(cudaStreamSynchronize(h->stream));
    h->pos_host = T;
    return QWC_OK;
}

// After a tensor-parallel prefill: every rank sends its shard of the decode state (GDN
// state and conv ring of its heads, the first T positions of its kv heads) to rank 0,
// which places them into a single-GPU handle on the same device; that handle then
// decodes from position T. Collective: every rank of the group calls it, rank 0 with its
// single-GPU handle, the others with null. All ranks walk the pieces in the same order,
// so the NCCL sends and receives pair up.
extern "C" int qwc_tp_set_timeout(qwc_handle* h, int ms) {
    if (!h || h->tp_world < 2 || ms <= 0) return fail(h, QWC_E_INVALID, "qwc_tp_set_timeout: needs a tensor-parallel handle and ms > 0");
    h->tp_timeout_ms = ms;
    return QWC_OK;
}

extern "C" int qwc_tp_allreduce_path(qwc_handle* h) {
    if (!h || h->tp_world < 2) return fail(h, QWC_E_INVALID, "qwc_tp_allreduce_path: needs a tensor-parallel handle");
    if (h->p2p) return 1;
    return h->p2p_off ? 0 : 2;
}

extern "C" int qwc_tp_gather_state(qwc_handle* tp, qwc_handle* full) {
    if (!tp || tp->tp_world < 2 || !tp->nccl)
        return fail(tp, QWC_E_INVALID, "qwc_tp_gather_state: needs a tensor-parallel handle");
    qwc_handle* h = tp;  // errors are reported on the tensor-parallel handle
    const bool root = tp->tp_rank == 0;
    const int T = tp->pos_host, W = tp->tp_world;
    // Each rank checks what it can see, then all ranks vote (minimum of the status codes)
    // before any send or receive is posted, so that either every rank transfers or none
    // does: a rank that returned early would leave its peers' transfers waiting forever.
    int bad = QWC_OK;
    std::string why;
    if (root) {
        if (!full || full->tp_world != 1 || full->device != tp->device) {
            bad = QWC_E_INVALID;
            why = "qwc_tp_gather_state: rank 0 needs a single-GPU handle on its device";
        } else if (full->H != tp->H || full->L != tp->L || full->KH != tp->gKH || full->VH != tp->gVH ||
                   full->NKV != tp->gNKV || full->NQ != tp->gNQ || full->kv_dtype != tp->kv_dtype) {
            bad = QWC_E_SHAPE;
            why = "qwc_tp_gather_state: the handles hold different models";
        } else if (T > full->max_ctx) {
            bad = QWC_E_CONTEXT;
            why = "qwc_tp_gather_state: prefix longer than max_context";
        }
    } else if (full) {
        bad = QWC_E_INVALID;
        why = "qwc_tp_gather_state: only rank 0 passes a destination handle";
    }
    CU(cudaSetDevice(tp->device));
    tp->h_pin[5] = bad;
    CU(cudaMemcpyAsync(tp->tp_vote, &tp->h_pin[5], sizeof(int), cudaMemcpyHostToDevice, tp->stream));
    int vrc = nccl_settle(tp, ncclAllReduce(tp->tp_vote, tp->tp_vote, 1, ncclInt32, ncclMin, tp->nccl, tp->stream),
                          "qwc_tp_gather_state: vote");
    if (vrc) return vrc;
    CU(cudaMemcpyAsync(&tp->h_pin[5], tp->tp_vote, sizeof(int), cudaMemcpyDeviceToHost, tp->stream));
    if ((vrc = stream_wait(tp, "qwc_tp_gather_state"))) return vrc;
    if (bad != QWC_OK) return fail(tp, bad, why);
    if (tp->h_pin[5] != QWC_OK)
        return fail(tp, tp->h_pin[5], "qwc_tp_gather_state: another rank of the group rejected the call");
    std::vector<qwc_tp_shard> sh(W);
    for (int r = 0; r < W; ++r) {
        int rc = qwc_tp_shard_of(&tp->cfg, r, W, &sh[r]);
        if (rc) return rc;
    }
    const int DK = tp->DK, DV = tp->DV, HD = tp->HD, kvb = tp->kv_bytes;
    const size_t hs = (size_t)DK * DV;  // one head of GDN state, floats
    // one piece: bytes at src (on rank `from`) to dst (on rank 0)
    int rc = QWC_OK;
    auto piece = [&](int from, const void* src, void* dst, size_t bytes) {
        if (rc || bytes == 0) return;
        if (from == 0) {
            if (root && cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, tp->stream) != cudaSuccess)
                rc = fail(tp, QWC_E_CUDA, "qwc_tp_gather_state: copy failed");
            return;
        }
        ncclResult_t r = ncclSuccess;
        if (root) r = ncclRecv(dst, bytes, ncclUint8, from, tp->nccl, tp->stream);
        else if (tp->tp_rank == from) r = ncclSend(src, bytes, ncclUint8, 0, tp->nccl, tp->stream);
        if (r != ncclSuccess) rc = fail(tp, QWC_E_CUDA, std::string("qwc_tp_gather_state: ") + ncclGetErrorString(r));
    };
    const qwc_tp_shard& me = sh[tp->tp_rank];
    ncclGroupStart();
    for (int gi = 0; gi < tp->n_gdn; ++gi) {
        for (int r = 0; r < W; ++r) {
            const bool mine = r == tp->tp_rank;
            // GDN state: the rank's v heads, one contiguous block
            const float* s_src = mine ? tp->st.gdn_state + (size_t)gi * me.n_vh * hs : nullptr;
            float* s_dst = root ? full->st.gdn_state + (size_t)gi * full->VH * hs + (size_t)sh[r].vh0 * hs : nullptr;
            piece(r, s_src, s_dst, (size_t)sh[r].n_vh * hs * 4);
            // conv ring [C][4]: q channels, k channels, v channels of the rank's heads
            const size_t KDl = (size_t)sh[r].n_kh * DK, VDl = (size_t)sh[r].n_vh * DV, Cl = 2 * KDl + VDl;
            const float* c_src = mine ? tp->st.conv_ring + (size_t)gi * Cl * 4 : nullptr;
            float* c_dst = root ? full->st.conv_ring + (size_t)gi * full->C * 4 : nullptr;
            const size_t q0 = (size_t)sh[r].kh0 * DK, k0 = (size_t)tp->gKD + q0,
                         v0 = 2 * (size_t)tp->gKD + (size_t)sh[r].vh0 * DV;
            piece(r, mine ? c_src : nullptr, root ? c_dst + q0 * 4 : nullptr, KDl * 16);
            piece(r, mine ? c_src + KDl * 4 : nullptr, root ? c_dst + k0 * 4 : nullptr, KDl * 16);
            piece(r, mine ? c_src + 2 * KDl * 4 : nullptr, root ? c_dst + v0 * 4 : nullptr, VDl * 16);
        }
    }
    const size_t kvl_tp = (size_t)2 * tp->NKV * tp->max_ctx * HD * kvb;
    const size_t kvl_full = root ? (size_t)2 * full->NKV * full->max_ctx * HD * kvb : 0;
    for (int ai = 0; ai < tp->n_attn; ++ai) {
        for (int which = 0; which < 2; ++which) {
            for (int kv = 0; kv < tp->gNKV; ++kv) {
                int from = -1;  // the first rank holding this kv head sends it
                for (int r = 0; r < W && from < 0; ++r)
                    if (kv >= sh[r].kv0 && kv < sh[r].kv0 + sh[r].n_kv) from = r;
                const bool mine = from == tp->tp_rank;
                const uint8_t* src = mine ? static_cast<const uint8_t*>(tp->st.kv) + kvl_tp * ai + which * (kvl_tp / 2) +
                                                (size_t)(kv - me.kv0) * tp->max_ctx * HD * kvb
                                          : nullptr;
                uint8_t* dst = root ? static_cast<uint8_t*>(full->st.kv) + kvl_full * ai + which * (kvl_full / 2) +
                                          (size_t)kv * full->max_ctx * HD * kvb
                                    : nullptr;
                piece(from, src, dst, (size_t)T * HD * kvb);
            }
        }
    }
    const ncclResult_t ge = ncclGroupEnd();
    if (rc) return rc;
    if ((rc = nccl_settle(tp, ge, "qwc_tp_gather_state"))) return rc;
    if ((rc = stream_wait(tp, "qwc_tp_gather_state"))) return rc;
    if (root) {
        full->h_pin[4] = T;
        CU(cudaMemcpyAsync(full->pos, &full->h_pin[4], sizeof(int), cudaMemcpyHostToDevice, full->stream));
        CU(cudaStreamSynchronize(full->stream));
        full->pos_host = T;
    }
    return QWC_OK;
}

// QwenForward::prefill semantics: stateless. A temporary state of T positions is
// allocated for the call; the handle's decode state and position are untouched.
static int forward_stateless(qwc_handle* h, const char* who, const int* ids, int T, float* logits_out, bool all,
                             float* hidden_out) {
    for (int i = 0; i < T; ++i)
        if (ids[i] < 0 || ids[i] >= h->V) return fail(h, QWC_E_INVALID, std::string(who) + ": token id out of range");
    if (T > h->max_ctx) return fail(h, QWC_E_CONTEXT, std::string(who) + ": T exceeds max_context");
    CU(cudaSetDevice(h->device));
    StateView tv;
    tv.max_ctx = T;
    const size_t gb = h->gdn_bytes, cb = h->conv_bytes;
    const size_t kb = (size_t)h->n_attn * 2 * h->NKV * (size_t)T * h->HD * h->kv_bytes;
    if (gb && cudaMalloc(&tv.gdn_state, gb) != cudaSuccess) return fail(h, QWC_E_OOM, "forward state allocation failed");
    if (cb && cudaMalloc(&tv.conv_ring, cb) != cudaSuccess) { cudaFree(tv.gdn_state); return fail(h, QWC_E_OOM, "forward state allocation failed"); }
    if (kb && cudaMalloc(&tv.kv, kb) != cudaSuccess) { cudaFree(tv.gdn_state); cudaFree(tv.conv_ring); return fail(h, QWC_E_OOM, "forward state allocation failed"); }
    int rc = QWC_OK;
    if ((gb && cudaMemsetAsync(tv.gdn_state, 0, gb, h->stream) != cudaSuccess) ||
        (cb && cudaMemsetAsync(tv.conv_ring, 0, cb, h->stream) != cudaSuccess))
        rc = fail(h, QWC_E_CUDA, "forward state clear failed");
    if (rc == QWC_OK) rc = pf_run(h, tv, ids, T, 0, logits_out, all, hidden_out);
    cudaStreamSynchronize(h->stream);
    cudaFree(tv.gdn_state);
    cudaFree(tv.conv_ring);
    cudaFree(tv.kv);
    return rc;
}

extern "C" int qwc_forward_logits(qwc_handle* h, const int* ids, int T, float* logits_out, int last_only) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_forward_logits: null handle");
    if (T <= 0 || !ids || !logits_out) return fail(h, QWC_E_INVALID, "qwc_forward_logits: invalid argument");
    return forward_stateless(h, "qwc_forward_logits", ids, T, logits_out, !last_only, nullptr);
}

extern "C" int qwc_forward_hidden(qwc_handle* h, const int* ids, int T, float* hidden_out) {
    if (!h) return fail(nullptr, QWC_E_INVALID, "qwc_forward_hidden: null handle");
    if (T <= 0 || !ids || !hidden_out) return fail(h, QWC_E_INVALID, "qwc_forward_hidden: invalid argument");
    return forward_stateless(h, "qwc_forward_hidden", ids, T, nullptr, false, hidden_out);
}

// ------------------------------------------------------------------ measurement API
extern "C" void* qwc_stream(const qwc_handle* h) { return h ? (void*)h->stream : nullptr; }

extern "C" int qwc_set_prompt(qwc_handle* h, const int* prompt, int n_prompt) {
    if (!h || n_prompt <= 0 || !prompt || n_prompt > h->max_ctx) return fail(h, QWC_E_INVALID, "qwc_set_prompt: invalid argument");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= h->V) return fail(h, QWC_E_INVALID, "qwc_set_prompt: token id out of range");
    CU(cudaSetDevice(h->device));
    CU(cudaMemcpyAsync(h->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, h->stream));
    CU(cudaStreamSynchronize(h->stream));
    return QWC_OK;
}

extern "C" int qwc_enqueue_greedy(qwc_handle* h, int n_prompt, int n_new) {
    if (!h || n_prompt <= 0 || n_new < 0 || h->tp_world > 1) return fail(h, QWC_E_INVALID, "qwc_enqueue_greedy: invalid argument");
    if ((long)n_prompt + n_new > h->max_ctx) return fail(h, QWC_E_CONTEXT, "qwc_enqueue_greedy: exceeds max_context");
    if (h->gdn_bytes) CU(cudaMemsetAsync(h->st.gdn_state, 0, h->gdn_bytes, h->stream));
    if (h->conv_bytes) CU(cudaMemsetAsync(h->st.conv_ring, 0, h->conv_bytes, h->stream));
    if (h->kvc_bytes) CU(cudaMemsetAsync(h->st.kv, 0, h->kvc_bytes, h->stream));
    CU(cudaMemsetAsync(h->pos, 0, sizeof(int), h->stream));
    h->h_pin[5] = n_prompt;
    CU(cudaMemcpyAsync(h->n_prompt, &h->h_pin[5], sizeof(int), cudaMemcpyHostToDevice, h->stream));
    for (int i = 0; i < n_prompt + n_new; ++i) {
        int rc = run_step(h);
        if (rc) return rc;
    }
    h->pos_host = n_prompt + n_new;
    return QWC_OK;
}

extern "C" int qwc_read_tokens(qwc_handle* h, int start, int n, int* out) {
    if (!h || start < 0 || n < 0 || (n > 0 && !out) || (long)start + n > h->max_ctx + 1)
        return fail(h, QWC_E_INVALID, "qwc_read_tokens: invalid argument");
    if (n > 0) CU(cudaMemcpyAsync(out, h->tokens + start, (size_t)n * 4, cudaMemcpyDeviceToHost, h->stream));
    return check_device_error(h);
}

extern "C" int qwc_profile_step(qwc_handle* h, int cap, int* kind, float* ms, int64_t* bytes) {
    if (!h || cap < 0 || (cap > 0 && (!kind || !ms || !bytes)) || h->tp_world > 1) return fail(h, QWC_E_INVALID, "qwc_profile_step: invalid argument");
    if (h->pos_host >= h->max_ctx) return fail(h, QWC_E_CONTEXT, "qwc_profile_step: context full");
    CU(cudaSetDevice(h->device));
    StepProfile prof;
    prof.cap = cap;
    prof.ev.resize((size_t)cap + 1);
    prof.kind.resize((size_t)cap);
    prof.bytes.resize((size_t)cap);
    for (auto& e : prof.ev) CU(cudaEventCreate(&e));
    h->h_pin[6] = h->max_ctx;
    int rc = QWC_OK;
    if (cudaMemcpyAsync(h->n_prompt, &h->h_pin[6], sizeof(int), cudaMemcpyHostToDevice, h->stream) != cudaSuccess)
        rc = fail(h, QWC_E_CUDA, "qwc_profile_step: copy failed");
    if (rc == QWC_OK && h->step_grid > 0) {
        // the persistent kernel: one launch, the whole step
        int64_t b = 0;
        for (const StepPhase& ph : h->step_host) b += phase_bytes(h, ph, h->pos_host);
        if (cudaEventRecord(prof.ev[0], h->stream) != cudaSuccess ||
            launch_decode_step(h->step, h->NQ / h->NKV, h->step_grid, h->stream) != cudaSuccess ||
            (cap > 0 && cudaEventRecord(prof.ev[1], h->stream) != cudaSuccess))
            rc = fail(h, QWC_E_CUDA, "qwc_profile_step: launch failed");
        if (cap > 0) {
            prof.kind[0] = QWC_K_DECODE_STEP;
            prof.bytes[0] = b;
        }
        prof.n = 1;
    } else if (rc == QWC_OK) {
        rc = enqueue_step(h, h->st, false, &prof, h->pos_host);
    }
    if (rc == QWC_OK) rc = check_device_error(h);
    int n = std::min(prof.n, cap);
    for (int i = 0; i < n && rc == QWC_OK; ++i) {
        float t = 0.f;
        cudaEventElapsedTime(&t, prof.ev[i], prof.ev[i + 1]);
        kind[i] = prof.kind[i];
        ms[i] = t;
        bytes[i] = prof.bytes[i];
    }
    for (auto& e : prof.ev) cudaEventDestroy(e);
    if (rc != QWC_OK) return rc;
    h->pos_host++;
    return prof.n;
}

extern "C" int qwc_trace_step(qwc_handle* h, int cap, int64_t* out) {
    if (!h || cap < 0 || (cap > 0 && !out)) return fail(h, QWC_E_INVALID, "qwc_trace_step: invalid argument");
    if (h->step_grid <= 0) return fail(h, QWC_E_INVALID, "qwc_trace_step: the persistent decode step is not in use");
    if (h->pos_host >= h->max_ctx) return fail(h, QWC_E_CONTEXT, "qwc_trace_step: context full");
    CU(cudaSetDevice(h->device));
    const int np = h->step.nphases, grid = h->step_grid;
    const size_t n = (size_t)grid * np * 8;
    const int need = 2 + np + (int)n;
    if (cap < need) return need;  // ask for a bigger buffer
    long long* d = nullptr;
    CU(cudaMalloc(&d, n * sizeof(long long)));
    CU(cudaMemset(d, 0, n * sizeof(long long)));
    StepParams sp = h->step;
    sp.trace = d;
    h->h_pin[6] = h->max_ctx;
    int rc = QWC_OK;
    if (cudaMemcpyAsync(h->n_prompt, &h->h_pin[6], sizeof(int), cudaMemcpyHostToDevice, h->stream) != cudaSuccess ||
        launch_decode_step(sp, h->NQ / h->NKV, grid, h->stream) != cudaSuccess)
        rc = fail(h, QWC_E_CUDA, "qwc_trace_step: launch failed");
    if (rc == QWC_OK) rc = check_device_error(h);
    if (rc == QWC_OK) {
        out[0] = grid;
        out[1] = np;
        for (int i = 0; i < np; ++i) out[2 + i] = h->step_kinds[i];
        if (cudaMemcpy(out + 2 + np, d, n * sizeof(long long), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = fail(h, QWC_E_CUDA, "qwc_trace_step: copy failed");
    }
    cudaFree(d);
    if (rc != QWC_OK) return rc;
    h->pos_host++;
    return need;
}

extern "C" int qwc_check_step_timeout(qwc_handle* h, int wait_ms) {
    if (!h || wait_ms <= 0 || wait_ms > 2000) return fail(h, QWC_E_INVALID, "qwc_check_step_timeout: invalid argument");
    if (h->step_grid <= 0) return fail(h, QWC_E_INVALID, "qwc_check_step_timeout: the persistent decode step is not in use");
    CU(cudaSetDevice(h->device));
    CU(cudaStreamSynchronize(h->stream));
    StepParams sp = h->step;
    sp.wait_ns = (unsigned long long)wait_ms * 1000000ull;
    sp.stall_cta = 0;  // CTA 0 never arrives at the first grid barrier
    if (launch_decode_step(sp, h->NQ / h->NKV, h->step_grid, h->stream) != cudaSuccess)
        return fail(h, QWC_E_CUDA, "qwc_check_step_timeout: launch failed");
    return check_device_error(h);  // QWC_E_DEVICE: the waits ran out and the step stopped
}

// ------------------------------------------------------------------ kernel-level API
static int* kernel_api_err() {
    int* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_kernel_api_error) != cudaSuccess) return nullptr;
    return p;
}

extern "C" int qwc_gemv_bf16(const uint16_t* W, const float* x, float* y, int out_dim, int in_dim, void* stream) {
    if (!W || !x || !y || out_dim <= 0 || in_dim <= 0 || in_dim % 8)
        return fail(nullptr, QWC_E_INVALID, "qwc_gemv_bf16: invalid argument");
    GemvParams p;
    p.W = W;
    p.rows = out_dim;
    p.in_dim = in_dim;
    p.x_len = in_dim;
    p.x = x;
    p.y = y;
    p.dev_err = kernel_api_err();
    cudaError_t e = launch_gemv(PRO_PLAIN, EPI_STORE, p, gemv_grid(out_dim), (cudaStream_t)stream, false);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_gemv_bf16: ") + cudaGetErrorString(e));
    return QWC_OK;
}

extern "C" int qwc_quantize_q8(const uint16_t* W, int8_t* Wq, float* scales, int out_dim, int in_dim, void* stream) {
    if (!W || !Wq || !scales || out_dim <= 0 || in_dim <= 0 || in_dim % 128)
        return fail(nullptr, QWC_E_INVALID, "qwc_quantize_q8: invalid argument (in_dim must be a multiple of 128)");
    cudaError_t e = launch_quantize_q8(W, Wq, scales, out_dim, in_dim, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_quantize_q8: ") + cudaGetErrorString(e));
    return QWC_OK;
}

extern "C" int qwc_gemv_q8(const int8_t* Wq, const float* scales, const float* x, float* y, int out_dim, int in_dim,
                           void* stream) {
    if (!Wq || !scales || !x || !y || out_dim <= 0 || in_dim <= 0 || in_dim % 512 || in_dim > 8192)
        return fail(nullptr, QWC_E_INVALID, "qwc_gemv_q8: invalid argument (in_dim a multiple of 512, at most 8192)");
    cudaError_t e = launch_gemv_q8(Wq, scales, x, y, out_dim, in_dim, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_gemv_q8: ") + cudaGetErrorString(e));
    return QWC_OK;
}

extern "C" int qwc_gemm_bf16(const uint16_t* W, const uint16_t* Xs, float* Y, int M, int N, int K, int accumulate,
                             void* stream) {
    if (!W || !Xs || !Y || M <= 0 || N <= 0 || K <= 0 || K % 64)
        return fail(nullptr, QWC_E_INVALID, "qwc_gemm_bf16: invalid argument");
    CUtensorMap mw, mx;
    if (tc_make_map(&mw, W, M, K, K) || tc_make_map(&mx, Xs, N, 2L * K, 2L * K))
        return fail(nullptr, QWC_E_INVALID, "qwc_gemm_bf16: tensor map creation failed (alignment)");
    TcGemmParams p;
    p.M = M;
    p.N = N;
    p.K = K;
    p.epi = accumulate ? TC_RESIDUAL : TC_STORE;
    p.y = Y;
    p.ldy = M;
    p.err = kernel_api_err();
    cudaError_t e = launch_tc_gemm(mw, mx, p, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_gemm_bf16: ") + cudaGetErrorString(e));
    return QWC_OK;
}

extern "C" size_t qwc_gdn_prefill_workspace(int KH, int VH, int T) {
    if (KH <= 0 || VH <= 0 || VH % KH || T <= 0) return 0;
    return pf_gdn_workspace_bytes(KH, VH, T);
}

extern "C" int qwc_gdn_prefill(const float* mixed, const float* a, const float* b, const float* conv_w,
                               const float* neg_exp_A, const float* dt_bias, float* conv_ring, float* state, float* out,
                               int KH, int VH, int T, int pos0, void* workspace, size_t workspace_bytes, void* stream) {
    if (!mixed || !a || !b || !conv_w || !neg_exp_A || !dt_bias || !conv_ring || !state || !out || KH <= 0 ||
        VH <= 0 || VH % KH || T <= 0 || pos0 < 0)
        return fail(nullptr, QWC_E_INVALID, "qwc_gdn_prefill: invalid argument");
    PfGdnArgs g;
    g.T = T;
    g.KH = KH;
    g.VH = VH;
    g.VD = VH * 128;
    g.C = 2 * KH * 128 + VH * 128;
    if (pf_gdn_carve(g, workspace, workspace_bytes))
        return fail(nullptr, QWC_E_INVALID, "qwc_gdn_prefill: workspace missing or smaller than qwc_gdn_prefill_workspace()");
    g.proj = mixed;
    g.ldp = g.C;
    g.a_in = a;
    g.b_in = b;
    g.ldab = VH;
    g.conv_w = conv_w;
    g.ring = conv_ring;
    g.neg_exp_A = neg_exp_A;
    g.dt_bias = dt_bias;
    g.state = state;
    g.out = out;
    g.p0 = pos0;
    cudaError_t e = pf_gdn(g, (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_gdn_prefill: ") + cudaGetErrorString(e));
    return QWC_OK;
}

extern "C" int qwc_gdn_decode_step(const float* mixed, const float* a, const float* b, const float* conv_w,
                                   const float* neg_exp_A, const float* dt_bias, float* conv_ring, float* state,
                                   float* out, int KH, int VH, int pos, void* stream) {
    if (!mixed || !a || !b || !conv_w || !neg_exp_A || !dt_bias || !conv_ring || !state || !out || KH <= 0 ||
        VH <= 0 || VH % KH || pos < 0)
        return fail(nullptr, QWC_E_INVALID, "qwc_gdn_decode_step: invalid argument");
    GdnDecodeParams p;
    p.mixed = mixed;
    p.a = a;
    p.b = b;
    p.conv_w = conv_w;
    p.neg_exp_A = neg_exp_A;
    p.dt_bias = dt_bias;
    p.conv_ring = conv_ring;
    p.state = state;
    p.out = out;
    p.pos_val = pos;
    p.KH = KH;
    p.VH = VH;
    cudaError_t e = launch_gdn_decode(p, (cudaStream_t)stream, false);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_gdn_decode_step: ") + cudaGetErrorString(e));
    return QWC_OK;
}

namespace {
struct AttnOpScratch {
    int device = -1;
    float* part_o = nullptr;
    float* part_ml = nullptr;
    unsigned* counters = nullptr;
    size_t cap_o = 0;
};
thread_local AttnOpScratch g_attn_op;
}  // namespace

extern "C" int qwc_attention_decode(const float* q, const float* gate, const void* k_cache, const void* v_cache,
                                    int kv_dtype, int NQ, int NKV, int max_ctx, int n_ctx, float* out, void* stream) {
    if (!q || !gate || !k_cache || !v_cache || !out || NKV <= 0 || NQ % NKV || n_ctx <= 0 || n_ctx > max_ctx ||
        (kv_dtype != QWC_DTYPE_F32 && kv_dtype != QWC_DTYPE_BF16))
        return fail(nullptr, QWC_E_INVALID, "qwc_attention_decode: invalid argument");
    AttnDecodeParams p;
    p.q_in = q;
    p.gate_in = gate;
    p.k_cache = const_cast<void*>(k_cache);
    p.v_cache = const_cast<void*>(v_cache);
    p.kv_bf16 = kv_dtype == QWC_DTYPE_BF16;
    p.max_ctx = max_ctx;
    p.n_ctx_val = n_ctx;
    p.NQ = NQ;
    p.NKV = NKV;
    // long caches: the block-per-warp kernel (lane = position for the scores) and a separate
    // combine; short ones: the per-position kernel shared with the decode step
    const bool long_ctx = n_ctx >= kAttnLongMin;
    p.nsplit = long_ctx ? attn_long_nsplit(n_ctx, NKV, NQ / NKV, kv_dtype == QWC_DTYPE_BF16) : attn_nsplit_for(n_ctx, NKV);
    p.out = out;
    const int grp = NQ / NKV;
    const size_t need_o = (size_t)NKV * p.nsplit * grp * 256;
    int dev = 0;
    cudaGetDevice(&dev);
    AttnOpScratch& s = g_attn_op;
    if (s.device != dev || s.cap_o < need_o) {
        // per-thread split-K workspace, grown on demand and kept for later calls
        if (s.part_o) { cudaFree(s.part_o); cudaFree(s.part_ml); cudaFree(s.counters); }
        s = AttnOpScratch();
        if (cudaMalloc(&s.part_o, need_o * 4) != cudaSuccess || cudaMalloc(&s.part_ml, need_o / 256 * 2 * 4) != cudaSuccess ||
            cudaMalloc(&s.counters, 64 * 4) != cudaSuccess)
            return fail(nullptr, QWC_E_OOM, "qwc_attention_decode: workspace allocation failed");
        cudaMemset(s.counters, 0, 64 * 4);
        s.device = dev;
        s.cap_o = need_o;
    }
    if (NKV > 64) return fail(nullptr, QWC_E_INVALID, "qwc_attention_decode: too many kv heads");
    p.part_o = s.part_o;
    p.part_ml = s.part_ml;
    p.counters = s.counters;
    cudaError_t e = long_ctx ? launch_attn_long(p, (cudaStream_t)stream) : launch_attn_decode(p, (cudaStream_t)stream, false);
    if (e != cudaSuccess) return fail(nullptr, QWC_E_CUDA, std::string("qwc_attention_decode: ") + cudaGetErrorString(e));
    return QWC_OK;
}
