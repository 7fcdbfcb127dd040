// Test/benchmark harness around the UNMODIFIED reference engine.
//
// TEST INFRASTRUCTURE ONLY: this file is linked with the reference's own sources
// (src/{memory_budget,inference_arenas,gguf_loader,config_loader,safetensors_loader,
// forward_pass,qwen_forward,qwen_model,tokenizer}.cpp, compiled where they lie) into
// oracle/_ref/libqwen_ref.so.  It replaces the reference's main.cpp, which needs a
// tokenizer vocabulary, with a C interface that feeds token ids directly, so that the
// tests (as the checker) and bench.py's reference arm can drive the reference's
// QwenModel::step / generate_greedy (src/qwen_model.cpp:211-255) and
// QwenForward::prefill (src/qwen_forward.cpp:154-206) from Python via ctypes.
#include <chrono>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "forward_pass.h"
#include "memory_budget.h"
#include "model_config.h"
#include "qwen_forward.h"
#include "qwen_model.h"
#include "safetensors_loader.h"

namespace {
struct RefHandle {
    ModelConfig cfg;
    SafeTensors st;
    std::unique_ptr<QwenModel> model;
    std::unique_ptr<QwenForward> fwd;
    int max_ctx = 0;
};
}  // namespace

extern "C" {

// Loads config.json + *.safetensors from model_dir (as main.cpp:21-27 does) and builds
// a QwenModel with the given max_context. Returns nullptr on failure.
void* ref_open(const char* model_dir, int max_context) {
    auto* h = new RefHandle();
    std::string dir(model_dir);
    load_model_config(dir + "/config.json", h->cfg);
    if (!h->st.load_model(dir)) { delete h; return nullptr; }
    h->max_ctx = max_context;
    h->model.reset(new QwenModel(h->st, h->cfg, max_context));
    if (!h->model->ok()) { delete h; return nullptr; }
    h->fwd.reset(new QwenForward(h->st, h->cfg));
    return h;
}

void ref_close(void* hp) { delete static_cast<RefHandle*>(hp); }

int ref_vocab(void* hp) { return static_cast<RefHandle*>(hp)->cfg.vocab_size; }
int ref_hidden(void* hp) { return static_cast<RefHandle*>(hp)->cfg.hidden_size; }
int ref_layers(void* hp) { return static_cast<RefHandle*>(hp)->cfg.n_layers_total; }

void ref_reset(void* hp) { static_cast<RefHandle*>(hp)->model->reset(); }
int ref_position(void* hp) { return static_cast<RefHandle*>(hp)->model->position(); }

// One QwenModel::step; copies the [vocab] logits out when logits != nullptr.
int ref_step(void* hp, int token, float* logits) {
    auto* h = static_cast<RefHandle*>(hp);
    const std::vector<float>& lg = h->model->step(token);
    if (logits) std::memcpy(logits, lg.data(), lg.size() * sizeof(float));
    return 0;
}

// QwenModel::generate_greedy; writes n_new ids to out. Returns the count produced.
int ref_generate_greedy(void* hp, const int* prompt, int n_prompt, int n_new, int* out) {
    auto* h = static_cast<RefHandle*>(hp);
    std::vector<int> p(prompt, prompt + n_prompt);
    std::vector<int> g = h->model->generate_greedy(p, n_new);
    for (size_t i = 0; i < g.size(); ++i) out[i] = g[i];
    return (int)g.size();
}

// QwenForward::prefill; logits is [T * vocab]. Returns 1 on success.
int ref_prefill(void* hp, const int* ids, int T, float* logits) {
    auto* h = static_cast<RefHandle*>(hp);
    std::vector<int> v(ids, ids + T);
    std::vector<float> out;
    if (!h->fwd->prefill(v, out)) return 0;
    std::memcpy(logits, out.data(), out.size() * sizeof(float));
    return 1;
}

// MemoryBudget as QwenModel reports it (qwen_model.cpp:83-87): 6 size_t values.
void ref_budget(void* hp, uint64_t* out6) {
    const MemoryBudget& b = static_cast<RefHandle*>(hp)->model->budget();
    out6[0] = b.weight_bytes; out6[1] = b.gdn_state_bytes; out6[2] = b.gdn_conv_bytes;
    out6[3] = b.kv_cache_bytes; out6[4] = b.activation_bytes; out6[5] = b.vision_scratch_bytes;
}

// compute_budget / solve_max_context straight from a config file.
int ref_compute_budget(const char* config_path, int bpw, int max_ctx, int kvb, uint64_t* out6) {
    ModelConfig cfg;
    if (!load_model_config(config_path, cfg)) return 0;
    MemoryBudget b = compute_budget(cfg, bpw, max_ctx, kvb);
    out6[0] = b.weight_bytes; out6[1] = b.gdn_state_bytes; out6[2] = b.gdn_conv_bytes;
    out6[3] = b.kv_cache_bytes; out6[4] = b.activation_bytes; out6[5] = b.vision_scratch_bytes;
    return 1;
}

int64_t ref_solve_max_context(const char* config_path, uint64_t ram, uint64_t wb, uint64_t gb,
                              uint64_t ab, uint64_t vb, uint64_t margin, int kvb) {
    ModelConfig cfg;
    if (!load_model_config(config_path, cfg)) return -2;
    return solve_max_context(cfg, ram, wb, gb, ab, vb, margin, kvb);
}

// ModelConfig fields after load_model_config, in a fixed order (ints then floats).
int ref_load_config(const char* config_path, int* ints16, double* dbl4) {
    ModelConfig c;
    int ok = load_model_config(config_path, c) ? 1 : 0;
    int v[16] = {c.hidden_size, c.n_layers_total, c.n_layers_gdn, c.n_layers_attn,
                 c.gdn_k_heads, c.gdn_v_heads, c.gdn_k_head_dim, c.gdn_v_head_dim,
                 c.gdn_conv_kernel, c.attn_q_heads, c.attn_kv_heads, c.attn_head_dim,
                 c.ffn_intermediate, c.vocab_size, c.attn_interval, c.tie_word_embeddings ? 1 : 0};
    std::memcpy(ints16, v, sizeof(v));
    dbl4[0] = c.rms_norm_eps; dbl4[1] = c.rope_theta; dbl4[2] = c.partial_rotary_factor;
    dbl4[3] = (double)c.native_max_context;
    return ok;
}

// ---- the reference's free kernels (include/forward_pass.h), for unit checks ----
void ref_matmul_bf16(const uint16_t* W, const float* x, float* y, int out_dim, int in_dim) {
    WeightView v; v.bf16 = W; v.numel = (int64_t)out_dim * in_dim;
    matmul(v, x, y, out_dim, in_dim);
}
void ref_rmsnorm(const float* x, const float* w, float* y, int n, float eps) { rmsnorm(x, w, y, n, eps); }
void ref_rmsnorm_gated(const float* x, const float* w, const float* g, float* y, int n, float eps) {
    rmsnorm_gated(x, w, g, y, n, eps);
}
void ref_l2norm(float* x, int n, float eps) { l2norm(x, n, eps); }
void ref_apply_rope(float* v, int rot, int pos, double theta) { apply_rope(v, rot, pos, theta); }

// Wall-clock seconds for n_new greedy steps after the prompt (generate_greedy).
double ref_time_generate(void* hp, const int* prompt, int n_prompt, int n_new, int* out) {
    auto t0 = std::chrono::steady_clock::now();
    ref_generate_greedy(hp, prompt, n_prompt, n_new, out);
    auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

}  // extern "C"
