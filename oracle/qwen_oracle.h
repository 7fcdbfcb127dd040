/* CPU restatement of the reference's fp32 Qwen3.5 forward pass -- TEST INFRASTRUCTURE.
 *
 * This is the checker that the CUDA path is compared against.  It is only ever
 * loaded by tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg.
 * It is never part of the product path.  Parity is pinned: tests/test_oracle_golden.py
 * checks it against golden vectors produced by the reference engine itself
 * (tests/golden/make_golden.py drives oracle/_ref/libqwen_ref.so, which is the
 * reference's own sources compiled here).
 *
 * Weights are registered by name (the Hugging Face names of the checkpoint) with
 * their on-disk dtype; small tensors are widened to fp32 once, matrices are read
 * in place as bf16 and widened per element inside the dot product, exactly as
 * SafeTensors::get_f32 / matmul(WeightView) do (src/safetensors_loader.cpp:252-278,
 * src/forward_pass.cpp:65-75).
 */
#ifndef QWEN_ORACLE_H
#define QWEN_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int hidden, layers, interval, ffn, vocab;
    int q_heads, kv_heads, head_dim, rot_dim;
    int k_heads, v_heads, k_dim, v_dim, conv_k;
    float eps;
    double theta;
} orc_config;

typedef struct orc_model orc_model;

orc_model* orc_create(const orc_config* cfg, int max_context);
void orc_destroy(orc_model* m);
/* dtype: 0 = F32, 1 = BF16. The data must outlive the model. */
int orc_set_tensor(orc_model* m, const char* name, int dtype, const void* data, int64_t numel);
/* Resolves every tensor; returns 0 on success, -1 (and the missing name) otherwise. */
int orc_finalize(orc_model* m, char* missing, int missing_len);

void orc_reset(orc_model* m);
int orc_position(const orc_model* m);
/* One incremental decode step (QwenModel::step). logits: [vocab] or NULL.
 * layer_hidden: [(layers+1) * hidden] residual stream after the embedding and after
 * each layer, or NULL. Returns 0, or -1 for a bad id / full context. */
int orc_step(orc_model* m, int token, float* logits, float* layer_hidden);
/* QwenModel::generate_greedy: reset, step the prompt, then n_new argmax steps. */
int orc_generate_greedy(orc_model* m, const int* prompt, int n_prompt, int n_new, int* out);
/* QwenForward::prefill (stateless): logits [T * vocab] (or NULL), layer_hidden
 * [(layers+1) * T * hidden] (or NULL), last_only: write only the last row of logits. */
int orc_prefill(orc_model* m, const int* ids, int T, float* logits, float* layer_hidden,
                int last_only);

/* ---- the free kernels of include/forward_pass.h ---- */
void orc_matmul_bf16(const uint16_t* W, const float* x, float* y, int out_dim, int in_dim);
void orc_rmsnorm(const float* x, const float* w, float* y, int n, float eps);
void orc_rmsnorm_gated(const float* x, const float* w, const float* g, float* y, int n, float eps);
void orc_l2norm(float* x, int n, float eps);
void orc_apply_rope(float* v, int rot, int pos, double theta);

/* ---- operator-level oracles for the two op benchmarks ----
 * GDN mixer core over a sequence (the part of gdn_step between the projections and
 * the gated norm, src/qwen_model.cpp:173-207): mixed [T][C] raw conv inputs, conv_w
 * [C][K], a/b raw gate inputs [T][VH], A_log/dt_bias [VH]; state [VH][DK][DV] in/out
 * (S layout of the reference), conv_state [C][K-1] in/out; out [T][VH][DV] (pre-norm). */
void orc_gdn_core(int T, int KH, int VH, int DK, int DV, int K,
                  const float* mixed, const float* conv_w, const float* a, const float* b,
                  const float* A_log, const float* dt_bias, float* state, float* conv_state,
                  float* out);
/* Attention for one query over positions 0..n_ctx-1 (src/qwen_model.cpp:134-150 after
 * the K/V append): q [NQ][HD] (already normed+roped), gate [NQ][HD], K/V cache
 * [n_ctx][NKV][HD]; out [NQ][HD] = softmax(qK^T/sqrt(HD)) V * sigmoid(gate). */
void orc_attention(int NQ, int NKV, int HD, int n_ctx, const float* q, const float* gate,
                   const float* kc, const float* vc, float* out);

#ifdef __cplusplus
}
#endif
#endif
