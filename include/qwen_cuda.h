/* libqwen_cuda -- C ABI of the B200 Qwen3.5 hybrid (Gated DeltaNet + gated attention)
 * forward pass.
 *
 * This is the drop-in boundary under the reference engine's C++ API. Each entry point
 * names the reference interface it replaces (paths inside the reference project).
 * The C++ classes of host/ (QwenModel, QwenForward) are thin wrappers over these
 * calls, and any FFI (ctypes, cgo, JNI) can bind them directly.
 *
 * Rules:
 *  - Every call returns an int status: QWC_OK (0) or a negative QWC_E* code. The
 *    message of the last failure on a handle is in qwc_last_error(handle); failures
 *    before a handle exists are in qwc_last_error(NULL).
 *  - One CUDA stream per handle. A handle is not thread-safe; use one host thread per
 *    handle (the reference objects are single-threaded as well).
 *  - Host buffers passed in are owned by the caller and only read/written during the
 *    call. Device buffers are owned by the handle and allocated once in qwc_create
 *    (weights, GDN recurrent and conv state, KV cache, scratch). qwc_step and
 *    qwc_generate_greedy allocate nothing.
 *  - No C++ or CUDA types cross this boundary; "stream" arguments of the kernel-level
 *    entry points are cudaStream_t passed as void* (NULL = default stream).
 */
#ifndef QWEN_CUDA_H
#define QWEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QWC_OK 0
#define QWC_E_INVALID (-1)     /* bad argument (null pointer, size, token id, ...) */
#define QWC_E_CUDA (-2)        /* a CUDA runtime call failed */
#define QWC_E_MISSING (-3)     /* a required tensor is absent from the checkpoint */
#define QWC_E_SHAPE (-4)       /* a tensor or config value has an unsupported shape */
#define QWC_E_CONTEXT (-5)     /* position would exceed max_context */
#define QWC_E_IO (-6)          /* a file could not be read or parsed */
#define QWC_E_DEVICE (-7)      /* a kernel reported an error (bounded wait expired) */
#define QWC_E_OOM (-8)         /* device allocation failed */

#define QWC_DTYPE_F32 0
#define QWC_DTYPE_BF16 1

/* ModelConfig (include/model_config.h:11-63), flattened to plain C. */
typedef struct {
    int hidden_size;           /* hidden_size */
    int n_layers_total;        /* num_hidden_layers */
    int n_layers_gdn;          /* derived: total - total / interval */
    int n_layers_attn;         /* derived: total / interval */
    int gdn_k_heads;           /* linear_num_key_heads */
    int gdn_v_heads;           /* linear_num_value_heads */
    int gdn_k_head_dim;        /* linear_key_head_dim */
    int gdn_v_head_dim;        /* linear_value_head_dim */
    int gdn_conv_kernel;       /* linear_conv_kernel_dim */
    int attn_q_heads;          /* num_attention_heads */
    int attn_kv_heads;         /* num_key_value_heads */
    int attn_head_dim;         /* head_dim */
    int ffn_intermediate;      /* intermediate_size */
    int vocab_size;            /* vocab_size */
    int native_max_context;    /* max_position_embeddings */
    int attn_interval;         /* full_attention_interval; layer L is attention iff (L+1)%interval==0 */
    int tie_word_embeddings;   /* tie_word_embeddings */
    float rms_norm_eps;        /* rms_norm_eps */
    float partial_rotary_factor; /* partial_rotary_factor */
    double rope_theta;         /* rope_theta */
    int64_t n_params;          /* derived, as load_model_config computes it */
} qwc_config;

/* One checkpoint tensor as it sits in host memory (a safetensors entry,
 * include/safetensors_loader.h:26-33). Matrices must be BF16; vectors may be F32 or BF16. */
typedef struct {
    const char* name;          /* Hugging Face name, e.g. model.language_model.norm.weight */
    int dtype;                 /* QWC_DTYPE_F32 or QWC_DTYPE_BF16 */
    int ndim;
    int64_t shape[4];
    const void* data;          /* host pointer, read during qwc_create only */
} qwc_tensor;

/* MemoryBudget (include/memory_budget.h:6-18): bytes per arena. */
typedef struct {
    uint64_t weight_bytes;
    uint64_t gdn_state_bytes;
    uint64_t gdn_conv_bytes;
    uint64_t kv_cache_bytes;
    uint64_t activation_bytes;
    uint64_t vision_scratch_bytes;
} qwc_budget;

typedef struct qwc_handle qwc_handle;

/* Head-wise tensor-parallel shard of one rank (no reference counterpart: the reference is
 * single-process). GDN k heads [kh0, kh0+n_kh) and v heads [vh0, vh0+n_vh) with their q/k/v
 * channels, z rows, b/a rows, conv channels, A_log/dt_bias and out_proj input columns;
 * attention q heads [q0, q0+n_q) with the kv heads [kv0, kv0+n_kv) they read (replicated
 * when world > attn_kv_heads) and the o_proj input columns; FFN intermediate rows
 * [i0, i0+n_i) of gate/up and the down_proj input columns. Embedding, norms and lm_head
 * are replicated. */
typedef struct {
    int kh0, n_kh, vh0, n_vh, q0, n_q, kv0, n_kv, i0, n_i;
} qwc_tp_shard;

/* ---------------------------------------------------------------- config / budget */

/* load_model_config (src/config_loader.cpp:59-108): fills *cfg from config.json
 * (text_config preferred); keys that are absent keep the Qwen3.5-0.8B defaults. Returns
 * QWC_E_IO (with defaults in *cfg) when the file cannot be read. */
int qwc_load_config(const char* config_json_path, qwc_config* cfg);

/* The ModelConfig defaults (include/model_config.h:11-63). */
void qwc_default_config(qwc_config* cfg);

/* compute_budget (src/memory_budget.cpp:30-54). */
int qwc_compute_budget(const qwc_config* cfg, int bytes_per_weight, int max_context,
                       int kv_bytes_per_elem, int max_vision_tiles, int vit_dim,
                       qwc_budget* out);

/* solve_max_context (src/memory_budget.cpp:56-81): -1 when the fixed costs do not fit. */
int64_t qwc_solve_max_context(const qwc_config* cfg, uint64_t ram_budget_bytes,
                              uint64_t weight_bytes, uint64_t gdn_state_bytes,
                              uint64_t activation_bytes, uint64_t vision_scratch_bytes,
                              uint64_t safety_margin_bytes, int kv_bytes_per_elem);

/* ---------------------------------------------------------------- model lifetime */

/* QwenModel::QwenModel (src/qwen_model.cpp:12-96): resolves every weight by name,
 * uploads them to `device` in the decode layout, and allocates all device arenas once
 * (sized by the memory equation). kv_dtype: QWC_DTYPE_F32 (the reference's cache
 * type) or QWC_DTYPE_BF16. Missing tensors -> QWC_E_MISSING with the name in the
 * error message. Weights are copied through pinned staging buffers (the caller's host
 * buffers, e.g. a file mapping, are read once; no full host copy is made).
 * max_context <= 0 plans the context from the device's free memory: solve_max_context
 * (src/memory_budget.cpp:56-81) over the free bytes with the weights and state as fixed
 * costs (qwc_max_context reports the chosen size); QWC_E_OOM when the model itself
 * does not fit. */
int qwc_create(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors,
               int max_context, int kv_dtype, int device, qwc_handle** out);

/* Convenience: load_model_config + SafeTensors::load_model (main.cpp:21-27) + qwc_create. */
int qwc_create_from_dir(const char* model_dir, int max_context, int kv_dtype, int device,
                        qwc_handle** out);

void qwc_destroy(qwc_handle* h);

/* Message of the last failure on h (or of the last handle-less failure if h is NULL). */
const char* qwc_last_error(const qwc_handle* h);

/* QwenModel::budget (include/qwen_model.h:31): the arenas as planned + allocated. */
int qwc_get_budget(const qwc_handle* h, qwc_budget* out);
int qwc_get_config(const qwc_handle* h, qwc_config* out);

/* ---------------------------------------------------------------- decode */

/* QwenModel::reset (src/qwen_model.cpp:98-104): zero KV, GDN and conv state; pos = 0. */
int qwc_reset(qwc_handle* h);

/* QwenModel::position (include/qwen_model.h:27). */
int qwc_position(const qwc_handle* h);

/* Test of the decode step's bounded waits (no reference counterpart): runs one step in
 * which one CTA never arrives at the first grid barrier, with every wait of the step
 * limited to wait_ms (1..2000). The other CTAs' waits run out, the kernel posts an error
 * code and returns, and the call returns QWC_E_DEVICE -- the path a real stall would
 * take, exercised without a fault. Nothing hangs; the decode state is then undefined:
 * call qwc_reset before the next step. */
int qwc_check_step_timeout(qwc_handle* h, int wait_ms);

/* The handle's context capacity (positions): the max_context it was created with, or the
 * planned one. Not in the reference (its callers pass the value they chose). */
int qwc_max_context(const qwc_handle* h);

/* QwenModel::step (src/qwen_model.cpp:211-239): one token through all layers (one CUDA
 * graph replay). logits_host: [vocab] floats or NULL; argmax_out: the greedy id
 * (lowest index among equal maxima) or NULL. */
int qwc_step(qwc_handle* h, int token, float* logits_host, int* argmax_out);

/* QwenModel::generate_greedy (src/qwen_model.cpp:241-255): reset, feed the prompt one
 * token at a time, then n_new greedy tokens; the argmax -> next-token feedback stays on
 * the device. out_tokens: n_new ids. */
int qwc_generate_greedy(qwc_handle* h, const int* prompt, int n_prompt, int n_new,
                        int* out_tokens);

/* ---------------------------------------------------------------- prefill */

/* QwenForward::prefill (src/qwen_forward.cpp:154-206): stateless forward pass over
 * ids[T]; writes T*vocab logits (or only the last row if last_only). The decode state of
 * h is not touched. */
int qwc_forward_logits(qwc_handle* h, const int* ids, int T, float* logits_out, int last_only);

/* The same stateless pass, returning the residual stream instead of logits (no reference
 * counterpart; a parity hook for the per-layer hidden states that QwenForward::prefill
 * keeps internally, src/qwen_forward.cpp:154-206): hidden_out [n_layers + 1][T][hidden],
 * slot 0 the embedding rows, slot l + 1 the stream after layer l (before the final norm). */
int qwc_forward_hidden(qwc_handle* h, const int* ids, int T, float* hidden_out);

/* Prefill that also seeds the decode state (the reference equivalent is stepping the
 * prompt through QwenModel::step, src/qwen_model.cpp:245): resets h, runs ids[T] and
 * leaves position() == T with KV / GDN / conv state filled. logits_out: the last
 * position's [vocab] logits when last_only != 0, else every position's [T][vocab]
 * (the lm_head then runs over all T rows), or NULL. */
int qwc_prefill(qwc_handle* h, const int* ids, int T, float* logits_out, int last_only);

/* ---------------------------------------------------------------- measurement */
/* No reference counterpart: hooks for timing the decode path without host round trips. */

/* The handle's CUDA stream (cudaStream_t as void*): record events on it to time work. */
void* qwc_stream(const qwc_handle* h);

/* Upload prompt ids to the device token buffer (synchronises). */
int qwc_set_prompt(qwc_handle* h, const int* prompt, int n_prompt);

/* Enqueue, without any host synchronisation, the device work of a greedy generation
 * whose n_prompt ids are already on the device (qwc_set_prompt): reset the state, then
 * n_prompt + n_new decode steps. Read the ids back with qwc_read_tokens. */
int qwc_enqueue_greedy(qwc_handle* h, int n_prompt, int n_new);

/* Copy device token ids [start, start+n) to host memory (synchronises; checks the
 * device error word). Position `start + i` holds the id fed at that position. */
int qwc_read_tokens(qwc_handle* h, int start, int n, int* out);

/* Runs ONE decode step eagerly (no graph, no programmatic launch) at the current
 * position with the token id already at that position, on the path qwc_step uses,
 * timing every kernel with CUDA events. For each launch i < cap: kind[i] (QWC_K_*),
 * ms[i], bytes[i] (algorithmic HBM bytes of that launch). With the persistent decode
 * kernel in use that is a single launch of kind QWC_K_DECODE_STEP; with
 * QWC_DECODE=kernels it is one launch per GEMV / mixer kernel. Returns the number of
 * launches (>= 0) or an error code. */
#define QWC_K_MIX_IN 0      /* norm + mixer input projection GEMV */
#define QWC_K_GDN 1         /* GDN conv + delta-rule recurrence */
#define QWC_K_ATTN 2        /* attention (norm/rope/append + split-K) */
#define QWC_K_MIX_OUT 3     /* mixer output projection GEMV + residual */
#define QWC_K_GATE_UP 4     /* norm + gate/up GEMV + SwiGLU */
#define QWC_K_DOWN 5        /* down GEMV + residual */
#define QWC_K_LM_HEAD 6     /* final norm + lm_head GEMV + argmax */
#define QWC_K_DECODE_STEP 7 /* the persistent kernel: the whole step in one launch */
int qwc_profile_step(qwc_handle* h, int cap, int* kind, float* ms, int64_t* bytes);

/* Runs ONE step of the persistent decode kernel (the one the CUDA graph replays) eagerly
 * at the current position, recording device timestamps (ns) per CTA and phase. out
 * receives: [0] grid size G, [1] phase count P, [2..2+P) the QWC_K_* kind of each phase,
 * then G*P*8 values, CTA-major, phase-minor: stamps of phase start, barrier passed,
 * GEMV prologue done, phase end (every warp of the CTA done, just before it arrives at
 * the next grid barrier); then for GEMV phases the ns warp 0 spent waiting on weight
 * slots and the slot count, for attention phases stamps after its prologue, main loop,
 * warp merge and split combine.
 * Returns the number of int64 values needed (when cap is too small nothing runs), or an
 * error code (QWC_E_INVALID when the persistent kernel is not in use). Allocates a
 * temporary device buffer. */
int qwc_trace_step(qwc_handle* h, int cap, int64_t* out);

/* ---------------------------------------------------------------- tensor parallel */

/* The shard of `rank` among `world` ranks; QWC_E_SHAPE when the model does not divide
 * (GDN heads, q heads and the FFN width must divide by world, the per-rank FFN width by 64,
 * and world must divide the kv heads or be a multiple of them). */
int qwc_tp_shard_of(const qwc_config* cfg, int rank, int world, qwc_tp_shard* out);

/* NCCL unique id (128 bytes) that rank 0 creates and sends to the other ranks (the caller's
 * own transport, e.g. torch.distributed), before every rank calls qwc_create_tp. */
int qwc_tp_unique_id(void* out, int bytes);

/* As qwc_create, for rank `rank` of a `world`-rank tensor-parallel group on one node: the
 * handle holds only its shard (qwc_tp_shard_of) and an NCCL communicator over the ranks
 * (every rank calls this concurrently). Such a handle serves the batched forward pass
 * (qwc_forward_logits, qwc_prefill) with an all-reduce of the [T][hidden] partial sums
 * after each mixer output projection and each down_proj; decode (qwc_step and the
 * generation calls) needs a single-GPU handle and returns QWC_E_INVALID. */
int qwc_create_tp(const qwc_config* cfg, const qwc_tensor* tensors, int n_tensors, int max_context,
                  int kv_dtype, int device, int rank, int world, const void* unique_id,
                  qwc_handle** out);
int qwc_create_from_dir_tp(const char* model_dir, int max_context, int kv_dtype, int device, int rank,
                           int world, const void* unique_id, qwc_handle** out);

/* Bound, in milliseconds, on every wait of a tensor-parallel handle for its group (default
 * 300000, or QWC_TP_TIMEOUT_MS at creation). The communicator is non-blocking; when a wait
 * runs out -- a rank died or never joined the collective -- the handle aborts it, so that
 * its kernels stop waiting, and the call returns QWC_E_DEVICE; the handle then refuses
 * further batched passes (destroy it and build the group again). No reference
 * counterpart (the reference runs on one CPU). */
int qwc_tp_set_timeout(qwc_handle* h, int ms);

/* Which all-reduce a tensor-parallel handle's batched passes use after the residual
 * projections: 1 = the library's peer-memory all-reduce (every rank's residual buffer
 * mapped into the others' address space over NVLink), 0 = NCCL's all-reduce
 * (QWC_TP_ALLREDUCE=nccl, or the group could not set the peer mappings up), 2 = not
 * decided yet (the first batched pass decides, collectively). QWC_E_INVALID for a
 * single-GPU handle. */
int qwc_tp_allreduce_path(qwc_handle* h);

/* After qwc_prefill on a tensor-parallel group: gathers every rank's shard of the decode
 * state (GDN state and conv ring of its heads, KV of its kv heads for the T prefilled
 * positions) into `full`, a single-GPU handle of the same model on rank 0's device, over
 * the group's NCCL communicator; `full` then decodes from position T (qwc_step).
 * Collective: every rank calls it, rank 0 with `full`, the others with NULL. */
int qwc_tp_gather_state(qwc_handle* tp, qwc_handle* full);

/* ---------------------------------------------------------------- kernel level */

/* matmul(const WeightView&, ...) (src/forward_pass.cpp:65-75) on device memory:
 * y[out_dim] = W[out_dim, in_dim](bf16, row-major) . x[in_dim](fp32), fp32 accumulate.
 * in_dim must be a multiple of 8 and W 16-byte aligned. */
int qwc_gemv_bf16(const uint16_t* W, const float* x, float* y, int out_dim, int in_dim,
                  void* stream);

/* Int8 weights for the decode GEMV (no reference implementation: the reference names
 * 8/4-bit weights as its next step for decode speed, README.md:80-81). A GEMV at batch 1
 * streams its weights once per token, so 1-byte codes halve the bytes of the bf16 path.
 * Format: codes Wq[out_dim][in_dim] int8 and one fp32 scale per row and 128-column group,
 * scales[out_dim][in_dim / 128], w ~= q * scale.
 * qwc_quantize_q8: from bf16 W on the device: scale = max |w| / 127 over the group,
 *   q = round-to-nearest-even(w / scale) in [-127, 127] (0 codes for an all-zero group);
 *   in_dim a multiple of 128.
 * qwc_gemv_q8: y = dequant(W) . x in fp32 (per lane: the group's scale times the fp32 sum
 *   of its codes times x); in_dim a multiple of 512, at most 8192. */
int qwc_quantize_q8(const uint16_t* W, int8_t* Wq, float* scales, int out_dim, int in_dim, void* stream);
int qwc_gemv_q8(const int8_t* Wq, const float* scales, const float* x, float* y, int out_dim, int in_dim,
                void* stream);

/* The projections of QwenForward::prefill (src/qwen_forward.cpp:154-206, each row a
 * matmul of src/forward_pass.cpp:65-75) for N tokens at once on the tensor cores:
 * Y[N][M] (=, or += when accumulate) sum_k X[n][k] W[m][k], W bf16 [M][K] row-major,
 * X given as bf16 pairs Xs[N][2K] with Xs[n][k] = bf16(x), Xs[n][K+k] = bf16(x - that)
 * so that hi + lo carries x to ~2^-17 relative; fp32 accumulation. K must be a multiple
 * of 64; W and Xs 16-byte aligned. Device pointers; asynchronous on `stream`. */
int qwc_gemm_bf16(const uint16_t* W, const uint16_t* Xs, float* Y, int M, int N, int K, int accumulate,
                  void* stream);

/* The decode GDN mixer core of gdn_step (src/qwen_model.cpp:173-207) for one token on
 * device memory, as used by step(): conv over the rolling state, SiLU, l2norm(q,k),
 * gates, delta-rule update of S and o = S^T q (before the gated norm).
 *   mixed [C] raw conv input (C = 2*KH*DK + VH*DV), a/b [VH] raw gate inputs,
 *   conv_w [C][K] fp32, neg_exp_A [VH] = -exp(A_log), dt_bias [VH],
 *   conv_ring [C][K] fp32 rolling state addressed by pos % K (zero at pos 0),
 *   state [VH][DK][DV] fp32 (the reference's S layout), out [VH][DV].
 * DK = DV = 128 and K = 4 are supported. */
int qwc_gdn_decode_step(const float* mixed, const float* a, const float* b,
                        const float* conv_w, const float* neg_exp_A, const float* dt_bias,
                        float* conv_ring, float* state, float* out, int KH, int VH, int pos,
                        void* stream);

/* The GDN mixer core of QwenForward::prefill's mix_gdn (src/qwen_forward.cpp:83-152; per
 * token the arithmetic of gdn_step, src/qwen_model.cpp:173-207) for T tokens at positions
 * pos0..pos0+T-1, continuing from conv_ring / state and leaving them as T calls of
 * qwc_gdn_decode_step would: mixed [T][C] raw conv inputs, a/b [T][VH] raw gate inputs,
 * out [T][VH][DV] (before the gated norm). The recurrence runs in the chunked WY form
 * (64-token chunks). workspace: device scratch of at least
 * qwc_gdn_prefill_workspace(KH, VH, T) bytes. DK = DV = 128, K = 4. */
size_t qwc_gdn_prefill_workspace(int KH, int VH, int T);
int qwc_gdn_prefill(const float* mixed, const float* a, const float* b, const float* conv_w,
                    const float* neg_exp_A, const float* dt_bias, float* conv_ring, float* state,
                    float* out, int KH, int VH, int T, int pos0, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Attention of one query over a KV cache on device memory (the loop of attn_step,
 * src/qwen_model.cpp:134-150): q [NQ][HD] (normed and roped), gate [NQ][HD],
 * K/V cache [NKV][max_ctx][HD] of kv_dtype, positions 0..n_ctx-1; out [NQ][HD] =
 * softmax(q K^T / sqrt(HD)) V * sigmoid(gate). HD = 256 is supported. From 2048 cached
 * positions on, a block-per-warp split kernel (bf16 caches: K/V staged through shared
 * memory) and a second, combining kernel run on `stream`. */
int qwc_attention_decode(const float* q, const float* gate, const void* k_cache,
                         const void* v_cache, int kv_dtype, int NQ, int NKV, int max_ctx,
                         int n_ctx, float* out, void* stream);

/* No counterpart in the reference. Same computation and arguments as
 * qwc_attention_decode, for callers that must not allocate device memory while they
 * run: a plugin whose host application owns all device memory through its own pool, or
 * a latency-critical loop that cannot afford cudaMalloc's implicit synchronisation.
 * qwc_attention_decode grows a per-thread split-K workspace with cudaMalloc on first
 * use; this variant instead uses a fixed 4 MiB array in device global memory that the
 * library reserves on every GPU that loads it (held until the process exits), and calls
 * no cudaMalloc, cudaFree or other allocating routine.
 *  - Limit: the workspace, 256 B + NQ * nsplit * 1032 B (nsplit = number of context
 *    splits, n_ctx / 32 rounded up, at most 2 per SM: 296 on a B200), must fit 4 MiB;
 *    larger requests
 *    return QWC_E_INVALID with the sizes in qwc_last_error(NULL). NKV <= 64.
 *  - The first call on each device looks up the array's device address (with that
 *    device current). With lazy module loading (the CUDA default) that first call may
 *    also load the library's device code and so reserve the array: a caller that must
 *    not allocate at all makes its first call during its own set-up, before any stream
 *    capture.
 *  - It always runs the per-position split kernel that qwc_attention_decode uses below
 *    2048 cached positions; on longer caches it is slower than qwc_attention_decode,
 *    which switches to its block-per-warp kernel there (results agree to rounding).
 *  - Every call on a device shares the one array: calls that overlap on the GPU (on
 *    different streams, or from different host threads) race and give wrong results.
 *    The split counters are cleared on `stream` at the start of each call. */
int qwc_attention_decode_noalloc(const float* q, const float* gate, const void* k_cache,
                                 const void* v_cache, int kv_dtype, int NQ, int NKV,
                                 int max_ctx, int n_ctx, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QWEN_CUDA_H */
