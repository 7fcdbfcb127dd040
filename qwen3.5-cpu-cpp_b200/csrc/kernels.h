// Internal launch interface of the sm_100a kernels (not part of the C ABI).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

namespace qwc {

// ------------------------------------------------------------------ GEMV family
// y = W . x with W bf16 [rows][in_dim] row-major, x fp32, fp32 accumulation: the
// reference's matmul(WeightView) (src/forward_pass.cpp:44-75), streamed from HBM by
// 1-D bulk TMA into a shared-memory ring, with the neighbouring elementwise work of
// the decode step fused as a prologue (how x is formed) and an epilogue (where the
// row results go).
enum GemvPro : int {
    PRO_PLAIN = 0,        // x = x_in
    PRO_RMSNORM = 1,      // x = rmsnorm(x_in) * (1 + w)            (forward_pass.cpp:77-84)
    PRO_EMBED_RMSNORM = 2,// x_in = embedding row of tokens[*pos]; CTA 0 stores it in hidden
    PRO_GATED_NORM = 3,   // x = w * (o * rsqrt(mean_head(o^2)+eps)) * silu(z)  (:86-93)
    PRO_ATTN_COMBINE = 4, // x = the split-K attention partials combined, * sigmoid(gate)
                          // (persistent step only; attn_step :134-150)
};
enum GemvEpi : int {
    EPI_STORE = 0,        // y[r] = acc
    EPI_RESIDUAL = 1,     // y[r] += acc                               (qwen_model.cpp:223,232)
    EPI_SWIGLU = 2,       // row r = [gate_r | up_r] (2*x_len long): y[r] = silu(g)*u (:227-231)
    EPI_ARGMAX = 3,       // y[r] = acc (logits) + greedy argmax over all rows (:249-251)
};

struct GemvParams {
    const uint16_t* W = nullptr;
    int rows = 0;
    int in_dim = 0;          // row length in elements
    int x_len = 0;           // length of x (in_dim, or in_dim/2 for EPI_SWIGLU)
    const float* x = nullptr;
    const float* norm_w = nullptr;  // PRO_RMSNORM: (1+w) [x_len]; PRO_GATED_NORM: w [gn_dim]
    const float* z = nullptr;       // PRO_GATED_NORM: gate input [x_len]
    int gn_dim = 128;
    float eps = 1e-6f;
    // PRO_EMBED_RMSNORM
    const uint16_t* embed = nullptr;
    const int* tokens = nullptr;    // token at position p is tokens[p]
    const int* pos = nullptr;
    int vocab = 0;
    float* hidden_out = nullptr;
    // output
    float* y = nullptr;
    // EPI_ARGMAX
    float* am_val = nullptr;        // [gridDim] per-CTA partials
    int* am_idx = nullptr;
    unsigned* am_counter = nullptr; // zero between launches (the last CTA resets it)
    int* argmax_out = nullptr;      // final id
    int* tokens_out = nullptr;      // if non-null: tokens_out[*pos + 1] = id when *pos+1 >= *n_prompt
    const int* n_prompt = nullptr;
    int* pos_inout = nullptr;       // if non-null: ++*pos_inout by the last CTA
    int max_ctx = 0;
    int slots_per_warp = 6;         // ring depth (set by the launcher)
    int* dev_err = nullptr;         // device error word (bounded waits, bad token)
    // PRO_ATTN_COMBINE: partials of the attention phase (AttnDecodeParams with
    // defer_combine), gate = x (the attention projection, [q | gate] per head), pos
    const float* part_o = nullptr;
    const float* part_ml = nullptr;
    int nsplit = 1, nq = 0, nkv = 0;
    int min_chunk = 32;             // positions per attention split at least (as the splits)
};

size_t gemv_smem_bytes(const GemvParams& p);
cudaError_t launch_gemv(int pro, int epi, GemvParams p, int grid, cudaStream_t s, bool pdl);
int gemv_grid(int rows, int per_sm = 1);

// Int8-weight GEMV (gemv_q8.cu): codes [rows][in_dim] int8 + fp32 scales [rows][in_dim/128];
// in_dim a multiple of 512 (<= 8192) for the GEMV, of 128 for the quantiser.
cudaError_t launch_quantize_q8(const uint16_t* W, int8_t* Wq, float* scales, int rows, int in_dim, cudaStream_t s);
cudaError_t launch_gemv_q8(const int8_t* W, const float* scales, const float* x, float* y, int rows, int in_dim,
                           cudaStream_t s);

// ------------------------------------------------------------------ GDN decode
// One token of the Gated DeltaNet mixer core (qwen_model.cpp:173-207): causal conv over
// the rolling state + SiLU, l2norm(q,k), gates, delta-rule update, o = S^T q.
struct GdnDecodeParams {
    const float* mixed = nullptr;   // [C] = [q KD | k KD | v VD]
    const float* a = nullptr;       // [VH]
    const float* b = nullptr;       // [VH]
    const float* conv_w = nullptr;  // [C][4]
    const float* neg_exp_A = nullptr;  // [VH]
    const float* dt_bias = nullptr;    // [VH]
    float* conv_ring = nullptr;     // [C][4], slot pos % 4 receives the new input
    float* state = nullptr;         // [VH][DK][DV]
    float* out = nullptr;           // [VH][DV]
    const int* pos_ptr = nullptr;   // device position (or nullptr: use pos_val)
    int pos_val = 0;
    int KH = 0, VH = 0;
};
cudaError_t launch_gdn_decode(const GdnDecodeParams& p, cudaStream_t s, bool pdl);

// ------------------------------------------------------------------ attention decode
// Split-K flash decode over the KV cache with the q/k norm + partial RoPE + KV append
// of attn_step (qwen_model.cpp:118-150) fused in, and the sigmoid output gate applied by
// the CTA that combines the splits.
struct AttnDecodeParams {
    const float* proj = nullptr;    // decode: [NQ][2*HD] ([q|gate] per head), [NKV][HD] k, [NKV][HD] v
    const float* q_in = nullptr;    // op mode: q [NQ][HD] (normed+roped); proj == nullptr
    const float* gate_in = nullptr; // op mode: gate [NQ][HD]
    const float* qn1 = nullptr;     // (1+w) q_norm [HD]
    const float* kn1 = nullptr;     // (1+w) k_norm [HD]
    const float* rope_cs = nullptr;   // [max_ctx][rot/2][2] (cos, sin) of pos * theta^(-2i/rot)
    void* k_cache = nullptr;        // [NKV][max_ctx][HD]
    void* v_cache = nullptr;
    int kv_bf16 = 0;
    int max_ctx = 0;
    const int* pos_ptr = nullptr;   // decode: position of the new token (n_ctx = pos+1)
    int n_ctx_val = 0;              // op mode: number of cached positions
    float* part_o = nullptr;        // [NKV][nsplit][GRP][HD]
    float* part_ml = nullptr;       // [NKV][nsplit][GRP][2]
    unsigned* counters = nullptr;   // [NKV], zero between launches
    float* out = nullptr;           // [NQ][HD]
    int NQ = 0, NKV = 0, rot = 64, nsplit = 1;
    float eps = 1e-6f;
    int defer_combine = 0;          // every split only publishes its partial; the consumer
                                    // of `out` combines them (PRO_ATTN_COMBINE)
    int min_chunk = 32;             // positions per split at least
};
cudaError_t launch_attn_decode(const AttnDecodeParams& p, cudaStream_t s, bool pdl);
int attn_nsplit_for(int max_ctx, int nkv);
// Op mode over long caches (attn_long.cu): splits of whole 256-position rounds, then a
// separate combine kernel; q_in / gate_in, part_o / part_ml sized for attn_long_nsplit.
constexpr int kAttnLongMin = 2048;
int attn_long_nsplit(int n_ctx, int nkv, int grp, int kv_bf16);
cudaError_t launch_attn_long(const AttnDecodeParams& p, cudaStream_t s);

// ------------------------------------------------------------------ persistent step
// One launch = one decode step: a list of phases run by a cooperative grid of one CTA
// per SM with grid-wide barriers between them (decode_step.cu).
enum PhaseType : int { PH_GEMV = 0, PH_GDN = 1, PH_ATTN = 2 };
struct alignas(16) StepPhase {
    int type = PH_GEMV, pro = 0, epi = 0, pad = 0;
    GemvParams g;
    GdnDecodeParams d;
    AttnDecodeParams a;
};
struct StepParams {
    const StepPhase* phases = nullptr;  // device array
    int nphases = 0;
    unsigned long long* bar = nullptr;  // arrival counter, zero between steps
    unsigned* done = nullptr;           // end-of-step ticket, zero between steps
    int* dev_err = nullptr;
    int nslot = 4;                      // ring slots per warp (4 KB each)
    int xs_max = 0;                     // largest GEMV x length (floats)
    unsigned long long wait_ns = 0;     // limit of every wait of the step (0: kWaitLimitNs)
    int stall_cta = -1;                 // test only: this CTA withholds its first grid arrival
    long long* trace = nullptr;         // optional [grid][nphases][8] globaltimer stamps / counters
};
static_assert(sizeof(StepPhase) % 16 == 0, "staged as int4");
int step_slots(int xs_max, int grp, int nphases);
size_t step_smem_bytes(int nslot, int xs_max, int nphases);
int decode_step_max_grid(int grp, int nslot, int xs_max, int nphases);  // 0: not co-resident
cudaError_t launch_decode_step(const StepParams& sp, int grp, int grid, cudaStream_t s);

int num_sms();

// ------------------------------------------------------------------ tensor-core GEMM
// Batched forward pass (tc_gemm.cu): Y[n][m] (op)= sum_k X[n][k] W[m][k] over N tokens,
// W bf16 [M][K], X carried as bf16 hi/lo pairs [N][ld] (hi at [0,K), lo at [K,2K)).
enum TcEpi : int {
    TC_STORE = 0,        // y[n][m] = acc
    TC_RESIDUAL = 1,     // y[n][m] += acc
    TC_SWIGLU_SPLIT = 2, // rows alternate gate_i/up_i: ys[n][i], ys[n][split_k+i] = hi/lo of silu(g)*u
};
struct TcGemmParams {
    int M = 0, N = 0, K = 0;
    int epi = TC_STORE;
    float* y = nullptr;
    long ldy = 0;
    uint16_t* ys = nullptr;
    long ldys = 0;
    int split_k = 0;
    int* err = nullptr;
};
// Tensor map of a row-major bf16 matrix [rows][cols] with row stride ld (elements), in
// 128 x 64 boxes with the 128-byte swizzle. Returns 0 on success.
int tc_make_map(CUtensorMap* map, const void* base, long rows, long cols, long ld);
// The same with boxes of `box_rows` rows (x 64 columns).
int tc_make_map_box(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_rows);
cudaError_t launch_tc_gemm(const CUtensorMap& mapW, const CUtensorMap& mapX, const TcGemmParams& p, cudaStream_t s);

// ------------------------------------------------------------------ prefill kernels
// Token-parallel pieces of the batched forward pass over a chunk of T tokens at
// positions p0.. (prefill.cu). Activation inputs of the GEMMs are written as hi/lo pairs.
cudaError_t pf_embed(const int* ids, int T, const uint16_t* embed, int H, int V, float* hid, int* err, cudaStream_t s);
cudaError_t pf_rmsnorm_split(const float* x, long ldx, int rows, const float* w1, int H, float eps, uint16_t* xs,
                             long ldxs, cudaStream_t s);
struct PfGdnArgs {
    const float* proj = nullptr;  // [T][ldp]: the C conv inputs (q | k | v) first
    long ldp = 0;
    const float* a_in = nullptr;  // [T][ldab] raw a gate inputs
    const float* b_in = nullptr;  // [T][ldab] raw b gate inputs
    long ldab = 0;
    const float* conv_w = nullptr;
    float* ring = nullptr;        // [C][4], read then updated
    const float* neg_exp_A = nullptr;
    const float* dt_bias = nullptr;
    float* qn = nullptr;          // scratch [T][KD]
    float* kn = nullptr;          // scratch [T][KD]
    float* vc = nullptr;          // scratch [T][VD]
    float* glog = nullptr;        // scratch [T][VH] log decay
    float* beta = nullptr;        // scratch [T][VH]
    float* U = nullptr;           // scratch [VH][T][128]  (chunked WY form)
    float* W = nullptr;           // scratch [VH][ceil(T/64)][128][64]  W^T per chunk
    uint16_t* QG = nullptr;       // scratch [VH][2][ceil(T/64)*64][128] bf16 pairs
    float* KD = nullptr;          // scratch [VH][T][128]
    uint16_t* P = nullptr;        // scratch [VH][ceil(T/64)][2][64][64] bf16 pairs
    float* gC = nullptr;          // scratch [VH][ceil(T/64)]
    uint16_t* ST = nullptr;       // scratch [VH][ceil(T/64)][2][128][128] bf16 pairs
    uint16_t* ET = nullptr;       // scratch [VH][ceil(T/64)][2][128][64] bf16 pairs
    int* err = nullptr;           // device error word of the tensor-core kernel
    cudaEvent_t ev_state0 = nullptr, ev_state1 = nullptr;  // optional: recorded around the state pass
    float* state = nullptr;       // [VH][DK][DV], read then updated
    float* out = nullptr;         // [T][VD]
    int T = 0, p0 = 0, KH = 0, VH = 0, C = 0, VD = 0;
};
cudaError_t pf_gdn(const PfGdnArgs& a, cudaStream_t s);
// Scratch of pf_gdn for T tokens, and its carving into the args' scratch pointers.
size_t pf_gdn_workspace_bytes(int KH, int VH, int T);
int pf_gdn_carve(PfGdnArgs& a, void* ws, size_t bytes);
cudaError_t pf_gated_norm_split(const float* o, long ldo, const float* z, long ldz, const float* w, int T, int nh,
                                float eps, uint16_t* xs, long ldxs, cudaStream_t s);
struct PfAttnArgs {
    const float* proj = nullptr;  // [T][ldp]: NQ x [q | gate], NKV x k, NKV x v
    long ldp = 0;
    const float* qn1 = nullptr;
    const float* kn1 = nullptr;
    const float* rope_cs = nullptr;
    float* qbuf = nullptr;        // scratch [T][NQ][HD]
    void* k_cache = nullptr;
    void* v_cache = nullptr;
    int kv_bf16 = 0, max_ctx = 0, p0 = 0, T = 0, NQ = 0, NKV = 0, rot = 64;
    float eps = 1e-6f;
    uint16_t* xs = nullptr;       // output [T][ldxs], K = NQ*HD
    long ldxs = 0;
    // tensor-core attention operands (bf16 pairs): K split [NKV][ctx_pad][512] and V^T
    // split [NKV][2][256][ctx_pad] of this layer (persist across chunks), V split scratch
    // [NKV][T][512] of the chunk
    uint16_t* ksplit = nullptr;
    uint16_t* vt = nullptr;
    uint16_t* vsplit = nullptr;
    int ctx_pad = 0;
    float* part_o = nullptr;      // key-split partials of the tensor-core attention
    float* part_ml = nullptr;
    int part_splits = 0;
    int* err = nullptr;
};
cudaError_t pf_attention(const PfAttnArgs& a, cudaStream_t s);
struct PfFattnArgs {
    const float* qbuf = nullptr;
    const float* proj = nullptr;
    long ldp = 0;
    uint16_t* xs = nullptr;
    long ldxs = 0;
    const uint16_t* ksplit = nullptr;
    uint16_t* vt = nullptr;
    const uint16_t* vsplit = nullptr;
    int T = 0, p0 = 0, NQ = 0, NKV = 0, ctx_pad = 0;
    // key-split partials (pf_fattn_splits(...) > 1): [splits][T][NQ][HD] and [splits][T][NQ][2]
    float* part_o = nullptr;
    float* part_ml = nullptr;
    int part_splits = 0;
    int* err = nullptr;
};
cudaError_t pf_fattn(const PfFattnArgs& a, cudaStream_t s);
// Key splits pf_fattn uses for a chunk of T queries at positions p0.. (grows with p0).
int pf_fattn_splits(int T, int p0, int NQ, int NKV);
constexpr int kFattnMaxSplits = 16;

// Peer-memory all-reduce of the tensor-parallel residual stream (tp_p2p.cu).
constexpr int kP2pMaxRanks = 8;
struct P2pPtrs {
    unsigned long long* flags[kP2pMaxRanks];  // every rank's barrier flags, as mapped here
    float* data[kP2pMaxRanks];                // every rank's residual buffer, as mapped here
    int world, rank;
};
struct P2pGroup;
// Collective over the group: every rank allocates an exportable buffer of data_bytes,
// exchanges it with the others (abstract Unix sockets named by `group` and `gen`, bounded
// by timeout_ms) and maps theirs. Returns 0, or -1 with `why` (nothing left allocated).
int p2p_setup(P2pGroup** out, int rank, int world, int device, uint64_t group, int gen, size_t data_bytes,
              int timeout_ms, std::string& why);
void p2p_destroy(P2pGroup* g);
float* p2p_local_data(P2pGroup* g);
size_t p2p_capacity_floats(const P2pGroup* g);
// In-place sum of n floats over the group's buffers (barrier, reduce, barrier); `epoch`
// advances by 2 and must advance identically on every rank.
cudaError_t p2p_allreduce(P2pGroup* g, size_t n, unsigned long long& epoch, unsigned long long wait_ns, int* err,
                          cudaStream_t s);

// Records a handle-less failure message (what qwc_last_error(NULL) returns).
void set_api_error(const char* msg);

}  // namespace qwc
