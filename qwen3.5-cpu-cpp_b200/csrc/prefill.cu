// Token-parallel kernels of the batched forward pass (prefill) of a chunk of T tokens at
// positions p0 .. p0+T-1. They continue from the decode state (KV cache, GDN state and
// conv ring) and leave it exactly where T decode steps would: the chunk's K/V rows are
// in the cache, the GDN state has absorbed the chunk, the conv ring holds its last
// inputs. The projections between them are tensor-core GEMMs (tc_gemm.cu), whose
// activation inputs these kernels write as bf16 hi/lo pairs.
//
// Reference: QwenForward::prefill (src/qwen_forward.cpp:154-206) with mix_gdn (:83-152)
// and mix_attention (:20-80); the per-token arithmetic is that of QwenModel::gdn_step /
// attn_step (src/qwen_model.cpp:106-209), in the same order as the decode kernels.
#include "attn_body.cuh"
#include "common.cuh"
#include "gdn_body.cuh"
#include "tc_util.cuh"
#include "kernels.h"

#include <cstdlib>

namespace qwc {

constexpr int kPT = 256;  // threads of the token-parallel kernels

// x = hi + lo as bf16 pair, stored at row[i] and row[K + i]
__device__ __forceinline__ void store_split(uint16_t* row, int K, int i, float v) {
    const uint16_t hi = f2bf(v);
    row[i] = hi;
    row[K + i] = f2bf(v - __uint_as_float((uint32_t)hi << 16));
}

// Sum over the block (kPT threads) in double.
__device__ __forceinline__ double block_sum_d(double v, double* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double s = 0.0;
#pragma unroll
    for (int w = 0; w < kPT / 32; ++w) s += red[w];
    return s;
}

// ---------------------------------------------------------------- embedding
__global__ void __launch_bounds__(kPT) k_pf_embed(const int* ids, const uint16_t* embed, int H, int V, float* hid,
                                                   int* err) {
    const int t = blockIdx.x;
    int tok = ids[t];
    if (tok < 0 || tok >= V) {
        if (threadIdx.x == 0) post_error(err, DEV_BAD_TOKEN);
        tok = 0;
    }
    const uint16_t* e = embed + (size_t)tok * H;
    float* o = hid + (size_t)t * H;
    for (int i = threadIdx.x; i < H; i += kPT) o[i] = __uint_as_float((uint32_t)e[i] << 16);
}

// ---------------------------------------------------------------- RMSNorm -> split
// xs[t] = split(x[t] * inv_rms * w1), w1 = 1 + weight (rmsnorm, forward_pass.cpp:77-84).
__global__ void __launch_bounds__(kPT) k_pf_rmsnorm_split(const float* x, long ldx, const float* w1, int H, float eps,
                                                           uint16_t* xs, long ldxs) {
    __shared__ double red[kPT / 32];
    const float* r = x + (size_t)blockIdx.x * ldx;
    double ss = 0.0;
    for (int i = threadIdx.x; i < H; i += kPT) ss += (double)r[i] * r[i];
    ss = block_sum_d(ss, red);
    const float inv = 1.0f / sqrtf((float)(ss / H) + eps);
    uint16_t* o = xs + (size_t)blockIdx.x * ldxs;
    for (int i = threadIdx.x; i < H; i += kPT) store_split(o, H, i, r[i] * inv * w1[i]);
}

// ---------------------------------------------------------------- GDN input preparation
// Per token: causal depthwise conv (K=4) over the qkv channels, continuing from the conv
// ring for positions before the chunk, SiLU; l2norm of q and k per head (q also scaled by
// 1/sqrt(DK)); the gates g = -exp(A_log) softplus(a + dt_bias) (decay exp(g)), beta = sigmoid(b).
struct PfGdnPrep {
    const float* proj;    // [T][ldp]: the C conv inputs (q | k | v) first
    long ldp;
    const float* a_in;    // [T][ldab] raw a gate inputs (VH)
    const float* b_in;    // [T][ldab] raw b gate inputs (VH)
    long ldab;
    const float* conv_w;  // [C][4]
    const float* ring;    // [C][4] (read only here)
    const float* neg_exp_A;
    const float* dt_bias;
    float* qn;            // [T][KD]
    float* kn;            // [T][KD]
    float* vc;            // [T][VD]
    float* glog;          // [T][VH] g (the decay is exp(g))
    float* beta;          // [T][VH]
    int p0, KH, VH, C, VD;
};
// CTA = (16 tokens, one q / k / v head vector), thread = channel. The thread reads its channel's inputs for the 3 positions before the tile and
// the tile's 16 tokens once (sliding conv window in registers, every row read once instead
// of four times); the l2norm sums of squares are reduced per token across the 128 channels
// (double, like the per-token kernel). Blocks with y = 2 KH + VH form the gates.
constexpr int kPrepT = 16;
__global__ void __launch_bounds__(128) k_pf_gdn_prep_tiled(const PfGdnPrep p, int T) {
    __shared__ double red[4][kPrepT];
    const int tb = blockIdx.x * kPrepT, v = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int KD = p.KH * 128, nvec = 2 * p.KH + p.VH;
    if (v == nvec) {
        for (int i = tid; i < kPrepT * p.VH; i += 128) {
            const int t = tb + i / p.VH, h = i % p.VH;
            if (t >= T) continue;
            const float bv = p.b_in[(size_t)t * p.ldab + h], av = p.a_in[(size_t)t * p.ldab + h];
            p.glog[(size_t)t * p.VH + h] = p.neg_exp_A[h] * softplus_f(av + p.dt_bias[h]);
            p.beta[(size_t)t * p.VH + h] = sigmoid_f(bv);
        }
        return;
    }
    const int kind = v < p.KH ? 0 : (v < 2 * p.KH ? 1 : 2);
    const int head = kind == 0 ? v : (kind == 1 ? v - p.KH : v - 2 * p.KH);
    const int c = (kind == 0 ? head * 128 : (kind == 1 ? KD + head * 128 : 2 * KD + head * 128)) + tid;
    float x[kPrepT + 3];  // inputs at tb-3 .. tb+15
#pragma unroll
    for (int d = 0; d < kPrepT + 3; ++d) {
        const int tt = tb - 3 + d;
        if (tt >= 0) {
            x[d] = tt < T ? p.proj[(size_t)tt * p.ldp + c] : 0.f;
        } else {
            const int pos = p.p0 + tt;
            x[d] = pos >= 0 ? p.ring[(size_t)c * 4 + (pos & 3)] : 0.f;
        }
    }
    const float4 w = reinterpret_cast<const float4*>(p.conv_w)[c];
    float val[kPrepT];
#pragma unroll
    for (int i = 0; i < kPrepT; ++i) {
        float acc = 0.f;
        acc += w.x * x[i];
        acc += w.y * x[i + 1];
        acc += w.z * x[i + 2];
        acc += w.w * x[i + 3];
        val[i] = silu_f(acc);
    }
    if (kind < 2) {
#pragma unroll
        for (int i = 0; i < kPrepT; ++i) {
            double ss = (double)val[i] * val[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp][i] = ss;
        }
        __syncthreads();
        float* dst = (kind == 0 ? p.qn : p.kn) + head * 128 + tid;
#pragma unroll
        for (int i = 0; i < kPrepT; ++i) {
            const int t = tb + i;
            if (t >= T) break;
            const double ss = red[0][i] + red[1][i] + red[2][i] + red[3][i];
            float xo = val[i] * (1.0f / sqrtf((float)ss + 1e-6f));
            if (kind == 0) xo = xo * (1.0f / sqrtf(128.0f));
            dst[(size_t)t * KD] = xo;
        }
    } else {
        float* dst = p.vc + head * 128 + tid;
#pragma unroll
        for (int i = 0; i < kPrepT; ++i) {
            const int t = tb + i;
            if (t >= T) break;
            dst[(size_t)t * p.VD] = val[i];
        }
    }
}

// Conv ring after the chunk: slot (pos & 3) holds the input at pos for the last (up to)
// four positions of the chunk. Runs after k_pf_gdn_prep has read the old ring.
__global__ void k_pf_conv_ring(const float* proj, long ldp, int T, int p0, int C, float* ring) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    for (int t = (T > 4 ? T - 4 : 0); t < T; ++t) ring[(size_t)c * 4 + ((p0 + t) & 3)] = proj[(size_t)t * ldp + c];
}

// ---------------------------------------------------------------- GDN recurrence, chunked
// The delta rule of gdn_step (qwen_model.cpp:199-205), per value head, in the order
//   S_t = a_t S_{t-1};  e_t = v_t - S_t^T k_t;  S_t += b_t k_t e_t^T;  o_t = S_t^T q_t
// (a_t = exp(g_t) the decay, b_t = beta_t), is evaluated for chunks of C = 64 tokens in
// the WY form. With G_i = g_1 + .. + g_i inside the chunk, gamma_i = exp(G_i) and S0 the
// state entering the chunk:
//   e_i = v_i - gamma_i S0^T k_i - sum_{j<i} exp(G_i - G_j) b_j (k_i . k_j) e_j
//   => (I + L) E = V - Gamma K S0,  L[i][j] = exp(G_i - G_j) b_j (k_i . k_j), j < i
//   => E = U - W S0 with U = (I + L)^-1 V, W = (I + L)^-1 Gamma K  (forward substitution)
//   o_i = gamma_i S0^T q_i + sum_{j<=i} P[i][j] e_j,  P[i][j] = exp(G_i - G_j) b_j (q_i . k_j)
//   S_C = gamma_C S0 + sum_i Kd_i e_i^T,  Kd_i = b_i exp(G_C - G_i) k_i
// Every exponent is a difference G_i - G_j <= 0 (or a G_i <= 0), so nothing overflows.
// Kernel A (parallel over chunks and heads, tcgen05) builds U, W, Gamma Q, Kd, P and
// gamma_C, with U = T V and W = T Gamma K from the explicit T = (I + L)^-1; kernel B1
// (sequential over chunks, parallel over heads and 16-column slices of S, CUDA cores)
// applies E = U - W S, S = gamma_C S + Kd^T E and keeps the state entering each chunk;
// kernel B2 (parallel over chunks and heads, tcgen05) forms O = (Gamma Q) S_c + P E.
constexpr int kGC = 64;            // tokens per chunk
constexpr uint32_t kT128 = 128 * 128;  // bytes of a 128-row x 64-column bf16 tile
constexpr uint32_t kT64 = 64 * 128;    // bytes of a 64-row x 64-column bf16 tile
constexpr int kGP = 128 + 4;       // padded row stride of 128-wide shared tiles

struct PfGdnChunk {
    const float* qn;     // [T][KD]
    const float* kn;     // [T][KD]
    const float* vc;     // [T][VD]
    const float* glog;   // [T][VH] g = log of the decay
    const float* beta;   // [T][VH]
    float* U;            // [VH][T][128]
    float* W;            // [VH][nch][128 key dims][64 tokens]  W^T per chunk
    uint16_t* QG;        // [VH][hi|lo][Tpad][128]  gamma_i q_i as bf16 pairs
    float* KD;           // [VH][T][128]  b_i exp(G_C - G_i) k_i
    uint16_t* P;         // [VH][nch][hi|lo][64][64] bf16 pairs
    float* gC;           // [VH][nch]
    uint16_t* ST;        // [VH][nch][hi|lo][DV][DK] transposed state entering each chunk, bf16 pairs
    uint16_t* ET;        // [VH][nch][hi|lo][DV][64]  E^T of each chunk, bf16 pairs
    float* state;        // [VH][DK][DV]
    float* out;          // [T][VD]
    int T, KH, VH, VD;
};
// x -> bf16 hi and lo (x = hi + lo within 2^-17 |x|)
__device__ __forceinline__ void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    hi = f2bf(x);
    lo = f2bf(x - bf16lo(hi));
}

// Kernel A on the tensor cores, CTA = (chunk, value head), 128 threads (thread = TMEM lane):
//   1. [K; Q] (128 x 128) times K^T -> [K K^T; Q K^T] (128 x 64) in TMEM: 24 MMAs M128 N64
//      K16 over bf16 pairs (hi hi + hi lo + lo hi);
//   2. rows 0-63 -> L (strictly lower, decay- and beta-weighted) into shared memory, rows
//      64-127 -> P as bf16 pairs to global (threads 64-127), while threads 0-63 each solve
//      one column of T = (I + L)^-1 by right-looking substitution in registers;
//   3. U^T = V^T T^T and W^T = (Gamma K)^T T^T (128 x 64 each): 2 x 12 MMAs; rows written
//      out as U and W. Kd, Gamma Q and gamma_C are formed on the way in.
// Shared operand tiles are K-major with 128-byte rows (64 bf16) and 128-byte swizzle.
constexpr uint32_t kA_KQ = 4 * kT128;               // [K; Q] tiles [hi|lo][dims 0-63 | 64-127]
constexpr uint32_t kA_T = 2 * kT64;                 // T tiles [hi|lo]
constexpr uint32_t kA_V = 2 * kT128;                // V^T tiles [hi|lo]
constexpr uint32_t kA_G = 2 * kT128;                // (Gamma K)^T tiles [hi|lo]
constexpr int kLtP = kGC;                           // row stride of L^T (floats)
// fp32 staging of the chunk's k and v rows [2][64][132], alive only while the operand tiles
// are built; it shares its space with T and L^T, which are written later
constexpr uint32_t kA_Stage = 2u * kGC * kGP * 4;
constexpr uint32_t kA_Late = kA_T + (uint32_t)(kGC * kLtP * 4);
constexpr uint32_t kA_Shared = kA_Stage > kA_Late ? kA_Stage : kA_Late;
constexpr size_t kGdnATcSmem = kA_KQ + kA_V + kA_G + kA_Shared + (size_t)(2 * kGC) * 4 + 1024 + 64;
__device__ __forceinline__ void cp16z(void* dst, const void* src, bool pred) {
    const int nb = pred ? 16 : 0;  // 0: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(nb) : "memory");
}
// byte offset of element (row, col) in a 128-byte-swizzled K-major tile
__device__ __forceinline__ uint32_t sw_off(int row, int col) {
    return (uint32_t)row * 128u + (uint32_t)((((col >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}
__global__ void __launch_bounds__(128, 1) k_pf_gdn_chunk_a_tc(const PfGdnChunk p, int* err) {
    extern __shared__ uint8_t sa_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sa_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* AKQ = sm;
    uint8_t* AV = AKQ + kA_KQ;
    uint8_t* AG = AV + kA_V;
    uint8_t* TB = AG + kA_G;
    float* Lt = reinterpret_cast<float*>(TB + kA_T);  // L^T: Lt[m][i] = L[i][m]
    float* Kst = reinterpret_cast<float*>(TB);        // staging k rows [64][132] (phase 0 only)
    float* Vst = Kst + kGC * kGP;                     // staging v rows [64][132] (phase 0 only)
    float* Qst = reinterpret_cast<float*>(AV);        // staging q rows [64][128] until V^T is built
    float* Gc = reinterpret_cast<float*>(TB + kA_Shared);
    float* Bs = Gc + kGC;
    uint64_t* bar = reinterpret_cast<uint64_t*>(Bs + kGC);
    uint64_t* mma1 = bar;
    uint64_t* mma2 = bar + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
    const int c = blockIdx.x, vh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nch = gridDim.x;
    const int rep = p.VH / p.KH, kh = vh / rep, KD = p.KH * 128;
    const int t0 = c * kGC, n = min(kGC, p.T - t0);
    if (tid == 0) {
        mbar_init(mma1, 1);
        mbar_init(mma2, 1);
        fence_mbar_init();
    }
    // q, k and v rows of the chunk -> shared memory (many copies in flight; rows past the chunk: 0)
    for (int e = tid; e < kGC * 32; e += 128) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        const size_t t = (size_t)(t0 + (i < n ? i : 0));
        cp16z(Kst + i * kGP + c4, p.kn + t * KD + kh * 128 + c4, i < n);
        cp16z(Vst + i * kGP + c4, p.vc + t * p.VD + vh * 128 + c4, i < n);
        cp16z(Qst + i * 128 + c4, p.qn + t * KD + kh * 128 + c4, i < n);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    if (warp == 0) tc::tmem_alloc(tmem_slot, 256);
    if (warp == 1) {
        // inclusive prefix sum of g over the chunk (two values per lane); beta
        const int i0 = 2 * lane;
        const float ga = i0 < n ? p.glog[(size_t)(t0 + i0) * p.VH + vh] : 0.f;
        const float gb = i0 + 1 < n ? p.glog[(size_t)(t0 + i0 + 1) * p.VH + vh] : 0.f;
        float sum = ga + gb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float up = __shfl_up_sync(0xffffffffu, sum, o);
            if (lane >= o) sum += up;
        }
        const float excl = sum - (ga + gb);
        Gc[i0] = excl + ga;
        Gc[i0 + 1] = excl + ga + gb;
        Bs[i0] = i0 < n ? p.beta[(size_t)(t0 + i0) * p.VH + vh] : 0.f;
        Bs[i0 + 1] = i0 + 1 < n ? p.beta[(size_t)(t0 + i0 + 1) * p.VH + vh] : 0.f;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    const float GC = Gc[n - 1];
    // ---- operands: [K; Q] rows (row-major), Kd and Gamma Q to global
    const size_t hrow = ((size_t)vh * p.T + t0) * 128;
    const size_t qrow = (size_t)nch * kGC;
    for (int e = tid; e < kGC * 32; e += 128) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        const float4 k4 = *reinterpret_cast<const float4*>(Kst + i * kGP + c4);
        const float4 q4 = *reinterpret_cast<const float4*>(Qst + i * 128 + c4);
        uint32_t kh2[2], kl2[2], qh2[2], ql2[2];
        tc::split2(k4.x, k4.y, kh2[0], kl2[0]);
        tc::split2(k4.z, k4.w, kh2[1], kl2[1]);
        tc::split2(q4.x, q4.y, qh2[0], ql2[0]);
        tc::split2(q4.z, q4.w, qh2[1], ql2[1]);
        const int kc = c4 >> 6, col = c4 & 63;
        *reinterpret_cast<uint2*>(AKQ + (0 * 2 + kc) * kT128 + sw_off(i, col)) = make_uint2(kh2[0], kh2[1]);
        *reinterpret_cast<uint2*>(AKQ + (1 * 2 + kc) * kT128 + sw_off(i, col)) = make_uint2(kl2[0], kl2[1]);
        *reinterpret_cast<uint2*>(AKQ + (0 * 2 + kc) * kT128 + sw_off(64 + i, col)) = make_uint2(qh2[0], qh2[1]);
        *reinterpret_cast<uint2*>(AKQ + (1 * 2 + kc) * kT128 + sw_off(64 + i, col)) = make_uint2(ql2[0], ql2[1]);
        if (i < n) {
            const float fd = Bs[i] * expf(GC - Gc[i]), fg = expf(Gc[i]);
            *reinterpret_cast<float4*>(p.KD + hrow + (size_t)i * 128 + c4) =
                make_float4(fd * k4.x, fd * k4.y, fd * k4.z, fd * k4.w);
            uint32_t gh[2], gl[2];
            tc::split2(fg * q4.x, fg * q4.y, gh[0], gl[0]);
            tc::split2(fg * q4.z, fg * q4.w, gh[1], gl[1]);
            uint16_t* qg = p.QG + ((size_t)vh * 2 * qrow + t0 + i) * 128 + c4;
            *reinterpret_cast<uint2*>(qg) = make_uint2(gh[0], gh[1]);
            *reinterpret_cast<uint2*>(qg + qrow * 128) = make_uint2(gl[0], gl[1]);
        }
    }
    __syncthreads();  // every read of the staged q is done before V^T overwrites it
    // ---- V^T and (Gamma K)^T: thread = value / key dim, 8 tokens per 16-byte segment
    for (int g = 0; g < 8; ++g) {
        float v8[8], k8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = g * 8 + u;
            v8[u] = Vst[i * kGP + tid];
            k8[u] = expf(Gc[i]) * Kst[i * kGP + tid];
        }
        uint32_t vh4[4], vl4[4], kh4[4], kl4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            tc::split2(v8[2 * u], v8[2 * u + 1], vh4[u], vl4[u]);
            tc::split2(k8[2 * u], k8[2 * u + 1], kh4[u], kl4[u]);
        }
        const uint32_t o = sw_off(tid, g * 8);
        *reinterpret_cast<uint4*>(AV + o) = make_uint4(vh4[0], vh4[1], vh4[2], vh4[3]);
        *reinterpret_cast<uint4*>(AV + kT128 + o) = make_uint4(vl4[0], vl4[1], vl4[2], vl4[3]);
        *reinterpret_cast<uint4*>(AG + o) = make_uint4(kh4[0], kh4[1], kh4[2], kh4[3]);
        *reinterpret_cast<uint4*>(AG + kT128 + o) = make_uint4(kl4[0], kl4[1], kl4[2], kl4[3]);
    }
    if (tid == 0) p.gC[(size_t)vh * nch + c] = expf(GC);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    constexpr uint32_t idesc = tc::idesc_bf16(128, 64);
    const uint32_t akq = smem_u32(AKQ), tb = smem_u32(TB), av = smem_u32(AV), ag = smem_u32(AG);
    if (tid == 0) {
        // [K K^T; Q K^T]: B = the first 64 rows (the K rows) of the same tiles
        for (int kc = 0; kc < 2; ++kc) {
            const uint64_t ah = tc::desc128(akq + kc * kT128), al = tc::desc128(akq + (2 + kc) * kT128);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                tc::mma_ss(tmem, ah + adv, ah + adv, idesc, (kc | ks) != 0 ? 1u : 0u);
                tc::mma_ss(tmem, ah + adv, al + adv, idesc, 1u);
                tc::mma_ss(tmem, al + adv, ah + adv, idesc, 1u);
            }
        }
        tc::commit(mma1);
    }
    bool ok = mbar_wait_bounded(mma1, 0u, err, DEV_TC_EPI_TIMEOUT);
    ok = __all_sync(0xffffffffu, ok);
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    if (ok) {
        tc::fence_after();
        uint32_t r[4][16];
#pragma unroll
        for (int q = 0; q < 4; ++q) tc::ld16_nowait(trow + q * 16, r[q]);
        tc::ld_wait();
        const int i = tid & 63;
        const float Gi = Gc[i];
        if (tid < 64) {
            // L[i][j] = exp(G_i - G_j) b_j (k_i . k_j) for j < i (rows past the chunk: 0)
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const float f = (j < i && i < n) ? expf(Gi - Gc[j]) * Bs[j] : 0.f;
                Lt[j * kLtP + i] = f * __uint_as_float(r[j >> 4][j & 15]);
            }
        } else {
            // P[i][j] = exp(G_i - G_j) b_j (q_i . k_j) for j <= i, as bf16 pairs
            uint16_t* Pg = p.P + (((size_t)vh * nch + c) * 2 * kGC + i) * kGC;
#pragma unroll
            for (int j0 = 0; j0 < 64; j0 += 8) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = j0 + 2 * u;
                    const float f0 = (j <= i && i < n) ? expf(Gi - Gc[j]) * Bs[j] : 0.f;
                    const float f1 = (j + 1 <= i && i < n) ? expf(Gi - Gc[j + 1]) * Bs[j + 1] : 0.f;
                    tc::split2(f0 * __uint_as_float(r[j >> 4][j & 15]), f1 * __uint_as_float(r[(j + 1) >> 4][(j + 1) & 15]),
                               hw[u], lw[u]);
                }
                *reinterpret_cast<uint4*>(Pg + j0) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4*>(Pg + kGC * kGC + j0) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
        }
    }
    if (tid < 64) asm volatile("bar.sync 1, 64;" ::: "memory");  // threads 0-63: L^T complete
    if (ok && tid < 64) {
        // column j = tid of T = (I + L)^-1: t = e_j, then for m = 0..62: t_i -= L[i][m] t_m (i > m)
        const int j = tid;
        float t[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) t[i] = (i == j) ? 1.f : 0.f;
#pragma unroll
        for (int m = 0; m < 63; ++m) {
            const float tm = t[m];
            const float* lc = Lt + m * kLtP;
#pragma unroll
            for (int i = m + 1; i < 64; ++i) t[i] -= lc[i] * tm;
        }
        // T as the B operand of step 3: row i, column (K index) m = j
#pragma unroll
        for (int i = 0; i < 64; ++i) {
            uint16_t hi, lo;
            split_bf16(t[i], hi, lo);
            const uint32_t o = sw_off(i, j);
            *reinterpret_cast<uint16_t*>(TB + o) = hi;
            *reinterpret_cast<uint16_t*>(TB + kT64 + o) = lo;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0) {
        if (ok) {
            const uint64_t bh = tc::desc128(tb), bl = tc::desc128(tb + kT64);
            const uint64_t vhd = tc::desc128(av), vld = tc::desc128(av + kT128);
            const uint64_t ghd = tc::desc128(ag), gld = tc::desc128(ag + kT128);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                tc::mma_ss(tmem + 64, vhd + adv, bh + adv, idesc, ks != 0 ? 1u : 0u);
                tc::mma_ss(tmem + 64, vhd + adv, bl + adv, idesc, 1u);
                tc::mma_ss(tmem + 64, vld + adv, bh + adv, idesc, 1u);
                tc::mma_ss(tmem + 128, ghd + adv, bh + adv, idesc, ks != 0 ? 1u : 0u);
                tc::mma_ss(tmem + 128, ghd + adv, bl + adv, idesc, 1u);
                tc::mma_ss(tmem + 128, gld + adv, bh + adv, idesc, 1u);
            }
        }
        tc::commit(mma2);
    }
    ok = mbar_wait_bounded(mma2, 0u, err, DEV_TC_EPI_TIMEOUT) && ok;
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
        tc::fence_after();
        // row tid of U^T / W^T = column tid of U / W
        // W is kept transposed per chunk (row = key dim, 64 tokens; rows past the chunk's
        // tokens are zero), so this thread's row is 256 contiguous bytes
        float* wt = p.W + (((size_t)vh * nch + c) * 128 + tid) * kGC;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
            uint32_t ru[16], rw[16];
            tc::ld16_nowait(trow + 64 + q * 16, ru);
            tc::ld16_nowait(trow + 128 + q * 16, rw);
            tc::ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int i = q * 16 + e;
                if (i < n) p.U[hrow + (size_t)i * 128 + tid] = __uint_as_float(ru[e]);
            }
#pragma unroll
            for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<uint4*>(wt + q * 16 + e) = make_uint4(rw[e], rw[e + 1], rw[e + 2], rw[e + 3]);
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, 256);
    }
}

// Kernel B1: the state recurrence across chunks, S_{c+1} = gamma_C S_c + Kd^T (U - W S_c).
// Columns of S evolve independently, so each CTA owns a (value head, WS-column slice) and
// walks the chunks in order; the next chunk's W, Kd and U slice are fetched (cp.async)
// while the current one is applied. For the output kernel B2 it writes the state entering
// every chunk and E = U - W S_c, both transposed (value dims as rows) as bf16 pairs; then
// the final state.
//
// The walk is sequential, so a launch takes (chunks x per-chunk time) however few CTAs
// it has. The arithmetic per chunk is proportional to WS and the fetch is not: with many
// value heads (one GPU) 16-column slices fill the SMs; a tensor-parallel rank holds VH / N
// heads, and narrower slices (8, 4 columns) give it as many CTAs and a shorter chunk step.
// Shared-memory strides (floats), chosen so that the float4 reads of the two products take
// the fewest wavefronts: in E = U - W S a warp reads W^T rows kq (the key-dim split) x 2
// token quads and S rows kq x the slice's column quads; in the update, Kd rows kh x 4
// key-dim quads and E rows kh x the column quads. A W^T stride = 8 (mod 32) banks, a Kd
// stride = 16 (mod 32) and unpadded S rows put those sets on distinct bank groups (with the
// earlier strides 68 / 132 / WS + 4, 39 % of the shared-memory wavefronts of a launch were
// bank conflicts and short-scoreboard stalls were 45 % of the samples). E and U keep WS + 4:
// E is also read transposed (one token per lane) for its bf16-pair copy.
constexpr int kWtP = kGC + 8;          // W^T rows
constexpr int kKdP = 128 + 16;         // Kd rows
template <int WS>
struct GdnStateCfg {
    static constexpr int P = WS + 4;                                // stride of the E and U tiles
    static constexpr int PS = WS;                                   // stride of the S tile
    static constexpr int Buf = 128 * kWtP + kGC * kKdP + kGC * P;   // floats per chunk buffer: W^T, Kd, U slice
    static constexpr size_t Smem = (size_t)(2 * Buf + 128 * PS + kGC * P) * 4;
    static constexpr int KS = 64 / WS;   // E = U - W S: lanes sharing one 4 x 4 tile (key-dim split)
    static constexpr int KH = 32 / WS;   // S update: lanes sharing one 4 x 4 tile (token split)
    static_assert(WS == 4 || WS == 8 || WS == 16, "state slice width");
};
__device__ __forceinline__ void cp16(float* dst, const float* src, bool pred) {
    const uint32_t d = smem_u32(dst);
    const int n = pred ? 16 : 0;  // 0: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
template <int WS>
__global__ void __launch_bounds__(256) k_pf_gdn_state(const PfGdnChunk p) {
    using C = GdnStateCfg<WS>;
    constexpr int P = C::P, PS = C::PS, KS = C::KS, KH = C::KH, Q4 = WS / 4;
    extern __shared__ __align__(16) float sb[];
    float* Ssm = sb + 2 * C::Buf;        // [128][PS]
    float* Esm = Ssm + 128 * PS;         // [64][P]
    const int vh = blockIdx.x / (128 / WS), sl = blockIdx.x % (128 / WS), tid = threadIdx.x;
    const int nch = (p.T + kGC - 1) / kGC;
    float* Sg = p.state + (size_t)vh * 128 * 128 + sl * WS;
    for (int e = tid; e < 128 * Q4; e += 256) {
        const int r = e / Q4, c4 = (e % Q4) * 4;
        *reinterpret_cast<float4*>(Ssm + r * PS + c4) = *reinterpret_cast<const float4*>(Sg + (size_t)r * 128 + c4);
    }
    auto fetch = [&](int c) {
        float* B = sb + (c & 1) * C::Buf;
        const int t0 = c * kGC, n = min(kGC, p.T - t0);
        const size_t hrow = ((size_t)vh * p.T + t0) * 128;
        const float* wt = p.W + ((size_t)vh * nch + c) * 128 * kGC;
        for (int e = tid; e < 128 * (kGC / 4); e += 256) {  // W^T rows: all 64 tokens (zeros past n)
            const int r = e >> 4, c4 = (e & 15) * 4;
            cp16(B + r * kWtP + c4, wt + (size_t)r * kGC + c4, true);
        }
        float* Bk = B + 128 * kWtP;
        for (int e = tid; e < kGC * 32; e += 256) {
            const int i = e >> 5, c4 = (e & 31) * 4;
            const size_t off = hrow + (size_t)(i < n ? i : 0) * 128 + c4;
            cp16(Bk + i * kKdP + c4, p.KD + off, i < n);
        }
        for (int e = tid; e < kGC * Q4; e += 256) {
            const int i = e / Q4, c4 = (e % Q4) * 4;
            cp16(Bk + kGC * kKdP + i * P + c4, p.U + hrow + (size_t)(i < n ? i : 0) * 128 + sl * WS + c4, i < n);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(0);
    // E: 4 x 4 tile (rows ei.., columns ec..) over every KS-th key dim (kq = lane % KS), the
    // KS partial tiles summed across lanes; state update: 4 x 4 tile (key dims sr.., columns
    // sc..) over every KH-th token (kh = lane % KH), summed across the KH lanes
    const int kq = tid % KS, et = tid / KS, ei = (et / Q4) * 4, ec = (et % Q4) * 4;
    const int kh = tid % KH, stl = tid / KH, sr = (stl / Q4) * 4, sc = (stl % Q4) * 4;
    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            fetch(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // chunk c's operands and the state are visible to every thread
        const float* Wts = sb + (c & 1) * C::Buf;  // W^T [128][kWtP]
        const float* Ksm = Wts + 128 * kWtP;         // Kd [64][kKdP]
        const float* Usm = Ksm + kGC * kKdP;          // U slice [64][P]
        // the state entering chunk c, transposed (rows = value dims) as bf16 pairs, for the
        // output kernel: thread -> key dim k = tid % 128 and WS / 2 value dims from
        // (tid / 128) WS / 2 (a warp's stores cover 32 consecutive key dims)
        {
            constexpr int V = WS / 2;
            const int k = tid & 127, d0 = (tid >> 7) * V;
            uint16_t* st = p.ST + (((size_t)vh * nch + c) * 2 * 128 + sl * WS + d0) * 128 + k;
            float v[V];
            if constexpr (V % 4 == 0) {  // vector reads of the row (fewer wavefronts than scalars)
#pragma unroll
                for (int q = 0; q < V / 4; ++q) {
                    const float4 f = *reinterpret_cast<const float4*>(Ssm + k * PS + d0 + 4 * q);
                    v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int u = 0; u < V; ++u) v[u] = Ssm[k * PS + d0 + u];
            }
#pragma unroll
            for (int u = 0; u < V; ++u) {
                uint16_t hi, lo;
                split_bf16(v[u], hi, lo);
                st[u * 128] = hi;
                st[128 * 128 + u * 128] = lo;
            }
        }
        // E = U - W S
        {
            float acc[4][4];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
            for (int it = 0; it < 128 / KS; ++it) {
                const int r = it * KS + kq;
                const float4 w4 = *reinterpret_cast<const float4*>(Wts + r * kWtP + ei);
                const float4 s4 = *reinterpret_cast<const float4*>(Ssm + r * PS + ec);
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int x = 0; x < 4; ++x)
#pragma unroll
                    for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(wv[x], sv[y], acc[x][y]);
            }
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y)
#pragma unroll
                    for (int o = 1; o < KS; o <<= 1) acc[x][y] += __shfl_xor_sync(0xffffffffu, acc[x][y], o);
            // lane kq < 4 of the group stores row ei + kq of the tile
            if (kq < 4) {
                const float4 u4 = *reinterpret_cast<const float4*>(Usm + (ei + kq) * P + ec);
                float rowv[4];
#pragma unroll
                for (int y = 0; y < 4; ++y)
                    rowv[y] = kq == 0 ? acc[0][y] : (kq == 1 ? acc[1][y] : (kq == 2 ? acc[2][y] : acc[3][y]));
                *reinterpret_cast<float4*>(Esm + (ei + kq) * P + ec) =
                    make_float4(u4.x - rowv[0], u4.y - rowv[1], u4.z - rowv[2], u4.w - rowv[3]);
            }
        }
        __syncthreads();  // E complete; every read of S for E done
        // E^T of the slice as bf16 pairs (rows = value dims, 64 token columns; rows past the
        // chunk's tokens are zero): thread -> token j = tid % 64 and WS / 4 value dims from
        // (tid / 64) WS / 4
        {
            const int j = tid & 63, d0 = (tid >> 6) * Q4;
            uint16_t* et = p.ET + (((size_t)vh * nch + c) * 2 * 128 + sl * WS + d0) * kGC + j;
#pragma unroll
            for (int u = 0; u < Q4; ++u) {
                uint16_t hi, lo;
                split_bf16(Esm[j * P + d0 + u], hi, lo);
                et[u * kGC] = hi;
                et[128 * kGC + u * kGC] = lo;
            }
        }
        // S = gamma_C S + Kd^T E (each lane group reads and writes only its own S tile here)
        {
            const float gC = p.gC[(size_t)vh * nch + c];
            float acc[4][4];
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
            for (int it = 0; it < kGC / KH; ++it) {  // rows past the chunk's tokens are zero
                const int i = it * KH + kh;
                const float4 k4 = *reinterpret_cast<const float4*>(Ksm + i * kKdP + sr);
                const float4 e4 = *reinterpret_cast<const float4*>(Esm + i * P + sc);
                const float kv4[4] = {k4.x, k4.y, k4.z, k4.w}, ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
                for (int x = 0; x < 4; ++x)
#pragma unroll
                    for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(kv4[x], ev[y], acc[x][y]);
            }
#pragma unroll
            for (int x = 0; x < 4; ++x)
#pragma unroll
                for (int y = 0; y < 4; ++y)
#pragma unroll
                    for (int o = 1; o < KH; o <<= 1) acc[x][y] += __shfl_xor_sync(0xffffffffu, acc[x][y], o);
            // the tile's 4 rows over the KH lanes of the group: RPL rows each (lanes past the
            // 4 rows idle)
            constexpr int RPL = KH >= 4 ? 1 : 4 / KH;
#pragma unroll
            for (int x2 = 0; x2 < RPL; ++x2) {
                const int x = kh * RPL + x2;
                if (x < 4) {
                    float* srow = Ssm + (sr + x) * PS + sc;
                    const float4 s4 = *reinterpret_cast<const float4*>(srow);
                    float a[4];
#pragma unroll
                    for (int y = 0; y < 4; ++y)
                        a[y] = x == 0 ? acc[0][y] : (x == 1 ? acc[1][y] : (x == 2 ? acc[2][y] : acc[3][y]));
                    *reinterpret_cast<float4*>(srow) =
                        make_float4(gC * s4.x + a[0], gC * s4.y + a[1], gC * s4.z + a[2], gC * s4.w + a[3]);
                }
            }
        }
        __syncthreads();  // new S visible; chunk c's buffer free for the fetch of chunk c + 2
    }
    for (int e = tid; e < 128 * Q4; e += 256) {
        const int r = e / Q4, c4 = (e % Q4) * 4;
        *reinterpret_cast<float4*>(Sg + (size_t)r * 128 + c4) = *reinterpret_cast<const float4*>(Ssm + r * PS + c4);
    }
}

// Column-slice width of the state pass: the narrowest of 16 / 8 / 4 that keeps about a
// wave of CTAs (QWC_GDN_STATE_COLS forces one).
static int gdn_state_cols(int VH) {
    const char* e = std::getenv("QWC_GDN_STATE_COLS");
    const int forced = e ? std::atoi(e) : 0;
    if (forced == 4 || forced == 8 || forced == 16) return forced;
    int cols = 16;
    while (cols > 4 && VH * (128 / cols) * 2 <= num_sms()) cols /= 2;
    return cols;
}

// Kernel B2 on the tensor cores: per (chunk, value head) the outputs, transposed,
//   O^T [128 value dims][64 tokens] = S_c^T (Gamma Q)^T + E^T P^T,
// each product with bf16-pair operands taken three times (hi hi + hi lo + lo hi) into an
// fp32 accumulator in tensor memory (64 columns): 24 + 12 MMAs of M128 N64 K16. Operands
// arrive by TMA (no multicast), all K-major with 128-byte swizzle: S_c^T [128][128] and
// E^T [128][64] as A, Gamma Q [64 tokens][128] and P [64][64] as B. Thread = value dim
// (its TMEM lane) in the epilogue; a warp's 32 lanes store 32 consecutive outputs.
constexpr uint32_t kGdnOutBytes = 4 * kT128 + 4 * kT64 + 2 * kT128 + 2 * kT64;
constexpr size_t kGdnOutSmem = kGdnOutBytes + 1024 + 64;
__global__ void __launch_bounds__(128, 1)
    k_pf_gdn_out_tc(const __grid_constant__ CUtensorMap mST, const __grid_constant__ CUtensorMap mQG,
                    const __grid_constant__ CUtensorMap mET, const __grid_constant__ CUtensorMap mP, const PfGdnChunk p,
                    int* err) {
    extern __shared__ uint8_t so_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(so_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* A1 = sm;                // S^T tiles [hi|lo][key dims 0-63 | 64-127]
    uint8_t* B1 = A1 + 4 * kT128;    // Gamma Q tiles [hi|lo][key dims 0-63 | 64-127]
    uint8_t* A2 = B1 + 4 * kT64;     // E^T tiles [hi|lo]
    uint8_t* B2 = A2 + 2 * kT128;    // P tiles [hi|lo]
    uint64_t* bar = reinterpret_cast<uint64_t*>(B2 + 2 * kT64);
    uint64_t* full = bar;
    uint64_t* done = bar + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 2);
    int* s_ok = reinterpret_cast<int*>(tmem_slot + 1);
    const int c = blockIdx.x, vh = blockIdx.y, nch = gridDim.x, tid = threadIdx.x, warp = tid >> 5;
    const int t0 = c * kGC, n = min(kGC, p.T - t0), Tpad = nch * kGC;
    if (tid == 0) {
        mbar_init(full, 1);
        mbar_init(done, 1);
        *s_ok = 1;
        fence_mbar_init();
    }
    if (warp == 0) tc::tmem_alloc(tmem_slot, 64);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) {
        mbar_arrive_expect_tx(full, kGdnOutBytes);
        const int rs = (vh * nch + c) * 2 * 128;  // hi row of S^T / E^T
        const int rq = vh * 2 * Tpad + t0;        // hi row of Gamma Q
        const int rp = (vh * nch + c) * 2 * kGC;  // hi row of P
        for (int hl = 0; hl < 2; ++hl) {
            for (int kc = 0; kc < 2; ++kc) {
                tc::tma2d(A1 + (hl * 2 + kc) * kT128, &mST, kc * 64, rs + hl * 128, full);
                tc::tma2d(B1 + (hl * 2 + kc) * kT64, &mQG, kc * 64, rq + hl * Tpad, full);
            }
            tc::tma2d(A2 + hl * kT128, &mET, 0, rs + hl * 128, full);
            tc::tma2d(B2 + hl * kT64, &mP, 0, rp + hl * kGC, full);
        }
        if (mbar_wait_bounded(full, 0u, err, DEV_TC_MMA_TIMEOUT)) {
            tc::fence_after();
            constexpr uint32_t idesc = tc::idesc_bf16(128, 64);
            const uint32_t a1 = smem_u32(A1), b1 = smem_u32(B1), a2 = smem_u32(A2), b2 = smem_u32(B2);
            for (int kc = 0; kc < 2; ++kc) {
                const uint64_t ah = tc::desc128(a1 + kc * kT128), al = tc::desc128(a1 + (2 + kc) * kT128);
                const uint64_t bh = tc::desc128(b1 + kc * kT64), bl = tc::desc128(b1 + (2 + kc) * kT64);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                    tc::mma_ss(tmem, ah + adv, bh + adv, idesc, (kc | ks) != 0 ? 1u : 0u);
                    tc::mma_ss(tmem, ah + adv, bl + adv, idesc, 1u);
                    tc::mma_ss(tmem, al + adv, bh + adv, idesc, 1u);
                }
            }
            const uint64_t ah = tc::desc128(a2), al = tc::desc128(a2 + kT128);
            const uint64_t bh = tc::desc128(b2), bl = tc::desc128(b2 + kT64);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                tc::mma_ss(tmem, ah + adv, bh + adv, idesc, 1u);
                tc::mma_ss(tmem, ah + adv, bl + adv, idesc, 1u);
                tc::mma_ss(tmem, al + adv, bh + adv, idesc, 1u);
            }
        } else {
            *reinterpret_cast<volatile int*>(s_ok) = 0;
            mbar_wait_bounded(full, 0u, err, DEV_TC_DRAIN_TIMEOUT);  // loads in flight land first
        }
        tc::commit(done);  // arrives once every MMA above has completed
    }
    bool ok = mbar_wait_bounded(done, 0u, err, DEV_TC_EPI_TIMEOUT);
    ok = __all_sync(0xffffffffu, ok && *reinterpret_cast<volatile int*>(s_ok) != 0);
    if (ok) {
        tc::fence_after();
        const int dv = warp * 32 + (tid & 31);
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
        float* o = p.out + (size_t)t0 * p.VD + vh * 128 + dv;
#pragma unroll 1
        for (int q = 0; q < 4; ++q) {
            uint32_t r[16];
            tc::ld16_nowait(taddr + q * 16, r);
            tc::ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int t = q * 16 + e;
                if (t < n) o[(size_t)t * p.VD] = __uint_as_float(r[e]);
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, 64);
    }
}

// ---------------------------------------------------------------- gated RMSNorm -> split
// xs[t][h*D + i] = split(w[i] * (o[i] * inv_rms(o_h)) * silu(z[i])) (rmsnorm_gated,
// forward_pass.cpp:86-93); one warp per head.
__global__ void __launch_bounds__(kPT) k_pf_gated_norm_split(const float* o, long ldo, const float* z, long ldz,
                                                              const float* w, int nh, float eps, uint16_t* xs,
                                                              long ldxs) {
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = nh * 128;
    for (int h = warp; h < nh; h += kPT / 32) {
        const float* oo = o + (size_t)t * ldo + h * 128;
        const float* zz = z + (size_t)t * ldz + h * 128;
        float ov[4], zv[4];
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            ov[j] = oo[lane + 32 * j];
            zv[j] = zz[lane + 32 * j];
            ss += (double)ov[j] * ov[j];
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
        const float inv = 1.0f / sqrtf((float)(ss / 128) + eps);
        uint16_t* row = xs + (size_t)t * ldxs;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = lane + 32 * j;
            store_split(row, K, h * 128 + i, w[i] * (ov[j] * inv) * silu_f(zv[j]));
        }
    }
}

// ---------------------------------------------------------------- attention preparation
// Per token: q heads normalised ((1+w) q_norm) and rotated into qbuf; k normalised and
// rotated, v raw, both appended to the cache at position p0 + t (attn_step,
// qwen_model.cpp:118-132). One warp per head vector (warp_norm_rope of the decode kernel).
struct PfAttnPrep {
    const float* proj;  // [T][ldp]: NQ x [q 256 | gate 256], NKV x k, NKV x v
    long ldp;
    const float* qn1;
    const float* kn1;
    const float* rope_cs;  // [max_ctx][rot/2][2]
    float* qbuf;           // [T][NQ][HD]
    void* k_cache;         // [NKV][max_ctx][HD]
    void* v_cache;
    int kv_bf16, max_ctx, p0, NQ, NKV, rot;
    float eps;
    // tensor-core attention operands (null: not written): K as bf16 pairs
    // [NKV][ctx_pad][hi 256 | lo 256], V likewise [NKV][T][hi | lo] for this chunk
    uint16_t* ksplit;
    uint16_t* vsplit;
    int ctx_pad, T;
};
// 8 values -> bf16 hi at dst[0..8), lo at dst[256..264) (16-byte stores)
__device__ __forceinline__ void store_split8(uint16_t* dst, const float (&x)[8]) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint16_t h0 = f2bf(x[2 * e]), h1 = f2bf(x[2 * e + 1]);
        const uint16_t l0 = f2bf(x[2 * e] - bf16lo(h0)), l1 = f2bf(x[2 * e + 1] - bf16lo(h1));
        hw[e] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        lw[e] = (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(dst + kHD) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}
__global__ void __launch_bounds__(kPT) k_pf_attn_prep(const PfAttnPrep p) {
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = p.p0 + t;
    const float* row = p.proj + (size_t)t * p.ldp;
    const float* cs = p.rope_cs + (size_t)pos * p.rot;
    for (int v = warp; v < p.NQ + 2 * p.NKV; v += kPT / 32) {
        const float* src;
        if (v < p.NQ) src = row + (size_t)v * 2 * kHD;
        else if (v < p.NQ + p.NKV) src = row + (size_t)p.NQ * 2 * kHD + (size_t)(v - p.NQ) * kHD;
        else src = row + (size_t)p.NQ * 2 * kHD + (size_t)p.NKV * kHD + (size_t)(v - p.NQ - p.NKV) * kHD;
        float x[8];
        const float4 a = reinterpret_cast<const float4*>(src + lane * 8)[0];
        const float4 b = reinterpret_cast<const float4*>(src + lane * 8)[1];
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        if (v < p.NQ + p.NKV) warp_norm_rope(x, v < p.NQ ? p.qn1 : p.kn1, p.eps, p.rot, cs);
        if (v < p.NQ) {
            float4* d = reinterpret_cast<float4*>(p.qbuf + ((size_t)t * p.NQ + v) * kHD + lane * 8);
            d[0] = make_float4(x[0], x[1], x[2], x[3]);
            d[1] = make_float4(x[4], x[5], x[6], x[7]);
        } else {
            const int kv = v < p.NQ + p.NKV ? v - p.NQ : v - p.NQ - p.NKV;
            void* cache = v < p.NQ + p.NKV ? p.k_cache : p.v_cache;
            const size_t off = ((size_t)kv * p.max_ctx + pos) * kHD + lane * 8;
            if (p.ksplit) {
                // the split carries the value the cache holds (bf16-rounded for a bf16 cache)
                float y[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = p.kv_bf16 ? bf16lo(f2bf(x[e])) : x[e];
                uint16_t* dst = v < p.NQ + p.NKV ? p.ksplit + ((size_t)kv * p.ctx_pad + pos) * 2 * kHD
                                                 : p.vsplit + ((size_t)kv * p.T + t) * 2 * kHD;
                store_split8(dst + lane * 8, y);
            }
            if (p.kv_bf16) {
                uint4 u;
                u.x = (uint32_t)f2bf(x[0]) | ((uint32_t)f2bf(x[1]) << 16);
                u.y = (uint32_t)f2bf(x[2]) | ((uint32_t)f2bf(x[3]) << 16);
                u.z = (uint32_t)f2bf(x[4]) | ((uint32_t)f2bf(x[5]) << 16);
                u.w = (uint32_t)f2bf(x[6]) | ((uint32_t)f2bf(x[7]) << 16);
                *reinterpret_cast<uint4*>(static_cast<uint16_t*>(cache) + off) = u;
            } else {
                float4* d = reinterpret_cast<float4*>(static_cast<float*>(cache) + off);
                d[0] = make_float4(x[0], x[1], x[2], x[3]);
                d[1] = make_float4(x[4], x[5], x[6], x[7]);
            }
        }
    }
}

// ---------------------------------------------------------------- causal attention
// CTA = (kv head, block of 64/GRP query tokens): 64 query rows (GRP heads x tokens),
// key tiles of 32 positions through shared memory, online softmax per row in fp32
// (softmax(q K^T / sqrt(HD)) over positions <= the query's, attn_step :134-149), then the
// sigmoid gate (:150); the result is written as hi/lo pairs for o_proj.
struct PfAttn {
    const float* qbuf;   // [T][NQ][HD]
    const float* proj;   // gate source: [T][ldp], head h gate at h*2*HD + HD
    long ldp;
    const void* k_cache;
    const void* v_cache;
    int kv_bf16, max_ctx, p0, T, NQ, NKV;
    uint16_t* xs;        // [T][ldxs], K = NQ*HD
    long ldxs;
};
// Row strides of 260 floats: float4 reads of 8 rows that are 1 (K) or 2 (Q) apart hit
// distinct bank groups.
constexpr int kAR = 64, kAK = 32, kKPad = kHD + 4;
constexpr size_t kAttnSmem = (size_t)(kAR * kKPad + kAK * kKPad + kAK * kHD + kAR * (kAK + 1) + 3 * kAR) * 4;
template <int GRP>
__global__ void __launch_bounds__(256, 1) k_pf_attn(const PfAttn p) {
    constexpr int BQT = kAR / GRP;  // query tokens per CTA
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                     // [64][260]
    float* Ks = Qs + kAR * kKPad;       // [32][260]
    float* Vs = Ks + kAK * kKPad;       // [32][256]
    float* Ps = Vs + kAK * kHD;         // [64][33]
    float* row_m = Ps + kAR * (kAK + 1);
    float* row_l = row_m + kAR;
    float* row_sc = row_l + kAR;
    const int tid = threadIdx.x;
    const int kv = blockIdx.x, t0 = blockIdx.y * BQT;
    const float scale = 1.0f / sqrtf((float)kHD);
    // rows: r = g * BQT + i  (query head kv*GRP + g, token t0 + i)
    for (int e = tid; e < kAR * (kHD / 4); e += 256) {
        const int r = e / (kHD / 4), c4 = e % (kHD / 4);
        const int g = r / BQT, i = r % BQT, t = t0 + i;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < p.T) v = reinterpret_cast<const float4*>(p.qbuf + ((size_t)t * p.NQ + kv * GRP + g) * kHD)[c4];
        reinterpret_cast<float4*>(Qs + r * kKPad)[c4] = v;
    }
    if (tid < kAR) { row_m[tid] = -INFINITY; row_l[tid] = 0.f; }
    // output accumulators: rows ro..ro+3, columns c = cb*4 + 64*j (+0..3)
    const int ro = (tid >> 4) * 4, cb = tid & 15;
    float acc[4][16];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 16; ++b) acc[a][b] = 0.f;
    const int last_t = min(t0 + BQT, p.T) - 1;
    const int n_keys = p.p0 + last_t + 1;  // keys 0 .. p0 + last_t
    const size_t kvbase = (size_t)kv * p.max_ctx * kHD;
    // score tiling: rows 2*(tid>>3) .. +1, keys (tid&7) + 8b for b < 4
    const int sr = (tid >> 3) * 2, kq = tid & 7;
    for (int k0 = 0; k0 < n_keys; k0 += kAK) {
        __syncthreads();  // previous tile fully consumed
        for (int e = tid; e < kAK * (kHD / 8); e += 256) {
            const int j = e / (kHD / 8), c8 = (e % (kHD / 8)) * 8;
            float kk[8], vv[8];
            if (k0 + j < n_keys) {
                load8(p.k_cache, p.kv_bf16, kvbase + (size_t)(k0 + j) * kHD + c8, kk);
                load8(p.v_cache, p.kv_bf16, kvbase + (size_t)(k0 + j) * kHD + c8, vv);
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) { kk[q] = 0.f; vv[q] = 0.f; }
            }
            float4* kd = reinterpret_cast<float4*>(Ks + j * kKPad + c8);
            kd[0] = make_float4(kk[0], kk[1], kk[2], kk[3]);
            kd[1] = make_float4(kk[4], kk[5], kk[6], kk[7]);
            float4* vd = reinterpret_cast<float4*>(Vs + j * kHD + c8);
            vd[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
            vd[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
        }
        __syncthreads();
        // scores
        float s[2][4];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) s[a][b] = 0.f;
#pragma unroll 4
        for (int d = 0; d < kHD; d += 4) {
            const float4 q0 = *reinterpret_cast<const float4*>(Qs + sr * kKPad + d);
            const float4 q1 = *reinterpret_cast<const float4*>(Qs + (sr + 1) * kKPad + d);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const float4 kk = *reinterpret_cast<const float4*>(Ks + (kq + 8 * b) * kKPad + d);
                s[0][b] += q0.x * kk.x + q0.y * kk.y + q0.z * kk.z + q0.w * kk.w;
                s[1][b] += q1.x * kk.x + q1.y * kk.y + q1.z * kk.z + q1.w * kk.w;
            }
        }
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            const int r = sr + a, t = t0 + r % BQT, qpos = p.p0 + t;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int kp = k0 + kq + 8 * b;
                Ps[r * (kAK + 1) + kq + 8 * b] = (kp <= qpos && t < p.T) ? s[a][b] * scale : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax: 4 threads per row, 8 keys each
        {
            const int r = tid >> 2, part = tid & 3;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; ++j) mx = fmaxf(mx, Ps[r * (kAK + 1) + part * 8 + j]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            const float mo = row_m[r];
            const float mn = fmaxf(mo, mx);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float& sv = Ps[r * (kAK + 1) + part * 8 + j];
                const float e = sv == -INFINITY ? 0.f : expf(sv - mn);
                sv = e;
                sum += e;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            __syncwarp();
            if (part == 0) {
                const float corr = (mo == -INFINITY) ? 0.f : expf(mo - mn);
                row_sc[r] = corr;
                row_l[r] = row_l[r] * corr + sum;
                row_m[r] = mn;
            }
        }
        __syncthreads();
        // O = O * corr + P V
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const float c = row_sc[ro + a];
#pragma unroll
            for (int b = 0; b < 16; ++b) acc[a][b] *= c;
        }
        for (int j = 0; j < kAK; ++j) {
            float pv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pv[a] = Ps[(ro + a) * (kAK + 1) + j];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(Vs + j * kHD + cb * 4 + 64 * q);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    acc[a][4 * q] += pv[a] * v.x;
                    acc[a][4 * q + 1] += pv[a] * v.y;
                    acc[a][4 * q + 2] += pv[a] * v.z;
                    acc[a][4 * q + 3] += pv[a] * v.w;
                }
            }
        }
    }
    __syncthreads();
    const int K = p.NQ * kHD;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int r = ro + a, g = r / BQT, t = t0 + r % BQT;
        if (t >= p.T) continue;
        const int h = kv * GRP + g;
        const float inv_l = 1.0f / row_l[r];
        const float* gate = p.proj + (size_t)t * p.ldp + (size_t)h * 2 * kHD + kHD;
        uint16_t* row = p.xs + (size_t)t * p.ldxs;
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int c = cb * 4 + 64 * q + e;
                store_split(row, K, h * kHD + c, acc[a][4 * q + e] * inv_l * sigmoid_f(gate[c]));
            }
    }
}

// ---------------------------------------------------------------- launchers
cudaError_t pf_embed(const int* ids, int T, const uint16_t* embed, int H, int V, float* hid, int* err,
                     cudaStream_t s) {
    k_pf_embed<<<T, kPT, 0, s>>>(ids, embed, H, V, hid, err);
    return cudaGetLastError();
}
cudaError_t pf_rmsnorm_split(const float* x, long ldx, int rows, const float* w1, int H, float eps, uint16_t* xs,
                             long ldxs, cudaStream_t s) {
    k_pf_rmsnorm_split<<<rows, kPT, 0, s>>>(x, ldx, w1, H, eps, xs, ldxs);
    return cudaGetLastError();
}
cudaError_t pf_gdn(const PfGdnArgs& a, cudaStream_t s) {
    if (a.VH % a.KH) return cudaErrorInvalidValue;
    PfGdnPrep pp{a.proj, a.ldp, a.a_in, a.b_in, a.ldab, a.conv_w, a.ring, a.neg_exp_A, a.dt_bias, a.qn, a.kn, a.vc,
                 a.glog, a.beta, a.p0, a.KH, a.VH, a.C, a.VD};
    k_pf_gdn_prep_tiled<<<dim3((a.T + kPrepT - 1) / kPrepT, 2 * a.KH + a.VH + 1), 128, 0, s>>>(pp, a.T);
    k_pf_conv_ring<<<(a.C + 255) / 256, 256, 0, s>>>(a.proj, a.ldp, a.T, a.p0, a.C, a.ring);
    if (!a.ST || !a.ET || !a.QG || !a.P) return cudaErrorInvalidValue;
    PfGdnChunk ck{a.qn, a.kn, a.vc, a.glog, a.beta, a.U, a.W, a.QG, a.KD, a.P, a.gC, a.ST, a.ET, a.state, a.out,
                  a.T, a.KH, a.VH, a.VD};
    {
        cudaError_t e = cudaFuncSetAttribute(k_pf_gdn_chunk_a_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdnATcSmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_state<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GdnStateCfg<16>::Smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_state<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GdnStateCfg<8>::Smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_state<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GdnStateCfg<4>::Smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_out_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdnOutSmem);
        if (e != cudaSuccess) return e;
    }
    const int nch = (a.T + kGC - 1) / kGC;
    const long Tpad = (long)nch * kGC, pl = (long)a.VH * nch * 2;
    CUtensorMap mST, mQG, mET, mP;
    if (tc_make_map_box(&mST, a.ST, pl * 128, 128, 128, 128) || tc_make_map_box(&mQG, a.QG, 2L * a.VH * Tpad, 128, 128, 64) ||
        tc_make_map_box(&mET, a.ET, pl * 128, kGC, kGC, 128) || tc_make_map_box(&mP, a.P, pl * kGC, kGC, kGC, 64))
        return cudaErrorInvalidValue;
    k_pf_gdn_chunk_a_tc<<<dim3(nch, a.VH), 128, kGdnATcSmem, s>>>(ck, a.err);
    if (a.ev_state0) cudaEventRecord(a.ev_state0, s);
    switch (gdn_state_cols(a.VH)) {
        case 4: k_pf_gdn_state<4><<<a.VH * 32, 256, GdnStateCfg<4>::Smem, s>>>(ck); break;
        case 8: k_pf_gdn_state<8><<<a.VH * 16, 256, GdnStateCfg<8>::Smem, s>>>(ck); break;
        default: k_pf_gdn_state<16><<<a.VH * 8, 256, GdnStateCfg<16>::Smem, s>>>(ck); break;
    }
    if (a.ev_state1) cudaEventRecord(a.ev_state1, s);
    k_pf_gdn_out_tc<<<dim3(nch, a.VH), 128, kGdnOutSmem, s>>>(mST, mQG, mET, mP, ck, a.err);
    return cudaGetLastError();
}
// scratch pieces of pf_gdn in bytes, in carving order
static void gdn_pieces(int KH, int VH, int T, size_t (&b)[13]) {
    const size_t t = (size_t)T, nch = (t + kGC - 1) / kGC, KD = (size_t)KH * 128, VD = (size_t)VH * 128;
    const size_t vh = (size_t)VH;
    const size_t v[13] = {t * KD * 4, t * KD * 4, t * VD * 4,            // qn, kn, vc
                          t * VD * 4, nch * kGC * VD * 4,                // U, W^T per chunk
                          vh * 2 * nch * kGC * 128 * 2,                  // Gamma Q pairs
                          t * VD * 4,                                    // Kd
                          t * vh * 4, t * vh * 4,                        // glog, beta
                          vh * nch * 2 * kGC * kGC * 2,                  // P pairs
                          vh * nch * 4,                                  // gamma_C
                          vh * nch * 2 * 128 * 128 * 2,                  // S^T pairs per chunk
                          vh * nch * 2 * 128 * kGC * 2};                 // E^T pairs per chunk
    for (int i = 0; i < 13; ++i) b[i] = (v[i] + 255) / 256 * 256;
}
size_t pf_gdn_workspace_bytes(int KH, int VH, int T) {
    size_t b[13], sum = 0;
    gdn_pieces(KH, VH, T, b);
    for (size_t x : b) sum += x;
    return sum;
}
int pf_gdn_carve(PfGdnArgs& a, void* ws, size_t bytes) {
    if (!ws || bytes < pf_gdn_workspace_bytes(a.KH, a.VH, a.T)) return -1;
    size_t b[13];
    gdn_pieces(a.KH, a.VH, a.T, b);
    uint8_t* base = static_cast<uint8_t*>(ws);
    void* ptr[13];
    for (int i = 0; i < 13; ++i) {
        ptr[i] = base;
        base += b[i];
    }
    a.qn = static_cast<float*>(ptr[0]);
    a.kn = static_cast<float*>(ptr[1]);
    a.vc = static_cast<float*>(ptr[2]);
    a.U = static_cast<float*>(ptr[3]);
    a.W = static_cast<float*>(ptr[4]);
    a.QG = static_cast<uint16_t*>(ptr[5]);
    a.KD = static_cast<float*>(ptr[6]);
    a.glog = static_cast<float*>(ptr[7]);
    a.beta = static_cast<float*>(ptr[8]);
    a.P = static_cast<uint16_t*>(ptr[9]);
    a.gC = static_cast<float*>(ptr[10]);
    a.ST = static_cast<uint16_t*>(ptr[11]);
    a.ET = static_cast<uint16_t*>(ptr[12]);
    return 0;
}

cudaError_t pf_gated_norm_split(const float* o, long ldo, const float* z, long ldz, const float* w, int T, int nh,
                                float eps, uint16_t* xs, long ldxs, cudaStream_t s) {
    k_pf_gated_norm_split<<<T, kPT, 0, s>>>(o, ldo, z, ldz, w, nh, eps, xs, ldxs);
    return cudaGetLastError();
}
cudaError_t pf_attention(const PfAttnArgs& a, cudaStream_t s) {
    if (a.rot > kHD || a.rot % 16 || a.NKV <= 0 || a.NQ % a.NKV) return cudaErrorInvalidValue;
    const bool tc = a.ksplit != nullptr;
    if (tc && (!a.vt || !a.vsplit || a.ctx_pad % 64 || a.p0 + a.T > a.ctx_pad)) return cudaErrorInvalidValue;
    PfAttnPrep pp{a.proj, a.ldp, a.qn1, a.kn1, a.rope_cs, a.qbuf, a.k_cache, a.v_cache,
                  a.kv_bf16, a.max_ctx, a.p0, a.NQ, a.NKV, a.rot, a.eps,
                  a.ksplit, a.vsplit, a.ctx_pad, a.T};
    k_pf_attn_prep<<<a.T, kPT, 0, s>>>(pp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (tc) {
        PfFattnArgs f;
        f.qbuf = a.qbuf;
        f.proj = a.proj;
        f.ldp = a.ldp;
        f.xs = a.xs;
        f.ldxs = a.ldxs;
        f.ksplit = a.ksplit;
        f.vt = a.vt;
        f.vsplit = a.vsplit;
        f.T = a.T;
        f.p0 = a.p0;
        f.NQ = a.NQ;
        f.NKV = a.NKV;
        f.ctx_pad = a.ctx_pad;
        f.part_o = a.part_o;
        f.part_ml = a.part_ml;
        f.part_splits = a.part_splits;
        f.err = a.err;
        return pf_fattn(f, s);
    }
    PfAttn at{a.qbuf, a.proj, a.ldp, a.k_cache, a.v_cache, a.kv_bf16, a.max_ctx, a.p0, a.T, a.NQ, a.NKV, a.xs, a.ldxs};
    const int grp = a.NQ / a.NKV;
    auto go = [&](auto kern, int bqt) -> cudaError_t {
        cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnSmem);
        if (e2 != cudaSuccess) return e2;
        dim3 grid(a.NKV, (a.T + bqt - 1) / bqt);
        kern<<<grid, 256, kAttnSmem, s>>>(at);
        return cudaGetLastError();
    };
    switch (grp) {
        case 1: return go(k_pf_attn<1>, kAR / 1);
        case 2: return go(k_pf_attn<2>, kAR / 2);
        case 4: return go(k_pf_attn<4>, kAR / 4);
        case 8: return go(k_pf_attn<8>, kAR / 8);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qwc
