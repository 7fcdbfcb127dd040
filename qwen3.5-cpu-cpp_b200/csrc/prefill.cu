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
#include "kernels.h"

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
// One warp per 128-channel head vector (q heads, k heads, v heads), 4 channels per lane.
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
__global__ void __launch_bounds__(kPT) k_pf_gdn_prep(const PfGdnPrep p) {
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KD = p.KH * 128;
    const int nvec = 2 * p.KH + p.VH;
    for (int v = warp; v < nvec; v += kPT / 32) {
        const int kind = v < p.KH ? 0 : (v < 2 * p.KH ? 1 : 2);
        const int head = kind == 0 ? v : (kind == 1 ? v - p.KH : v - 2 * p.KH);
        const int c0 = kind == 0 ? head * 128 : (kind == 1 ? KD + head * 128 : 2 * KD + head * 128);
        float val[4];
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = c0 + lane + 32 * j;
            // inputs at positions pos-3 .. pos (pos = p0 + t)
            float xin[4];
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int tt = t - 3 + d;
                if (tt >= 0) {
                    xin[d] = p.proj[(size_t)tt * p.ldp + c];
                } else {
                    const int pos = p.p0 + tt;
                    xin[d] = pos >= 0 ? p.ring[(size_t)c * 4 + (pos & 3)] : 0.f;
                }
            }
            const float4 w = reinterpret_cast<const float4*>(p.conv_w)[c];
            float acc = 0.f;
            acc += w.x * xin[0];
            acc += w.y * xin[1];
            acc += w.z * xin[2];
            acc += w.w * xin[3];
            val[j] = silu_f(acc);
            ss += (double)val[j] * val[j];
        }
        if (kind < 2) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.0f / sqrtf((float)ss + 1e-6f);
            float* dst = (kind == 0 ? p.qn : p.kn) + (size_t)t * KD + head * 128;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float x = val[j] * inv;
                if (kind == 0) x = x * (1.0f / sqrtf(128.0f));
                dst[lane + 32 * j] = x;
            }
        } else {
            float* dst = p.vc + (size_t)t * p.VD + head * 128;
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = val[j];
        }
    }
    for (int h = threadIdx.x; h < p.VH; h += kPT) {
        const float bv = p.b_in[(size_t)t * p.ldab + h], av = p.a_in[(size_t)t * p.ldab + h];
        const float g = p.neg_exp_A[h] * softplus_f(av + p.dt_bias[h]);
        p.glog[(size_t)t * p.VH + h] = g;  // log of the decay exp(g)
        p.beta[(size_t)t * p.VH + h] = sigmoid_f(bv);
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
// Kernel A (parallel over chunks and heads) builds U, W, Gamma Q, Kd, P and gamma_C;
// kernel B1 (sequential over chunks, parallel over heads and 16-column slices of S) applies
// E = U - W S, S = gamma_C S + Kd^T E and keeps the state entering each chunk; kernel B2
// (parallel over chunks and heads) forms O = (Gamma Q) S_c + P E. fp32 on CUDA cores.
constexpr int kGC = 64;            // tokens per chunk
constexpr int kGP = 128 + 4;       // padded row stride of 128-wide shared tiles
constexpr int kGLP = kGC + 1;      // padded row stride of 64 x 64 shared tiles
constexpr size_t kGdnASmem = (size_t)(3 * kGC * kGP + 2 * kGC * kGLP + 2 * kGC) * 4;

struct PfGdnChunk {
    const float* qn;     // [T][KD]
    const float* kn;     // [T][KD]
    const float* vc;     // [T][VD]
    const float* glog;   // [T][VH] g = log of the decay
    const float* beta;   // [T][VH]
    float* U;            // [VH][T][128]
    float* W;            // [VH][T][128]
    float* QG;           // [VH][T][128]  gamma_i q_i
    float* KD;           // [VH][T][128]  b_i exp(G_C - G_i) k_i
    float* P;            // [VH][nch][64][64]
    float* gC;           // [VH][nch]
    float* Sc;           // [VH][nch][DK][DV] state entering each chunk
    float* state;        // [VH][DK][DV]
    float* out;          // [T][VD]
    int T, KH, VH, VD;
};

__global__ void __launch_bounds__(256) k_pf_gdn_chunk_a(const PfGdnChunk p) {
    extern __shared__ __align__(16) float sa[];
    float* Ks = sa;                 // [64][132] k, later Gamma K -> W
    float* Qs = Ks + kGC * kGP;     // [64][132]
    float* Vs = Qs + kGC * kGP;     // [64][132] v -> U
    float* Ls = Vs + kGC * kGP;     // [64][65]
    float* Ps = Ls + kGC * kGLP;    // [64][65]
    float* Gc = Ps + kGC * kGLP;    // [64]
    float* Bs = Gc + kGC;           // [64]
    const int c = blockIdx.x, vh = blockIdx.y, tid = threadIdx.x;
    const int nch = gridDim.x;
    const int rep = p.VH / p.KH, kh = vh / rep, KD = p.KH * 128;
    const int t0 = c * kGC, n = min(kGC, p.T - t0);
    for (int e = tid; e < kGC * 32; e += 256) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f), q4 = k4, v4 = k4;
        if (i < n) {
            const size_t t = (size_t)(t0 + i);
            k4 = *reinterpret_cast<const float4*>(p.kn + t * KD + kh * 128 + c4);
            q4 = *reinterpret_cast<const float4*>(p.qn + t * KD + kh * 128 + c4);
            v4 = *reinterpret_cast<const float4*>(p.vc + t * p.VD + vh * 128 + c4);
        }
        *reinterpret_cast<float4*>(Ks + i * kGP + c4) = k4;
        *reinterpret_cast<float4*>(Qs + i * kGP + c4) = q4;
        *reinterpret_cast<float4*>(Vs + i * kGP + c4) = v4;
    }
    if (tid < 32) {
        // inclusive prefix sum of g over the chunk (two values per lane)
        const int i0 = 2 * tid;
        const float ga = i0 < n ? p.glog[(size_t)(t0 + i0) * p.VH + vh] : 0.f;
        const float gb = i0 + 1 < n ? p.glog[(size_t)(t0 + i0 + 1) * p.VH + vh] : 0.f;
        float sum = ga + gb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float up = __shfl_up_sync(0xffffffffu, sum, o);
            if (tid >= o) sum += up;
        }
        const float excl = sum - (ga + gb);
        Gc[i0] = excl + ga;
        Gc[i0 + 1] = excl + ga + gb;
        Bs[i0] = i0 < n ? p.beta[(size_t)(t0 + i0) * p.VH + vh] : 0.f;
        Bs[i0 + 1] = i0 + 1 < n ? p.beta[(size_t)(t0 + i0 + 1) * p.VH + vh] : 0.f;
    }
    __syncthreads();
    // KK and QK, 4 x 4 register tiles: rows 4*(tid>>4).., columns (tid&15) + 16*b
    {
        const int i0 = (tid >> 4) * 4, jq = tid & 15;
        float kk[4][4], qk[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) { kk[a][b] = 0.f; qk[a][b] = 0.f; }
        for (int d = 0; d < 128; d += 4) {
            float4 ki[4], qi[4], kj[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                ki[a] = *reinterpret_cast<const float4*>(Ks + (i0 + a) * kGP + d);
                qi[a] = *reinterpret_cast<const float4*>(Qs + (i0 + a) * kGP + d);
            }
#pragma unroll
            for (int b = 0; b < 4; ++b) kj[b] = *reinterpret_cast<const float4*>(Ks + (jq + 16 * b) * kGP + d);
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    kk[a][b] += ki[a].x * kj[b].x + ki[a].y * kj[b].y + ki[a].z * kj[b].z + ki[a].w * kj[b].w;
                    qk[a][b] += qi[a].x * kj[b].x + qi[a].y * kj[b].y + qi[a].z * kj[b].z + qi[a].w * kj[b].w;
                }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int i = i0 + a, j = jq + 16 * b;
                const float f = (j <= i && i < n) ? expf(Gc[i] - Gc[j]) * Bs[j] : 0.f;
                Ls[i * kGLP + j] = j < i ? f * kk[a][b] : 0.f;
                Ps[i * kGLP + j] = f * qk[a][b];
            }
    }
    __syncthreads();
    // outputs that need the raw k and q: Kd, Gamma Q, P, gamma_C; then Ks <- Gamma K
    const float GC = Gc[n - 1];
    const size_t hrow = ((size_t)vh * p.T + t0) * 128;
    for (int e = tid; e < kGC * 32; e += 256) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        if (i >= n) continue;
        const float4 k4 = *reinterpret_cast<const float4*>(Ks + i * kGP + c4);
        const float4 q4 = *reinterpret_cast<const float4*>(Qs + i * kGP + c4);
        const float fd = Bs[i] * expf(GC - Gc[i]), fg = expf(Gc[i]);
        *reinterpret_cast<float4*>(p.KD + hrow + (size_t)i * 128 + c4) =
            make_float4(fd * k4.x, fd * k4.y, fd * k4.z, fd * k4.w);
        *reinterpret_cast<float4*>(p.QG + hrow + (size_t)i * 128 + c4) =
            make_float4(fg * q4.x, fg * q4.y, fg * q4.z, fg * q4.w);
    }
    float* Pg = p.P + ((size_t)vh * nch + c) * kGC * kGC;
    for (int e = tid; e < kGC * kGC; e += 256) Pg[e] = Ps[(e >> 6) * kGLP + (e & 63)];
    if (tid == 0) p.gC[(size_t)vh * nch + c] = expf(GC);
    __syncthreads();
    for (int e = tid; e < kGC * 128; e += 256) {
        const int i = e >> 7, col = e & 127;
        Ks[i * kGP + col] *= expf(Gc[i]);
    }
    __syncthreads();
    // forward substitution: U (columns of V) on threads 0-127, W (columns of Gamma K) on 128-255
    {
        float* M = tid < 128 ? Vs : Ks;
        const int col = tid & 127;
        for (int i = 1; i < n; ++i) {
            float acc = M[i * kGP + col];
            for (int m = 0; m < i; ++m) acc -= Ls[i * kGLP + m] * M[m * kGP + col];
            M[i * kGP + col] = acc;
            __syncthreads();
        }
    }
    for (int e = tid; e < kGC * 32; e += 256) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        if (i >= n) continue;
        *reinterpret_cast<float4*>(p.U + hrow + (size_t)i * 128 + c4) = *reinterpret_cast<const float4*>(Vs + i * kGP + c4);
        *reinterpret_cast<float4*>(p.W + hrow + (size_t)i * 128 + c4) = *reinterpret_cast<const float4*>(Ks + i * kGP + c4);
    }
}

// Kernel B1: the state recurrence across chunks, S_{c+1} = gamma_C S_c + Kd^T (U - W S_c).
// Columns of S evolve independently, so each CTA owns a (value head, 16-column slice) and
// walks the chunks in order; the next chunk's W, Kd and U slice are fetched (cp.async)
// while the current one is applied. It writes the state entering every chunk (for the
// output kernel B2), E = U - W S_c in place of U, and the final state.
constexpr int kGS1 = 16;             // columns of S per CTA
constexpr int kGS1P = kGS1 + 4;      // padded stride of [.][16] tiles
constexpr int kB1Buf = 2 * kGC * kGP + kGC * kGS1P;  // floats per chunk buffer: W, Kd, U slice
constexpr size_t kGdnB1Smem = (size_t)(2 * kB1Buf + 128 * kGS1P + kGC * kGS1P) * 4;
__device__ __forceinline__ void cp16(float* dst, const float* src, bool pred) {
    const uint32_t d = smem_u32(dst);
    const int n = pred ? 16 : 0;  // 0: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__global__ void __launch_bounds__(256) k_pf_gdn_state(const PfGdnChunk p) {
    extern __shared__ __align__(16) float sb[];
    float* Ssm = sb + 2 * kB1Buf;        // [128][20]
    float* Esm = Ssm + 128 * kGS1P;      // [64][20]
    const int vh = blockIdx.x / (128 / kGS1), sl = blockIdx.x % (128 / kGS1), tid = threadIdx.x;
    const int nch = (p.T + kGC - 1) / kGC;
    float* Sg = p.state + (size_t)vh * 128 * 128 + sl * kGS1;
    for (int e = tid; e < 128 * (kGS1 / 4); e += 256) {
        const int r = e / (kGS1 / 4), c4 = (e % (kGS1 / 4)) * 4;
        *reinterpret_cast<float4*>(Ssm + r * kGS1P + c4) = *reinterpret_cast<const float4*>(Sg + (size_t)r * 128 + c4);
    }
    auto fetch = [&](int c) {
        float* B = sb + (c & 1) * kB1Buf;
        const int t0 = c * kGC, n = min(kGC, p.T - t0);
        const size_t hrow = ((size_t)vh * p.T + t0) * 128;
        for (int e = tid; e < kGC * 32; e += 256) {
            const int i = e >> 5, c4 = (e & 31) * 4;
            const size_t off = hrow + (size_t)(i < n ? i : 0) * 128 + c4;
            cp16(B + i * kGP + c4, p.W + off, i < n);
            cp16(B + kGC * kGP + i * kGP + c4, p.KD + off, i < n);
        }
        for (int e = tid; e < kGC * (kGS1 / 4); e += 256) {
            const int i = e / (kGS1 / 4), c4 = (e % (kGS1 / 4)) * 4;
            cp16(B + 2 * kGC * kGP + i * kGS1P + c4, p.U + hrow + (size_t)(i < n ? i : 0) * 128 + sl * kGS1 + c4, i < n);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    fetch(0);
    // E tile: row tid >> 2, columns 4 (tid & 3) .. +3; state tile: row tid >> 1, columns 8 (tid & 1) .. +7
    const int ei = tid >> 2, ec = (tid & 3) * 4;
    const int sr = tid >> 1, sc = (tid & 1) * 8;
    for (int c = 0; c < nch; ++c) {
        const int t0 = c * kGC, n = min(kGC, p.T - t0);
        const size_t hrow = ((size_t)vh * p.T + t0) * 128;
        if (c + 1 < nch) {
            fetch(c + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // chunk c's operands and the state are visible to every thread
        const float* Wsm = sb + (c & 1) * kB1Buf;
        const float* Ksm = Wsm + kGC * kGP;
        const float* Usm = Ksm + kGC * kGP;
        // the state entering chunk c, for the output kernel
        float* Scg = p.Sc + ((size_t)vh * nch + c) * 128 * 128 + sl * kGS1;
        for (int e = tid; e < 128 * (kGS1 / 4); e += 256) {
            const int r = e / (kGS1 / 4), c4 = (e % (kGS1 / 4)) * 4;
            *reinterpret_cast<float4*>(Scg + (size_t)r * 128 + c4) = *reinterpret_cast<const float4*>(Ssm + r * kGS1P + c4);
        }
        // E = U - W S
        {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            for (int r = 0; r < 128; ++r) {
                const float w = Wsm[ei * kGP + r];
                const float4 s4 = *reinterpret_cast<const float4*>(Ssm + r * kGS1P + ec);
                acc[0] += w * s4.x; acc[1] += w * s4.y; acc[2] += w * s4.z; acc[3] += w * s4.w;
            }
            const float4 u4 = *reinterpret_cast<const float4*>(Usm + ei * kGS1P + ec);
            const float4 e4 = make_float4(u4.x - acc[0], u4.y - acc[1], u4.z - acc[2], u4.w - acc[3]);
            *reinterpret_cast<float4*>(Esm + ei * kGS1P + ec) = e4;
            if (ei < n) *reinterpret_cast<float4*>(p.U + hrow + (size_t)ei * 128 + sl * kGS1 + ec) = e4;
        }
        __syncthreads();  // E complete; every read of S for E done
        // S = gamma_C S + Kd^T E (each thread reads and writes only its own S entries here)
        {
            const float gC = p.gC[(size_t)vh * nch + c];
            float acc[8];
            const float4 s0 = *reinterpret_cast<const float4*>(Ssm + sr * kGS1P + sc);
            const float4 s1 = *reinterpret_cast<const float4*>(Ssm + sr * kGS1P + sc + 4);
            acc[0] = gC * s0.x; acc[1] = gC * s0.y; acc[2] = gC * s0.z; acc[3] = gC * s0.w;
            acc[4] = gC * s1.x; acc[5] = gC * s1.y; acc[6] = gC * s1.z; acc[7] = gC * s1.w;
            for (int i = 0; i < n; ++i) {
                const float kd = Ksm[i * kGP + sr];
                const float4 e0 = *reinterpret_cast<const float4*>(Esm + i * kGS1P + sc);
                const float4 e1 = *reinterpret_cast<const float4*>(Esm + i * kGS1P + sc + 4);
                acc[0] += kd * e0.x; acc[1] += kd * e0.y; acc[2] += kd * e0.z; acc[3] += kd * e0.w;
                acc[4] += kd * e1.x; acc[5] += kd * e1.y; acc[6] += kd * e1.z; acc[7] += kd * e1.w;
            }
            *reinterpret_cast<float4*>(Ssm + sr * kGS1P + sc) = make_float4(acc[0], acc[1], acc[2], acc[3]);
            *reinterpret_cast<float4*>(Ssm + sr * kGS1P + sc + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
        }
        __syncthreads();  // new S visible; chunk c's buffer free for the fetch of chunk c + 2
    }
    for (int e = tid; e < 128 * (kGS1 / 4); e += 256) {
        const int r = e / (kGS1 / 4), c4 = (e % (kGS1 / 4)) * 4;
        *reinterpret_cast<float4*>(Sg + (size_t)r * 128 + c4) = *reinterpret_cast<const float4*>(Ssm + r * kGS1P + c4);
    }
}

// Kernel B2: outputs of every chunk in parallel, O = (Gamma Q) S_c + P E; CTA = (chunk,
// value head, 64-column half), 4 x 4 output tile per thread.
constexpr int kGOP = 64 + 4;
constexpr size_t kGdnB2Smem = (size_t)(128 * kGOP + kGC * kGP + kGC * kGLP + kGC * kGOP) * 4;
__global__ void __launch_bounds__(256) k_pf_gdn_out(const PfGdnChunk p) {
    extern __shared__ __align__(16) float so[];
    float* Ssm = so;                     // [128][68]
    float* Qsm = Ssm + 128 * kGOP;       // [64][132]
    float* Psm = Qsm + kGC * kGP;        // [64][65]
    float* Esm = Psm + kGC * kGLP;       // [64][68]
    const int c = blockIdx.x, vh = blockIdx.y, half = blockIdx.z, tid = threadIdx.x;
    const int nch = gridDim.x;
    const int t0 = c * kGC, n = min(kGC, p.T - t0);
    const size_t hrow = ((size_t)vh * p.T + t0) * 128;
    const float* Scg = p.Sc + ((size_t)vh * nch + c) * 128 * 128 + half * 64;
    for (int e = tid; e < 128 * 16; e += 256) {
        const int r = e >> 4, c4 = (e & 15) * 4;
        *reinterpret_cast<float4*>(Ssm + r * kGOP + c4) = *reinterpret_cast<const float4*>(Scg + (size_t)r * 128 + c4);
    }
    for (int e = tid; e < kGC * 32; e += 256) {
        const int i = e >> 5, c4 = (e & 31) * 4;
        float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n) q4 = *reinterpret_cast<const float4*>(p.QG + hrow + (size_t)i * 128 + c4);
        *reinterpret_cast<float4*>(Qsm + i * kGP + c4) = q4;
    }
    for (int e = tid; e < kGC * 16; e += 256) {
        const int i = e >> 4, c4 = (e & 15) * 4;
        float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < n) e4 = *reinterpret_cast<const float4*>(p.U + hrow + (size_t)i * 128 + half * 64 + c4);
        *reinterpret_cast<float4*>(Esm + i * kGOP + c4) = e4;
    }
    const float* Pg = p.P + ((size_t)vh * nch + c) * kGC * kGC;
    for (int e = tid; e < kGC * kGC; e += 256) Psm[(e >> 6) * kGLP + (e & 63)] = Pg[e];
    __syncthreads();
    const int oi = (tid >> 4) * 4, oc = (tid & 15) * 4;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
    for (int r = 0; r < 128; ++r) {
        const float4 s4 = *reinterpret_cast<const float4*>(Ssm + r * kGOP + oc);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const float q = Qsm[(oi + a) * kGP + r];
            acc[a][0] += q * s4.x; acc[a][1] += q * s4.y; acc[a][2] += q * s4.z; acc[a][3] += q * s4.w;
        }
    }
    for (int j = 0; j <= oi + 3; ++j) {  // P is lower triangular (zero above the diagonal)
        const float4 e4 = *reinterpret_cast<const float4*>(Esm + j * kGOP + oc);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const float pv = Psm[(oi + a) * kGLP + j];
            acc[a][0] += pv * e4.x; acc[a][1] += pv * e4.y; acc[a][2] += pv * e4.z; acc[a][3] += pv * e4.w;
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int i = oi + a;
        if (i < n)
            *reinterpret_cast<float4*>(p.out + (size_t)(t0 + i) * p.VD + vh * 128 + half * 64 + oc) =
                make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
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

// ---------------------------------------------------------------- y += x
__global__ void k_pf_add(float* y, const float* x, size_t n) {
    const size_t i = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        float4 a = *reinterpret_cast<float4*>(y + i);
        const float4 b = *reinterpret_cast<const float4*>(x + i);
        a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
        *reinterpret_cast<float4*>(y + i) = a;
    } else {
        for (size_t j = i; j < n; ++j) y[j] += x[j];
    }
}

// ---------------------------------------------------------------- launchers
cudaError_t pf_add(float* y, const float* x, size_t n, cudaStream_t s) {
    const size_t threads = (n + 3) / 4;
    k_pf_add<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(y, x, n);
    return cudaGetLastError();
}
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
    k_pf_gdn_prep<<<a.T, kPT, 0, s>>>(pp);
    k_pf_conv_ring<<<(a.C + 255) / 256, 256, 0, s>>>(a.proj, a.ldp, a.T, a.p0, a.C, a.ring);
    if (!a.Sc) return cudaErrorInvalidValue;
    PfGdnChunk ck{a.qn, a.kn, a.vc, a.glog, a.beta, a.U, a.W, a.QG, a.KD, a.P, a.gC, a.Sc, a.state, a.out,
                  a.T, a.KH, a.VH, a.VD};
    {
        cudaError_t e = cudaFuncSetAttribute(k_pf_gdn_chunk_a, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdnASmem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_state, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdnB1Smem);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_pf_gdn_out, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGdnB2Smem);
        if (e != cudaSuccess) return e;
    }
    const int nch = (a.T + kGC - 1) / kGC;
    k_pf_gdn_chunk_a<<<dim3(nch, a.VH), 256, kGdnASmem, s>>>(ck);
    k_pf_gdn_state<<<a.VH * (128 / kGS1), 256, kGdnB1Smem, s>>>(ck);
    k_pf_gdn_out<<<dim3(nch, a.VH, 2), 256, kGdnB2Smem, s>>>(ck);
    return cudaGetLastError();
}
size_t pf_gdn_workspace_bytes(int KH, int VH, int T) {
    const size_t t = (size_t)T, nch = (t + kGC - 1) / kGC, KD = (size_t)KH * 128, VD = (size_t)VH * 128;
    auto r = [](size_t b) { return (b + 255) / 256 * 256; };
    return 2 * r(t * KD * 4) + 5 * r(t * VD * 4) + 2 * r(t * VH * 4) + r(VH * nch * kGC * kGC * 4) + r(VH * nch * 4) +
           r(VH * nch * 128 * 128 * 4);
}
int pf_gdn_carve(PfGdnArgs& a, void* ws, size_t bytes) {
    const size_t t = (size_t)a.T, nch = (t + kGC - 1) / kGC, KD = (size_t)a.KH * 128, VD = (size_t)a.VH * 128;
    if (!ws || bytes < pf_gdn_workspace_bytes(a.KH, a.VH, a.T)) return -1;
    uint8_t* b = static_cast<uint8_t*>(ws);
    size_t off = 0;
    auto take = [&](size_t n) {
        float* f = reinterpret_cast<float*>(b + off);
        off += (n * 4 + 255) / 256 * 256;
        return f;
    };
    a.qn = take(t * KD);
    a.kn = take(t * KD);
    a.vc = take(t * VD);
    a.U = take(t * VD);
    a.W = take(t * VD);
    a.QG = take(t * VD);
    a.KD = take(t * VD);
    a.glog = take(t * a.VH);
    a.beta = take(t * a.VH);
    a.P = take(a.VH * nch * kGC * kGC);
    a.gC = take(a.VH * nch);
    a.Sc = take(a.VH * nch * 128 * 128);
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
