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
// 1/sqrt(DK)); the gates decay = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b).
// One warp per 128-channel head vector (q heads, k heads, v heads), 4 channels per lane.
struct PfGdnPrep {
    const float* proj;    // [T][ldp]: qkv C | z VD | b VH | a VH
    long ldp;
    const float* conv_w;  // [C][4]
    const float* ring;    // [C][4] (read only here)
    const float* neg_exp_A;
    const float* dt_bias;
    float* qn;            // [T][KD]
    float* kn;            // [T][KD]
    float* vc;            // [T][VD]
    float* decay;         // [T][VH]
    float* beta;          // [T][VH]
    int p0, KH, VH, C, VD;
};
__global__ void __launch_bounds__(kPT) k_pf_gdn_prep(const PfGdnPrep p) {
    const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KD = p.KH * 128;
    const int nvec = 2 * p.KH + p.VH;
    const float* row = p.proj + (size_t)t * p.ldp;
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
        const float bv = row[p.C + p.VD + h], av = row[p.C + p.VD + p.VH + h];
        const float g = p.neg_exp_A[h] * softplus_f(av + p.dt_bias[h]);
        p.decay[(size_t)t * p.VH + h] = expf(g);
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

// ---------------------------------------------------------------- GDN recurrence
// One (value head, 16-column slice) per CTA of 128 threads; thread r owns row r of the
// slice of S (16 fp32 in registers). The chunk's tokens are processed in order with the
// delta rule of gdn_step (qwen_model.cpp:199-205), exactly as the decode item does;
// the inputs of the next 8 tokens are loaded while the current 8 are processed.
struct PfGdnScan {
    const float* qn;
    const float* kn;
    const float* vc;
    const float* decay;
    const float* beta;
    float* state;  // [VH][DK][DV]
    float* out;    // [T][VD]
    int T, KH, VH, VD;
};
constexpr int kScanAhead = 8;
__global__ void __launch_bounds__(128) k_pf_gdn_scan(const PfGdnScan p) {
    __shared__ float red16[2][4][16];  // [0]: S^T k partials, [1]: S^T q partials
    __shared__ float s_d[16];
    const int vh = blockIdx.x >> 3, vs = blockIdx.x & 7;
    const int r = threadIdx.x, warp = r >> 5, lane = r & 31;
    const int rep = p.VH / p.KH, kh = vh / rep, KD = p.KH * 128;
    float S[16];
    float* Srow = p.state + ((size_t)vh * 128 + r) * 128 + vs * 16;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 v = reinterpret_cast<const float4*>(Srow)[i];
        S[4 * i] = v.x; S[4 * i + 1] = v.y; S[4 * i + 2] = v.z; S[4 * i + 3] = v.w;
    }
    const int sidx = scatter_index(lane);
    // per-token inputs of this thread: q[r], k[r], (v[col] for r < 16), decay, beta
    float cq[kScanAhead], ck[kScanAhead], cv[kScanAhead], cdec[kScanAhead], cbeta[kScanAhead];
    auto load = [&](int t0, float* q, float* k, float* v, float* dec, float* be) {
#pragma unroll
        for (int i = 0; i < kScanAhead; ++i) {
            const int t = t0 + i;
            const bool in = t < p.T;
            q[i] = in ? p.qn[(size_t)t * KD + kh * 128 + r] : 0.f;
            k[i] = in ? p.kn[(size_t)t * KD + kh * 128 + r] : 0.f;
            v[i] = (in && r < 16) ? p.vc[(size_t)t * p.VD + vh * 128 + vs * 16 + r] : 0.f;
            dec[i] = in ? p.decay[(size_t)t * p.VH + vh] : 0.f;
            be[i] = in ? p.beta[(size_t)t * p.VH + vh] : 0.f;
        }
    };
    load(0, cq, ck, cv, cdec, cbeta);
    for (int t0 = 0; t0 < p.T; t0 += kScanAhead) {
        float nq[kScanAhead], nk[kScanAhead], nv[kScanAhead], ndec[kScanAhead], nbeta[kScanAhead];
        load(t0 + kScanAhead, nq, nk, nv, ndec, nbeta);
#pragma unroll
        for (int i = 0; i < kScanAhead; ++i) {
            const int t = t0 + i;
            if (t >= p.T) break;  // uniform
            const float decay = cdec[i], k = ck[i], q = cq[i];
            float part[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                S[j] *= decay;
                part[j] = S[j] * k;
            }
            // Barriers: (1) km partials written; (2) d written (km partials read);
            // (3) o partials written. The next token writes km partials only after (3),
            // when d and the previous km partials are no longer read, and its o partials
            // only after its own (2), when this token's o partials have been read.
            float rr = reduce_scatter16(part, lane);
            if ((lane & 1) == 0) red16[0][warp][sidx] = rr;
            __syncthreads();
            if (r < 16) {
                const float km = (red16[0][0][r] + red16[0][1][r]) + (red16[0][2][r] + red16[0][3][r]);
                s_d[r] = (cv[i] - km) * cbeta[i];
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                S[j] += k * s_d[j];
                part[j] = S[j] * q;
            }
            rr = reduce_scatter16(part, lane);
            if ((lane & 1) == 0) red16[1][warp][sidx] = rr;
            __syncthreads();
            if (r < 16)
                p.out[(size_t)t * p.VD + vh * 128 + vs * 16 + r] =
                    (red16[1][0][r] + red16[1][1][r]) + (red16[1][2][r] + red16[1][3][r]);
        }
#pragma unroll
        for (int i = 0; i < kScanAhead; ++i) {
            cq[i] = nq[i]; ck[i] = nk[i]; cv[i] = nv[i]; cdec[i] = ndec[i]; cbeta[i] = nbeta[i];
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(Srow)[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
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
};
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
    PfGdnPrep pp{a.proj, a.ldp, a.conv_w, a.ring, a.neg_exp_A, a.dt_bias, a.qn, a.kn, a.vc, a.decay, a.beta,
                 a.p0, a.KH, a.VH, a.C, a.VD};
    k_pf_gdn_prep<<<a.T, kPT, 0, s>>>(pp);
    k_pf_conv_ring<<<(a.C + 255) / 256, 256, 0, s>>>(a.proj, a.ldp, a.T, a.p0, a.C, a.ring);
    PfGdnScan sc{a.qn, a.kn, a.vc, a.decay, a.beta, a.state, a.out, a.T, a.KH, a.VH, a.VD};
    k_pf_gdn_scan<<<a.VH * 8, 128, 0, s>>>(sc);
    return cudaGetLastError();
}
cudaError_t pf_gated_norm_split(const float* o, long ldo, const float* z, long ldz, const float* w, int T, int nh,
                                float eps, uint16_t* xs, long ldxs, cudaStream_t s) {
    k_pf_gated_norm_split<<<T, kPT, 0, s>>>(o, ldo, z, ldz, w, nh, eps, xs, ldxs);
    return cudaGetLastError();
}
cudaError_t pf_attention(const PfAttnArgs& a, cudaStream_t s) {
    if (a.rot > kHD || a.rot % 16 || a.NKV <= 0 || a.NQ % a.NKV) return cudaErrorInvalidValue;
    PfAttnPrep pp{a.proj, a.ldp, a.qn1, a.kn1, a.rope_cs, a.qbuf, a.k_cache, a.v_cache,
                  a.kv_bf16, a.max_ctx, a.p0, a.NQ, a.NKV, a.rot, a.eps};
    k_pf_attn_prep<<<a.T, kPT, 0, s>>>(pp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
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
