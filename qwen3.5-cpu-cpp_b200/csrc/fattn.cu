// Causal gated GQA attention of the batched forward pass (prefill) on the tcgen05 tensor
// cores: softmax(q K^T / sqrt(HD)) V over positions <= the query's, times sigmoid(gate)
// (attn_step, src/qwen_model.cpp:134-150; mix_attention, src/qwen_forward.cpp:20-80).
//
// Precision: the reference computes in fp32. Every fp32 operand is carried as a bf16 pair
// (x = hi + lo, |x - hi - lo| <= 2^-17 |x|) and each product is taken three times,
//   S = Qh Kh + Qh Kl + Ql Kh,     O += Ph Vh + Ph Vl + Pl Vh,
// with fp32 accumulation in tensor memory: the dropped lo x lo term is ~2^-16 relative.
//
// CTA = (kv head, block of 128 query rows = GRP q heads x 128/GRP tokens), 160 threads:
//   warps 0-3  one query row per thread (= its TMEM lane): load and split the row's q,
//              online softmax over each 64-key block read from TMEM (tcgen05.ld), P as bf16
//              pairs into shared memory (128-byte swizzle, K-major), O rescaled in TMEM
//              (tcgen05.ld / st) when the row max grows; at the end O / l * sigmoid(gate)
//              written as the hi/lo input of o_proj.
//   warp 4     allocates 512 TMEM columns (S: 64, O: 256); one lane issues the TMA loads
//              (no multicast) and the MMAs: per key block K (split, 64 KB) -> 48 MMAs
//              M=128 N=64 K=16 -> S; the same 64 KB buffer then takes V^T (split) -> after
//              the softmax warps publish P, 12 MMAs M=128 N=256 K=16 -> O.
// Shared memory: Q pairs 128 KB (resident), K / V^T block 64 KB, P pairs 32 KB.
// K and V reach this kernel as bf16 pairs written by the attention prep kernel: K split
// row-major [kv][pos][hi 256 | lo 256], V split and transposed [kv][hi|lo][256 dims][pos],
// so that every operand is K-major. Every wait is bounded.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace qwc {
namespace {

constexpr int kM = 128, kN = 64, kHD = 256, kThreads = 160;
constexpr uint32_t kQTile = kM * 128;         // 128 rows x 64 dims bf16
constexpr uint32_t kQBytes = 8 * kQTile;      // 4 dim chunks x (hi, lo)
constexpr uint32_t kKTile = kN * 128;         // 64 keys x 64 dims bf16
constexpr uint32_t kKVBytes = 8 * kKTile;     // K: 4 chunks x (hi, lo); V^T: (hi, lo) x 256 x 64
constexpr uint32_t kPTile = kM * 128;         // 128 rows x 64 keys bf16
constexpr size_t kSmem = kQBytes + kKVBytes + 2 * kPTile + 1024 + 256;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;
constexpr uint32_t kIdescS =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
constexpr uint32_t kIdescO =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kHD >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
static_assert(kSmem <= 232448, "shared memory of the attention CTA");

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint64_t desc128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
        "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
        "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ uint16_t bf16r(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// Write 8 consecutive values (K index 8s .. 8s+7) of row `row` into a K-major 128-byte
// swizzled tile as bf16 hi and lo: 16-byte segment s of the row lives at s ^ (row % 8).
__device__ __forceinline__ void put8(uint8_t* hi_tile, uint8_t* lo_tile, int row, int s, const float (&v)[8]) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint16_t h0 = bf16r(v[2 * e]), h1 = bf16r(v[2 * e + 1]);
        const uint16_t l0 = bf16r(v[2 * e] - bf16f(h0)), l1 = bf16r(v[2 * e + 1] - bf16f(h1));
        h[e] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        l[e] = (uint32_t)l0 | ((uint32_t)l1 << 16);
    }
    const uint32_t off = (uint32_t)row * 128 + (uint32_t)((s ^ (row & 7)) * 16);
    *reinterpret_cast<uint4*>(hi_tile + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo_tile + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

struct FAParams {
    const float* qbuf;   // [T][NQ][HD] normed + roped queries of the chunk
    const float* proj;   // [T][ldp]: head h gate at h*2*HD + HD
    long ldp;
    uint16_t* xs;        // output [T][ldxs], K = NQ*HD, hi/lo
    long ldxs;
    int T, p0, NQ, NKV, grp, ctx_pad;
    int* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    k_pf_fattn(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapVt, const FAParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;
    uint8_t* KV = sm + kQBytes;
    uint8_t* Ph = KV + kKVBytes;
    uint8_t* Pl = Ph + kPTile;
    uint64_t* bar = reinterpret_cast<uint64_t*>(Pl + kPTile);
    uint64_t* kv_full = bar + 0;
    uint64_t* kv_free = bar + 1;
    uint64_t* s_full = bar + 2;
    uint64_t* p_full = bar + 3;
    uint64_t* pv_done = bar + 4;
    uint64_t* mma_done = bar + 5;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 6);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv = blockIdx.x, qb = blockIdx.y;
    const int bqt = kM / p.grp;  // tokens per CTA
    const int t_last = min((qb + 1) * bqt, p.T) - 1;
    const int nkb = (p.p0 + t_last) / kN + 1;  // causal: key blocks up to the last query
    const float scale = 1.0f / sqrtf((float)kHD);

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        mbar_init(kv_free, 1);
        mbar_init(s_full, 1);
        mbar_init(p_full, 4);
        mbar_init(pv_done, 1);
        mbar_init(mma_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // query rows: thread rho (< 128) = TMEM lane rho; row rho = (head g, token i)
    const int rho = threadIdx.x;
    const int g = rho / bqt, ti = qb * bqt + (rho % bqt);
    const int h = kv * p.grp + g;
    const bool valid = warp < 4 && ti < p.T;
    const int qpos = p.p0 + ti;
    if (warp < 4) {
        const float* q = p.qbuf + ((size_t)(valid ? ti : 0) * p.NQ + h) * kHD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int s = 0; s < 8; ++s) {
                float v[8];
                if (valid) {
                    const float4 a = *reinterpret_cast<const float4*>(q + c * 64 + s * 8);
                    const float4 b = *reinterpret_cast<const float4*>(q + c * 64 + s * 8 + 4);
                    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = 0.f;
                }
                put8(Qs + (c * 2) * kQTile, Qs + (c * 2 + 1) * kQTile, rho, s, v);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(s_abort) != 0; };
    auto give_up = [&](int code) {
        post_error(p.err, code);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
    };

    if (warp == 4) {
        if (lane == 0) {
            // -------------------------------------------------- TMA + MMA issuer
            const uint32_t q0 = smem_u32(Qs), kv0 = smem_u32(KV), ph0 = smem_u32(Ph), pl0 = smem_u32(Pl);
            int pending = -1;  // parity of a kv_full phase whose TMA loads may still be in flight
            for (int kb = 0; kb < nkb && !aborted(); ++kb) {
                const uint32_t par = (uint32_t)(kb & 1);
                // K block (the buffer is free: the previous PV MMAs have completed)
                if (kb > 0 && !mbar_wait_bounded(pv_done, par ^ 1u, p.err, DEV_TC_MMA_TIMEOUT)) { give_up(DEV_TC_MMA_TIMEOUT); break; }
                mbar_arrive_expect_tx(kv_full, kKVBytes);
                for (int c = 0; c < 4; ++c)
                    for (int hl = 0; hl < 2; ++hl)
                        tma2d(KV + (c * 2 + hl) * kKTile, &mapK, hl * kHD + c * 64, kv * p.ctx_pad + kb * kN, kv_full);
                pending = 0;
                if (!mbar_wait_bounded(kv_full, 0u, p.err, DEV_TC_MMA_TIMEOUT)) { give_up(DEV_TC_MMA_TIMEOUT); break; }
                pending = -1;
                fence_after();
                // S = Qh Kh + Qh Kl + Ql Kh over 4 dim chunks x 4 k-steps
                for (int c = 0; c < 4; ++c) {
                    const uint64_t ah = desc128(q0 + (c * 2) * kQTile), al = desc128(q0 + (c * 2 + 1) * kQTile);
                    const uint64_t bh = desc128(kv0 + (c * 2) * kKTile), bl = desc128(kv0 + (c * 2 + 1) * kKTile);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                        mma(tmem + kColS, ah + adv, bh + adv, kIdescS, (c | ks) != 0 ? 1u : 0u);
                        mma(tmem + kColS, ah + adv, bl + adv, kIdescS, 1u);
                        mma(tmem + kColS, al + adv, bh + adv, kIdescS, 1u);
                    }
                }
                commit(s_full);
                commit(kv_free);
                if (!mbar_wait_bounded(kv_free, par, p.err, DEV_TC_MMA_TIMEOUT)) { give_up(DEV_TC_MMA_TIMEOUT); break; }
                // V^T block into the same buffer: hi rows d at [0, 32 KB), lo at [32, 64 KB)
                mbar_arrive_expect_tx(kv_full, kKVBytes);
                for (int hl = 0; hl < 2; ++hl)
                    for (int dc = 0; dc < 4; ++dc)
                        tma2d(KV + hl * 4 * kKTile + dc * kKTile, &mapVt, kb * kN, (kv * 2 + hl) * kHD + dc * 64, kv_full);
                pending = 1;
                if (!mbar_wait_bounded(kv_full, 1u, p.err, DEV_TC_MMA_TIMEOUT)) { give_up(DEV_TC_MMA_TIMEOUT); break; }
                pending = -1;
                if (!mbar_wait_bounded(p_full, par, p.err, DEV_TC_MMA_TIMEOUT)) { give_up(DEV_TC_MMA_TIMEOUT); break; }
                fence_after();
                // O += Ph Vh + Ph Vl + Pl Vh over 4 k-steps of 16 keys
                const uint64_t vh = desc128(kv0), vl = desc128(kv0 + 4 * kKTile);
                const uint64_t pa = desc128(ph0), pb = desc128(pl0);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                    mma(tmem + kColO, pa + adv, vh + adv, kIdescO, (kb | ks) != 0 ? 1u : 0u);
                    mma(tmem + kColO, pa + adv, vl + adv, kIdescO, 1u);
                    mma(tmem + kColO, pb + adv, vh + adv, kIdescO, 1u);
                }
                commit(pv_done);
            }
            // before the CTA exits: the loads in flight have landed and every MMA has completed
            if (pending >= 0) mbar_wait_bounded(kv_full, (uint32_t)pending, p.err, DEV_TC_DRAIN_TIMEOUT);
            commit(mma_done);
            mbar_wait_bounded(mma_done, 0u, p.err, DEV_TC_DRAIN_TIMEOUT);
        }
    } else {
        // -------------------------------------------------- softmax rows
        const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const uint32_t par = (uint32_t)(kb & 1);
            ok = mbar_wait_bounded(s_full, par, p.err, DEV_TC_EPI_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok && !aborted());
            if (!ok) {
                if (lane == 0) give_up(DEV_TC_EPI_TIMEOUT);
                break;
            }
            fence_after();
            float s[64];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float v[16];
                ld16(trow + kColS + c * 16, v);
#pragma unroll
                for (int e = 0; e < 16; ++e) s[c * 16 + e] = v[e];
            }
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int key = kb * kN + j;
                s[j] = (valid && key <= qpos) ? s[j] * scale : -INFINITY;
                mx = fmaxf(mx, s[j]);
            }
            const float mn = fmaxf(m, mx);
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
            float sum = 0.f;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                s[j] = (s[j] == -INFINITY) ? 0.f : expf(s[j] - mn);
                sum += s[j];
            }
            l = l * corr + sum;
            m = mn;
            // P as bf16 pairs (the previous PV MMAs, which read P, completed before S did)
#pragma unroll
            for (int sg = 0; sg < 8; ++sg) {
                float v[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = s[sg * 8 + e];
                put8(Ph, Pl, rho, sg, v);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            // rescale O when a row's max grew (warp-uniform: tcgen05.ld / st are warp-wide)
            if (kb > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < kHD / 16; ++c) {
                    float v[16];
                    ld16(trow + kColO + c * 16, v);
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[e] *= corr;
                    st16(trow + kColO + c * 16, v);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
        }
        if (ok && nkb > 0) {
            ok = mbar_wait_bounded(pv_done, (uint32_t)((nkb - 1) & 1), p.err, DEV_TC_EPI_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok && !aborted());
        }
        if (ok) {
            fence_after();
            const int K = p.NQ * kHD;
            uint16_t* row = p.xs + (size_t)(valid ? ti : 0) * p.ldxs;
            const float* gate = p.proj + (size_t)(valid ? ti : 0) * p.ldp + (size_t)h * 2 * kHD + kHD;
            const float inv_l = 1.0f / l;
#pragma unroll 1
            for (int c = 0; c < kHD / 16; ++c) {
                float v[16];
                ld16(trow + kColO + c * 16, v);
                if (valid) {
                    uint32_t hw[8], lw[8];
#pragma unroll
                    for (int e = 0; e < 16; e += 2) {
                        const float x0 = v[e] * inv_l * sigmoid_f(gate[c * 16 + e]);
                        const float x1 = v[e + 1] * inv_l * sigmoid_f(gate[c * 16 + e + 1]);
                        const uint16_t h0 = bf16r(x0), h1 = bf16r(x1);
                        hw[e / 2] = (uint32_t)h0 | ((uint32_t)h1 << 16);
                        lw[e / 2] = (uint32_t)bf16r(x0 - bf16f(h0)) | ((uint32_t)bf16r(x1 - bf16f(h1)) << 16);
                    }
                    uint4* dh = reinterpret_cast<uint4*>(row + h * kHD + c * 16);
                    uint4* dl = reinterpret_cast<uint4*>(row + K + h * kHD + c * 16);
                    dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                    dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
                    dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 4) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// V split rows [kv][pos][hi 256 | lo 256] (positions p0..p0+T-1) -> transposed
// [kv][hi|lo][256][ctx_pad], through 32 x 32 shared-memory tiles.
__global__ void k_pf_vt(const uint16_t* vsplit, uint16_t* vt, int T, int p0, int ctx_pad) {
    __shared__ uint16_t tile[32][33];
    const int kv = blockIdx.z, col0 = blockIdx.y * 32;  // col in [0, 512): hl * 256 + d
    const int t0 = blockIdx.x * 32;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    for (int r = ty; r < 32; r += 8) {
        const int t = t0 + r;
        tile[r][tx] = t < T ? vsplit[((size_t)kv * T + t) * 512 + col0 + tx] : (uint16_t)0;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int col = col0 + r;  // hl * 256 + d
        const int t = t0 + tx;
        if (t < T) vt[((size_t)kv * 512 + col) * ctx_pad + p0 + t] = tile[tx][r];
    }
}

}  // namespace

cudaError_t pf_fattn(const PfFattnArgs& a, cudaStream_t s) {
    if (a.NKV <= 0 || a.NQ % a.NKV) return cudaErrorInvalidValue;
    const int grp = a.NQ / a.NKV;
    if (grp != 1 && grp != 2 && grp != 4 && grp != 8) return cudaErrorInvalidValue;
    dim3 tb(32, 8), tg((a.T + 31) / 32, 512 / 32, a.NKV);
    k_pf_vt<<<tg, tb, 0, s>>>(a.vsplit, a.vt, a.T, a.p0, a.ctx_pad);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    CUtensorMap mk, mv;
    if (tc_make_map_box(&mk, a.ksplit, (long)a.NKV * a.ctx_pad, 512, 512, kN) ||
        tc_make_map_box(&mv, a.vt, (long)a.NKV * 512, a.ctx_pad, a.ctx_pad, 64))
        return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(k_pf_fattn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
    if (e != cudaSuccess) return e;
    FAParams p;
    p.qbuf = a.qbuf;
    p.proj = a.proj;
    p.ldp = a.ldp;
    p.xs = a.xs;
    p.ldxs = a.ldxs;
    p.T = a.T;
    p.p0 = a.p0;
    p.NQ = a.NQ;
    p.NKV = a.NKV;
    p.grp = grp;
    p.ctx_pad = a.ctx_pad;
    p.err = a.err;
    dim3 grid(a.NKV, (a.T + (kM / grp) - 1) / (kM / grp));
    k_pf_fattn<<<grid, kThreads, kSmem, s>>>(mk, mv, p);
    return cudaGetLastError();
}

}  // namespace qwc
