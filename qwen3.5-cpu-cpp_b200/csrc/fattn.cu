// Causal gated GQA attention of the batched forward pass (prefill) on the tcgen05 tensor
// cores: softmax(q K^T / sqrt(HD)) V over positions <= the query's, times sigmoid(gate)
// (attn_step, src/qwen_model.cpp:134-150; mix_attention, src/qwen_forward.cpp:20-80).
//
// Precision: the reference computes in fp32. Every fp32 operand is carried as a bf16 pair
// (x = hi + lo, |x - hi - lo| <= 2^-17 |x|) and each product is taken three times,
//   S = Qh Kh + Qh Kl + Ql Kh,     O += Ph Vh + Ph Vl + Pl Vh,
// with fp32 accumulation in tensor memory: the dropped lo x lo term is ~2^-16 relative.
//
// CTA = (kv head, block of 128 query rows = GRP q heads x 128/GRP tokens), 224 threads:
//   warps 0-3  one query row per thread (= its TMEM lane): split the row's q (hi to shared
//              memory, lo to tensor memory); per 64-key block read S from TMEM, online
//              softmax in the log2 domain, write P as bf16 pairs back over S in TMEM. The
//              running max is raised (and O rescaled in TMEM) only when a block's max
//              exceeds it by more than 8 (a factor 256): P stays <= 256, and O / l is the
//              same quotient. At the end O / l * sigmoid(gate) -> the hi/lo input of o_proj.
//   warp 4     allocates the 512 TMEM columns; one lane issues the MMAs in the order
//              S(0) S(1) PV(0) S(2) PV(1) ..., so that S(kb+1) runs on the tensor cores
//              while the softmax works on block kb.
//   warp 5     one lane loads K blocks (TMA, no multicast) into the K buffer once the S MMAs
//              of the previous block have read it.
//   warp 6     one lane loads V^T blocks into the V buffer once PV of the previous block
//              has completed.
// Tensor memory: S / P double buffer (2 x 64 columns: S fp32, then P hi in the first 32
// and P lo in the next 32 as packed bf16), Q lo (128 columns), O (256 columns).
// Shared memory: Q hi 64 KB, K block 64 KB (4 dim chunks x hi/lo), V^T block 64 KB.
// K and V reach this kernel as bf16 pairs written by the attention prep kernel: K split
// row-major [kv][pos][hi 256 | lo 256], V split and transposed [kv][hi|lo][256 dims][pos],
// so that every shared-memory operand is K-major. Every wait is bounded.
//
// Key splits. One CTA per (kv head, query block) gives NKV * T / (128 / GRP) CTAs: 256 for
// a 4096-token chunk of the 2B shape on one GPU, but 32 on each rank of an 8-way tensor-
// parallel group (one q head per rank), where a long context then runs on a fifth of the
// SMs. The grid's third dimension therefore splits each CTA's key blocks into `nsplit`
// contiguous ranges; a split CTA leaves its unnormalised O, running max m (log2 units)
// and sum l per row in a workspace, and k_pf_fattn_combine merges the splits of a row,
//   M = max_s m_s,  O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s,
// before the gate and the bf16-pair split (the split-K combine of the decode attention).
// Rotated key order (each CTA starting at a different block, to spread L2 reads of a
// short context) is used only while the layer's K / V operands fit in L2; over a long
// context every CTA of a kv head walks the same blocks in the same order, so each block
// is read from HBM once and served from L2 to the others.
#include "common.cuh"
#include "kernels.h"
#include "tc_util.cuh"

#include <algorithm>
#include <cstdlib>

namespace qwc {
namespace {

constexpr int kM = 128, kN = 64, kHD = 256, kThreads = 224;
constexpr uint32_t kQTile = kM * 128;     // 128 rows x 64 dims bf16
constexpr uint32_t kQBytes = 4 * kQTile;  // Q hi: 4 dim chunks
constexpr uint32_t kKTile = kN * 128;     // 64 keys x 64 dims bf16
constexpr uint32_t kKVBytes = 8 * kKTile; // K: 4 chunks x (hi, lo); V^T: (hi, lo) x 256 x 64
constexpr size_t kSmem = kQBytes + 2 * kKVBytes + 1024 + 256;
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColQl = 128, kColO = 256;  // S / P buffer b at kColS + 64 b
constexpr uint32_t kIdescS =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kN >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
constexpr uint32_t kIdescO =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kHD >> 3) << 17) | ((uint32_t)(kM >> 4) << 24);
constexpr float kRescaleLog2 = 8.0f;
constexpr int kFattnWaves = 2, kFattnMinBlocks = 32;
constexpr size_t kFattnRotateBytes = 48ull << 20;
static_assert(kSmem <= 232448, "shared memory of the attention CTA");

using namespace tc;

struct FAParams {
    const float* qbuf;   // [T][NQ][HD] normed + roped queries of the chunk
    const float* proj;   // [T][ldp]: head h gate at h*2*HD + HD
    long ldp;
    uint16_t* xs;        // output [T][ldxs], K = NQ*HD, hi/lo
    long ldxs;
    int T, p0, NQ, NKV, grp, ctx_pad;
    int nsplit, rotate;  // key ranges per query block; rotated key order (short contexts)
    float* part_o;       // nsplit > 1: [nsplit][T][NQ][HD] unnormalised O
    float* part_ml;      //             [nsplit][T][NQ][2] running max (log2 units), sum
    int* err;
};

// Key blocks [lo, hi) of split `s` of a query block whose causal range has nkb blocks.
__host__ __device__ inline void fattn_split_range(int nkb, int nsplit, int s, int& lo, int& hi) {
    const int len = (nkb + nsplit - 1) / nsplit;
    lo = s * len;
    hi = lo + len < nkb ? lo + len : nkb;
}

__global__ void __launch_bounds__(kThreads, 1)
    k_pf_fattn(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapVt, const FAParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;
    uint8_t* Kb = sm + kQBytes;
    uint8_t* Vb = Kb + kKVBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(Vb + kKVBytes);
    uint64_t* k_full = bar + 0;
    uint64_t* k_free = bar + 1;
    uint64_t* v_full = bar + 2;
    uint64_t* pv_done = bar + 3;  // also: V buffer free
    uint64_t* s_full = bar + 4;   // [2]
    uint64_t* p_full = bar + 6;   // [2]
    uint64_t* mma_done = bar + 8;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 9);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kv = blockIdx.x;
    const int qb = gridDim.y - 1 - blockIdx.y;  // longest causal rows first
    const int bqt = kM / p.grp;                 // tokens per CTA
    const int t_last = min((qb + 1) * bqt, p.T) - 1;
    const int nkb_all = (p.p0 + t_last) / kN + 1;  // causal: key blocks up to the last query
    int kb_lo, kb_hi;
    fattn_split_range(nkb_all, p.nsplit, blockIdx.z, kb_lo, kb_hi);
    const int nkb = kb_hi - kb_lo;
    if (nkb <= 0) return;  // an empty split (short causal range): the combine skips it
    // Short contexts: each CTA walks its key blocks from a different start (the online
    // softmax does not depend on the order), so that the CTAs of a kv head do not all
    // read the same block from L2 at the same time. Long contexts: the same order for all.
    const int rot = p.rotate ? (qb * 13 + kv * 7) % nkb : 0;
    auto blk = [&](int kb) { return kb_lo + (kb + rot < nkb ? kb + rot : kb + rot - nkb); };

    if (threadIdx.x == 0) {
        mbar_init(k_full, 1);
        mbar_init(k_free, 1);
        mbar_init(v_full, 1);
        mbar_init(pv_done, 1);
        mbar_init(&s_full[0], 1);
        mbar_init(&s_full[1], 1);
        mbar_init(&p_full[0], 4);
        mbar_init(&p_full[1], 4);
        mbar_init(mma_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

    // query rows: thread rho (< 128) = TMEM lane rho; row rho = (head g, token i)
    const int rho = threadIdx.x;
    const int g = rho / bqt, ti = qb * bqt + (rho % bqt);
    const int h = kv * p.grp + g;
    const bool valid = warp < 4 && ti < p.T;
    const int qpos = p.p0 + ti;
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    if (warp < 4) {
        const float* q = p.qbuf + ((size_t)(valid ? ti : 0) * p.NQ + h) * kHD;
#pragma unroll 1
        for (int gq = 0; gq < 8; ++gq) {  // 32 dims per step
            uint32_t lo[16];
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
                float v[8];
                if (valid) {
                    const float4 a = *reinterpret_cast<const float4*>(q + gq * 32 + s4 * 8);
                    const float4 b = *reinterpret_cast<const float4*>(q + gq * 32 + s4 * 8 + 4);
                    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = 0.f;
                }
                uint32_t hi[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split2(v[2 * e], v[2 * e + 1], hi[e], lo[s4 * 4 + e]);
                // 16-byte segment s of a 128-byte swizzled row lives at s ^ (row % 8)
                const int c = gq >> 1, seg = (gq & 1) * 4 + s4;
                *reinterpret_cast<uint4*>(Qs + c * kQTile + rho * 128 + ((seg ^ (rho & 7)) * 16)) =
                    make_uint4(hi[0], hi[1], hi[2], hi[3]);
            }
            st16(trow + kColQl + gq * 16, lo);
        }
        st_wait();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
    }
    fence_before();
    __syncthreads();
    fence_after();
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(s_abort) != 0; };
    auto give_up = [&](int code) {
        post_error(p.err, code);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
    };

    if (warp == 5) {
        if (lane == 0) {
            // -------------------------------------------------- K loader
            int pending = -1;  // parity of a k_full phase whose loads may still be in flight
            for (int kb = 0; kb < nkb && !aborted(); ++kb) {
                if (kb > 0 && !mbar_wait_bounded(k_free, (uint32_t)((kb - 1) & 1), p.err, DEV_TC_PRODUCER_TIMEOUT)) {
                    give_up(DEV_TC_PRODUCER_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(k_full, kKVBytes);
                for (int c = 0; c < 4; ++c)
                    for (int hl = 0; hl < 2; ++hl)
                        tma2d(Kb + (c * 2 + hl) * kKTile, &mapK, hl * kHD + c * 64, kv * p.ctx_pad + blk(kb) * kN,
                              k_full);
                pending = kb & 1;
            }
            // one load at most is outstanding (the previous one was consumed before this issue)
            if (pending >= 0) mbar_wait_bounded(k_full, (uint32_t)pending, p.err, DEV_TC_DRAIN_TIMEOUT);
        }
    } else if (warp == 6) {
        if (lane == 0) {
            // -------------------------------------------------- V^T loader
            int pending = -1;
            for (int kb = 0; kb < nkb && !aborted(); ++kb) {
                if (kb > 0 && !mbar_wait_bounded(pv_done, (uint32_t)((kb - 1) & 1), p.err, DEV_TC_PRODUCER_TIMEOUT)) {
                    give_up(DEV_TC_PRODUCER_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(v_full, kKVBytes);
                // hi rows d at [0, 32 KB), lo at [32, 64 KB)
                for (int hl = 0; hl < 2; ++hl)
                    for (int dc = 0; dc < 4; ++dc)
                        tma2d(Vb + hl * 4 * kKTile + dc * kKTile, &mapVt, blk(kb) * kN, (kv * 2 + hl) * kHD + dc * 64,
                              v_full);
                pending = kb & 1;
            }
            if (pending >= 0) mbar_wait_bounded(v_full, (uint32_t)pending, p.err, DEV_TC_DRAIN_TIMEOUT);
        }
    } else if (warp == 4) {
        if (lane == 0) {
            // -------------------------------------------------- MMA issuer
            const uint32_t q0 = smem_u32(Qs), k0 = smem_u32(Kb), v0 = smem_u32(Vb);
            auto issue_s = [&](int kb) -> bool {
                if (!mbar_wait_bounded(k_full, (uint32_t)(kb & 1), p.err, DEV_TC_MMA_TIMEOUT)) return false;
                fence_after();
                const uint32_t d = tmem + kColS + 64u * (uint32_t)(kb & 1);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint64_t ah = desc128(q0 + c * kQTile);
                    const uint64_t bh = desc128(k0 + (c * 2) * kKTile), bl = desc128(k0 + (c * 2 + 1) * kKTile);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                        const uint32_t al = tmem + kColQl + (uint32_t)(c * 32 + ks * 8);
                        mma_ss(d, ah + adv, bh + adv, kIdescS, (c | ks) != 0 ? 1u : 0u);
                        mma_ss(d, ah + adv, bl + adv, kIdescS, 1u);
                        mma_ts(d, al, bh + adv, kIdescS, 1u);
                    }
                }
                commit(&s_full[kb & 1]);
                commit(k_free);
                return true;
            };
            bool ok = issue_s(0);
            for (int kb = 0; ok && kb < nkb; ++kb) {
                if (aborted()) { ok = false; break; }
                if (kb + 1 < nkb && !(ok = issue_s(kb + 1))) break;
                if (!mbar_wait_bounded(&p_full[kb & 1], (uint32_t)((kb >> 1) & 1), p.err, DEV_TC_MMA_TIMEOUT) ||
                    !mbar_wait_bounded(v_full, (uint32_t)(kb & 1), p.err, DEV_TC_MMA_TIMEOUT)) {
                    ok = false;
                    break;
                }
                fence_after();
                // O += Ph Vh + Ph Vl + Pl Vh over 4 k-steps of 16 keys; P hi / lo in TMEM
                const uint32_t pb = tmem + kColS + 64u * (uint32_t)(kb & 1);
                const uint64_t vh = desc128(v0), vl = desc128(v0 + 4 * kKTile);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t adv = (uint64_t)((ks * 32) >> 4);
                    const uint32_t ph = pb + (uint32_t)(ks * 8), pl = pb + 32u + (uint32_t)(ks * 8);
                    mma_ts(tmem + kColO, ph, vh + adv, kIdescO, (kb | ks) != 0 ? 1u : 0u);
                    mma_ts(tmem + kColO, ph, vl + adv, kIdescO, 1u);
                    mma_ts(tmem + kColO, pl, vh + adv, kIdescO, 1u);
                }
                commit(pv_done);
            }
            if (!ok) give_up(DEV_TC_MMA_TIMEOUT);
            // before the CTA exits every MMA has completed
            commit(mma_done);
            mbar_wait_bounded(mma_done, 0u, p.err, DEV_TC_DRAIN_TIMEOUT);
        }
    } else {
        // -------------------------------------------------- softmax rows
        const float scale2 = 1.4426950408889634f / sqrtf((float)kHD);  // log2(e) / sqrt(HD)
        float m = -INFINITY, l = 0.f;  // running max (log2 units) and sum
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int b = kb & 1;
            ok = mbar_wait_bounded(&s_full[b], (uint32_t)((kb >> 1) & 1), p.err, DEV_TC_EPI_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok && !aborted());
            if (!ok) {
                if (lane == 0) give_up(DEV_TC_EPI_TIMEOUT);
                break;
            }
            fence_after();
            const uint32_t sb = trow + kColS + 64u * (uint32_t)b;
            uint32_t r[4][16];
#pragma unroll
            for (int c = 0; c < 4; ++c) ld16_nowait(sb + c * 16, r[c]);
            ld_wait();
            float s[64];
            float mx = -INFINITY;
            const int key0 = blk(kb) * kN;
            const bool full = valid && key0 + kN - 1 <= qpos;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const float x = __uint_as_float(r[j >> 4][j & 15]) * scale2;
                s[j] = (full || (valid && key0 + j <= qpos)) ? x : -INFINITY;
                mx = fmaxf(mx, s[j]);
            }
            const bool need = mx > m + kRescaleLog2;
            float corr = 1.f;
            if (need) {
                corr = (m == -INFINITY) ? 0.f : exp2f(m - mx);
                m = mx;
            }
            const float mref = (m == -INFINITY) ? 0.f : m;
            float sum = 0.f;
            uint32_t ph[32], pl[32];
#pragma unroll
            for (int j = 0; j < 64; j += 2) {
                const float a = exp2f(s[j] - mref), c2 = exp2f(s[j + 1] - mref);
                sum += a + c2;
                split2(a, c2, ph[j >> 1], pl[j >> 1]);
            }
            l = l * corr + sum;
            if (kb > 0) {
                // every completion of pv_done is confirmed in order, so that each parity
                // wait names one phase; PV(kb - 1) done also frees O for the rescale
                ok = mbar_wait_bounded(pv_done, (uint32_t)((kb - 1) & 1), p.err, DEV_TC_EPI_TIMEOUT);
                ok = __all_sync(0xffffffffu, ok && !aborted());
                if (!ok) {
                    if (lane == 0) give_up(DEV_TC_EPI_TIMEOUT);
                    break;
                }
                if (__any_sync(0xffffffffu, need)) {
                    fence_after();
#pragma unroll 1
                    for (int c = 0; c < kHD / 16; ++c) {
                        uint32_t o[16];
                        ld16_nowait(trow + kColO + c * 16, o);
                        ld_wait();
#pragma unroll
                        for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
                        st16(trow + kColO + c * 16, o);
                    }
                }
            }
            // P over S(kb): hi in columns 0-31, lo in 32-63 of the buffer
            st16(sb, &ph[0]);
            st16(sb + 16, &ph[16]);
            st16(sb + 32, &pl[0]);
            st16(sb + 48, &pl[16]);
            st_wait();
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[b]);
        }
        if (ok) {
            ok = mbar_wait_bounded(pv_done, (uint32_t)((nkb - 1) & 1), p.err, DEV_TC_EPI_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok && !aborted());
            if (!ok && lane == 0) give_up(DEV_TC_EPI_TIMEOUT);
        }
        if (ok && p.nsplit > 1) {
            // partial of this key range: unnormalised O, m, l (combined by k_pf_fattn_combine)
            fence_after();
            const size_t prow = ((size_t)blockIdx.z * p.T + (valid ? ti : 0)) * p.NQ + h;
            float* po = p.part_o + prow * kHD;
#pragma unroll 1
            for (int c = 0; c < kHD / 16; ++c) {
                uint32_t o[16];
                ld16_nowait(trow + kColO + c * 16, o);
                ld_wait();
                if (valid) {
                    float4* d4 = reinterpret_cast<float4*>(po + c * 16);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        d4[e] = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                            __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
                }
            }
            if (valid) *reinterpret_cast<float2*>(p.part_ml + prow * 2) = make_float2(m, l);
        } else if (ok) {
            fence_after();
            const int K = p.NQ * kHD;
            uint16_t* row = p.xs + (size_t)(valid ? ti : 0) * p.ldxs;
            const float* gate = p.proj + (size_t)(valid ? ti : 0) * p.ldp + (size_t)h * 2 * kHD + kHD;
            const float inv_l = 1.0f / l;
#pragma unroll 1
            for (int c = 0; c < kHD / 16; ++c) {
                uint32_t o[16];
                ld16_nowait(trow + kColO + c * 16, o);
                ld_wait();
                if (valid) {
                    uint32_t hw[8], lw[8];
#pragma unroll
                    for (int e = 0; e < 16; e += 2) {
                        const float x0 = __uint_as_float(o[e]) * inv_l * sigmoid_f(gate[c * 16 + e]);
                        const float x1 = __uint_as_float(o[e + 1]) * inv_l * sigmoid_f(gate[c * 16 + e + 1]);
                        split2(x0, x1, hw[e / 2], lw[e / 2]);
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

// Merges the key-range partials of each (token, q head) row: one warp per row, lane l
// holding dims 8l..8l+7; then O / l * sigmoid(gate) as the bf16 pair o_proj reads.
__global__ void __launch_bounds__(256) k_pf_fattn_combine(const FAParams p) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= p.T * p.NQ) return;
    const int ti = row / p.NQ, h = row % p.NQ;
    const int bqt = kM / p.grp, qb = ti / bqt;
    const int t_last = min((qb + 1) * bqt, p.T) - 1;
    const int nkb_all = (p.p0 + t_last) / kN + 1;
    float M = -INFINITY;
    int ns = 0;
    for (int s2 = 0; s2 < p.nsplit; ++s2) {
        int lo, hi;
        fattn_split_range(nkb_all, p.nsplit, s2, lo, hi);
        if (lo >= hi) break;
        M = fmaxf(M, p.part_ml[(((size_t)s2 * p.T + ti) * p.NQ + h) * 2]);
        ++ns;
    }
    float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s2 = 0; s2 < ns; ++s2) {
        const size_t prow = ((size_t)s2 * p.T + ti) * p.NQ + h;
        const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + prow * 2);
        if (ml.x == -INFINITY) continue;  // every key of this range is after the query
        const float f = exp2f(ml.x - M);
        L += ml.y * f;
        const float4* po = reinterpret_cast<const float4*>(p.part_o + prow * kHD + lane * 8);
        const float4 a = po[0], b = po[1];
        o[0] += a.x * f; o[1] += a.y * f; o[2] += a.z * f; o[3] += a.w * f;
        o[4] += b.x * f; o[5] += b.y * f; o[6] += b.z * f; o[7] += b.w * f;
    }
    const float inv_l = 1.0f / L;
    const float* gate = p.proj + (size_t)ti * p.ldp + (size_t)h * 2 * kHD + kHD + lane * 8;
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
        const float x0 = o[e] * inv_l * sigmoid_f(gate[e]);
        const float x1 = o[e + 1] * inv_l * sigmoid_f(gate[e + 1]);
        split2(x0, x1, hw[e / 2], lw[e / 2]);
    }
    const int K = p.NQ * kHD;
    uint16_t* xrow = p.xs + (size_t)ti * p.ldxs;
    *reinterpret_cast<uint4*>(xrow + h * kHD + lane * 8) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(xrow + K + h * kHD + lane * 8) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
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
    p.nsplit = pf_fattn_splits(a.T, a.p0, a.NQ, a.NKV);
    p.part_o = a.part_o;
    p.part_ml = a.part_ml;
    if (p.nsplit > 1 && (!a.part_o || !a.part_ml || a.part_splits < p.nsplit)) return cudaErrorInvalidValue;
    // K and V pairs of the layer: NKV * ctx_pad * (1 KB + 1 KB)
    p.rotate = (size_t)a.NKV * a.ctx_pad * 2048 <= kFattnRotateBytes ? 1 : 0;
    dim3 grid(a.NKV, (a.T + (kM / grp) - 1) / (kM / grp), p.nsplit);
    k_pf_fattn<<<grid, kThreads, kSmem, s>>>(mk, mv, p);
    e = cudaGetLastError();
    if (e != cudaSuccess || p.nsplit == 1) return e;
    k_pf_fattn_combine<<<(a.T * a.NQ + 7) / 8, 256, 0, s>>>(p);
    return cudaGetLastError();
}

// Key splits of one launch. A launch with at least one CTA per SM is not split (measured:
// splitting the 256 CTAs of a one-GPU 2B chunk made the 131072-token pass 0.8 % slower);
// one with fewer (a tensor-parallel rank's few q heads) gets enough splits for about
// kFattnWaves waves, each split at least kFattnMinBlocks key blocks (the query load and
// the epilogue amortised), at most kFattnMaxSplits. QWC_FATTN_SPLITS=n forces n.
int pf_fattn_splits(int T, int p0, int NQ, int NKV) {
    const char* env = std::getenv("QWC_FATTN_SPLITS");  // read per call, like the other prefill switches
    const int forced = env ? std::max(0, std::atoi(env)) : 0;
    if (T <= 0 || NKV <= 0 || NQ % NKV) return 1;
    const int grp = NQ / NKV, bqt = kM / grp;
    const int base = NKV * ((T + bqt - 1) / bqt);
    const int nkb_max = (p0 + T - 1) / kN + 1;
    if (forced > 0) return std::min(forced, kFattnMaxSplits);
    if (base >= num_sms()) return 1;
    int n = (kFattnWaves * num_sms() + base - 1) / base;
    n = std::min(n, std::max(1, nkb_max / kFattnMinBlocks));
    return std::max(1, std::min(n, kFattnMaxSplits));
}

}  // namespace qwc
