// Tensor-core GEMM of the batched forward pass (prefill): for T tokens,
//   Y[n][m] (op)= sum_k X[n][k] * W[m][k]      n < T tokens, m < M output features
// with W the bf16 weight matrix [M][K] (row-major, as stored) and X the fp32 activations.
//
// Precision: the reference multiplies bf16 weights by fp32 activations in fp32
// (forward_pass.cpp:44-75). The tensor cores take bf16 x bf16 products, so every
// activation is carried as an exact-ish pair x = hi + lo of bf16 values (hi = bf16(x),
// lo = bf16(x - hi); |x - hi - lo| <= 2^-17 |x|). Both halves are multiplied by the same
// weight tile and accumulated in fp32 in tensor memory, so Y carries ~16 significant
// bits of every product instead of bf16's 8 -- the error stays well inside the parity
// tolerance while the FLOPs run on tcgen05. Activations live in HBM as [T][2K] bf16
// (hi in columns [0, K), lo in [K, 2K)) and are written in that form by the kernels
// that produce them.
//
// Kernel: one CTA per SM, persistent over 256 x 128 output tiles (256 features x 128
// tokens; feature tile outer, token tile inner, so concurrent CTAs share a weight tile
// through L2). Two 128-row weight tiles share every hi / lo activation tile, so a 64 KB
// stage carries 8 MFLOP.
//   warp 0 (one lane)  TMA producer: 2-D tiled loads (128-byte swizzle) of the two weight
//                      tiles (128 x 64 each) and the hi / lo activation tiles (128 x 64
//                      each) into a 3-stage ring; every CTA loads its own tiles.
//   warp 1             allocates 512 TMEM columns (two tiles in flight, each two fp32
//                      accumulators of 128 x 128); one lane issues tcgen05.mma (M=128,
//                      N=128, K=16, kind::f16, bf16 in, fp32 accumulate) from shared-memory
//                      descriptors and commits each stage back to the producer and each
//                      finished tile to the epilogue.
//   warps 2-9          epilogue: tcgen05.ld of their 32 TMEM lanes (= output features) of
//                      one of the tile's two accumulators (warps 2-5 the first, 6-9 the
//                      second), store / residual add / SwiGLU + hi-lo split, coalesced
//                      across the warp (consecutive features of one token).
// Every wait is bounded: on a timeout the kernel posts an error code and all roles stop.
#include "common.cuh"
#include "kernels.h"
#include "tc_util.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace qwc {

constexpr int kTM = 128, kTN = 128, kTK = 64, kTStages = 3, kTEpiWarps = 8, kTThreads = 64 + 32 * kTEpiWarps;
constexpr int kTileRows = 2 * kTM;               // features per output tile
constexpr uint32_t kTileABytes = kTM * kTK * 2;  // 16 KB
constexpr uint32_t kTileBBytes = kTN * kTK * 2;  // 16 KB
constexpr uint32_t kStageBytes = 2 * kTileABytes + 2 * kTileBBytes;
constexpr int kAccCols = 2 * kTN;                // columns of one tile's two accumulators
constexpr int kTmemCols = 2 * kAccCols;
constexpr size_t kTcSmem = (size_t)kTStages * kStageBytes + 1024 /* align */ + 256 /* barriers */;

// Instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, M=128, N=128.
constexpr uint32_t kIdesc = tc::idesc_bf16(kTM, kTN);

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    tc::ld16_nowait(taddr, r);
    tc::ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// fp32 -> bf16 bits, round to nearest even (finite inputs)
__device__ __forceinline__ uint16_t bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(kTThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap mapW, const __grid_constant__ CUtensorMap mapX,
              const TcGemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kTStages * kStageBytes);
    uint64_t* empty = full + kTStages;
    uint64_t* acc_full = empty + kTStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* mma_done = acc_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    int* s_abort = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntm = (p.M + kTileRows - 1) / kTileRows, ntn = (p.N + kTN - 1) / kTN, ntiles = ntm * ntn;
    const int nkb = p.K / kTK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], kTEpiWarps);
        }
        mbar_init(mma_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(tmem_slot, kTmemCols);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = *tmem_slot;
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(s_abort) != 0; };
    auto abort_with = [&](int code) {
        post_error(p.err, code);
        *reinterpret_cast<volatile int*>(s_abort) = 1;
    };

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------ TMA producer
        long kc = 0;
        for (int tile = blockIdx.x; tile < ntiles && !aborted(); tile += gridDim.x) {
            const int m0 = (tile / ntn) * kTileRows, n0 = (tile % ntn) * kTN;
            for (int kb = 0; kb < nkb; ++kb, ++kc) {
                const int s = (int)(kc % kTStages);
                const uint32_t ph = (uint32_t)((kc / kTStages) & 1);
                if (!mbar_wait_bounded(&empty[s], ph ^ 1u, p.err, DEV_TC_PRODUCER_TIMEOUT)) { abort_with(DEV_TC_PRODUCER_TIMEOUT); break; }
                uint8_t* st = smem + (size_t)s * kStageBytes;
                mbar_arrive_expect_tx(&full[s], kStageBytes);
                // rows past M (a partial or empty second weight tile) read as zero
                tc::tma2d(st, &mapW, kb * kTK, m0, &full[s]);
                tc::tma2d(st + kTileABytes, &mapW, kb * kTK, m0 + kTM, &full[s]);
                tc::tma2d(st + 2 * kTileABytes, &mapX, kb * kTK, n0, &full[s]);
                tc::tma2d(st + 2 * kTileABytes + kTileBBytes, &mapX, p.K + kb * kTK, n0, &full[s]);
            }
        }
        // every stage issued has been consumed (its MMAs completed) before the CTA exits
        for (long k = (kc > kTStages ? kc - kTStages : 0); k < kc; ++k) {
            const int s = (int)(k % kTStages);
            if (!mbar_wait_bounded(&empty[s], (uint32_t)((k / kTStages) & 1), p.err, DEV_TC_DRAIN_TIMEOUT)) break;
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------ MMA issuer
        long kc = 0;
        int it = 0;
        const uint32_t sbase = smem_u32(smem);
        for (int tile = blockIdx.x; tile < ntiles && !aborted(); tile += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1);
            if (!mbar_wait_bounded(&acc_empty[buf], (use & 1u) ^ 1u, p.err, DEV_TC_MMA_TIMEOUT)) { abort_with(DEV_TC_MMA_TIMEOUT); break; }
            tc::fence_after();
            const uint32_t d0 = tmem + (uint32_t)(buf * kAccCols), d1 = d0 + kTN;
            bool ok = true;
            for (int kb = 0; kb < nkb; ++kb, ++kc) {
                const int s = (int)(kc % kTStages);
                const uint32_t ph = (uint32_t)((kc / kTStages) & 1);
                if (!mbar_wait_bounded(&full[s], ph, p.err, DEV_TC_MMA_TIMEOUT)) { ok = false; break; }
                tc::fence_after();
                const uint32_t a0 = sbase + (uint32_t)s * kStageBytes;
                const uint64_t da0 = tc::desc128(a0), da1 = tc::desc128(a0 + kTileABytes),
                               dh = tc::desc128(a0 + 2 * kTileABytes), dl = tc::desc128(a0 + 2 * kTileABytes + kTileBBytes);
#pragma unroll
                for (int ks = 0; ks < kTK / 16; ++ks) {
                    const uint64_t adv = (uint64_t)((ks * 32) >> 4);  // +32 bytes along K
                    const uint32_t first = (kb | ks) != 0 ? 1u : 0u;
                    tc::mma_ss(d0, da0 + adv, dh + adv, kIdesc, first);
                    tc::mma_ss(d0, da0 + adv, dl + adv, kIdesc, 1u);
                    tc::mma_ss(d1, da1 + adv, dh + adv, kIdesc, first);
                    tc::mma_ss(d1, da1 + adv, dl + adv, kIdesc, 1u);
                }
                tc::commit(&empty[s]);  // stage free once these MMAs have read it
            }
            if (!ok) { abort_with(DEV_TC_MMA_TIMEOUT); break; }
            tc::commit(&acc_full[buf]);  // accumulator complete
        }
        tc::commit(mma_done);
        mbar_wait_bounded(mma_done, 0u, p.err, DEV_TC_DRAIN_TIMEOUT);
    } else if (warp >= 2) {
        // ------------------------------------------------ epilogue
        const int q = warp & 3;           // TMEM lanes 32q..32q+31 belong to this warp
        const int half = (warp - 2) >> 2;  // accumulator (weight tile) of this warp
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const int buf = it & 1;
            const uint32_t use = (uint32_t)(it >> 1);
            bool ok = mbar_wait_bounded(&acc_full[buf], use & 1u, p.err, DEV_TC_EPI_TIMEOUT);
            ok = __all_sync(0xffffffffu, ok && !aborted());
            if (!ok) break;
            tc::fence_after();
            const int n0 = (tile % ntn) * kTN;
            for (int c = half * kTN; c < (half + 1) * kTN; c += 16) {
                // columns [0, 128): features m0 + lane row; [128, 256): the second weight tile
                const int m = (tile / ntn) * kTileRows + (c >= kTN ? kTM : 0) + 32 * q + lane;
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * kAccCols);
                float v[16];
                tmem_ld16(taddr + (uint32_t)c, v);
                if (p.epi == TC_SWIGLU_SPLIT) {
                    // rows alternate gate_i (even lane) / up_i (odd lane): the pair swaps
                    // halves so that the even lane forms tokens 0-7 and the odd lane 8-15
                    const bool odd = (lane & 1) != 0;
                    float g8[8], u8[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float send = odd ? v[e] : v[8 + e];
                        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        g8[e] = odd ? recv : v[e];
                        u8[e] = odd ? v[8 + e] : recv;
                    }
                    const int nb = n0 + (c & (kTN - 1)) + (odd ? 8 : 0);
                    if ((m | 1) < p.M) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            if (nb + e < p.N) {
                                const float g = g8[e];
                                const float a = g * __frcp_rn(1.0f + __expf(-g)) * u8[e];
                                const uint16_t hi = bf16_rne(a);
                                const uint16_t lo = bf16_rne(a - __uint_as_float((uint32_t)hi << 16));
                                uint16_t* row = p.ys + (size_t)(nb + e) * p.ldys;
                                row[m >> 1] = hi;
                                row[p.split_k + (m >> 1)] = lo;
                            }
                        }
                    }
                } else if (m < p.M) {
                    const int nb = n0 + (c & (kTN - 1));
                    float* dst = p.y + (size_t)nb * p.ldy + m;
                    if (p.epi == TC_RESIDUAL) {
                        // all 16 residual loads in flight before the adds (one dependent
                        // round trip per 16 tokens instead of one per token)
                        float r[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) r[j] = nb + j < p.N ? dst[(size_t)j * p.ldy] : 0.f;
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (nb + j < p.N) dst[(size_t)j * p.ldy] = r[j] + v[j];
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (nb + j < p.N) dst[(size_t)j * p.ldy] = v[j];
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D bf16 tensor map over a row-major [rows][cols] matrix (row stride ld elements),
// boxes of 128 rows x 64 columns in the 128-byte swizzle; out-of-range rows read as zero.
int tc_make_map(CUtensorMap* map, const void* base, long rows, long cols, long ld) {
    return tc_make_map_box(map, base, rows, cols, ld, kTM);
}

int tc_make_map_box(CUtensorMap* map, const void* base, long rows, long cols, long ld, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return -1;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16 || rows <= 0 || cols <= 0 || ld < cols) return -2;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    if (box_rows <= 0 || box_rows > 256) return -2;
    const cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -3;
}

cudaError_t launch_tc_gemm(const CUtensorMap& mapW, const CUtensorMap& mapX, const TcGemmParams& p,
                           cudaStream_t s) {
    if (p.M <= 0 || p.N <= 0 || p.K <= 0 || p.K % kTK) return cudaErrorInvalidValue;
    if (p.epi == TC_SWIGLU_SPLIT ? (!p.ys || p.M % 2) : !p.y) return cudaErrorInvalidValue;
    static bool attr_done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_tc_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmem);
        if (e != cudaSuccess) return e;
        attr_done[dev] = true;
    }
    const long ntiles = (long)((p.M + kTileRows - 1) / kTileRows) * ((p.N + kTN - 1) / kTN);
    const int grid = (int)std::min<long>(ntiles, num_sms());
    k_tc_gemm<<<grid, kTThreads, kTcSmem, s>>>(mapW, mapX, p);
    return cudaGetLastError();
}

}  // namespace qwc
