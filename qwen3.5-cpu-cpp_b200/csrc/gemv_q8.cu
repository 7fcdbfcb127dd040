// Int8-weight decode GEMV: y = W x with W stored as int8 codes plus one fp32 scale per
// row and 128-column group (w ~= q * scale), x and y fp32, fp32 accumulation.
//
// The reference streams bf16 weights (src/forward_pass.cpp:44-75) and names 8/4-bit
// weights as its next lever for decode speed: a GEMV at batch 1 is bound by the bytes of
// W, so int8 codes halve them (1 B per weight + 4 B per 128 weights). There is no
// reference implementation of the format, so parity is defined against the restated
// arithmetic (dequantise, then the reference's fp32 dot product) rather than against the
// reference's outputs.
//
// Quantisation (qwc_quantize_q8): scale = max |w| / 127 over the group (fp32, from the
// exact bf16 values), q = round-to-nearest-even(w / scale) clamped to [-127, 127]; an
// all-zero group has scale 0 and codes 0.
//
// GEMV kernel: rows split into balanced contiguous ranges, one per warp of a grid of
// 2 x SM CTAs (8 warps each). A warp walks its rows; each lane loads 16 codes (one uint4)
// per 512-column slice of a row, so a 1024-column row is two fully coalesced 512 B loads,
// and keeps up to kRowsInFlight rows of loads outstanding. Lane l's 16 codes belong to
// group (slice * 512 + 16 l) / 128, whose scale multiplies the lane's partial sum before
// the warp reduction: y[r] = sum_lanes scale_l * sum_k q_k x_k.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace qwc {

constexpr int kQ8Warps = 8;
constexpr int kQ8Threads = kQ8Warps * 32;
constexpr int kQ8Group = 128;       // columns per scale
constexpr int kRowsInFlight = 4;    // rows of loads a warp keeps outstanding
constexpr int kQ8MaxIn = 8192;      // x staged in shared memory (32 KB)

__device__ __forceinline__ uint4 ld_stream_q8(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// sum over the 16 signed bytes of w times x[0..15]
__device__ __forceinline__ float dot16_q8(uint4 w, const float* x) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 xv = *reinterpret_cast<const float4*>(x + 4 * i);
        acc = fmaf((float)(int8_t)(u[i] & 0xffu), xv.x, acc);
        acc = fmaf((float)(int8_t)((u[i] >> 8) & 0xffu), xv.y, acc);
        acc = fmaf((float)(int8_t)((u[i] >> 16) & 0xffu), xv.z, acc);
        acc = fmaf((float)(int8_t)(u[i] >> 24), xv.w, acc);
    }
    return acc;
}

__global__ void __launch_bounds__(kQ8Threads, 2)
    k_gemv_q8(const int8_t* __restrict__ W, const float* __restrict__ scales, const float* __restrict__ x,
              float* __restrict__ y, int rows, int in_dim) {
    __shared__ __align__(16) float xs[kQ8MaxIn];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid * 4; i < in_dim; i += kQ8Threads * 4)
        *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
    __syncthreads();
    const long long nw = (long long)gridDim.x * kQ8Warps, gw = (long long)blockIdx.x * kQ8Warps + warp;
    const int r0 = (int)(rows * gw / nw), r1 = (int)(rows * (gw + 1) / nw);
    const int slices = in_dim / 512, ng = in_dim / kQ8Group;
    for (int rb = r0; rb < r1; rb += kRowsInFlight) {
        const int nr = min(kRowsInFlight, r1 - rb);
        float part[kRowsInFlight];
#pragma unroll
        for (int j = 0; j < kRowsInFlight; ++j) part[j] = 0.f;
        for (int s0 = 0; s0 < slices; s0 += 2) {
            // two slices of up to kRowsInFlight rows: every load issued before any use
            uint4 w[kRowsInFlight][2];
            float sc[kRowsInFlight][2];
#pragma unroll
            for (int j = 0; j < kRowsInFlight; ++j)
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    const int sl = s0 + t;
                    if (j < nr && sl < slices) {
                        const size_t r = (size_t)(rb + j);
                        w[j][t] = ld_stream_q8(W + r * in_dim + (size_t)sl * 512 + lane * 16);
                        sc[j][t] = __ldg(scales + r * ng + (sl * 512 + lane * 16) / kQ8Group);
                    } else {
                        w[j][t] = make_uint4(0u, 0u, 0u, 0u);
                        sc[j][t] = 0.f;
                    }
                }
#pragma unroll
            for (int j = 0; j < kRowsInFlight; ++j)
#pragma unroll
                for (int t = 0; t < 2; ++t)
                    if (s0 + t < slices) part[j] = fmaf(sc[j][t], dot16_q8(w[j][t], xs + (s0 + t) * 512 + lane * 16), part[j]);
        }
#pragma unroll
        for (int j = 0; j < kRowsInFlight; ++j) {
            const float v = warp_sum(part[j]);
            if (lane == 0 && j < nr) y[rb + j] = v;
        }
    }
}

// One warp per (row, group): scale = max |w| / 127, codes = rne(w / scale) in [-127, 127].
__global__ void __launch_bounds__(256) k_quantize_q8(const uint16_t* __restrict__ W, int8_t* __restrict__ Wq,
                                                     float* __restrict__ scales, int rows, int in_dim) {
    const int ng = in_dim / kQ8Group;
    const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= (long long)rows * ng) return;
    const int lane = threadIdx.x & 31;
    const long long r = item / ng, g = item % ng;
    const uint16_t* src = W + r * in_dim + g * kQ8Group + lane * 4;
    float v[4], m = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[i] = __uint_as_float((uint32_t)src[i] << 16);
        m = fmaxf(m, fabsf(v[i]));
    }
    m = warp_max(m);
    const float scale = m / 127.0f;
    int8_t* dst = Wq + r * in_dim + g * kQ8Group + lane * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float q = scale > 0.f ? rintf(v[i] / scale) : 0.f;
        q = fminf(fmaxf(q, -127.f), 127.f);
        dst[i] = (int8_t)q;
    }
    if (lane == 0) scales[item] = scale;
}

cudaError_t launch_quantize_q8(const uint16_t* W, int8_t* Wq, float* scales, int rows, int in_dim, cudaStream_t s) {
    if (rows <= 0 || in_dim <= 0 || in_dim % kQ8Group) return cudaErrorInvalidValue;
    const long long items = (long long)rows * (in_dim / kQ8Group);
    k_quantize_q8<<<(unsigned)((items + 7) / 8), 256, 0, s>>>(W, Wq, scales, rows, in_dim);
    return cudaGetLastError();
}

cudaError_t launch_gemv_q8(const int8_t* W, const float* scales, const float* x, float* y, int rows, int in_dim,
                           cudaStream_t s) {
    if (rows <= 0 || in_dim <= 0 || in_dim % 512 || in_dim > kQ8MaxIn) return cudaErrorInvalidValue;
    const int grid = std::min(2 * num_sms(), std::max(1, (rows + kQ8Warps - 1) / kQ8Warps));
    k_gemv_q8<<<grid, kQ8Threads, 0, s>>>(W, scales, x, y, rows, in_dim);
    return cudaGetLastError();
}

}  // namespace qwc
