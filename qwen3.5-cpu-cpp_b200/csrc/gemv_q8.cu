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
// 2 x SM CTAs (8 warps each). A warp walks its rows in batches of kRowsInFlight rows x two
// 512-column slices; each lane loads 16 codes (one uint4) per slice of a row, so a
// 1024-column row is two fully coalesced 512 B loads, and the next batch's loads are
// issued before the current batch is consumed (two register buffers). Lane l's 16 codes
// belong to group (slice * 512 + 16 l) / 128, whose scale multiplies the lane's partial
// sum before the warp reduction: y[r] = sum_lanes scale_l * sum_k q_k x_k.
//
// What bounds it: every code needs a conversion and an FMA, and every slice needs 64 B of
// x per lane from shared memory. x is therefore read once per slice into registers and
// used for all rows of the batch (reading it per row made shared memory the limit at
// ~1.8 TB/s), the shared copy is padded by 4 floats per 32 so the lanes' 16-float runs
// fall in distinct banks, and codes are converted with the exponent-bias construction
// (below) instead of the slower integer-to-float conversion unit.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace qwc {

constexpr int kQ8Warps = 8;
constexpr int kQ8Threads = kQ8Warps * 32;
constexpr int kQ8Group = 128;       // columns per scale
constexpr int kRowsInFlight = 4;    // rows of loads a warp keeps outstanding
constexpr int kQ8MaxIn = 8192;      // x staged in shared memory (36 KB with padding)

__device__ __forceinline__ uint4 ld_stream_q8(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Signed byte -> fp32 by the exponent-bias construction: with the sign bit flipped the
// byte is the unsigned u = q + 128, and the fp32 bit pattern 0x4B0000uu is exactly
// 2^23 + u (the ulp of 2^23 is 1), so subtracting 2^23 + 128 leaves q exactly. One byte
// permute and one add per code, both on the full-rate pipes.
constexpr float kQ8Bias = 8388736.0f;  // 2^23 + 128
__device__ __forceinline__ float q8_code(uint32_t flipped, uint32_t sel) {
    return __uint_as_float(__byte_perm(flipped, 0x4B000000u, sel)) - kQ8Bias;
}
// sum over the 16 signed bytes of w times xv[0..3] (16 floats), in byte order
__device__ __forceinline__ float dot16_q8(uint4 w, const float4 (&xv)[4]) {
    const uint32_t u[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc = fmaf(q8_code(u[i], 0x7540), xv[i].x, acc);
        acc = fmaf(q8_code(u[i], 0x7541), xv[i].y, acc);
        acc = fmaf(q8_code(u[i], 0x7542), xv[i].z, acc);
        acc = fmaf(q8_code(u[i], 0x7543), xv[i].w, acc);
    }
    return acc;
}
// Shared-memory index of x[e]: 4 floats of padding after every 32.
__device__ __forceinline__ int q8_xpad(int e) { return e + ((e >> 5) << 2); }

// One batch: kRowsInFlight rows x two 512-column slices of this lane's codes and scales.
struct Q8Batch {
    uint4 w[kRowsInFlight][2];
    float sc[kRowsInFlight][2];
};
__device__ __forceinline__ void q8_issue(Q8Batch& B, const int8_t* __restrict__ W, const float* __restrict__ scales,
                                         int rb, int r1, int s0, int slices, int in_dim, int ng, int lane) {
#pragma unroll
    for (int j = 0; j < kRowsInFlight; ++j)
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int sl = s0 + t;
            if (rb + j < r1 && sl < slices) {
                const size_t r = (size_t)(rb + j);
                B.w[j][t] = ld_stream_q8(W + r * in_dim + (size_t)sl * 512 + lane * 16);
                B.sc[j][t] = __ldg(scales + r * ng + (sl * 512 + lane * 16) / kQ8Group);
            } else {
                B.w[j][t] = make_uint4(0u, 0u, 0u, 0u);
                B.sc[j][t] = 0.f;
            }
        }
}

// Folds batch `bi` (row block rb, slices s0, s0+1) into the partial sums; at the end of a
// row block, reduces them and writes the rows. Per slice the lane's 16 x values are read
// once and used for every row of the batch.
__device__ __forceinline__ void q8_consume(const Q8Batch& B, float (&part)[kRowsInFlight], const float* xs, int bi,
                                           int spb, int r0, int r1, int slices, int lane, float* __restrict__ y) {
    const int rb = r0 + (bi / spb) * kRowsInFlight, s0 = (bi % spb) * 2;
    float dot[kRowsInFlight][2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        float4 xv[4];
        const int e0 = (s0 + t) * 512 + lane * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            xv[i] = s0 + t < slices ? *reinterpret_cast<const float4*>(xs + q8_xpad(e0 + 4 * i))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < kRowsInFlight; ++j) dot[j][t] = dot16_q8(B.w[j][t], xv);
    }
#pragma unroll
    for (int j = 0; j < kRowsInFlight; ++j)
#pragma unroll
        for (int t = 0; t < 2; ++t)
            if (s0 + t < slices) part[j] = fmaf(B.sc[j][t], dot[j][t], part[j]);
    if (bi % spb == spb - 1) {  // the row block is complete
#pragma unroll
        for (int j = 0; j < kRowsInFlight; ++j) {
            const float v = warp_sum(part[j]);
            if (lane == 0 && rb + j < r1) y[rb + j] = v;
            part[j] = 0.f;
        }
    }
}

__global__ void __launch_bounds__(kQ8Threads, 2)
    k_gemv_q8(const int8_t* __restrict__ W, const float* __restrict__ scales, const float* __restrict__ x,
              float* __restrict__ y, int rows, int in_dim) {
    extern __shared__ __align__(16) float xs[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long nw = (long long)gridDim.x * kQ8Warps, gw = (long long)blockIdx.x * kQ8Warps + warp;
    const int r0 = (int)(rows * gw / nw), r1 = (int)(rows * (gw + 1) / nw);
    const int slices = in_dim / 512, ng = in_dim / kQ8Group;
    const int spb = (slices + 1) / 2;  // batches per row block (two slices each)
    const int nbatch = ((r1 - r0 + kRowsInFlight - 1) / kRowsInFlight) * spb;
    // batch i covers row block i / spb and slices 2 (i % spb), +1
    auto issue = [&](Q8Batch& B, int i) {
        q8_issue(B, W, scales, r0 + (i / spb) * kRowsInFlight, r1, (i % spb) * 2, slices, in_dim, ng, lane);
    };
    // two register buffers, named (not indexed) so they stay in registers; the first
    // batch's codes do not depend on x and are issued before x is staged
    Q8Batch A, B;
    if (nbatch > 0) issue(A, 0);
    for (int i = tid * 4; i < in_dim; i += kQ8Threads * 4)
        *reinterpret_cast<float4*>(xs + q8_xpad(i)) = *reinterpret_cast<const float4*>(x + i);
    __syncthreads();
    float part[kRowsInFlight];
#pragma unroll
    for (int j = 0; j < kRowsInFlight; ++j) part[j] = 0.f;
    for (int bi = 0; bi < nbatch; bi += 2) {
        if (bi + 1 < nbatch) issue(B, bi + 1);  // next batch in flight while this one is used
        q8_consume(A, part, xs, bi, spb, r0, r1, slices, lane, y);
        if (bi + 1 >= nbatch) break;
        if (bi + 2 < nbatch) issue(A, bi + 2);
        q8_consume(B, part, xs, bi + 1, spb, r0, r1, slices, lane, y);
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
    const size_t smem = (size_t)(in_dim + in_dim / 8) * sizeof(float);  // q8_xpad(in_dim - 1) < in_dim * 9 / 8
    k_gemv_q8<<<grid, kQ8Threads, smem, s>>>(W, scales, x, y, rows, in_dim);
    return cudaGetLastError();
}

}  // namespace qwc
