// Peer-memory all-reduce of the tensor-parallel residual stream.
//
// After each row-parallel projection (out_proj / o_proj / down_proj) every rank holds a
// partial [T][H] (rank 0's already includes the residual) that must be summed across the
// group and left, identical, on every rank. NCCL's all-reduce of the 32-64 MB messages ran
// at about 300 GB/s of bus bandwidth on 8 GPUs. Here each rank's residual buffer is
// mapped into every other rank's address space and the sum is taken with plain loads and
// stores over NVLink in two steps of one kernel (a "two-shot" all-reduce):
//   rank r sums slice r of every rank's buffer, in rank order 0..N-1 (the same value on
//   every rank, run to run), and stores the sum into slice r of every rank's buffer;
// between cross-rank barriers before (every rank's projection is complete) and after
// (every rank's stores have landed). Per rank it moves (N-1)/N of the buffer in each
// direction of its links, like a ring, in one pass instead of 2 (N-1) steps.
//
// Memory: each buffer is a driver virtual-memory allocation exported as a POSIX file
// descriptor; the descriptors travel to the other ranks over abstract Unix sockets named
// after the group's NCCL id (exchange_fds, host/src/fd_exchange.cpp), and every rank
// imports and maps the others. An imported
// allocation stays alive while it is mapped, so a rank that exits does not unmap the
// others' view of its memory. No multicast object is created. Before use, every rank
// reads a token each peer wrote into its buffer through the mapping (a host-driven copy),
// and the engine has the group vote on the result: all ranks use the peer path or none.
//
// Barriers: a one-warp kernel; lane q stores the barrier's epoch into rank q's flag array
// at this rank's slot (release, system scope) after a system-scope fence, then polls this
// rank's own array until every slot holds the epoch (acquire). Every wait is bounded: on
// expiry the kernel posts DEV_TP_BARRIER_TIMEOUT, the reduction kernel that follows sees
// the error word and touches no peer memory, and the host aborts the group.
#include "common.cuh"
#include "kernels.h"
#include "../host/src/fd_exchange.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <unistd.h>

#include <cstring>

namespace qwc {

namespace {

constexpr size_t kP2pHeader = 256;  // [0, 64): flags[8] (epochs); [128, 136): the setup token
constexpr uint32_t kP2pMagic = 0x71776332u;  // in the setup token
static_assert(kP2pMaxRanks <= kFdExchangeMaxRanks, "descriptor exchange group size");

struct DriverFns {
    PFN_cuMemCreate_v10020 create = nullptr;
    PFN_cuMemRelease_v10020 release = nullptr;
    PFN_cuMemAddressReserve_v10020 reserve = nullptr;
    PFN_cuMemAddressFree_v10020 addr_free = nullptr;
    PFN_cuMemMap_v10020 map = nullptr;
    PFN_cuMemUnmap_v10020 unmap = nullptr;
    PFN_cuMemSetAccess_v10020 set_access = nullptr;
    PFN_cuMemExportToShareableHandle_v10020 export_h = nullptr;
    PFN_cuMemImportFromShareableHandle_v10020 import_h = nullptr;
    PFN_cuMemGetAllocationGranularity_v10020 granularity = nullptr;
    bool ok = false;
};
template <class F>
bool entry(const char* name, F& fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &f, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return false;
    fn = reinterpret_cast<F>(f);
    return true;
}
const DriverFns& drv() {
    static DriverFns d = [] {
        DriverFns x;
        x.ok = entry("cuMemCreate", x.create) && entry("cuMemRelease", x.release) &&
               entry("cuMemAddressReserve", x.reserve) && entry("cuMemAddressFree", x.addr_free) &&
               entry("cuMemMap", x.map) && entry("cuMemUnmap", x.unmap) && entry("cuMemSetAccess", x.set_access) &&
               entry("cuMemExportToShareableHandle", x.export_h) &&
               entry("cuMemImportFromShareableHandle", x.import_h) &&
               entry("cuMemGetAllocationGranularity", x.granularity);
        return x;
    }();
    return d;
}

struct Mapping {
    CUmemGenericAllocationHandle handle = 0;
    CUdeviceptr va = 0;
    size_t size = 0;
};
void unmap(Mapping& m) {
    const DriverFns& d = drv();
    if (m.va) {
        d.unmap(m.va, m.size);
        d.addr_free(m.va, m.size);
    }
    if (m.handle) d.release(m.handle);
    m = Mapping();
}
// Maps allocation `h` into a fresh address range with read/write access for `device`. On
// failure nothing stays reserved or mapped, `m` is left empty and the caller still owns `h`.
bool map_handle(Mapping& m, CUmemGenericAllocationHandle h, size_t size, int device) {
    const DriverFns& d = drv();
    m = Mapping();
    CUdeviceptr va = 0;
    if (d.reserve(&va, size, 0, 0, 0) != CUDA_SUCCESS) return false;
    if (d.map(va, size, 0, h, 0) != CUDA_SUCCESS) {
        d.addr_free(va, size);
        return false;
    }
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    if (d.set_access(va, size, &acc, 1) != CUDA_SUCCESS) {
        d.unmap(va, size);
        d.addr_free(va, size);
        return false;
    }
    m.handle = h;
    m.va = va;
    m.size = size;
    return true;
}

}  // namespace

struct P2pGroup {
    int rank = 0, world = 1, device = 0;
    size_t bytes = 0;  // per-rank allocation (header + data)
    Mapping map[kP2pMaxRanks];  // [rank]: own allocation at map[rank]
    P2pPtrs ptrs{};
};

void p2p_destroy(P2pGroup* g) {
    if (!g) return;
    for (int q = 0; q < g->world; ++q) unmap(g->map[q]);
    delete g;
}

float* p2p_local_data(P2pGroup* g) { return g->ptrs.data[g->rank]; }
size_t p2p_capacity_floats(const P2pGroup* g) { return (g->bytes - kP2pHeader) / sizeof(float); }

int p2p_setup(P2pGroup** out, int rank, int world, int device, uint64_t group, int gen, size_t data_bytes,
              int timeout_ms, std::string& why) {
    *out = nullptr;
    const DriverFns& d = drv();
    if (!d.ok) {
        why = "driver virtual-memory entry points unavailable";
        return -1;
    }
    if (world < 2 || world > kP2pMaxRanks || rank < 0 || rank >= world) {
        why = "group size outside 2..8";
        return -1;
    }
    P2pGroup* g = new P2pGroup;
    g->rank = rank;
    g->world = world;
    g->device = device;
    auto bail = [&](const std::string& w) {
        why = w;
        p2p_destroy(g);
        return -1;
    };
    // ---- own allocation, exportable as a file descriptor
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = device;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    if (d.granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || gran == 0)
        return bail("cuMemGetAllocationGranularity failed");
    g->bytes = (kP2pHeader + data_bytes + gran - 1) / gran * gran;
    CUmemGenericAllocationHandle own = 0;
    if (d.create(&own, g->bytes, &prop, 0) != CUDA_SUCCESS) return bail("cuMemCreate failed");
    if (!map_handle(g->map[rank], own, g->bytes, device)) {
        d.release(own);
        return bail("mapping the own allocation failed");
    }
    // zero flags, write this rank's token (read by the peers through their mappings)
    uint8_t* base = reinterpret_cast<uint8_t*>(g->map[rank].va);
    const uint64_t token = ((uint64_t)kP2pMagic << 32) ^ ((uint64_t)gen << 8) ^ (uint64_t)rank;
    if (cudaMemset(base, 0, kP2pHeader) != cudaSuccess ||
        cudaMemcpy(base + 128, &token, sizeof(token), cudaMemcpyHostToDevice) != cudaSuccess)
        return bail("initialising the own allocation failed");
    int fd = -1;
    if (d.export_h(&fd, own, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) != CUDA_SUCCESS || fd < 0)
        return bail("cuMemExportToShareableHandle failed");
    // ---- exchange descriptors with the other ranks (bounded by timeout_ms)
    int fds[kP2pMaxRanks];
    uint64_t sizes[kP2pMaxRanks];
    const bool ok_x = exchange_fds(group, gen, rank, world, fd, (uint64_t)g->bytes, timeout_ms, fds, sizes, why);
    close(fd);
    if (!ok_x) return bail(why);
    bool ok = true;
    // ---- import and map every peer's allocation
    for (int q = 0; q < world && ok; ++q) {
        if (q == rank) continue;
        CUmemGenericAllocationHandle ph = 0;
        if (d.import_h(&ph, reinterpret_cast<void*>((uintptr_t)fds[q]), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) !=
            CUDA_SUCCESS) {
            ok = false;
            why = "cuMemImportFromShareableHandle failed for rank " + std::to_string(q);
            break;
        }
        if (!map_handle(g->map[q], ph, sizes[q], device)) {
            d.release(ph);
            ok = false;
            why = "mapping rank " + std::to_string(q) + "'s allocation failed";
        }
    }
    for (int q = 0; q < world; ++q)
        if (fds[q] >= 0) close(fds[q]);
    if (!ok) return bail(why);
    // ---- every peer's token through the mapping
    for (int q = 0; q < world; ++q) {
        uint64_t t = 0;
        const uint64_t want = ((uint64_t)kP2pMagic << 32) ^ ((uint64_t)gen << 8) ^ (uint64_t)q;
        if (cudaMemcpy(&t, reinterpret_cast<uint8_t*>(g->map[q].va) + 128, sizeof(t), cudaMemcpyDeviceToHost) !=
                cudaSuccess ||
            t != want)
            return bail("rank " + std::to_string(q) + "'s buffer is not readable through the mapping");
    }
    for (int q = 0; q < world; ++q) {
        g->ptrs.flags[q] = reinterpret_cast<unsigned long long*>(g->map[q].va);
        g->ptrs.data[q] = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(g->map[q].va) + kP2pHeader);
    }
    g->ptrs.world = world;
    g->ptrs.rank = rank;
    *out = g;
    return 0;
}

// ---------------------------------------------------------------------- kernels
__global__ void k_p2p_barrier(const P2pPtrs P, unsigned long long epoch, unsigned long long wait_ns, int* err) {
    const int lane = threadIdx.x;
    // the projection's stores (earlier kernels on this stream) and, for the closing
    // barrier, the reduction's stores into the peers' buffers, before the signal
    asm volatile("fence.sc.sys;" ::: "memory");
    __syncwarp();
    if (lane < P.world) {
        unsigned long long* slot = P.flags[lane] + P.rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(slot), "l"(epoch) : "memory");
        const unsigned long long* f = P.flags[P.rank] + lane;
        const volatile int* e = err;
        const unsigned long long t0 = globaltimer_ns();
        for (unsigned it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
            if (v >= epoch) break;
            // an earlier barrier of this pass ran out: the group is already lost, do not
            // wait again (every later barrier of the pass returns at once)
            if ((it & 63u) == 0 && *e != 0) break;
            if (globaltimer_ns() - t0 > wait_ns) {
                post_error(err, DEV_TP_BARRIER_TIMEOUT);
                break;
            }
        }
    }
    __syncwarp();
}

__device__ __forceinline__ float4 ld_cg4(const float* p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ void st_cg4(float* p, float4 v) {
    asm volatile("st.global.cg.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Slice `rank` of n floats (n % 4 == 0): sum over the ranks' buffers in rank order, the
// sum stored into every rank's buffer. Skipped entirely after a barrier error. Each thread
// takes two elements a grid stride apart with all their loads issued first (peer loads
// cross NVLink: more of them in flight).
__global__ void __launch_bounds__(256) k_p2p_reduce(const P2pPtrs P, long long n4, const int* err) {
    if (*reinterpret_cast<const volatile int*>(err) != 0) return;
    const long long per = (n4 + P.world - 1) / P.world;
    const long long a = (long long)P.rank * per, b = a + per < n4 ? a + per : n4;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = a + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < b; i += 2 * stride) {
        const long long i2 = i + stride;
        const bool two = i2 < b;
        float4 v[2][kP2pMaxRanks];
#pragma unroll
        for (int q = 0; q < kP2pMaxRanks; ++q)
            if (q < P.world) {
                v[0][q] = ld_cg4(P.data[q] + 4 * i);
                if (two) v[1][q] = ld_cg4(P.data[q] + 4 * i2);
            }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (u == 1 && !two) break;
            float4 s = v[u][0];
#pragma unroll
            for (int q = 1; q < kP2pMaxRanks; ++q)
                if (q < P.world) {
                    s.x += v[u][q].x;
                    s.y += v[u][q].y;
                    s.z += v[u][q].z;
                    s.w += v[u][q].w;
                }
            const long long e = u == 0 ? i : i2;
#pragma unroll
            for (int q = 0; q < kP2pMaxRanks; ++q)
                if (q < P.world) st_cg4(P.data[q] + 4 * e, s);
        }
    }
}

cudaError_t p2p_allreduce(P2pGroup* g, size_t n, unsigned long long& epoch, unsigned long long wait_ns, int* err,
                          cudaStream_t s) {
    if (n % 4 || n > p2p_capacity_floats(g)) return cudaErrorInvalidValue;
    k_p2p_barrier<<<1, 32, 0, s>>>(g->ptrs, ++epoch, wait_ns, err);
    k_p2p_reduce<<<2 * num_sms(), 256, 0, s>>>(g->ptrs, (long long)(n / 4), err);
    k_p2p_barrier<<<1, 32, 0, s>>>(g->ptrs, ++epoch, wait_ns, err);
    return cudaGetLastError();
}

}  // namespace qwc
