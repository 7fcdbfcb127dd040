// Persistent decode-step kernel: one launch runs a whole QwenModel::step()
// (src/qwen_model.cpp:211-239) -- embedding, every layer, final norm, lm_head and the
// greedy argmax -- as a sequence of phases separated by grid-wide barriers.
//
// Why: at batch 1 every projection is a small GEMV (1-17 MB). As separate kernels each
// one pays a launch plus several dependent memory round trips after its input is ready,
// and can keep only ~64 KB of weights in flight per SM in registers. Here one CTA per SM
// lives for the whole step. Eight consumer warps compute; each owns a contiguous range
// of every GEMV's rows and reads them from its own ring of 4 KB shared-memory slots. A
// ninth, producer warp fills the rings with 1-D bulk TMA copies (cp.async.bulk, L2
// evict-first): its lane w walks consumer w's rows of every GEMV phase of the step in
// order and refills a slot as soon as the consumer releases it (empty / full mbarrier
// pair per slot). The producer never waits for a phase barrier -- weights never depend
// on activations -- so HBM keeps streaming while the grid waits, while the GDN recurrence
// and the attention run and while activations are exchanged, and the consumers never
// spend time issuing copies (an issuing thread is held ~0.4 us per copy).
//
// Phase types (descriptors built once on the host, in global memory, staged per phase
// in shared memory):
//   GEMV  y = W x with the fused prologues/epilogues of the GEMV family (kernels.h);
//         rows split into NC balanced CTA ranges, each into 8 balanced warp ranges;
//         a warp's range is one contiguous byte stream consumed in 512 B groups.
//   GDN   the recurrent mixer core (gdn_body.cuh), one (value head, 16-column) item per
//         CTA on warps 0-3; the state slice is loaded before the barrier.
//   ATTN  split-K decode attention (attn_body.cuh), one (kv head, split) item per CTA.
// Each phase body is a separate non-inlined function so that it gets its own register
// allocation (one inlined body would spill the others' hot loops).
//
// Barrier: every CTA adds 1 to a 64-bit arrival counter after a phase (release); phase p
// may start when the counter reaches p * NC (acquire). The last CTA to finish the step
// resets it. CTA-level synchronisation inside the step is a named barrier over the 256
// consumer threads (the producer warp runs its own loop). All waits are bounded (they
// post an error code and stop the step instead of hanging), and the kernel is launched
// cooperatively, so all CTAs are co-resident.
#include "attn_body.cuh"
#include "gdn_body.cuh"

#include <algorithm>
#include <type_traits>

namespace qwc {

constexpr int kSW = 8;                 // consumer warps per CTA (each owns GEMV rows)
constexpr int kSThreads = kSW * 32;    // consumer threads
constexpr int kBlockThreads = kSThreads + 32;  // + the producer warp
constexpr int kChunkBytes = 4096;      // one ring slot = one bulk copy
constexpr int kGroupBytes = 512;       // 32 lanes x 16 B
constexpr int kGroupsPerChunk = kChunkBytes / kGroupBytes;
constexpr int kMaxSlots = 8;

// Compact per-phase stream description kept in shared memory for the issue cursor.
struct PhaseBrief {
    const uint16_t* W;  // nullptr: not a GEMV phase
    int rows, in_dim;
};

// Consumer cursor of one warp's ring, kept in shared memory between phases.
struct RingState {
    int consumed;         // chunks consumed so far
    int cslot;            // slot of the next chunk to consume
    uint32_t cpar;        // full-barrier parity of that slot
};

// Block-shared bookkeeping of the step kernel.
struct StepShared {
    uint8_t* ring;        // [kSW][nslot][kChunkBytes]
    float* xs;            // GEMV input vector
    uint64_t* full;       // [kSW][nslot] mbarriers: slot filled (producer -> consumer)
    uint64_t* empty;      // [kSW][nslot] mbarriers: slot released (consumer -> producer)
    int issued[kSW];      // chunks the producer issued per consumer warp
    PhaseBrief* brief;    // [nphases]
    StepPhase* ph;        // staged descriptor of the current phase
    RingState rings[kSW];
    double red_d[kSW];
    float rv[kSW];
    int ri[kSW];
    int s_last;
    int abort;            // CTA-uniform: an error was posted
};

struct StepSmem {
    size_t ring, xs, bars, brief, phase, total;
};
static __host__ __device__ inline StepSmem step_smem_plan(int nslot, int xs_max, int nphases) {
    StepSmem s;
    s.ring = 0;
    s.xs = (size_t)kSW * nslot * kChunkBytes;
    s.bars = s.xs + (((size_t)xs_max * 4 + 127) / 128) * 128;
    s.brief = s.bars + (((size_t)2 * kSW * nslot * 8 + 15) / 16) * 16;
    s.phase = s.brief + (((size_t)nphases * sizeof(PhaseBrief) + 127) / 128) * 128;
    s.total = s.phase + ((sizeof(StepPhase) + 127) / 128) * 128;
    return s;
}

// rows [a, b) of warp w in CTA c for a GEMV phase
__device__ __forceinline__ void warp_rows(int rows, int c, int nc, int w, int& a, int& b) {
    const int r0 = (int)((long long)rows * c / nc), r1 = (int)((long long)rows * (c + 1) / nc);
    const int nr = r1 - r0;
    a = r0 + (int)((long long)nr * w / kSW);
    b = r0 + (int)((long long)nr * (w + 1) / kSW);
}

// dot of 8 bf16 weights (one uint4) with 8 fp32 x values in shared memory
__device__ __forceinline__ float dot8s(uint4 w, const float* x, float acc) {
    const float4 x0 = *reinterpret_cast<const float4*>(x);
    const float4 x1 = *reinterpret_cast<const float4*>(x + 4);
    acc = fmaf(bf16lo(w.x), x0.x, acc);
    acc = fmaf(bf16hi(w.x), x0.y, acc);
    acc = fmaf(bf16lo(w.y), x0.z, acc);
    acc = fmaf(bf16hi(w.y), x0.w, acc);
    acc = fmaf(bf16lo(w.z), x1.x, acc);
    acc = fmaf(bf16hi(w.z), x1.y, acc);
    acc = fmaf(bf16lo(w.w), x1.z, acc);
    acc = fmaf(bf16hi(w.w), x1.w, acc);
    return acc;
}

__device__ __forceinline__ unsigned long long step_wait_ns(const StepParams& sp) {
    return sp.wait_ns ? sp.wait_ns : kWaitLimitNs;
}

__device__ __forceinline__ bool step_aborted(const StepParams& sp) {
    return *reinterpret_cast<const volatile int*>(sp.dev_err) != 0;
}

__device__ __forceinline__ void trace_mark(const StepParams& sp, int c, int p, int k) {
    if (sp.trace && threadIdx.x == 0)
        sp.trace[((size_t)c * sp.nphases + p) * 8 + k] = (long long)globaltimer_ns();
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Barrier over the 256 consumer threads (named barrier 3); the producer warp is not in it.
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 3, 256;" ::: "memory"); }

// mbarrier wait that also gives up once another CTA has posted an error
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, uint32_t parity, const StepParams& sp, int err) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0 && step_aborted(sp)) return false;
        if (globaltimer_ns() - t0 > step_wait_ns(sp)) {
            post_error(sp.dev_err, err);
            return false;
        }
    }
}

// Producer warp: lane w streams consumer warp w's rows of every GEMV phase of the step,
// in phase order, into that warp's ring, refilling a slot as soon as it is released.
__device__ __noinline__ void producer(StepShared& S, const StepParams sp, int c, int nc) {
    const int w = threadIdx.x & 31;
    if (w >= kSW) return;
    const int nslot = sp.nslot;
    uint8_t* ring = S.ring + (size_t)w * nslot * kChunkBytes;
    uint64_t* full = S.full + w * nslot;
    uint64_t* empty = S.empty + w * nslot;
    const uint64_t pol = l2_policy_evict_first();
    int issued = 0;
    bool ok = true;
    for (int p = 0; p < sp.nphases && ok; ++p) {
        const PhaseBrief bf = S.brief[p];
        if (!bf.W) continue;
        int a, b;
        warp_rows(bf.rows, c, nc, w, a, b);
        const long long bytes = (long long)(b - a) * bf.in_dim * 2;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(bf.W + (size_t)a * bf.in_dim);
        for (long long off = 0; off < bytes; off += kChunkBytes) {
            const int slot = issued % nslot;
            const uint32_t ph = (uint32_t)((issued / nslot) & 1);
            if (!mbar_wait_or_abort(&empty[slot], ph ^ 1u, sp, DEV_GEMV_EMPTY_TIMEOUT)) {
                ok = false;
                break;
            }
            const uint32_t len = (uint32_t)min((long long)kChunkBytes, bytes - off);
            mbar_arrive_expect_tx(&full[slot], len);
            bulk_g2s_hint(ring + (size_t)slot * kChunkBytes, src + off, len, &full[slot], pol);
            ++issued;
        }
    }
    S.issued[w] = issued;
}

// Grid barrier: all CTAs finished phase p-1 (acquire of the arrival counter, which every
// CTA bumps with a release after its CTA barrier). Leaves S.abort CTA-uniform.
//
// The poll is the critical path of every phase, so each iteration is one acquire load of
// the counter and nothing else: the error word is read once, issued together with the
// first poll (its value is only needed after the wait), and again every 16 iterations of
// a long wait. An error posted while this barrier is pending stops the CTA at the next one.
__device__ __noinline__ void grid_wait(StepShared& S, const StepParams sp, int p, int c, int nc) {
    const int tid = threadIdx.x;
    if (tid == 0) {
        const int err0 = *reinterpret_cast<const volatile int*>(sp.dev_err);  // in flight with the poll
        int ab = 0;
        if (p > 0) {
            const unsigned long long target = (unsigned long long)p * nc;
            if (ld_acquire_u64(sp.bar) < target) {
                const unsigned long long t0 = globaltimer_ns();
                for (unsigned it = 1; ld_acquire_u64(sp.bar) < target; ++it) {
                    if ((it & 15u) != 0) continue;
                    if (step_aborted(sp)) { ab = 1; break; }
                    if (globaltimer_ns() - t0 > step_wait_ns(sp)) {
                        post_error(sp.dev_err, DEV_STEP_BARRIER_TIMEOUT);
                        ab = 1;
                        break;
                    }
                }
            }
        }
        S.abort = (ab || err0 != 0) ? 1 : 0;
    }
    cta_sync();
    trace_mark(sp, c, p, 1);
}

// ---------------------------------------------------------------------- GEMV streams
// One warp's weight stream of a GEMV phase: read-only context and the cursor state that
// persists across phases. The stream functions are separate non-inlined templates (one
// per epilogue / shape) so that each gets its own register allocation; they copy what
// they need into registers on entry and write the state back on exit.
struct StreamCtx {
    const uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    const float* xs;
    float* y;
    int nslot, b, bytes, in, xlen;
    bool trace;
};
struct StreamState {
    RingState r;
    int row, res_base;
    float res, best;
    int best_idx;
    long long waited_ns;
    int nchunks;
};

// Registers of a stream: the cursor and the epilogue state.
struct StreamRegs {
    const uint8_t* ring;
    uint64_t* full;
    uint64_t* empty;
    float* y;
    int nslot, b, lane;
    bool trace;
    RingState r;
    int row, res_base;
    float res, best;
    int best_idx;
    long long waited_ns;
    int nchunks;

    __device__ __forceinline__ StreamRegs(const StreamCtx& cx, const StreamState& st) {
        ring = cx.ring; full = cx.full; empty = cx.empty; y = cx.y;
        nslot = cx.nslot; b = cx.b; trace = cx.trace; lane = threadIdx.x & 31;
        r = st.r; row = st.row; res_base = st.res_base; res = st.res; best = st.best;
        best_idx = st.best_idx; waited_ns = st.waited_ns; nchunks = st.nchunks;
    }
    __device__ __forceinline__ void save(StreamState& st) const {
        st.r = r; st.row = row; st.res_base = res_base; st.res = res; st.best = best;
        st.best_idx = best_idx; st.waited_ns = waited_ns; st.nchunks = nchunks;
    }
    __device__ __forceinline__ bool next_chunk(const uint4*& wv, const StepParams& sp) {
        const unsigned long long tw = trace ? globaltimer_ns() : 0ull;
        if (!mbar_wait_or_abort(&full[r.cslot], r.cpar, sp, DEV_GEMV_FULL_TIMEOUT)) return false;
        if (trace) {
            waited_ns += (long long)(globaltimer_ns() - tw);
            ++nchunks;
        }
        wv = reinterpret_cast<const uint4*>(ring + (size_t)r.cslot * kChunkBytes);
        return true;
    }
    __device__ __forceinline__ void release_chunk() {
        __syncwarp();  // every lane's reads of the slot are done
        if (lane == 0) mbar_arrive(&empty[r.cslot]);
        ++r.consumed;
        if (++r.cslot == nslot) { r.cslot = 0; r.cpar ^= 1u; }
    }
    // epilogue of one finished row (lane 0 stores); residuals prefetched 32 rows at a time
    template <int EPI>
    __device__ __forceinline__ void finish_row(float sum, float su) {
        float resv = 0.f;
        if constexpr (EPI == EPI_RESIDUAL) {
            if (row - res_base >= 32) {
                res_base += 32;
                res = (res_base + lane < b) ? y[res_base + lane] : 0.f;
            }
            resv = __shfl_sync(0xffffffffu, res, row - res_base);
        }
        if (lane == 0) {
            if constexpr (EPI == EPI_STORE) y[row] = sum;
            else if constexpr (EPI == EPI_RESIDUAL) y[row] = resv + sum;
            else if constexpr (EPI == EPI_SWIGLU) y[row] = silu_f(sum) * su;
            else {
                y[row] = sum;
                if (sum > best) { best = sum; best_idx = row; }
            }
        }
        ++row;
    }
};

// Specialised stream: GPR groups per row, x (XG groups of 256) in registers. Chunks hold 8
// groups and start on a row boundary (GPR divides 8), so each group's x slice, gate/up
// half and row end are compile-time.
template <int EPI, int GPR, int XG>
__device__ __noinline__ void stream_fast_fn(const StreamCtx& cx, StreamState& state, const StepParams sp) {
    StreamRegs R(cx, state);
    const int lane = R.lane;
    const int bytes = cx.bytes;
    float xr[XG][8];
#pragma unroll
    for (int k = 0; k < XG; ++k) {
        const float4 v0 = *reinterpret_cast<const float4*>(cx.xs + k * 256 + lane * 8);
        const float4 v1 = *reinterpret_cast<const float4*>(cx.xs + k * 256 + lane * 8 + 4);
        xr[k][0] = v0.x; xr[k][1] = v0.y; xr[k][2] = v0.z; xr[k][3] = v0.w;
        xr[k][4] = v1.x; xr[k][5] = v1.y; xr[k][6] = v1.z; xr[k][7] = v1.w;
    }
    float acc = 0.f, acc_u = 0.f;
    for (int off = 0; off < bytes; off += kChunkBytes) {
        const uint4* wv;
        if (!R.next_chunk(wv, sp)) break;
        const int ng = min(kChunkBytes, bytes - off) / kGroupBytes;
        uint4 w[kGroupsPerChunk];
#pragma unroll
        for (int gi = 0; gi < kGroupsPerChunk; ++gi)
            w[gi] = gi < ng ? wv[gi * 32 + lane] : make_uint4(0u, 0u, 0u, 0u);
        float pt[kGroupsPerChunk];
#pragma unroll
        for (int gi = 0; gi < kGroupsPerChunk; ++gi) {
            const float* xx = xr[gi % XG];
            float d = 0.f;
            d = fmaf(bf16lo(w[gi].x), xx[0], d);
            d = fmaf(bf16hi(w[gi].x), xx[1], d);
            d = fmaf(bf16lo(w[gi].y), xx[2], d);
            d = fmaf(bf16hi(w[gi].y), xx[3], d);
            d = fmaf(bf16lo(w[gi].z), xx[4], d);
            d = fmaf(bf16hi(w[gi].z), xx[5], d);
            d = fmaf(bf16lo(w[gi].w), xx[6], d);
            d = fmaf(bf16hi(w[gi].w), xx[7], d);
            pt[gi] = d;
        }
#pragma unroll
        for (int gi = 0; gi < kGroupsPerChunk; ++gi) {
            if (gi < ng) {
                const int qq = gi % GPR;  // position of the group in its row
                if (EPI == EPI_SWIGLU && qq >= XG) acc_u += pt[gi];
                else acc += pt[gi];
                if (qq == GPR - 1) {
                    const float sum = warp_sum(acc);
                    const float su = EPI == EPI_SWIGLU ? warp_sum(acc_u) : 0.f;
                    R.template finish_row<EPI>(sum, su);
                    acc = 0.f;
                    acc_u = 0.f;
                }
            }
        }
        R.release_chunk();
    }
    R.save(state);
}

// Generic stream: x from shared memory, row position tracked at run time.
template <int EPI>
__device__ __noinline__ void stream_generic_fn(const StreamCtx& cx, StreamState& state, const StepParams sp) {
    StreamRegs R(cx, state);
    const int lane = R.lane;
    const int bytes = cx.bytes, xlen = cx.xlen;
    const float* xs = cx.xs;
    const int gpr = cx.in >> 8;
    int q = 0;
    float acc = 0.f, acc_u = 0.f;
    for (int off = 0; off < bytes; off += kChunkBytes) {
        const uint4* wv;
        if (!R.next_chunk(wv, sp)) break;
        const int ng = min(kChunkBytes, bytes - off) / kGroupBytes;
#pragma unroll 4
        for (int gi = 0; gi < ng; ++gi) {
            const uint4 w = wv[gi * 32 + lane];
            const int col = q * 256 + lane * 8;
            if (EPI == EPI_SWIGLU && col >= xlen) acc_u = dot8s(w, xs + (col - xlen), acc_u);
            else acc = dot8s(w, xs + col, acc);
            if (q == gpr - 1) {
                const float sum = warp_sum(acc);
                const float su = EPI == EPI_SWIGLU ? warp_sum(acc_u) : 0.f;
                R.template finish_row<EPI>(sum, su);
                acc = 0.f;
                acc_u = 0.f;
                q = 0;
            } else {
                ++q;
            }
        }
        R.release_chunk();
    }
    R.save(state);
}

// ---------------------------------------------------------------------- GEMV phase
__device__ __noinline__ void gemv_phase(StepShared& S, const StepParams sp, int p, int c, int nc) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const StepPhase& ph = *S.ph;
    const int pro = ph.pro, epi = ph.epi;
    const int xlen = ph.g.x_len, in = ph.g.in_dim;
    float* const y = ph.g.y;
    float* const xs = S.xs;
    const float eps = ph.g.eps;

    // ---- norm weights do not depend on the previous phase: load them before the barrier
    constexpr int kV = 4096 / (4 * kSThreads);  // float4 per thread: x_len <= 4096 (checked on the host)
    float4 wv[kV];
    if (pro == PRO_RMSNORM || pro == PRO_EMBED_RMSNORM) load_vec4<kV>(ph.g.norm_w, xlen, tid, kSThreads, wv);
    grid_wait(S, sp, p, c, nc);
    if (S.abort) return;

    // ---- prologue: x into shared memory, every load issued before any use
    if (pro == PRO_ATTN_COMBINE) {
        // The attention phase left one partial (max, sum, unnormalised output) per split;
        // warp h combines q head h (lane l: dims 8l..8l+7) exactly as the split-K combine
        // of the attention kernel does, then applies the sigmoid gate.
        const GemvParams& g = ph.g;
        const int grp = g.nq / g.nkv;
        const int n_ctx = *g.pos + 1;
        int n_act = (n_ctx + g.min_chunk - 1) / g.min_chunk;
        if (n_act > g.nsplit) n_act = g.nsplit;
        for (int h = warp; h < g.nq; h += kSW) {
            const int kv = h / grp, gg = h % grp;
            const float* gt = g.x + (size_t)h * 2 * kHD + kHD + lane * 8;  // gate of head h
            const float4 ga = *reinterpret_cast<const float4*>(gt), gb = *reinterpret_cast<const float4*>(gt + 4);
            float M = -INFINITY;
            for (int s2 = 0; s2 < n_act; ++s2)
                M = fmaxf(M, __ldcg(&g.part_ml[((size_t)(kv * g.nsplit + s2) * grp + gg) * 2]));
            float L = 0.f, o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 8
            for (int s2 = 0; s2 < n_act; ++s2) {
                const size_t pi = (size_t)(kv * g.nsplit + s2) * grp + gg;
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(g.part_ml) + pi);
                const float4* po = reinterpret_cast<const float4*>(g.part_o + pi * kHD + lane * 8);
                const float4 va = __ldcg(po), vb = __ldcg(po + 1);
                const float f = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M);
                L += ml.y * f;
                o[0] += va.x * f; o[1] += va.y * f; o[2] += va.z * f; o[3] += va.w * f;
                o[4] += vb.x * f; o[5] += vb.y * f; o[6] += vb.z * f; o[7] += vb.w * f;
            }
            const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) xs[(size_t)h * kHD + lane * 8 + e] = (o[e] / L) * sigmoid_f(gv[e]);
        }
        cta_sync();
    } else if (pro == PRO_GATED_NORM) {
        // one warp per head of gn_dim values: w * (o * inv_head) * silu(z)
        const int D = ph.g.gn_dim, nh = xlen / D;
        const float* x0 = ph.g.x;
        const float* z0 = ph.g.z;
        const float* nw = ph.g.norm_w;
        // heads warp, warp + 8, ... (up to kGnHeads per warp): every load of all of them is
        // issued before the first reduction, one memory round trip for the prologue
        constexpr int kGnHeads = 4;
        for (int h0 = warp; h0 < nh; h0 += kSW * kGnHeads) {
            float ov[kGnHeads][4], zv[kGnHeads][4], wv4[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int i = lane + 32 * k;
                wv4[k] = i < D ? nw[i] : 0.f;
            }
#pragma unroll
            for (int j = 0; j < kGnHeads; ++j) {
                const int h = h0 + j * kSW;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int i = lane + 32 * k;
                    const bool in_r = h < nh && i < D;
                    ov[j][k] = in_r ? x0[(size_t)h * D + i] : 0.f;
                    zv[j][k] = in_r ? z0[(size_t)h * D + i] : 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < kGnHeads; ++j) {
                const int h = h0 + j * kSW;
                if (h >= nh) break;
                double ss = 0.0;
#pragma unroll
                for (int k = 0; k < 4; ++k) ss += (double)ov[j][k] * ov[j][k];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
                const float inv = 1.0f / sqrtf((float)(ss / D) + eps);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int i = lane + 32 * k;
                    if (i < D) xs[(size_t)h * D + i] = wv4[k] * (ov[j][k] * inv) * silu_f(zv[j][k]);
                }
            }
        }
        cta_sync();
    } else {
        const float* src = ph.g.x;
        if (pro == PRO_EMBED_RMSNORM) {
            int tok = ph.g.tokens[*ph.g.pos];
            if (tok < 0 || tok >= ph.g.vocab) {
                if (tid == 0) post_error(sp.dev_err, DEV_BAD_TOKEN);
                tok = 0;
            }
            const uint16_t* erow = ph.g.embed + (size_t)tok * xlen;
            float* hout = ph.g.hidden_out;
            for (int i = tid; i < xlen; i += kSThreads) {
                const float v = __uint_as_float((uint32_t)erow[i] << 16);
                xs[i] = v;
                if (c == 0) hout[i] = v;
            }
            cta_sync();
            src = xs;
        }
        // x in registers: one round trip per kV * 4 * kSThreads elements
        const int n4 = xlen >> 2;
        float4* xs4 = reinterpret_cast<float4*>(xs);
        if (pro == PRO_PLAIN) {
            for (int base = 0; base < n4; base += kV * kSThreads) {
                float4 xv[kV];
                load_vec4<kV>(src + 4 * base, 4 * min(n4 - base, kV * kSThreads), tid, kSThreads, xv);
#pragma unroll
                for (int k = 0; k < kV; ++k) {
                    const int i = base + tid + k * kSThreads;
                    if (i < n4) xs4[i] = xv[k];
                }
            }
        } else {  // RMSNORM (xlen <= 4096: checked when the phases are built)
            float4 xv[kV];
            load_vec4<kV>(src, xlen, tid, kSThreads, xv);
            double ss = 0.0;
#pragma unroll
            for (int k = 0; k < kV; ++k)
                ss += (double)xv[k].x * xv[k].x + (double)xv[k].y * xv[k].y + (double)xv[k].z * xv[k].z +
                      (double)xv[k].w * xv[k].w;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) S.red_d[warp] = ss;
            cta_sync();
            ss = 0.0;
#pragma unroll
            for (int w = 0; w < kSW; ++w) ss += S.red_d[w];
            const float inv = 1.0f / sqrtf((float)(ss / xlen) + eps);
#pragma unroll
            for (int k = 0; k < kV; ++k) {
                const int i = tid + k * kSThreads;
                if (i < n4) {
                    float4 v = xv[k];
                    v.x = v.x * inv * wv[k].x;
                    v.y = v.y * inv * wv[k].y;
                    v.z = v.z * inv * wv[k].z;
                    v.w = v.w * inv * wv[k].w;
                    xs4[i] = v;
                }
            }
        }
        cta_sync();
    }
    trace_mark(sp, c, p, 2);

    // ---- this warp's weight stream
    int a, b;
    warp_rows(ph.g.rows, c, nc, warp, a, b);
    StreamCtx cx;
    cx.ring = S.ring + (size_t)warp * sp.nslot * kChunkBytes;
    cx.full = S.full + warp * sp.nslot;
    cx.empty = S.empty + warp * sp.nslot;
    cx.xs = xs;
    cx.y = y;
    cx.nslot = sp.nslot;
    cx.b = b;
    cx.bytes = (b - a) * in * 2;
    cx.in = in;
    cx.xlen = xlen;
    cx.trace = sp.trace != nullptr;
    StreamState st;
    st.r = S.rings[warp];
    st.row = a;
    st.res_base = a;
    st.res = (epi == EPI_RESIDUAL && a + lane < b) ? y[a + lane] : 0.f;
    st.best = -INFINITY;
    st.best_idx = 0x7fffffff;
    st.waited_ns = 0;
    st.nchunks = 0;
    const int gpr = in >> 8, xg = xlen >> 8;
    const bool fast = (epi == EPI_SWIGLU) ? (gpr == 8 && xg == 4) : (gpr == 4 && xg == 4);
    switch (epi) {
        case EPI_STORE:
            fast ? stream_fast_fn<EPI_STORE, 4, 4>(cx, st, sp) : stream_generic_fn<EPI_STORE>(cx, st, sp);
            break;
        case EPI_RESIDUAL:
            fast ? stream_fast_fn<EPI_RESIDUAL, 4, 4>(cx, st, sp) : stream_generic_fn<EPI_RESIDUAL>(cx, st, sp);
            break;
        case EPI_SWIGLU:
            fast ? stream_fast_fn<EPI_SWIGLU, 8, 4>(cx, st, sp) : stream_generic_fn<EPI_SWIGLU>(cx, st, sp);
            break;
        default:
            fast ? stream_fast_fn<EPI_ARGMAX, 4, 4>(cx, st, sp) : stream_generic_fn<EPI_ARGMAX>(cx, st, sp);
            break;
    }
    const float best = st.best;
    const int best_idx = st.best_idx;
    __syncwarp();
    if (lane == 0) S.rings[warp] = st.r;
    if (sp.trace && tid == 0) {
        sp.trace[((size_t)c * sp.nphases + p) * 8 + 4] = st.waited_ns;
        sp.trace[((size_t)c * sp.nphases + p) * 8 + 5] = st.nchunks;
    }

    if (epi == EPI_ARGMAX) {
        // CTA argmax (larger wins, ties -> lower index), then the grid ticket
        const GemvParams& g = ph.g;
        if (lane == 0) { S.rv[warp] = best; S.ri[warp] = best_idx; }
        cta_sync();
        if (tid == 0) {
            float bv = S.rv[0];
            int bi = S.ri[0];
            for (int w = 1; w < kSW; ++w)
                if (S.rv[w] > bv || (S.rv[w] == bv && S.ri[w] < bi)) { bv = S.rv[w]; bi = S.ri[w]; }
            g.am_val[c] = bv;
            g.am_idx[c] = bi;
            __threadfence();
            S.s_last = (atomicAdd(g.am_counter, 1u) == (unsigned)nc - 1) ? 1 : 0;
        }
        cta_sync();
        if (S.s_last) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int k = tid; k < nc; k += kSThreads) {
                const float v = __ldcg(&g.am_val[k]);
                const int i = __ldcg(&g.am_idx[k]);
                if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            cta_sync();
            if (lane == 0) { S.rv[warp] = bv; S.ri[warp] = bi; }
            cta_sync();
            if (tid == 0) {
                bv = S.rv[0];
                bi = S.ri[0];
                for (int w = 1; w < kSW; ++w)
                    if (S.rv[w] > bv || (S.rv[w] == bv && S.ri[w] < bi)) { bv = S.rv[w]; bi = S.ri[w]; }
                if (bi == 0x7fffffff) bi = 0;
                if (g.argmax_out) *g.argmax_out = bi;
                if (g.pos_inout) {
                    const int pos = *g.pos_inout;
                    if (g.tokens_out && pos + 1 < g.max_ctx && pos + 1 >= *g.n_prompt) g.tokens_out[pos + 1] = bi;
                    *g.pos_inout = pos + 1;
                }
                *g.am_counter = 0u;
            }
        }
    }
}

// ---------------------------------------------------------------------- GDN phase
// Warps 0-3 run the item (state slice loaded before the barrier); all threads take
// part in the barrier.
__device__ __noinline__ void gdn_phase(StepShared& S, const StepParams sp, int p, int c, int nc) {
    const int tid = threadIdx.x, warp = tid >> 5;
    const GdnDecodeParams& d = S.ph->d;
    const int items = d.VH * (128 / 16);
    bool waited = false;
    if (warp < 4) {
        for (int it = c; it < items; it += nc) {
            const int vh = it >> 3, vs = it & 7;
            if (!waited) {
                gdn_decode_item(d, vh, vs, tid, [&] { grid_wait(S, sp, p, c, nc); });
                waited = true;
            } else {
                gdn_decode_item(d, vh, vs, tid, [] {});
            }
        }
    }
    if (warp >= 4 || c >= items) grid_wait(S, sp, p, c, nc);
}

// ---------------------------------------------------------------------- attention phase
template <int GRP>
__device__ __noinline__ void attn_phase(StepShared& S, const StepParams sp, int p, int c, int nc) {
    const AttnDecodeParams at = S.ph->a;
    const int items = at.NKV * at.nsplit;
    long long* marks = sp.trace ? sp.trace + ((size_t)c * sp.nphases + p) * 8 + 4 : nullptr;
    if (threadIdx.x >= kAttnThreads) return;  // the item runs on warps 0-7
    for (int it = c; it < items; it += nc) attn_decode_item<GRP>(at, it % at.NKV, it / at.NKV, marks);
}

template <int GRP>
__global__ void __launch_bounds__(kBlockThreads, 1) k_decode_step(const StepParams sp) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ StepShared S;
    const int tid = threadIdx.x;
    const int c = blockIdx.x, nc = gridDim.x;
    const StepSmem plan = step_smem_plan(sp.nslot, sp.xs_max, sp.nphases);
    const int nbar = kSW * sp.nslot;

    if (tid == 0) {
        S.ring = smem;
        S.xs = reinterpret_cast<float*>(smem + plan.xs);
        S.full = reinterpret_cast<uint64_t*>(smem + plan.bars);
        S.empty = S.full + nbar;
        S.brief = reinterpret_cast<PhaseBrief*>(smem + plan.brief);
        S.ph = reinterpret_cast<StepPhase*>(smem + plan.phase);
        S.abort = 0;
    }
    if (tid < kSW) {
        RingState r;
        r.consumed = 0;
        r.cslot = 0;
        r.cpar = 0;
        S.rings[tid] = r;
        S.issued[tid] = 0;
    }
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + plan.bars);
    for (int q = tid; q < 2 * nbar; q += kBlockThreads) mbar_init(&bars[q], 1);
    if (tid == 0) fence_mbar_init();
    PhaseBrief* brief = reinterpret_cast<PhaseBrief*>(smem + plan.brief);
    for (int q = tid; q < sp.nphases; q += kBlockThreads) {
        const StepPhase& g = sp.phases[q];
        PhaseBrief bf;
        bf.W = g.type == PH_GEMV ? g.g.W : nullptr;
        bf.rows = g.g.rows;
        bf.in_dim = g.g.in_dim;
        brief[q] = bf;
    }
    __syncthreads();

    if (tid >= kSThreads) {
        producer(S, sp, c, nc);
    } else {
        // The descriptor of phase p+1 is loaded into registers (one int4 per thread) while
        // phase p runs and stored to shared memory after it, so no CTA -- in particular not
        // the last one to arrive at a barrier -- waits for a descriptor load between phases.
        constexpr int kDesc16 = (int)(sizeof(StepPhase) / 16);
        static_assert(sizeof(StepPhase) % 16 == 0 && kDesc16 <= kSThreads, "descriptor staging");
        int4* ph16 = reinterpret_cast<int4*>(smem + plan.phase);
        const int4* desc = reinterpret_cast<const int4*>(sp.phases);
        if (tid < kDesc16) ph16[tid] = desc[tid];
        for (int p = 0; p < sp.nphases; ++p) {
            trace_mark(sp, c, p, 0);
            int4 next_desc = make_int4(0, 0, 0, 0);
            if (tid < kDesc16 && p + 1 < sp.nphases) next_desc = desc[(size_t)(p + 1) * kDesc16 + tid];
            cta_sync();  // this phase's descriptor is in shared memory
            const int type = reinterpret_cast<const StepPhase*>(ph16)->type;
            if (type == PH_GDN) {
                gdn_phase(S, sp, p, c, nc);
            } else if (type == PH_ATTN) {
                grid_wait(S, sp, p, c, nc);
                attn_phase<GRP>(S, sp, p, c, nc);
            } else {
                gemv_phase(S, sp, p, c, nc);  // waits for the grid after its weight-only loads
            }
            cta_sync();  // every warp is done (also ends every read of the staged descriptor)
            trace_mark(sp, c, p, 3);
            // (a test may have one CTA withhold its first arrival: every other CTA's bounded
            // wait then runs out and the step ends with an error, see qwc_check_step_timeout)
            if (p + 1 < sp.nphases && tid == 0 && !(p == 0 && c == sp.stall_cta))
                red_release_add_u64(sp.bar, 1ull);  // orders this CTA's writes before it
            if (tid < kDesc16 && p + 1 < sp.nphases) ph16[tid] = next_desc;
        }
    }
    __syncthreads();
    // After an error, copies the producer issued may still be in flight: wait for them
    // (bounded) before the CTA exits. On the normal path every issued copy was consumed.
    if (tid >= kSThreads && tid - kSThreads < kSW) {
        const int w = tid - kSThreads;
        const RingState r = S.rings[w];
        int slot = r.cslot;
        uint32_t par = r.cpar;
        for (int k = r.consumed; k < S.issued[w]; ++k) {
            if (!mbar_wait_bounded(&S.full[w * sp.nslot + slot], par, sp.dev_err, DEV_GEMV_DRAIN_TIMEOUT)) break;
            if (++slot == sp.nslot) { slot = 0; par ^= 1u; }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(sp.done, 1u) == (unsigned)nc - 1) {  // last CTA of the step
            *sp.bar = 0ull;
            *sp.done = 0u;
        }
    }
}

size_t step_smem_bytes(int nslot, int xs_max, int nphases) { return step_smem_plan(nslot, xs_max, nphases).total; }

int step_slots(int xs_max, int grp, int nphases) {
    // static shared memory: StepShared + the attention body (grows with the GQA group)
    const size_t static_bytes = sizeof(StepShared) + (size_t)grp * 1024 + 2048 + 8192 + 2048 + 1024;
    const size_t budget = 227 * 1024 - static_bytes;
    int n = kMaxSlots;
    while (n > 2 && step_smem_plan(n, xs_max, nphases).total > budget) --n;
    return n;
}

template <int GRP>
static cudaError_t launch_step_t(const StepParams& sp, int grid, cudaStream_t s) {
    const size_t smem = step_smem_bytes(sp.nslot, sp.xs_max, sp.nphases);
    auto kern = k_decode_step<GRP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kBlockThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, sp);
}

cudaError_t launch_decode_step(const StepParams& sp, int grp, int grid, cudaStream_t s) {
    switch (grp) {
        case 1: return launch_step_t<1>(sp, grid, s);
        case 2: return launch_step_t<2>(sp, grid, s);
        case 4: return launch_step_t<4>(sp, grid, s);
        case 8: return launch_step_t<8>(sp, grid, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int GRP>
static int max_grid_t(size_t smem) {
    int per_sm = 0;
    cudaFuncSetAttribute(k_decode_step<GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_step<GRP>, kBlockThreads, smem) != cudaSuccess)
        return 0;
    return per_sm >= 1 ? num_sms() : 0;  // one CTA per SM
}

int decode_step_max_grid(int grp, int nslot, int xs_max, int nphases) {
    const size_t smem = step_smem_bytes(nslot, xs_max, nphases);
    switch (grp) {
        case 1: return max_grid_t<1>(smem);
        case 2: return max_grid_t<2>(smem);
        case 4: return max_grid_t<4>(smem);
        case 8: return max_grid_t<8>(smem);
        default: return 0;
    }
}

}  // namespace qwc
