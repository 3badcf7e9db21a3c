// Binned push propagation: shared-memory target tiles fed through L2 bins.
//
// Why: a push step delivers one fp32 add per synaptic event to a random
// target. Done as red.global.add.f32 every event is one L2 atomic request,
// and on B200 the L2 serves ~1.9e11 such requests/s however many SMs issue
// them -- the atomic push kernel sits at that ceiling, well below what HBM
// could feed (8 B per event). Shared-memory atomics run ~4x faster, but then
// every target has to live in exactly one SM's shared memory.
//
// How: one persistent CTA per SM (cooperative launch: all resident). The
// rank's targets are split into `passes` contiguous ranges small enough that
// range/grid targets fit one CTA's shared memory; each pass has its own CSR
// slice (every presynaptic row, only the edges into the pass's range, local
// column ids), so no event is read twice. In a pass CTA c owns the fp32 tile
// [c*tile, (c+1)*tile) of the range. Its warps are split:
//  * router warps read the spiking rows of the current round (16-byte
//    evict-first loads of col_idx/weights) and append each event
//    (offset in tile, weight) to a shared-memory staging slot of its owner
//    tile; every chunk the staging is flushed with plain coalesced stores
//    into the sub-bin bins[buffer][owner][c] that only CTA c writes -- no
//    global atomics;
//  * drainer warps fold the sub-bins [buffer][c][*] of the previous round
//    into their shared tile with shared-memory atomics.
// Rounds are decoupled, not barriered: two monotonic counters count finished
// router rounds and finished drain rounds over all CTAs; routers may run
// nb - 1 rounds ahead of the slowest drainer (nb bin buffers), a drainer
// waits only for the routers of its round. Every wait is bounded: on expiry
// the kernel raises DevCounters::error and every CTA stops waiting, so the
// host reports an error instead of the GPU hanging. After a pass each CTA
// adds its tile into next_current. A sub-bin that overflows its capacity
// spills the excess through red.global.add into next_current (hence the
// write-back adds instead of storing); results are the same up to fp32
// reassociation.
#include "b200_device.cuh"
#include "b200_kernels.h"

#include <algorithm>
#include <mutex>

namespace b200 {
namespace {

using namespace dev;

constexpr int kRouterWarps = 12;
constexpr int kDrainWarps = 4;
constexpr int kThreads = 32 * (kRouterWarps + kDrainWarps);
constexpr int kRouterThreads = 32 * kRouterWarps;
constexpr int kDrainThreads = 32 * kDrainWarps;
constexpr int kChunkEdges = 256;  // edges a router warp handles between staging flushes
constexpr uint32_t kStage = 24;   // staged entries per destination tile

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Named barrier that also ANDs a per-thread predicate over the participants.
__device__ __forceinline__ bool named_sync_and(int id, int n, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(n)
        : "memory");
    return r != 0u;
}

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(unsigned long long *p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bounded wait for *p >= target. Gives up (and raises the error word) after
// `limit` polls, or at once if another CTA already raised it.
__device__ bool wait_geq(const unsigned long long *p, unsigned long long target, uint32_t limit,
                         uint32_t *err) {
    for (uint32_t it = 0; ld_acquire(p) < target; ++it) {
        if (*(volatile uint32_t *)err != 0u) return false;
        if (it >= limit) {
            atomicExch(err, 1u);
            return false;
        }
        __nanosleep(100);
    }
    return true;
}

struct Smem {
    float *tile;       // [tile]          the pass's targets owned by this CTA
    uint2 *stage;      // [grid][kStage]  staged events per destination
    uint32_t *scount;  // [grid]          staged entries per destination
    uint32_t *wcount;  // [grid]          entries written this round into my sub-bin of each destination
    uint32_t *sbase;   // [grid]          flush base per destination
    uint32_t *dcount;  // [grid]          drain: entries in each source's sub-bin
};

__device__ __forceinline__ Smem smem_layout(const BinLayout &L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem s;
    size_t o = 0;
    s.tile = reinterpret_cast<float *>(smem_raw + o);
    o += (size_t)L.tile * 4u;
    s.stage = reinterpret_cast<uint2 *>(smem_raw + o);
    o += (size_t)L.grid * kStage * 8u;
    s.scount = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += (size_t)L.grid * 4u;
    s.wcount = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += (size_t)L.grid * 4u;
    s.sbase = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += (size_t)L.grid * 4u;
    s.dcount = reinterpret_cast<uint32_t *>(smem_raw + o);
    return s;
}

struct RouteCtx {
    uint2 *sub;        // my sub-bin of destination 0 in this buffer; destination q at + q * q_stride
    size_t q_stride;   // grid * cap
    float *next_pass;  // next_current + pass offset
};

// Route one event (local target t within the pass, weight wv).
__device__ __forceinline__ void route(uint32_t t, float wv, const BinLayout &L, const Smem &S, const RouteCtx &R) {
    const uint32_t q = (uint32_t)(((uint64_t)t * L.div_magic) >> 40);  // t / tile, exact for t < 2^24
    const uint32_t off = t - q * L.tile;
    const uint32_t slot = atomicAdd(&S.scount[q], 1u);
    if (slot < kStage) {
        S.stage[q * kStage + slot] = make_uint2(off, __float_as_uint(wv));
    } else {
        // Staging full: write straight into my sub-bin of q.
        const uint32_t pos = atomicAdd(&S.wcount[q], 1u);
        if (pos < L.cap) R.sub[q * R.q_stride + pos] = make_uint2(off, __float_as_uint(wv));
        else red_add(R.next_pass + t, wv);
    }
}

// Route edges [p, p + n) with the whole warp: 16-byte loads for the 4-aligned
// body (both vectors of a lane issued before any routing), scalar head/tail.
__device__ __forceinline__ void route_range(uint64_t p, uint64_t n, const uint32_t *__restrict__ col,
                                            const float *__restrict__ w, const BinLayout &L, const Smem &S,
                                            const RouteCtx &R, unsigned lane) {
    const uint64_t e = p + n;
    uint64_t a = (p + 3) & ~(uint64_t)3;
    if (a > e) a = e;
    if (lane < a - p) route(col[p + lane], w[p + lane], L, S, R);
    const uint64_t nvec = (e - a) / 4;
    const uint4 *cv = reinterpret_cast<const uint4 *>(col + a);
    const float4 *wv = reinterpret_cast<const float4 *>(w + a);
    uint4 c0 = make_uint4(0, 0, 0, 0), c1 = c0;
    float4 x0 = make_float4(0, 0, 0, 0), x1 = x0;
    const bool h0 = lane < nvec, h1 = lane + 32 < nvec;
    if (h0) {
        c0 = __ldcs(cv + lane);
        x0 = __ldcs(wv + lane);
    }
    if (h1) {
        c1 = __ldcs(cv + lane + 32);
        x1 = __ldcs(wv + lane + 32);
    }
    if (h0) {
        route(c0.x, x0.x, L, S, R);
        route(c0.y, x0.y, L, S, R);
        route(c0.z, x0.z, L, S, R);
        route(c0.w, x0.w, L, S, R);
    }
    if (h1) {
        route(c1.x, x1.x, L, S, R);
        route(c1.y, x1.y, L, S, R);
        route(c1.z, x1.z, L, S, R);
        route(c1.w, x1.w, L, S, R);
    }
    const uint64_t t0 = a + nvec * 4;
    if (lane < e - t0) route(col[t0 + lane], w[t0 + lane], L, S, R);
}

template <typename TIdx>
__global__ void __launch_bounds__(kThreads, 1)
    propagate_binned_kernel(const TIdx *__restrict__ list, float *__restrict__ next, DevCounters *ctr, int parity,
                            int count_spikes, BinLayout L) {
    const Smem S = smem_layout(L);
    __shared__ uint32_t s_abort;
    const unsigned lane = lane_id();
    const unsigned warp = threadIdx.x >> 5;
    const uint32_t c = blockIdx.x;
    const uint32_t G = L.grid;
    const uint32_t S_rows = *(volatile uint32_t *)&ctr->list_count[parity];
    const uint32_t rows_round = G * L.rows_per_cta;
    const uint32_t rounds = (S_rows + rows_round - 1) / rows_round;
    unsigned long long *routed = L.sync;
    unsigned long long *drained = L.sync + 1;
    const size_t q_stride = (size_t)G * L.cap;       // one destination's sub-bins (all sources)
    const size_t buf_stride = (size_t)G * q_stride;  // one bin buffer

    if (threadIdx.x == 0) s_abort = 0u;
    for (uint32_t j = threadIdx.x; j < G; j += kThreads) S.scount[j] = 0u;
    unsigned long long events = 0;

    for (uint32_t pass = 0; pass < L.passes; ++pass) {
        const uint64_t *__restrict__ row_ptr = L.row_ptr[pass];
        const uint32_t *__restrict__ col = L.col[pass];
        const float *__restrict__ w = L.w[pass];
        float *next_pass = next + L.pass_lo[pass];
        for (uint32_t j = threadIdx.x; j < L.tile; j += kThreads) S.tile[j] = 0.0f;
        __syncthreads();
        if (warp < (unsigned)kRouterWarps) {
            // --------------------------------------------------- routers --
            const unsigned rw = warp;
            for (uint32_t k = 0; k < rounds; ++k) {
                const uint32_t g = pass * rounds + k;
                const uint32_t b = g % L.nb;
                const RouteCtx R{L.bins + b * buf_stride + (size_t)c * L.cap, q_stride, next_pass};
                if (threadIdx.x == 0 && g >= L.nb &&
                    !wait_geq(drained, (unsigned long long)G * (g - L.nb + 1), L.spin_limit, &ctr->error))
                    s_abort = 1u;
                for (uint32_t j = threadIdx.x; j < G; j += kRouterThreads) S.wcount[j] = 0u;
                named_sync(1, kRouterThreads);
                if (s_abort) break;
                const uint32_t r0 = k * rows_round + c * L.rows_per_cta;
                const uint32_t r1 = min(r0 + L.rows_per_cta, S_rows);
                uint32_t ri = r0 + rw;  // warp rw walks rows r0 + rw, + kRouterWarps, ...
                uint64_t pos = 0, end = 0;
                bool done = ri >= r1;
                if (!done) {
                    const uint64_t row = (uint64_t)list[ri];
                    pos = row_ptr[row];
                    end = row_ptr[row + 1];
                    events += end - pos;
                }
                for (;;) {
                    uint64_t budget = kChunkEdges;
                    while (!done && budget > 0) {
                        const uint64_t n = min(end - pos, budget);
                        if (n) route_range(pos, n, col, w, L, S, R, lane);
                        pos += n;
                        budget -= n;
                        if (pos == end) {
                            ri += kRouterWarps;
                            if (ri < r1) {
                                const uint64_t row = (uint64_t)list[ri];
                                pos = row_ptr[row];
                                end = row_ptr[row + 1];
                                events += end - pos;
                            } else {
                                done = true;
                            }
                        }
                    }
                    named_sync(1, kRouterThreads);
                    // Flush: reserve per destination in shared memory, then
                    // copy each destination's staged run with one warp.
                    for (uint32_t q = threadIdx.x; q < G; q += kRouterThreads) {
                        const uint32_t cnt = min(S.scount[q], kStage);
                        S.sbase[q] = S.wcount[q];
                        S.wcount[q] += cnt;
                    }
                    named_sync(1, kRouterThreads);
                    for (uint32_t q = rw; q < G; q += kRouterWarps) {
                        const uint32_t cnt = min(S.scount[q], kStage);
                        if (lane < cnt) {
                            const uint2 ent = S.stage[q * kStage + lane];
                            const uint32_t p = S.sbase[q] + lane;
                            if (p < L.cap) R.sub[q * q_stride + p] = ent;
                            else red_add(next_pass + (size_t)q * L.tile + ent.x, __uint_as_float(ent.y));
                        }
                        __syncwarp();
                        if (lane == 0) S.scount[q] = 0u;
                    }
                    if (named_sync_and(1, kRouterThreads, done)) break;
                }
                // Publish my sub-bin sizes for this round, then the round.
                uint32_t *counts = L.counts + (size_t)b * G * G;
                for (uint32_t q = threadIdx.x; q < G; q += kRouterThreads)
                    counts[(size_t)q * G + c] = min(S.wcount[q], L.cap);
                named_sync(1, kRouterThreads);
                if (threadIdx.x == 0) {
                    __threadfence();
                    red_release_add(routed, 1ull);
                }
            }
        } else {
            // -------------------------------------------------- drainers --
            const unsigned dt = threadIdx.x - kRouterThreads;
            const unsigned dw = dt >> 5;
            for (uint32_t k = 0; k < rounds; ++k) {
                const uint32_t g = pass * rounds + k;
                const uint32_t b = g % L.nb;
                if (dt == 0 && !wait_geq(routed, (unsigned long long)G * (g + 1), L.spin_limit, &ctr->error))
                    s_abort = 1u;
                named_sync(2, kDrainThreads);
                if (s_abort) break;
                const uint32_t *counts = L.counts + (size_t)b * G * G + (size_t)c * G;
                for (uint32_t src = dt; src < G; src += kDrainThreads) S.dcount[src] = __ldcg(counts + src);
                named_sync(2, kDrainThreads);
                const uint2 *mine = L.bins + b * buf_stride + (size_t)c * q_stride;
                for (uint32_t src = dw; src < G; src += kDrainWarps) {
                    const uint32_t cnt = S.dcount[src];
                    const uint2 *bin = mine + (size_t)src * L.cap;
                    uint32_t i = lane;
                    for (; i + 96u < cnt; i += 128u) {
                        const uint2 e0 = __ldcg(bin + i), e1 = __ldcg(bin + i + 32u);
                        const uint2 e2 = __ldcg(bin + i + 64u), e3 = __ldcg(bin + i + 96u);
                        atomicAdd(&S.tile[e0.x], __uint_as_float(e0.y));
                        atomicAdd(&S.tile[e1.x], __uint_as_float(e1.y));
                        atomicAdd(&S.tile[e2.x], __uint_as_float(e2.y));
                        atomicAdd(&S.tile[e3.x], __uint_as_float(e3.y));
                    }
                    for (; i < cnt; i += 32u) {
                        const uint2 e0 = __ldcg(bin + i);
                        atomicAdd(&S.tile[e0.x], __uint_as_float(e0.y));
                    }
                }
                named_sync(2, kDrainThreads);
                if (dt == 0) {
                    __threadfence();
                    red_release_add(drained, 1ull);
                }
            }
        }
        __syncthreads();
        // Write-back of this pass's tile: add (spilled reds may already be in
        // next_current; the last drain round waited for every router).
        const uint64_t t0 = (uint64_t)c * L.tile;
        const uint64_t len = L.pass_len[pass];
        for (uint32_t j = threadIdx.x; j < L.tile; j += kThreads) {
            const uint64_t t = t0 + j;
            const float v = S.tile[j];
            if (t < len && __float_as_uint(v) != 0u) next_pass[t] = __fadd_rn(next_pass[t], v);
        }
        __syncthreads();
    }
    block_add_u64(lane == 0 ? events : 0ull, &ctr->events);
    step_epilogue(ctr, parity, count_spikes, S_rows);
}

cudaError_t configure(const BinLayout &L, int idx_bits, void **fn_out) {
    static std::mutex mu;
    static uint32_t configured[64][2] = {};  // dynamic smem already allowed, per device and list width
    void *fn = idx_bits == 32 ? (void *)propagate_binned_kernel<uint32_t> : (void *)propagate_binned_kernel<uint64_t>;
    *fn_out = fn;
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaGetDevice(&dev);
    uint32_t &allowed = configured[dev & 63][idx_bits == 32 ? 0 : 1];
    if (allowed < L.smem_bytes) {
        const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.smem_bytes);
        if (e != cudaSuccess) return e;
        allowed = L.smem_bytes;
    }
    return cudaSuccess;
}

}  // namespace

bool binned_layout(int device, uint64_t n_local, uint64_t e_local, uint64_t n_rows, uint32_t force_passes,
                   BinLayout *L) {
    int optin = 0, coop = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop)
        return false;
    if (n_local == 0) return false;
    const uint32_t G = (uint32_t)sm_count(device);
    const size_t fixed = (size_t)G * kStage * 8 + (size_t)G * 16 + 2048;  // + static smem and slack
    if ((size_t)optin <= fixed + 4096) return false;
    const uint64_t tmax = ((optin - fixed) / 4) & ~(uint64_t)3;
    uint32_t passes = (uint32_t)((n_local + (uint64_t)G * tmax - 1) / ((uint64_t)G * tmax));
    if (force_passes > passes) passes = force_passes;
    if (passes == 0 || passes > kMaxBinPasses) return false;
    const uint64_t per_pass = (n_local + passes - 1) / passes;
    if (per_pass >= (1u << 24)) return false;  // offsets/divisions assume < 2^24 targets per pass
    uint64_t tile = (per_pass + G - 1) / G;
    tile = std::max<uint64_t>((tile + 3) & ~(uint64_t)3, 4);
    const double deg = n_rows ? (double)e_local / (double)n_rows / passes : 0.0;
    // ~8K events per tile per round: sub-bins average 8K / grid entries.
    const double per_tile = 8192.0;
    double rpc = deg > 0.0 ? per_tile / deg : 1e9;
    rpc = std::min(std::max(rpc, 1.0), 1e6);
    L->grid = G;
    L->nb = 3;
    L->passes = passes;
    for (uint32_t p = 0; p < passes; ++p) {
        L->pass_lo[p] = std::min<uint64_t>(n_local, p * per_pass);
        L->pass_len[p] = std::min<uint64_t>(n_local, (p + 1) * per_pass) - L->pass_lo[p];
    }
    L->tile = (uint32_t)tile;
    L->div_magic = ((1ull << 40) + tile - 1) / tile;
    L->rows_per_cta = (uint32_t)rpc;
    const double per_sub = per_tile / G;
    L->cap = (uint32_t)(((uint64_t)(3.0 * per_sub) + 64 + 31) & ~31ull);
    L->smem_bytes = (uint32_t)(tile * 4 + (size_t)G * kStage * 8 + (size_t)G * 16);
    L->spin_limit = 1u << 22;  // x ~100 ns naps: ~0.5 s before a wait is declared failed
    return true;
}

bool binned_fits(int device, const BinLayout &L) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    void *fn = nullptr;
    bool ok = configure(L, 32, &fn) == cudaSuccess && configure(L, 64, &fn) == cudaSuccess;
    int per_sm = 0;
    if (ok)
        ok = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, propagate_binned_kernel<uint32_t>, kThreads,
                                                           L.smem_bytes) == cudaSuccess &&
             per_sm >= 1 && (uint32_t)per_sm * (uint32_t)sm_count(device) >= L.grid;
    cudaGetLastError();
    if (prev != device) cudaSetDevice(prev);
    return ok;
}

cudaError_t launch_propagate_binned(cudaStream_t s, const void *list, int idx_bits, float *next, DevCounters *ctr,
                                    int parity, int count_spikes, const BinLayout &L) {
    cudaError_t e = cudaMemsetAsync(L.sync, 0, 2 * sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    void *fn = nullptr;
    if ((e = configure(L, idx_bits, &fn)) != cudaSuccess) return e;
    BinLayout Lc = L;
    void *args[] = {(void *)&list, (void *)&next, (void *)&ctr, (void *)&parity, (void *)&count_spikes, (void *)&Lc};
    return cudaLaunchCooperativeKernel(fn, dim3(L.grid), dim3(kThreads), args, L.smem_bytes, s);
}

}  // namespace b200
