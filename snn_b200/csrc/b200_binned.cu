// Binned push propagation: shared-memory target tiles fed through L2 bins.
//
// Why: a push step delivers one fp32 add per synaptic event to a random
// target. Done as red.global.add.f32 every event is one L2 atomic request,
// and on B200 the L2 serves ~1.9e11 such requests/s no matter how many SMs
// issue them -- the atomic-push kernel sits at that ceiling, far below HBM
// bandwidth (8 B/event read). Shared-memory atomics run ~4x faster, but a
// target must then live in one SM's shared memory.
//
// How: one persistent CTA per SM (cooperative launch, so all are resident).
// CTA c owns the targets [c*tile, (c+1)*tile) of the first `owned` local
// targets as an fp32 tile in shared memory. Its warps are split:
//  * router warps read the spiking rows of the current round (16-byte
//    evict-first loads of col_idx/weights) and, per event, append
//    (offset in tile, weight) to a shared-memory staging slot of the owning
//    tile; every chunk the staging is flushed into that tile's bin in global
//    memory (one atomic reservation per destination run, L2-resident bins);
//    events for targets >= owned go straight to L2 with red.global.add;
//  * drainer warps fold the bin of their own tile from the previous round
//    into the shared tile with shared-memory atomics.
// Rounds are decoupled, not barriered: two monotonic counters in global
// memory count finished router rounds and finished drain rounds over all
// CTAs; a router may run `nb - 1` rounds ahead of the slowest drainer (nb bin
// buffers), a drainer waits only for the routers of its round. Every wait is
// bounded: on expiry the kernel raises DevCounters::error and every CTA stops
// waiting, so the host reports an error instead of the GPU hanging.
// After the last round each CTA adds its tile into next_current (bins that
// overflow their capacity fall back to red.global.add into next_current, so
// the write-back is an add, not a store).
#include "b200_device.cuh"
#include "b200_kernels.h"

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
        __nanosleep(128);
    }
    return true;
}

struct Smem {
    // Layout of the dynamic shared memory: [tile floats | stage | scount].
    float *tile;
    uint2 *stage;
    uint32_t *scount;
};

__device__ __forceinline__ Smem smem_layout(const BinLayout &L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem s;
    s.tile = reinterpret_cast<float *>(smem_raw);
    s.stage = reinterpret_cast<uint2 *>(smem_raw + (size_t)L.tile * 4u);
    s.scount = reinterpret_cast<uint32_t *>(smem_raw + (size_t)L.tile * 4u + (size_t)L.grid * L.stage * 8u);
    return s;
}

// Route one event of local target c with weight wv.
__device__ __forceinline__ void route(uint32_t c, float wv, const BinLayout &L, const Smem &S, uint2 *bins,
                                      uint32_t *bin_count, float *next) {
    if (c < L.owned) {
        const uint32_t q = (uint32_t)(((uint64_t)c * L.div_magic) >> 40);  // c / tile (exact: c < 2^24)
        const uint32_t off = c - q * L.tile;
        const uint32_t slot = atomicAdd(&S.scount[q], 1u);
        const uint2 ent = make_uint2(off, __float_as_uint(wv));
        if (slot < L.stage) {
            S.stage[q * L.stage + slot] = ent;
        } else {
            const uint32_t pos = atomicAdd(&bin_count[q], 1u);
            if (pos < L.cap) bins[(size_t)q * L.cap + pos] = ent;
            else red_add(next + c, wv);
        }
    } else {
        red_add(next + c, wv);
    }
}

// Route edges [p, p + n) of the CSR with the whole warp (16-byte loads for the
// 4-aligned body, scalar head/tail).
__device__ __forceinline__ void route_range(uint64_t p, uint64_t n, const uint32_t *__restrict__ col,
                                            const float *__restrict__ w, const BinLayout &L, const Smem &S,
                                            uint2 *bins, uint32_t *bin_count, float *next, unsigned lane) {
    const uint64_t e = p + n;
    uint64_t a = (p + 3) & ~(uint64_t)3;
    if (a > e) a = e;
    if (lane < a - p) route(col[p + lane], w[p + lane], L, S, bins, bin_count, next);
    const uint64_t nvec = (e - a) / 4;
    const uint4 *cv = reinterpret_cast<const uint4 *>(col + a);
    const float4 *wv = reinterpret_cast<const float4 *>(w + a);
    // nvec <= kChunkEdges/4 = 64: at most two vectors per lane; load both first.
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
        route(c0.x, x0.x, L, S, bins, bin_count, next);
        route(c0.y, x0.y, L, S, bins, bin_count, next);
        route(c0.z, x0.z, L, S, bins, bin_count, next);
        route(c0.w, x0.w, L, S, bins, bin_count, next);
    }
    if (h1) {
        route(c1.x, x1.x, L, S, bins, bin_count, next);
        route(c1.y, x1.y, L, S, bins, bin_count, next);
        route(c1.z, x1.z, L, S, bins, bin_count, next);
        route(c1.w, x1.w, L, S, bins, bin_count, next);
    }
    const uint64_t t0 = a + nvec * 4;
    if (lane < e - t0) route(col[t0 + lane], w[t0 + lane], L, S, bins, bin_count, next);
}

template <typename TIdx>
__global__ void __launch_bounds__(kThreads, 1)
    propagate_binned_kernel(const TIdx *__restrict__ list, const uint64_t *__restrict__ row_ptr,
                            const uint32_t *__restrict__ col, const float *__restrict__ w, float *__restrict__ next,
                            DevCounters *ctr, int parity, int count_spikes, BinLayout L) {
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

    for (uint32_t j = threadIdx.x; j < L.tile; j += kThreads) S.tile[j] = 0.0f;
    for (uint32_t j = threadIdx.x; j < G; j += kThreads) S.scount[j] = 0u;
    if (threadIdx.x == 0) s_abort = 0u;
    __syncthreads();

    unsigned long long events = 0;
    if (warp < (unsigned)kRouterWarps) {
        // ------------------------------------------------------- routers --
        const unsigned rw = warp;
        for (uint32_t g = 0; g < rounds; ++g) {
            const uint32_t b = g % L.nb;
            uint2 *bins = L.bins + (size_t)b * G * L.cap;
            uint32_t *bin_count = L.bin_count + (size_t)b * G;
            if (threadIdx.x == 0 && g >= L.nb &&
                !wait_geq(drained, (unsigned long long)G * (g - L.nb + 1), L.spin_limit, &ctr->error))
                s_abort = 1u;
            named_sync(1, kRouterThreads);
            if (s_abort) break;
            const uint32_t r0 = g * rows_round + c * L.rows_per_cta;
            const uint32_t r1 = min(r0 + L.rows_per_cta, S_rows);
            // Warp rw walks rows r0 + rw, r0 + rw + kRouterWarps, ...
            uint32_t ri = r0 + rw;
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
                    if (n) route_range(pos, n, col, w, L, S, bins, bin_count, next, lane);
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
                // Flush: warp rw drains the staging of tiles rw, rw + kRouterWarps, ...
                for (uint32_t q = rw; q < G; q += kRouterWarps) {
                    const uint32_t cnt = min(S.scount[q], L.stage);
                    if (cnt == 0) continue;
                    uint32_t base = 0;
                    if (lane == 0) base = atomicAdd(&bin_count[q], cnt);
                    base = __shfl_sync(kFull, base, 0);
                    if (lane < cnt) {
                        const uint2 ent = S.stage[q * L.stage + lane];
                        if (base + lane < L.cap) bins[(size_t)q * L.cap + base + lane] = ent;
                        else red_add(next + (size_t)q * L.tile + ent.x, __uint_as_float(ent.y));
                    }
                    __syncwarp();
                    if (lane == 0) S.scount[q] = 0u;
                }
                if (named_sync_and(1, kRouterThreads, done)) break;
            }
            if (threadIdx.x == 0) {
                __threadfence();
                red_release_add(routed, 1ull);
            }
        }
    } else {
        // ------------------------------------------------------ drainers --
        const unsigned dt = threadIdx.x - kRouterThreads;
        for (uint32_t g = 0; g < rounds; ++g) {
            const uint32_t b = g % L.nb;
            if (dt == 0 && !wait_geq(routed, (unsigned long long)G * (g + 1), L.spin_limit, &ctr->error))
                s_abort = 1u;
            named_sync(2, kDrainThreads);
            if (s_abort) break;
            uint32_t *cnt_p = L.bin_count + (size_t)b * G + c;
            const uint32_t cnt = min(*(volatile uint32_t *)cnt_p, L.cap);
            const uint2 *bin = L.bins + ((size_t)b * G + c) * L.cap;
            uint32_t i = dt;
            for (; i + 3u * kDrainThreads < cnt; i += 4u * kDrainThreads) {
                const uint2 e0 = __ldcg(bin + i), e1 = __ldcg(bin + i + kDrainThreads);
                const uint2 e2 = __ldcg(bin + i + 2u * kDrainThreads), e3 = __ldcg(bin + i + 3u * kDrainThreads);
                atomicAdd(&S.tile[e0.x], __uint_as_float(e0.y));
                atomicAdd(&S.tile[e1.x], __uint_as_float(e1.y));
                atomicAdd(&S.tile[e2.x], __uint_as_float(e2.y));
                atomicAdd(&S.tile[e3.x], __uint_as_float(e3.y));
            }
            for (; i < cnt; i += kDrainThreads) {
                const uint2 e0 = __ldcg(bin + i);
                atomicAdd(&S.tile[e0.x], __uint_as_float(e0.y));
            }
            named_sync(2, kDrainThreads);
            if (dt == 0) {
                *cnt_p = 0u;
                __threadfence();
                red_release_add(drained, 1ull);
            }
        }
    }
    __syncthreads();
    // Write-back: add the tile into next_current (overflow reds may already
    // have landed there; the last drain round waited for every router).
    const uint64_t t0 = (uint64_t)c * L.tile;
    for (uint32_t j = threadIdx.x; j < L.tile; j += kThreads) {
        const uint64_t t = t0 + j;
        if (t < L.owned) {
            const float v = S.tile[j];
            if (v != 0.0f || __float_as_uint(v) != 0u) next[t] = __fadd_rn(next[t], v);
        }
    }
    block_add_u64(lane == 0 ? events : 0ull, &ctr->events);
    step_epilogue(ctr, parity, count_spikes, S_rows);
}

}  // namespace

uint32_t binned_threads() { return kThreads; }

bool binned_layout(int device, uint64_t n_local, uint64_t e_local, uint64_t n_rows, double owned_fraction,
                   BinLayout *L) {
    int optin = 0, coop = 0;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess || !coop)
        return false;
    if (n_local == 0 || n_local >= (1u << 24)) return false;  // offsets/divisions assume < 2^24 targets
    const uint32_t G = (uint32_t)sm_count(device);
    const uint32_t stage = 32;
    const size_t fixed = (size_t)G * stage * 8 + (size_t)G * 4 + 2048;  // + static smem and slack
    if ((size_t)optin <= fixed + 4096) return false;
    const uint64_t tmax = ((optin - fixed) / 4) & ~(uint64_t)3;
    uint64_t owned = (uint64_t)(owned_fraction * (double)n_local);
    owned = std::min<uint64_t>(std::min<uint64_t>(owned, n_local), (uint64_t)G * tmax);
    if (owned == 0) return false;
    uint64_t tile = (owned + G - 1) / G;
    tile = (tile + 3) & ~(uint64_t)3;
    const double deg = n_rows ? (double)e_local / (double)n_rows : 0.0;
    const double frac = (double)owned / (double)n_local;
    // ~12K binned events per tile per round.
    const double per_tile = 12288.0;
    double rpc = deg * frac > 0.0 ? per_tile / (deg * frac) : 1e9;
    if (rpc < 1.0) rpc = 1.0;
    if (rpc > 1e6) rpc = 1e6;
    L->grid = G;
    L->nb = 3;
    L->stage = stage;
    L->tile = (uint32_t)tile;
    L->owned = (uint32_t)owned;
    L->div_magic = ((1ull << 40) + tile - 1) / tile;
    L->rows_per_cta = (uint32_t)rpc;
    L->cap = (uint32_t)(1.5 * per_tile) + 2048u;
    L->smem_bytes = (uint32_t)(tile * 4 + (size_t)G * stage * 8 + (size_t)G * 4);
    L->spin_limit = 1u << 22;  // x ~128 ns naps: ~0.5 s before a wait is declared failed
    return true;
}

cudaError_t launch_propagate_binned(cudaStream_t s, const void *list, int idx_bits, const uint64_t *row_ptr,
                                    const uint32_t *col, const float *w, float *next, DevCounters *ctr, int parity,
                                    int count_spikes, const BinLayout &L) {
    static std::mutex mu;
    static bool configured[64][2] = {};
    cudaError_t e = cudaMemsetAsync(L.sync, 0, 2 * sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    void *fn = idx_bits == 32 ? (void *)propagate_binned_kernel<uint32_t> : (void *)propagate_binned_kernel<uint64_t>;
    {
        std::lock_guard<std::mutex> lock(mu);
        int dev = 0;
        cudaGetDevice(&dev);
        bool &done = configured[dev & 63][idx_bits == 32 ? 0 : 1];
        if (!done) {
            e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return e;
            done = true;
        }
    }
    BinLayout Lc = L;
    void *args[] = {(void *)&list, (void *)&row_ptr, (void *)&col, (void *)&w, (void *)&next,
                    (void *)&ctr, (void *)&parity, (void *)&count_spikes, (void *)&Lc};
    return cudaLaunchCooperativeKernel(fn, dim3(L.grid), dim3(kThreads), args, L.smem_bytes, s);
}

}  // namespace b200
