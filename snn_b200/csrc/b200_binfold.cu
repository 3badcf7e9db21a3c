// Bin-fold propagation: bit-exact (CSR-order) synaptic propagation whose cost
// follows the step's events, with no sort library and no host round trip.
//
// The serial CPU step adds, for every target, the weights of its spiking
// presynaptic rows in ascending (row, edge) order, starting from +0.0f
// (src/snn.c:898-906). Per step, on the device:
//  1. ordered compaction: the spike bitmap becomes the ascending spike list
//     (per-chunk popcounts, then every chunk writes its ids at its prefix),
//     and the step's event total (sum of the spiking rows' degrees) is added
//     to DevCounters::step_events[parity];
//  2. count: the spike list is cut into G contiguous slices, one per CTA;
//     each CTA counts its events per target tile (2^tile_bits consecutive
//     local targets) into hist[tile][cta];
//  3. an exclusive scan of hist (tile-major) gives every (tile, CTA) its
//     first slot in the event array;
//  4. scatter: every CTA walks its slice again in groups of rows (each warp
//     a run of consecutive rows, the warps in row order): per-warp counts per
//     tile, a prefix over the warps behind the CTA's cursor of each tile, then
//     every event (target within the tile, weight) is written to its slot;
//     equal tiles inside one round of 32 events are ranked in lane (= edge)
//     order (a shared-memory tag finds collisions, a ballot match over the
//     5-bit group id ranks them), so every tile keeps the global order;
//  5. fold: one CTA per tile keeps the tile's sums in shared memory; each
//     window of events is partitioned stably by owner warp (an eighth of the
//     tile each), then every warp applies its events in order, same-target
//     events of a round one after the other in lane order; last, the tile's
//     currents are written.
// A step whose events exceed the gate is a dense step: 2-5 do nothing
// and the pull kernel (launched behind the same device-side gate) runs.
// HBM per event: 4 B (count) + 8 B (scatter reads) + 8 B (scatter writes) +
// 8 B (fold reads), with 32-bit columns.
#include "b200_binfold.h"
#include "b200_device.cuh"

#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <mutex>
#include <vector>

namespace b200 {

namespace {

using namespace dev;

constexpr int kBfThreads = 256;
constexpr int kBfWarps = kBfThreads / 32;
constexpr uint32_t kChunkWords = 2048;  // bitmap words per compaction chunk (65,536 neurons)
constexpr int kWordsPerThread = kChunkWords / kBfThreads;
constexpr uint32_t kFoldWindow = 2048;  // events staged in shared memory per fold round

__device__ __forceinline__ bool dense_step(const DevCounters *ctr, int parity, unsigned long long gate) {
    return *(volatile const unsigned long long *)&ctr->step_events[parity] > gate;
}

// Block-wide exclusive scan of one u32 per thread; returns the thread's
// exclusive prefix, *total the block's sum. Every thread must call it.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *total) {
    __shared__ uint32_t s_warp[kBfWarps];
    const unsigned lane = lane_id(), warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(kFull, incl, d);
        if (lane >= (unsigned)d) incl += y;
    }
    if (lane == 31u) s_warp[warp] = incl;
    __syncthreads();
    uint32_t base = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kBfWarps; ++w) {
        const uint32_t t = s_warp[w];
        base += (w < (int)warp) ? t : 0u;
        tot += t;
    }
    __syncthreads();  // s_warp may be reused by the next call
    *total = tot;
    return base + incl - v;
}

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v) {
    __shared__ unsigned long long s_part[kBfWarps];
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(kFull, v, d);
    if (lane_id() == 0) s_part[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long t = 0;
#pragma unroll
    for (int w = 0; w < kBfWarps; ++w) t += s_part[w];
    __syncthreads();
    return t;
}

// ------------------------------------------------- ordered compaction ----
// Per-chunk popcounts of the (global) bitmap; also the popcount of this
// rank's own words [own_begin, own_end) into ctr->spikes. With a peer wait,
// every CTA first waits (bounded) for all ranks' flags of this step and
// gathers the other ranks' words into `bitmap` as it counts them.
__global__ void __launch_bounds__(kBfThreads) chunk_counts_kernel(uint32_t *__restrict__ bitmap, uint64_t words,
                                                                  uint32_t *__restrict__ ccnt, DevCounters *ctr,
                                                                  uint64_t own_begin, uint64_t own_end, PeerWait pw) {
    if (pw.nflags) {
        if (!block_peer_sync(pw, ctr)) return;
    }
    const uint64_t chunks = (words + kChunkWords - 1) / kChunkWords;
    unsigned long long own = 0;
    for (uint64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
        const uint64_t w0 = c * kChunkWords;
        uint32_t cnt = 0;
        for (uint32_t k = threadIdx.x; k < kChunkWords; k += kBfThreads) {
            const uint64_t wi = w0 + k;
            if (wi < words) {
                const uint32_t p = __popc(pw.nflags ? gather_word(pw, bitmap, wi) : __ldcg(bitmap + wi));
                cnt += p;
                if (wi >= own_begin && wi < own_end) own += p;
            }
        }
        uint32_t tot;
        block_exclusive_scan(cnt, &tot);
        if (threadIdx.x == 0) ccnt[c] = tot;
    }
    own = block_sum_u64(own);
    if (threadIdx.x == 0 && own) atomicAdd(&ctr->spikes, own);
}

// Each chunk writes its spiking ids ascending at the prefix of the chunks
// before it, so the list is globally ascending. The degrees of the written
// rows (batched states: row = id % batch_rows) are summed into
// step_events[parity]; the last chunk sets list_count[parity].
template <typename TIdx>
__global__ void __launch_bounds__(kBfThreads) compact_ordered_kernel(const uint32_t *__restrict__ bitmap,
                                                                     uint64_t words,
                                                                     const uint32_t *__restrict__ ccnt,
                                                                     TIdx *__restrict__ list, DevCounters *ctr,
                                                                     int parity, const uint64_t *__restrict__ row_ptr,
                                                                     uint64_t batch_rows) {
    if (*(volatile uint32_t *)&ctr->error != 0u) return;  // a peer wait expired: nothing to compact
    const uint64_t chunks = (words + kChunkWords - 1) / kChunkWords;
    unsigned long long events = 0;
    for (uint64_t c = blockIdx.x; c < chunks; c += gridDim.x) {
        uint32_t before = 0;
        for (uint64_t k = threadIdx.x; k < c; k += kBfThreads) before += ccnt[k];
        uint32_t prefix;
        block_exclusive_scan(before, &prefix);
        const uint64_t w0 = c * kChunkWords + (uint64_t)threadIdx.x * kWordsPerThread;
        uint32_t wv[kWordsPerThread];
        uint32_t cnt = 0;
#pragma unroll
        for (int j = 0; j < kWordsPerThread; ++j) {
            wv[j] = w0 + j < words ? __ldcg(bitmap + w0 + j) : 0u;
            cnt += __popc(wv[j]);
        }
        uint32_t tot;
        uint32_t pos = prefix + block_exclusive_scan(cnt, &tot);
#pragma unroll
        for (int j = 0; j < kWordsPerThread; ++j) {
            uint32_t m = wv[j];
            while (m) {
                const int b = __ffs(m) - 1;
                m &= m - 1u;
                const uint64_t id = (w0 + j) * 32u + (uint64_t)b;
                list[pos++] = (TIdx)id;
                const uint64_t row = batch_rows ? id % batch_rows : id;
                events += row_ptr[row + 1] - row_ptr[row];
            }
        }
        if (c == chunks - 1 && threadIdx.x == 0) ctr->list_count[parity] = prefix + tot;
    }
    events = block_sum_u64(events);
    if (threadIdx.x == 0 && events) atomicAdd(&ctr->step_events[parity], events);
}

// --------------------------------------------------------------- count ----
// CTA c owns list positions [count*c/G, count*(c+1)/G); hist[tile*G + c] =
// its events into each tile.
template <typename TIdx, typename TCol>
__global__ void __launch_bounds__(kBfThreads) binfold_count_kernel(const TIdx *__restrict__ list, DevCounters *ctr,
                                                                   int parity, const uint64_t *__restrict__ row_ptr,
                                                                   const TCol *__restrict__ col, uint64_t batch_rows,
                                                                   uint32_t tile_bits, uint32_t tiles,
                                                                   uint32_t *__restrict__ hist,
                                                                   unsigned long long gate) {
    extern __shared__ uint32_t s_cnt[];  // [tiles]
    if (dense_step(ctr, parity, gate)) return;
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    const unsigned lane = lane_id(), warp = threadIdx.x >> 5;
    for (uint32_t b = threadIdx.x; b < tiles; b += kBfThreads) s_cnt[b] = 0u;
    __syncthreads();
    const uint64_t G = gridDim.x;
    const uint64_t s0 = (uint64_t)count * blockIdx.x / G, s1 = (uint64_t)count * (blockIdx.x + 1) / G;
    for (uint64_t s = s0 + warp; s < s1; s += kBfWarps) {
        const uint64_t id = (uint64_t)list[s];
        const uint64_t row = batch_rows ? id % batch_rows : id;
        const uint64_t base = id - row;
        const uint64_t b = row_ptr[row], e = row_ptr[row + 1];
        for (uint64_t k0 = b + lane; k0 < e; k0 += 256u) {
            uint64_t c[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) c[u] = k0 + 32u * u < e ? (uint64_t)__ldg(col + k0 + 32u * u) : ~0ull;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (c[u] != ~0ull) atomicAdd(&s_cnt[(uint32_t)((base + c[u]) >> tile_bits)], 1u);
        }
    }
    __syncthreads();
    for (uint32_t b = threadIdx.x; b < tiles; b += kBfThreads) hist[(uint64_t)b * G + blockIdx.x] = s_cnt[b];
}

// ------------------------------------------------------------- scatter ----
// Same CTA slices as the count. The slice goes in groups of kScatterRows
// rows per warp, warp w taking the w-th run of consecutive rows of the group
// (so the warps are in row order): pass 1 counts each warp's events per tile,
// a prefix over the warps places them behind the CTA's cursor of each tile,
// pass 2 writes the events (equal tiles inside a round of 32 events ranked
// in lane = edge order), then the counters are cleared. All warps of a CTA
// append to one region per tile, so the partly written sectors waiting in L2
// number about CTAs x tiles.
constexpr uint32_t kScatterRows = 8;

template <typename TIdx, typename TCol>
__global__ void __launch_bounds__(kBfThreads) binfold_scatter_kernel(const TIdx *__restrict__ list, DevCounters *ctr,
                                                                     int parity, const uint64_t *__restrict__ row_ptr,
                                                                     const TCol *__restrict__ col,
                                                                     const float *__restrict__ w, uint64_t batch_rows,
                                                                     uint32_t tile_bits, uint32_t tiles,
                                                                     const uint32_t *__restrict__ offs,
                                                                     uint2 *__restrict__ bins,
                                                                     unsigned long long gate) {
    extern __shared__ uint32_t s_mem[];
    uint32_t *s_cur = s_mem;            // [tiles] this CTA's next slot of each tile
    uint32_t *s_w = s_mem + tiles;      // [warps][tiles] per-warp counts, then positions
    uint8_t *s_tag = reinterpret_cast<uint8_t *>(s_mem + (uint64_t)tiles * (kBfWarps + 1));  // [warps][tiles]
    if (dense_step(ctr, parity, gate)) return;
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    const unsigned lane = lane_id(), warp = threadIdx.x >> 5;
    const uint64_t G = gridDim.x;
    for (uint32_t b = threadIdx.x; b < tiles; b += kBfThreads) s_cur[b] = offs[(uint64_t)b * G + blockIdx.x];
    for (uint32_t b = threadIdx.x; b < tiles * kBfWarps; b += kBfThreads) s_w[b] = 0u;
    __syncthreads();
    const uint64_t s0 = (uint64_t)count * blockIdx.x / G, s1 = (uint64_t)count * (blockIdx.x + 1) / G;
    const uint32_t tmask = (1u << tile_bits) - 1u;
    uint32_t *my = s_w + (uint64_t)warp * tiles;
    uint8_t *tag = s_tag + (uint64_t)warp * tiles;
    for (uint64_t g0 = s0; g0 < s1; g0 += (uint64_t)kScatterRows * kBfWarps) {
        const uint64_t r0 = min(s1, g0 + (uint64_t)warp * kScatterRows);
        const uint64_t r1 = min(s1, r0 + kScatterRows);
        for (uint64_t s = r0; s < r1; ++s) {
            const uint64_t id = (uint64_t)list[s];
            const uint64_t row = batch_rows ? id % batch_rows : id;
            const uint64_t base = id - row;
            const uint64_t b = row_ptr[row], e = row_ptr[row + 1];
            for (uint64_t k0 = b + lane; k0 < e; k0 += 256u) {
                uint64_t c[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) c[u] = k0 + 32u * u < e ? (uint64_t)__ldg(col + k0 + 32u * u) : ~0ull;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (c[u] != ~0ull) atomicAdd(&my[(uint32_t)((base + c[u]) >> tile_bits)], 1u);
            }
        }
        __syncthreads();
        for (uint32_t t = threadIdx.x; t < tiles; t += kBfThreads) {
            uint32_t run = s_cur[t];
#pragma unroll
            for (int q = 0; q < kBfWarps; ++q) {
                const uint32_t x = s_w[(uint64_t)q * tiles + t];
                s_w[(uint64_t)q * tiles + t] = run;
                run += x;
            }
            s_cur[t] = run;
        }
        __syncthreads();
        for (uint64_t s = r0; s < r1; ++s) {
            const uint64_t id = (uint64_t)list[s];
            const uint64_t row = batch_rows ? id % batch_rows : id;
            const uint64_t base = id - row;
            const uint64_t b = row_ptr[row], e = row_ptr[row + 1];
            // Eight rounds of columns and weights in flight per lane, then the
            // eight rounds are ranked and written in order.
            for (uint64_t k0 = b; k0 < e; k0 += 256u) {
                uint32_t tv[8];
                float wv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const uint64_t k = k0 + 32u * u + lane;
                    tv[u] = k < e ? (uint32_t)(base + (uint64_t)__ldg(col + k)) : 0u;
                    wv[u] = k < e ? __ldcs(w + k) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (k0 + 32u * u >= e) break;  // warp-uniform
                    const bool act = k0 + 32u * u + lane < e;
                    const uint32_t t = tv[u];
                    const uint32_t tile = t >> tile_bits;
                    const uint32_t peers = group_by_key(tag, tile, act, lane);
                    const int leader = __ffs(peers) - 1;
                    uint32_t pos = 0;
                    if (act && lane == (unsigned)leader) pos = my[tile];
                    pos = __shfl_sync(kFull, pos, leader);
                    __syncwarp();
                    if (act && lane == (unsigned)leader) my[tile] = pos + (uint32_t)__popc(peers);
                    if (act) bins[pos + __popc(peers & lanemask_lt())] = make_uint2(t & tmask, __float_as_uint(wv[u]));
                }
            }
        }
        __syncthreads();
        for (uint32_t b = threadIdx.x; b < tiles * kBfWarps; b += kBfThreads) s_w[b] = 0u;
        __syncthreads();
    }
}

// ---------------------------------------------------------------- fold ----
// CTA per tile (grid-stride over tiles); warp w owns the tile's targets
// [w*T/8, (w+1)*T/8). Each window of events is first partitioned by owner,
// stably (warp w reads window positions [w*W/8, (w+1)*W/8) in rounds of 32;
// eight ballots rank every event among the equal-owner events before it),
// then every warp folds its own bucket in order: inside a round of 32, events
// for the same target are applied one after the other in lane order.
__global__ void __launch_bounds__(kBfThreads) binfold_fold_kernel(const uint2 *__restrict__ bins,
                                                                  const uint32_t *__restrict__ offs, uint32_t tiles,
                                                                  uint32_t grid_count, uint32_t tile_bits,
                                                                  uint64_t n_local, float *__restrict__ next,
                                                                  DevCounters *ctr, int parity,
                                                                  unsigned long long gate) {
    extern __shared__ __align__(16) unsigned char s_raw[];
    constexpr int kRounds = kFoldWindow / kBfWarps / 32;  // rounds of 32 events per warp per window
    const uint32_t T = 1u << tile_bits;
    float *acc = reinterpret_cast<float *>(s_raw);
    uint2 *sorted = reinterpret_cast<uint2 *>(s_raw + (size_t)T * 4);
    uint8_t *tag = reinterpret_cast<uint8_t *>(s_raw + (size_t)T * 4 + (size_t)kFoldWindow * 8);  // [T]
    __shared__ uint32_t s_cnt[kBfWarps][kBfWarps];  // [warp][owner] events in the warp's part
    __shared__ uint32_t s_pos[kBfWarps][kBfWarps];  // [warp][owner] first sorted position
    __shared__ uint32_t s_bucket[kBfWarps + 1];     // owner buckets in the sorted window
    if (dense_step(ctr, parity, gate)) return;
    const unsigned lane = lane_id(), warp = threadIdx.x >> 5;
    const uint32_t owner_shift = tile_bits - 3;
    const uint64_t G = grid_count;
    const uint32_t lt = lanemask_lt();
    for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const uint64_t lo = offs[(uint64_t)tile * G];
        const uint64_t hi = offs[(uint64_t)(tile + 1) * G];
        if (lo == hi) continue;  // no events: the tile's currents stay zero
        for (uint32_t t = threadIdx.x; t < T; t += kBfThreads) acc[t] = 0.0f;
        for (uint64_t w0 = lo; w0 < hi; w0 += kFoldWindow) {
            const uint32_t nwin = (uint32_t)min((uint64_t)kFoldWindow, hi - w0);
            // Partition: events of this warp's part, their owners and ranks.
            uint2 ev[kRounds];
            uint32_t rk[kRounds];
            if (lane < kBfWarps) s_cnt[warp][lane] = 0u;
            // Warp w partitions window positions [p0, p1), in order.
            const uint32_t p0 = nwin * warp / kBfWarps, p1 = nwin * (warp + 1) / kBfWarps;
#pragma unroll
            for (int j = 0; j < kRounds; ++j) {
                const uint32_t i = p0 + j * 32u + lane;
                ev[j] = i < p1 ? __ldcs(bins + w0 + i) : make_uint2(0u, 0u);
            }
            __syncwarp();
#pragma unroll
            for (int j = 0; j < kRounds; ++j) {
                if (p0 + j * 32u >= p1) break;  // warp-uniform
                const uint32_t i = p0 + j * 32u + lane;
                const bool act = i < p1;
                const uint32_t o = ev[j].x >> owner_shift;
                uint32_t peers = match_bits_n<3>(o, __ballot_sync(kFull, act));
                if (!act) peers = 1u << lane;
                const int leader = __ffs(peers) - 1;
                uint32_t base = 0;
                if (act && lane == (unsigned)leader) base = atomicAdd(&s_cnt[warp][o], (uint32_t)__popc(peers));
                base = __shfl_sync(kFull, base, leader);
                rk[j] = base + __popc(peers & lt);
            }
            __syncthreads();
            if (threadIdx.x < kBfWarps * kBfWarps) {
                const uint32_t o = threadIdx.x / kBfWarps, wq = threadIdx.x % kBfWarps;
                uint32_t p = 0;
                for (uint32_t o2 = 0; o2 < o; ++o2)
                    for (uint32_t w2 = 0; w2 < kBfWarps; ++w2) p += s_cnt[w2][o2];
                for (uint32_t w2 = 0; w2 < wq; ++w2) p += s_cnt[w2][o];
                s_pos[wq][o] = p;
                if (wq == 0) s_bucket[o] = p;
                if (threadIdx.x == 0) s_bucket[kBfWarps] = nwin;
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kRounds; ++j) {
                const uint32_t i = p0 + j * 32u + lane;
                if (i < p1) sorted[s_pos[warp][ev[j].x >> owner_shift] + rk[j]] = ev[j];
            }
            __syncthreads();
            // Fold this warp's bucket in order.
            const uint32_t b0 = s_bucket[warp], b1 = s_bucket[warp + 1];
            for (uint32_t i0 = b0; i0 < b1; i0 += 32u) {
                const uint32_t i = i0 + lane;
                const bool act = i < b1;
                const uint2 e = act ? sorted[i] : make_uint2(0u, 0u);
                const uint32_t peers = group_by_key(tag, e.x, act, lane);
                const int rank = __popc(peers & lt);
                const int rounds = (int)__reduce_max_sync(kFull, act ? (uint32_t)__popc(peers) : 0u);
                for (int r = 0; r < rounds; ++r) {
                    if (act && rank == r) acc[e.x] = __fadd_rn(acc[e.x], __uint_as_float(e.y));
                    __syncwarp();
                }
            }
            __syncthreads();
        }
        const uint64_t t0 = (uint64_t)tile << tile_bits;
        const uint32_t nt = (uint32_t)min((uint64_t)T, n_local - t0);
        for (uint32_t t = threadIdx.x; t < nt; t += kBfThreads) next[t0 + t] = acc[t];
        __syncthreads();
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) ctr->events += ctr->step_events[parity];
    step_epilogue(ctr, parity, 0, *(volatile uint32_t *)&ctr->list_count[parity]);
}

int fold_smem(uint32_t tile_bits) { return (int)(((size_t)5 << tile_bits) + (size_t)kFoldWindow * 8); }
int scatter_smem(uint32_t tiles) { return (int)((size_t)tiles * (kBfWarps + 1) * 4 + (size_t)tiles * kBfWarps); }

template <typename K>
void allow_smem(K kernel, int bytes) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

}  // namespace

bool binfold_plan(int device, uint64_t n_local, BinFoldPlan *plan) {
    // Tiles of 2^tile_bits targets, at most kBinFoldMaxTiles of them; a tile's
    // sums (4 B each) plus a fold window must fit one CTA's shared memory.
    uint32_t tb = 10;
    while (tb < 15 && ((n_local + (1ull << tb) - 1) >> tb) > kBinFoldMaxTiles) ++tb;
    const uint64_t tiles = (n_local + (1ull << tb) - 1) >> tb;
    if (tiles > kBinFoldMaxTiles || tiles == 0) return false;
    plan->tile_bits = tb;
    plan->tiles = (uint32_t)tiles;
    plan->grid = (uint32_t)sm_count(device) * 4u;
    plan->hist_entries = (uint64_t)plan->tiles * plan->grid + 1;
    plan->chunks = 0;
    return true;
}

uint32_t binfold_chunks(uint64_t words) { return (uint32_t)((words + kChunkWords - 1) / kChunkWords); }

cudaError_t binfold_scan(cudaStream_t s, const uint32_t *hist, uint32_t *offs, uint64_t n, void *temp,
                         size_t *temp_bytes) {
    return cub::DeviceScan::ExclusiveSum(temp, *temp_bytes, hist, offs, (int64_t)n, s);
}

void launch_compact_ordered(cudaStream_t s, int device, uint32_t *bitmap, uint64_t words, uint32_t *ccnt,
                            void *list, int idx_bits, DevCounters *ctr, int parity, uint64_t own_begin,
                            uint64_t own_end, const uint64_t *row_ptr, uint64_t batch_rows, const PeerWait *wait) {
    PeerWait pw{};
    if (wait) pw = *wait;
    const uint64_t chunks = binfold_chunks(words);
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(chunks, (uint64_t)sm_count(device) * 8));
    chunk_counts_kernel<<<grid, kBfThreads, 0, s>>>(bitmap, words, ccnt, ctr, own_begin, own_end, pw);
    if (idx_bits == 32)
        compact_ordered_kernel<uint32_t><<<grid, kBfThreads, 0, s>>>(bitmap, words, ccnt, (uint32_t *)list, ctr,
                                                                     parity, row_ptr, batch_rows);
    else
        compact_ordered_kernel<uint64_t><<<grid, kBfThreads, 0, s>>>(bitmap, words, ccnt, (uint64_t *)list, ctr,
                                                                     parity, row_ptr, batch_rows);
}

cudaError_t launch_binfold(cudaStream_t s, int device, const BinFoldPlan &p, const BinFoldBuffers &buf,
                           const void *list, int idx_bits, const uint64_t *row_ptr, const void *col, int col_bits,
                           const float *w, uint64_t batch_rows, uint64_t n_local, float *next, DevCounters *ctr,
                           int parity, unsigned long long gate) {
    static std::mutex mu;
    static bool attr_done[64] = {};
    const int ssm = scatter_smem(p.tiles), fsm = fold_smem(p.tile_bits);
#define B200_BF(TI, TC)                                                                                          \
    do {                                                                                                         \
        {                                                                                                        \
            std::lock_guard<std::mutex> lock(mu);                                                                \
            if (device >= 0 && device < 64 && !attr_done[device]) {                                             \
                allow_smem(binfold_scatter_kernel<uint32_t, uint32_t>, scatter_smem(kBinFoldMaxTiles));           \
                allow_smem(binfold_scatter_kernel<uint32_t, uint64_t>, scatter_smem(kBinFoldMaxTiles));           \
                allow_smem(binfold_scatter_kernel<uint64_t, uint32_t>, scatter_smem(kBinFoldMaxTiles));           \
                allow_smem(binfold_scatter_kernel<uint64_t, uint64_t>, scatter_smem(kBinFoldMaxTiles));           \
                allow_smem(binfold_fold_kernel, fold_smem(15));                                                  \
                attr_done[device] = true;                                                                        \
            }                                                                                                    \
        }                                                                                                        \
        binfold_count_kernel<TI, TC><<<p.grid, kBfThreads, (size_t)p.tiles * 4, s>>>(                            \
            (const TI *)list, ctr, parity, row_ptr, (const TC *)col, batch_rows, p.tile_bits, p.tiles, buf.hist, \
            gate);                                                                                               \
        size_t tb = buf.scan_bytes;                                                                              \
        const cudaError_t e = binfold_scan(s, buf.hist, buf.offs, p.hist_entries, buf.scan_temp, &tb);           \
        if (e != cudaSuccess) return e;                                                                          \
        binfold_scatter_kernel<TI, TC><<<p.grid, kBfThreads, ssm, s>>>(                                          \
            (const TI *)list, ctr, parity, row_ptr, (const TC *)col, w, batch_rows, p.tile_bits, p.tiles,        \
            buf.offs, buf.bins, gate);                                                                           \
    } while (0)
    if (idx_bits == 32 && col_bits == 32) B200_BF(uint32_t, uint32_t);
    else if (idx_bits == 32) B200_BF(uint32_t, uint64_t);
    else if (col_bits == 32) B200_BF(uint64_t, uint32_t);
    else B200_BF(uint64_t, uint64_t);
#undef B200_BF
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, binfold_fold_kernel, kBfThreads, fsm) != cudaSuccess ||
        per_sm <= 0)
        per_sm = 1;
    const int grid = (int)std::min<uint64_t>(p.tiles, (uint64_t)sm_count(device) * per_sm);
    binfold_fold_kernel<<<grid, kBfThreads, fsm, s>>>(buf.bins, buf.offs, p.tiles, p.grid, p.tile_bits, n_local,
                                                       next, ctr, parity, gate);
    return cudaGetLastError();
}

}  // namespace b200
