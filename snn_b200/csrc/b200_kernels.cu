// snn_b200 device kernels for sm_100a.
//
// The simulation step is HBM-bound integer/byte work plus fp32 adds, so the
// kernels are SIMT with wide vector loads, warp ballots and warp/block
// aggregated atomics; nothing here is a dense contraction, so there is no
// tensor-core path. Floating point follows the reference's bit-exactness rules
// (src/snn_cuda.cu:203-225, CMakeLists.txt:57-60): every LIF, injection and
// weight-generation operation is an explicitly rounded __fadd_rn / __fmul_rn /
// __fsub_rn, so no FMA contraction can change a bit, and the host's
// decay = expf(-dt/tau) is used as given.
#include "b200_kernels.h"
#include "b200_device.cuh"

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>
#include <thrust/iterator/transform_iterator.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

namespace b200 {

namespace {

using namespace dev;

constexpr uint64_t kGamma = 0x9e3779b97f4a7c15ull;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Draw d (1-based) of the splitmix64 stream seeded `seed` (src/snn.c:94-99:
// the state advances by gamma before every mix).
__device__ __forceinline__ uint64_t draw_at(uint64_t seed, uint64_t d) { return mix64(seed + d * kGamma); }

// src/snn.c:101-105: top 53 bits scaled to [0,1) in double, rounded to float.
__device__ __forceinline__ float unit_float(uint64_t r) {
    return __double2float_rn((double)(r >> 11) * (1.0 / 9007199254740992.0));
}

// src/snn.c:559-567: weight_min + span * u in float (no FMA), clamped.
__device__ __forceinline__ float lerp_weight(float wmin, float wmax, float u) {
    const float w = __fadd_rn(wmin, __fmul_rn(__fsub_rn(wmax, wmin), u));
    return w < wmax ? w : wmax;
}


template <typename T>
struct Vec16;
template <>
struct Vec16<uint32_t> {
    using type = uint4;
    static constexpr int n = 4;
};
template <>
struct Vec16<uint64_t> {
    using type = ulonglong2;
    static constexpr int n = 2;
};
template <int N>
struct FVec;
template <>
struct FVec<4> {
    using type = float4;
};
template <>
struct FVec<2> {
    using type = float2;
};

template <typename T>
__device__ __forceinline__ T vget(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint64_t cget(const ulonglong2 &v, int i) { return i == 0 ? v.x : v.y; }
__device__ __forceinline__ uint32_t cget(const uint4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ float fget(const float4 &v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ float fget(const float2 &v, int i) { return i == 0 ? v.x : v.y; }

// ---------------------------------------------------------------- init ----
__global__ void init_state_kernel(uint64_t n, float v_rest, float *v, float *cur0, float *cur1, float *ext,
                                  uint32_t *refr, uint8_t *spikes, uint64_t words, uint32_t *bitmap,
                                  DevCounters *ctr, uint8_t *kind_log) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    const uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (uint64_t i = t0; i < n; i += stride) {
        v[i] = v_rest;
        cur0[i] = 0.0f;
        cur1[i] = 0.0f;
        if (ext != nullptr) ext[i] = 0.0f;
        refr[i] = 0u;
        spikes[i] = 0u;
    }
    for (uint64_t i = t0; i < words; i += stride) bitmap[i] = 0u;
    if (t0 == 0 && ctr != nullptr) {
        ctr->list_count[0] = 0u;
        ctr->list_count[1] = 0u;
        ctr->error = 0u;
        ctr->spikes = 0ull;
        ctr->events = 0ull;
        ctr->stream_step = 0ull;
        ctr->pull_runs = 0ull;
        ctr->pull_events = 0ull;
        ctr->pull_spikes = 0ull;
        ctr->step_seq = 0ull;
        ctr->wait_ns = 0ull;
        ctr->wait_max_ns = 0ull;
        ctr->kind_log = kind_log;
        ctr->step_events[0] = 0ull;
        ctr->step_events[1] = 0ull;
    }
}

// ----------------------------------------------------------------- LIF ----
// One CTA owns a tile of ITERS*1024 consecutive neurons; each thread updates 4
// consecutive neurons per iteration with 16-byte loads/stores. The 4 fired
// flags of a lane form a nibble; 8 lanes OR their nibbles into one 32-bit
// bitmap word. Spiking ids are ranked with a warp scan + a per-iteration block
// scan, buffered ascending in shared memory, and appended to the global list
// with ONE atomic per tile (the list is ascending inside a tile).
constexpr int kLifThreads = 256;

__device__ __forceinline__ uint32_t lif_one(float &v, float &c, float in, uint32_t &r, const LifArgs &p) {
    // ((v_rest + (v - v_rest) * decay) + current) + in   (src/snn_cuda.cu:214)
    const float v_int =
        __fadd_rn(__fadd_rn(__fadd_rn(p.v_rest, __fmul_rn(__fsub_rn(v, p.v_rest), p.decay)), c), in);
    const uint32_t active = r == 0u;
    const uint32_t fired = active & (v_int >= p.v_threshold ? 1u : 0u);
    c = 0.0f;
    v = (active & (fired ^ 1u)) ? v_int : p.v_reset;
    r = fired ? p.refractory_steps : r - (uint32_t)(r != 0u);
    return fired;
}

template <bool HAS_EXT, bool WRITE_LIST, typename TIdx, int ITERS>
__global__ void __launch_bounds__(kLifThreads) lif_kernel(uint64_t n, LifArgs p, float *__restrict__ v,
                                                          float *__restrict__ cur,
                                                          const float *__restrict__ ext,
                                                          uint32_t *__restrict__ refr, uint8_t *__restrict__ spikes,
                                                          uint32_t *__restrict__ bitmap, TIdx *__restrict__ list,
                                                          uint64_t global_offset, DevCounters *ctr, int parity) {
    constexpr uint64_t kTile = (uint64_t)ITERS * kLifThreads * 4u;
    // The step's injection (stream order: already complete) has read the
    // index; advance it for the next step.
    if (p.stream_step != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *p.stream_step += 1ull;
    __shared__ TIdx sbuf[WRITE_LIST ? kTile : 1];
    __shared__ uint32_t warp_tot[kLifThreads / 32];
    __shared__ uint32_t s_base;
    const unsigned lane = lane_id();
    const unsigned warp = threadIdx.x >> 5;
    const uint64_t tiles = (n + kTile - 1) / kTile;
    for (uint64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        uint32_t block_off = 0;
        for (int it = 0; it < ITERS; ++it) {
            const uint64_t i0 = tile * kTile + (uint64_t)it * (kLifThreads * 4u) + threadIdx.x * 4u;
            uint32_t nib = 0;
            if (i0 + 3 < n) {
                float4 vv = *reinterpret_cast<const float4 *>(v + i0);
                float4 cc = *reinterpret_cast<const float4 *>(cur + i0);
                uint4 rr = *reinterpret_cast<const uint4 *>(refr + i0);
                float4 ee = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (HAS_EXT) {
                    ee = *reinterpret_cast<const float4 *>(ext + i0);
                    ee.x = __fmul_rn(ee.x, p.input_scale);
                    ee.y = __fmul_rn(ee.y, p.input_scale);
                    ee.z = __fmul_rn(ee.z, p.input_scale);
                    ee.w = __fmul_rn(ee.w, p.input_scale);
                }
                nib |= lif_one(vv.x, cc.x, ee.x, rr.x, p);
                nib |= lif_one(vv.y, cc.y, ee.y, rr.y, p) << 1;
                nib |= lif_one(vv.z, cc.z, ee.z, rr.z, p) << 2;
                nib |= lif_one(vv.w, cc.w, ee.w, rr.w, p) << 3;
                *reinterpret_cast<float4 *>(v + i0) = vv;
                *reinterpret_cast<float4 *>(cur + i0) = cc;
                *reinterpret_cast<uint4 *>(refr + i0) = rr;
                *reinterpret_cast<uint32_t *>(spikes + i0) =
                    (nib & 1u) | ((nib >> 1) & 1u) << 8 | ((nib >> 2) & 1u) << 16 | ((nib >> 3) & 1u) << 24;
            } else if (i0 < n) {
                for (int k = 0; k < 4; ++k) {
                    const uint64_t i = i0 + k;
                    if (i < n) {
                        float vv = v[i], cc = cur[i];
                        uint32_t rr = refr[i];
                        const float in = HAS_EXT ? __fmul_rn(ext[i], p.input_scale) : 0.0f;
                        const uint32_t f = lif_one(vv, cc, in, rr, p);
                        v[i] = vv;
                        cur[i] = cc;
                        refr[i] = rr;
                        spikes[i] = (uint8_t)f;
                        nib |= f << k;
                    }
                }
            }
            // 8 lanes x 4 neurons = one 32-bit bitmap word.
            uint32_t word = nib << (4u * (lane & 7u));
            word |= __shfl_xor_sync(kFull, word, 1);
            word |= __shfl_xor_sync(kFull, word, 2);
            word |= __shfl_xor_sync(kFull, word, 4);
            if ((lane & 7u) == 0u && i0 < n) bitmap[i0 >> 5] = word;
            if (WRITE_LIST) {
                const uint32_t cnt = __popc(nib);
                uint32_t incl = cnt;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const uint32_t y = __shfl_up_sync(kFull, incl, d);
                    if (lane >= (unsigned)d) incl += y;
                }
                if (lane == 31u) warp_tot[warp] = incl;
                __syncthreads();
                uint32_t wbase = block_off, total = 0;
#pragma unroll
                for (int w = 0; w < kLifThreads / 32; ++w) {
                    const uint32_t t = warp_tot[w];
                    wbase += (w < (int)warp) ? t : 0u;
                    total += t;
                }
                uint32_t pos = wbase + incl - cnt;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (nib & (1u << k)) sbuf[pos++] = (TIdx)(i0 + k);
                }
                __syncthreads();
                block_off += total;
            }
        }
        if (WRITE_LIST) {
            if (threadIdx.x == 0) s_base = block_off ? atomicAdd(&ctr->list_count[parity], block_off) : 0u;
            __syncthreads();
            const uint32_t base = s_base;
            for (uint32_t k = threadIdx.x; k < block_off; k += kLifThreads)
                list[base + k] = (TIdx)(sbuf[k] + global_offset);
            __syncthreads();
        }
    }
}

// Peer exchange publication, launched right after the LIF kernel on the same
// stream: the LIF kernel's words are complete and visible when it starts, and
// its release store of the step tag into this rank's flag slot of every rank
// lets the others read them after an acquire.
__global__ void publish_flags_kernel(PeerWait pw) {
    if (threadIdx.x < pw.nflags && pw.publish[threadIdx.x] != nullptr)
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(pw.publish[threadIdx.x]), "l"(pw.tag) : "memory");
}

// ---------------------------------------------------------- compaction ----
template <typename TIdx>
__global__ void __launch_bounds__(256) compact_kernel(uint32_t *__restrict__ bitmap, uint64_t words,
                                                      TIdx *__restrict__ list, DevCounters *ctr, int parity,
                                                      uint64_t own_begin, uint64_t own_end, PeerWait pw) {
    const unsigned lane = lane_id();
    if (pw.nflags) {
        // Wait (bounded) until every rank has published this step's slice.
        if (!block_peer_sync(pw, ctr)) return;
    }
    // Four words (16 bytes) per thread: the bitmap (words a multiple of 4)
    // and every rank's slice (slot_words a multiple of 4) are 16-byte
    // aligned, so a vector never straddles two owners.
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    const uint64_t vecs = words / 4;
    uint32_t own = 0;
    for (uint64_t base = (uint64_t)blockIdx.x * blockDim.x; base < vecs; base += stride) {
        const uint64_t vi = base + threadIdx.x;
        const uint64_t wi = vi * 4;
        uint4 q = make_uint4(0u, 0u, 0u, 0u);
        if (vi < vecs) q = pw.nflags ? gather_vec(pw, bitmap, wi) : __ldcg(reinterpret_cast<const uint4 *>(bitmap) + vi);
        const uint32_t cnt = __popc(q.x) + __popc(q.y) + __popc(q.z) + __popc(q.w);
        if (wi >= own_begin && wi < own_end) own += cnt;
        uint32_t incl = cnt;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t y = __shfl_up_sync(kFull, incl, d);
            if (lane >= (unsigned)d) incl += y;
        }
        const uint32_t total = __shfl_sync(kFull, incl, 31);
        uint32_t off = 0;
        if (lane == 31u && total) off = atomicAdd(&ctr->list_count[parity], total);
        off = __shfl_sync(kFull, off, 31);
        uint32_t pos = off + incl - cnt;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t m = j == 0 ? q.x : j == 1 ? q.y : j == 2 ? q.z : q.w;
            while (m) {
                const int b = __ffs(m) - 1;
                m &= m - 1u;
                list[pos++] = (TIdx)((wi + j) * 32u + (uint64_t)b);
            }
        }
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) own += __shfl_xor_sync(kFull, own, d);
    if (lane == 0 && own) atomicAdd(&ctr->spikes, (unsigned long long)own);
}

// ---------------------------------------------------------------- push ----
// Warp per spiking row (grid-stride over the list). The row's col_idx and
// weights are streamed with 16-byte evict-first loads (__ldcs: they are read
// once per step and must not push the L2-resident target currents out),
// software-pipelined one vector deep, and every edge issues a fire-and-forget
// red.global.add.f32 into next_current, which stays L2-resident.
template <typename TCol, int LANES = 32>
__device__ __forceinline__ void push_row(uint64_t b, uint64_t e, const TCol *__restrict__ col,
                                         const float *__restrict__ w, float *__restrict__ next, unsigned lane) {
    using V = typename Vec16<TCol>::type;
    constexpr int VN = Vec16<TCol>::n;
    using FV = typename FVec<VN>::type;
    uint64_t a = (b + (VN - 1)) & ~(uint64_t)(VN - 1);
    if (a > e) a = e;
    if (lane < a - b) red_add(next + col[b + lane], w[b + lane]);
    const uint64_t nvec = (e - a) / VN;
    const V *cv = reinterpret_cast<const V *>(col + a);
    const FV *wv = reinterpret_cast<const FV *>(w + a);
    uint64_t k = lane;
    V c0;
    FV x0;
    if (k < nvec) {
        c0 = __ldcs(cv + k);
        x0 = __ldcs(wv + k);
    }
    while (k < nvec) {
        const uint64_t k1 = k + (uint64_t)LANES;
        V c1;
        FV x1;
        if (k1 < nvec) {
            c1 = __ldcs(cv + k1);
            x1 = __ldcs(wv + k1);
        }
#pragma unroll
        for (int j = 0; j < VN; ++j) red_add(next + cget(c0, j), fget(x0, j));
        c0 = c1;
        x0 = x1;
        k = k1;
    }
    const uint64_t t0 = a + nvec * VN;
    if (lane < e - t0) red_add(next + col[t0 + lane], w[t0 + lane]);
}

// LANES lanes per spiking row (32: a warp; 16 or 8 for short rows, such as
// a shard's slice of a row, so that a warp has several rows in flight).
template <typename TIdx, typename TCol, int LANES>
__global__ void __launch_bounds__(256) propagate_push_kernel(const TIdx *__restrict__ list,
                                                             const uint64_t *__restrict__ row_ptr,
                                                             const TCol *__restrict__ col,
                                                             const float *__restrict__ w, float *__restrict__ next,
                                                             DevCounters *ctr, int parity, int count_spikes,
                                                             uint64_t batch_rows, uint32_t pull_above) {
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    if (pull_above && count > pull_above) return;  // dense step: the pull kernel runs
    const unsigned lane = lane_id() % LANES;
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) / LANES;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) / LANES;
    unsigned long long events = 0;
    for (uint64_t s = gwarp; s < count; s += nwarps) {
        uint64_t row = (uint64_t)list[s];
        float *dst = next;
        if (batch_rows) {  // batched states: sample (id / rows) adds into its own current slice
            const uint64_t r = row % batch_rows;
            dst = next + (row - r);
            row = r;
        }
        const uint64_t b = row_ptr[row];
        const uint64_t e = row_ptr[row + 1];
        events += e - b;
        push_row<TCol, LANES>(b, e, col, w, dst, lane);
    }
    block_add_u64(lane == 0 ? events : 0ull, &ctr->events);
    step_epilogue(ctr, parity, count_spikes, count);
}

// --------------------------------------------------------- ordered push ----
// Bit-exact propagation driven by the spike list (cost ~ events, not
// synapses). Every target must fold its contributions in CSR order, i.e. in
// ascending edge index (src/snn.c:898-906). Each step:
//  1. ordered_sdeg: sdeg[row] = out-degree of every spiking row;
//  2. exclusive scan of sdeg over all rows -> eoff[row]: the step's events
//     numbered densely in CSR order;
//  3. ordered_gen: every spiking row writes its (target, weight) pairs at
//     eoff[row] (coalesced runs), so the event array is in CSR order;
//  4. a stable LSD radix sort by target groups the events per target and
//     keeps each group in CSR order;
//  5. ordered_fold: the first event of every target's run folds the run
//     sequentially onto next[t].
// A step whose events exceed the buffer capacity runs 3-5 per row range.
template <typename TIdx>
__global__ void __launch_bounds__(256) ordered_sdeg_kernel(const TIdx *__restrict__ list, DevCounters *ctr,
                                                           int parity, const uint64_t *__restrict__ row_ptr,
                                                           uint32_t *__restrict__ sdeg, int clear,
                                                           uint64_t batch_rows) {
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s < count; s += stride) {
        const uint64_t id = (uint64_t)list[s];
        const uint64_t row = batch_rows ? id % batch_rows : id;
        sdeg[id] = clear ? 0u : (uint32_t)(row_ptr[row + 1] - row_ptr[row]);
    }
}

// Warp per spiking row of [row_lo, row_hi): copy the row's (target, weight)
// pairs to event slots eoff[row] - id_base onwards and clear its sdeg entry.
// Block 0 adds the step's events (eoff[rows]) and runs the step epilogue when
// asked.
template <typename TIdx, typename TCol>
__global__ void __launch_bounds__(256) ordered_gen_kernel(const TIdx *__restrict__ list, DevCounters *ctr, int parity,
                                                          uint64_t row_lo, uint64_t row_hi,
                                                          const uint64_t *__restrict__ row_ptr,
                                                          const TCol *__restrict__ col, const float *__restrict__ w,
                                                          const unsigned long long *__restrict__ eoff, uint64_t rows,
                                                          uint64_t id_base, uint32_t *__restrict__ sdeg,
                                                          uint32_t *__restrict__ keys, float *__restrict__ vals,
                                                          int epilogue, int count_spikes, uint64_t batch_rows) {
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t s = gwarp; s < count; s += nwarps) {
        const uint64_t id = (uint64_t)list[s];
        if (id < row_lo || id >= row_hi) continue;
        const uint64_t row = batch_rows ? id % batch_rows : id;
        const uint32_t base = (uint32_t)(id - row);  // batched: the sample's first neuron
        const uint64_t b = row_ptr[row], e = row_ptr[row + 1];
        const uint64_t d = eoff[id] - id_base - b;
        uint64_t k = b + lane;
        // Four rounds of loads in flight per lane, then their stores.
        for (; k + 96u < e; k += 128u) {
            uint32_t cv[4];
            float wv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                cv[u] = (uint32_t)__ldcs(col + k + 32u * u);
                wv[u] = __ldcs(w + k + 32u * u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                keys[d + k + 32u * u] = base + cv[u];
                vals[d + k + 32u * u] = wv[u];
            }
        }
        for (; k < e; k += 32u) {
            keys[d + k] = base + (uint32_t)col[k];
            vals[d + k] = __ldcs(w + k);
        }
        if (lane == 0) sdeg[id] = 0u;
    }
    if (epilogue) {
        if (blockIdx.x == 0 && threadIdx.x == 0) ctr->events += eoff[rows];
        step_epilogue(ctr, parity, count_spikes, count);
    }
}

// First position in [lo, hi) whose key is >= x (hi if none), for keys
// sorted in their bits above the fold group's and x a multiple of the group
// size: a 33-way search, one load per lane per round.
__device__ __forceinline__ uint64_t warp_lower_bound(const uint32_t *__restrict__ keys, uint64_t lo, uint64_t hi,
                                                     uint32_t x, unsigned lane) {
    while (hi - lo > 32u) {
        const uint64_t span = hi - lo;
        const uint64_t p = lo + span * (lane + 1u) / 33u;
        const uint32_t ge = __ballot_sync(kFull, keys[p] >= x);
        if (ge == 0u) {
            lo = __shfl_sync(kFull, p, 31) + 1u;
        } else {
            const int f = __ffs(ge) - 1;
            const uint64_t pf = __shfl_sync(kFull, p, f);
            const uint64_t pb = __shfl_sync(kFull, p, f > 0 ? f - 1 : 0);
            if (f > 0) lo = pb + 1u;
            hi = pf;
        }
    }
    const uint64_t q = lo + lane;
    const uint32_t ge = __ballot_sync(kFull, q < hi && keys[q] >= x);
    return ge ? lo + (uint64_t)(__ffs(ge) - 1) : hi;
}

// Group fold: the events are sorted stably by target >> GB only, so every
// group of 2^GB consecutive targets has its events contiguous and still in
// CSR order (one radix pass fewer than a full sort by target). A warp per
// group keeps the group's currents in shared memory (loaded from next, so
// successive row ranges accumulate) and applies the events 32 at a time in
// order: within a round of 32, the lowest pending lane of every target (a
// shared-memory atomicMin on a per-target tag) applies its event, then the
// next, so same-target events go in lane (= CSR) order. The next rounds'
// events are loaded while the current ones are applied.
template <int GB>
__global__ void __launch_bounds__(256) ordered_group_fold_kernel(uint64_t events, const uint32_t *__restrict__ keys,
                                                                 const float *__restrict__ vals,
                                                                 float *__restrict__ next, uint64_t n_targets) {
    constexpr uint32_t G = 1u << GB;
    constexpr int kAhead = 4;  // rounds of 32 events per load batch
    constexpr uint32_t kFree = 0xffffffffu;
    __shared__ float s_acc[8][G];
    __shared__ uint32_t s_tag[8][G];
    const unsigned lane = lane_id(), warp = threadIdx.x >> 5;
    float *acc = s_acc[warp];
    uint32_t *tag = s_tag[warp];
    for (uint32_t t = lane; t < G; t += 32u) tag[t] = kFree;
    __syncwarp();
    const uint64_t groups = (n_targets + G - 1) / G;
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t g = gwarp; g < groups; g += nwarps) {
        const uint32_t t0 = (uint32_t)(g * G);
        const uint64_t lo = warp_lower_bound(keys, 0, events, t0, lane);
        const uint64_t hi = g + 1 < groups ? warp_lower_bound(keys, lo, events, t0 + G, lane) : events;
        if (lo == hi) continue;  // warp-uniform: no events, currents untouched
        const uint32_t nt = (uint32_t)min((uint64_t)G, n_targets - t0);
        for (uint32_t t = lane; t < nt; t += 32u) acc[t] = next[t0 + t];
        uint32_t key[kAhead], nkey[kAhead];
        float v[kAhead], nv[kAhead];
#pragma unroll
        for (int j = 0; j < kAhead; ++j) {
            const uint64_t i = lo + 32u * j + lane;
            key[j] = i < hi ? __ldcs(keys + i) - t0 : 0u;
            v[j] = i < hi ? __ldcs(vals + i) : 0.0f;
        }
        __syncwarp();
        for (uint64_t i0 = lo; i0 < hi; i0 += 32u * kAhead) {
            const uint64_t n0 = i0 + 32u * kAhead;
#pragma unroll
            for (int j = 0; j < kAhead; ++j) {
                const uint64_t i = n0 + 32u * j + lane;
                nkey[j] = i < hi ? __ldcs(keys + i) - t0 : 0u;
                nv[j] = i < hi ? __ldcs(vals + i) : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < kAhead; ++j) {
                uint32_t pending = __ballot_sync(kFull, i0 + 32u * j + lane < hi);
                while (pending) {  // warp-uniform
                    const bool mine = (pending >> lane) & 1u;
                    if (mine) atomicMin(&tag[key[j]], lane);
                    __syncwarp();
                    const bool win = mine && tag[key[j]] == lane;
                    if (win) {  // a loser reading the freed tag sees no match
                        acc[key[j]] = __fadd_rn(acc[key[j]], v[j]);
                        tag[key[j]] = kFree;
                    }
                    __syncwarp();
                    pending &= ~__ballot_sync(kFull, win);
                }
            }
#pragma unroll
            for (int j = 0; j < kAhead; ++j) {
                key[j] = nkey[j];
                v[j] = nv[j];
            }
        }
        __syncwarp();
        for (uint32_t t = lane; t < nt; t += 32u) next[t0 + t] = acc[t];
        __syncwarp();
    }
}

// Warp per 32-event chunk of the target-sorted array; every run (one
// target's events) is folded in order onto next[target] by the chunk where
// it starts. A run shorter than 32 events is walked by the lane at its start
// (four events per round of loads); a longer run is walked by the whole warp,
// 32 events per coalesced load, folded through lane shuffles.
__global__ void __launch_bounds__(256) ordered_fold_kernel(uint64_t events, const uint32_t *__restrict__ keys,
                                                           const float *__restrict__ vals, float *__restrict__ next) {
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t c0 = gwarp * 32u; c0 < events; c0 += nwarps * 32u) {
        const uint64_t k = c0 + lane;
        const uint32_t key = k < events ? keys[k] : 0xffffffffu;
        const bool start = k < events && (k == 0 || keys[k - 1] != key);
        const bool longrun = start && k + 31 < events && keys[k + 31] == key;
        if (start && !longrun) {
            float acc = next[key];
            uint64_t j = k;
            bool more = true;
            while (more) {
                uint32_t kk[4];
                float vv[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint64_t q = j + u;
                    kk[u] = q < events ? keys[q] : ~key;
                    vv[u] = q < events ? vals[q] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (more && kk[u] == key) acc = __fadd_rn(acc, vv[u]);
                    else more = false;
                }
                j += 4;
            }
            next[key] = acc;
        }
        uint32_t longs = __ballot_sync(kFull, longrun);
        while (longs) {
            const int src = __ffs(longs) - 1;
            longs &= longs - 1u;
            const uint32_t t = __shfl_sync(kFull, key, src);
            float acc = next[t];
            for (uint64_t j = c0 + (uint64_t)src;; j += 32u) {
                const uint64_t q = j + lane;
                const bool in = q < events && keys[q] == t;
                const float v = in ? vals[q] : 0.0f;
                const uint32_t m = __ballot_sync(kFull, in);  // a prefix: runs are contiguous
                const int len = __popc(m);
                for (int i = 0; i < len; ++i) acc = __fadd_rn(acc, __shfl_sync(kFull, v, i));
                if (len < 32) break;
            }
            if (lane == 0) next[t] = acc;
        }
    }
}

// ----------------------------------------------------------- ordered pull ----
// The pull reads a sliced-ELL (SELL-32) CSC: local targets in blocks of 32;
// block b holds width_b = max in-degree of its targets slots per target,
// slot k of target t at sell_off[b] + k*32 + (t % 32), each slot an 8-byte
// (presynaptic id, weight bits) pair, so a warp (one lane per target) loads
// 256 contiguous bytes per slot row: every load is coalesced and every lane
// folds its own target. Each target's in-edges keep CSR order
// (ascending presynaptic row, ascending edge), and the lane folds the spiking
// ones in that order from +0.0f, exactly the serial CPU fold
// (src/snn.c:898-906); padding slots hold an all-ones id and are skipped.
// (The chunked variant below stores chunk-relative ids; its padding id
// points at a shared-memory word that is always zero.)
// Cost ~ local synapses whatever the firing, so it is taken on dense steps:
// when pull_above != 0 the kernel runs only if the step's spike count
// exceeds it (the push kernel, launched with the same gate, runs otherwise).
constexpr int kPullUnroll = 4;

template <typename TIdx>
__global__ void __launch_bounds__(256) propagate_pull_kernel(uint64_t n_local, const uint64_t *__restrict__ sell_off,
                                                             const uint2 *__restrict__ slots,
                                                             const uint32_t *__restrict__ bitmap,
                                                             float *__restrict__ next, const TIdx *__restrict__ list,
                                                             const uint32_t *__restrict__ out_degree,
                                                             DevCounters *ctr, int parity, int count_spikes,
                                                             uint32_t pull_above, int events_gate,
                                                             unsigned long long events_above) {
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    if (pull_above && count <= pull_above) return;  // sparse step: the push kernel runs
    if (events_gate && *(volatile unsigned long long *)&ctr->step_events[parity] <= events_above) return;
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    const uint64_t blocks = (n_local + 31) / 32;
    for (uint64_t blk = gwarp; blk < blocks; blk += nwarps) {
        const uint64_t base = sell_off[blk];
        const uint64_t width = (sell_off[blk + 1] - base) / 32;
        const uint2 *sp = slots + base + lane;
        float acc = 0.0f;
        uint64_t k = 0;
        for (; k + kPullUnroll <= width; k += kPullUnroll) {
            uint2 q[kPullUnroll];
#pragma unroll
            for (int j = 0; j < kPullUnroll; ++j) q[j] = __ldcs(sp + (k + j) * 32u);
#pragma unroll
            for (int j = 0; j < kPullUnroll; ++j)
                if (q[j].x != 0xffffffffu && ((__ldg(bitmap + (q[j].x >> 5)) >> (q[j].x & 31u)) & 1u))
                    acc = __fadd_rn(acc, __uint_as_float(q[j].y));
        }
        for (; k < width; ++k) {
            const uint2 q = sp[k * 32u];
            if (q.x != 0xffffffffu && ((__ldg(bitmap + (q.x >> 5)) >> (q.x & 31u)) & 1u))
                acc = __fadd_rn(acc, __uint_as_float(q.y));
        }
        const uint64_t t = blk * 32u + lane;
        if (t < n_local) next[t] = acc;
    }
    // Event statistics: out-degree (towards this rank) of every spiking row.
    const uint64_t gthread = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    unsigned long long events = 0;
    for (uint64_t s = gthread; s < count; s += nthreads) events += out_degree[(uint64_t)list[s]];
    block_add_u64(events, &ctr->events);
    block_add_u64(events, &ctr->pull_events);
    if (blockIdx.x == 0 && threadIdx.x == 0) ctr->pull_runs += 1ull;
    step_epilogue(ctr, parity, count_spikes, count, 1);
}

// Chunked variant (the default when the layout was built chunked): the
// presynaptic ids are cut into chunks of kPullChunkWords bitmap words
// (1.8M neurons) and every (block, chunk) has its own slot run, so a CTA can
// stage one chunk of the bitmap in shared memory and serve every spike-bit
// lookup from there instead of from L1/L2 (one sector per lookup). A CTA
// takes sweeps of 32 warps x 4 blocks; each lane keeps its 4 targets' sums
// in registers across the chunks, which are visited in ascending order, so
// the fold order is still ascending presynaptic row, ascending edge.
constexpr uint32_t kPullChunkWords = 56320;  // 220 KB of shared memory (+1 zero word)
constexpr int kPullSmemThreads = 1024;
constexpr int kPullBlocksPerWarp = 4;
constexpr int kPullSmemUnroll = 8;  // slot loads in flight per lane

template <typename TIdx>
__global__ void __launch_bounds__(kPullSmemThreads, 1)
    propagate_pull_smem_kernel(uint64_t n_local, uint32_t chunks, uint64_t chunk_words,
                               const uint64_t *__restrict__ sell_off, const uint2 *__restrict__ slots,
                               const uint32_t *__restrict__ bitmap, uint64_t words, float *__restrict__ next,
                               const TIdx *__restrict__ list, const uint32_t *__restrict__ out_degree,
                               DevCounters *ctr, int parity, int count_spikes, uint32_t pull_above,
                               int events_gate, unsigned long long events_above) {
    extern __shared__ __align__(16) uint32_t s_bits[];  // chunk_words + 1 (the last word: zero, for padding)
    const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
    if (pull_above && count <= pull_above) return;  // sparse step: the push kernel runs
    if (events_gate && *(volatile unsigned long long *)&ctr->step_events[parity] <= events_above) return;
    const unsigned lane = lane_id();
    const unsigned warp = threadIdx.x >> 5;
    const uint64_t blocks = (n_local + 31) / 32;
    constexpr uint64_t kWarps = kPullSmemThreads / 32;
    constexpr uint64_t kSweep = kWarps * kPullBlocksPerWarp;
    // Each CTA owns an equal contiguous range of target blocks, visited in
    // sweeps of up to kSweep blocks; inside a sweep block j of warp w is
    // sweep_base + j * kWarps + w, so a short last sweep still spreads over
    // the warps.
    const uint64_t c_lo = blocks * blockIdx.x / gridDim.x, c_hi = blocks * (blockIdx.x + 1) / gridDim.x;
    for (uint64_t sb = c_lo; sb < c_hi; sb += kSweep) {
        float acc[kPullBlocksPerWarp];
#pragma unroll
        for (int j = 0; j < kPullBlocksPerWarp; ++j) acc[j] = 0.0f;
        for (uint32_t c = 0; c < chunks; ++c) {
            const uint64_t w0 = (uint64_t)c * chunk_words;
            const uint64_t cw = words - w0 < chunk_words ? words - w0 : chunk_words;
            __syncthreads();  // every warp is done with the previous chunk
            const uint32_t *src = bitmap + w0;
            if ((((uintptr_t)src) & 15u) == 0) {
                const uint64_t cw4 = cw / 4;
                for (uint64_t i = threadIdx.x; i < cw4; i += blockDim.x)
                    reinterpret_cast<uint4 *>(s_bits)[i] = __ldcg(reinterpret_cast<const uint4 *>(src) + i);
                for (uint64_t i = cw4 * 4 + threadIdx.x; i < cw; i += blockDim.x) s_bits[i] = __ldcg(src + i);
            } else {
                for (uint64_t i = threadIdx.x; i < cw; i += blockDim.x) s_bits[i] = __ldcg(src + i);
            }
            if (threadIdx.x == 0) s_bits[chunk_words] = 0u;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < kPullBlocksPerWarp; ++j) {
                const uint64_t b = sb + (uint64_t)j * kWarps + warp;
                if (b >= c_hi) break;
                const uint64_t base = sell_off[b * chunks + c];
                const uint64_t width = (sell_off[b * chunks + c + 1] - base) / 32;
                const uint2 *sp = slots + base + lane;
                float a = acc[j];
                uint64_t k = 0;
                // Software-pipelined: the next group's slots are in flight
                // while this group's bits are looked up and folded.
                uint2 q[kPullSmemUnroll];
                bool have = kPullSmemUnroll <= width;
                if (have) {
#pragma unroll
                    for (int u = 0; u < kPullSmemUnroll; ++u) q[u] = __ldcs(sp + (uint64_t)u * 32u);
                }
                while (have) {
                    const uint64_t kn = k + kPullSmemUnroll;
                    const bool more = kn + kPullSmemUnroll <= width;
                    uint2 qn[kPullSmemUnroll];
                    if (more) {
#pragma unroll
                        for (int u = 0; u < kPullSmemUnroll; ++u) qn[u] = __ldcs(sp + (kn + u) * 32u);
                    }
#pragma unroll
                    for (int u = 0; u < kPullSmemUnroll; ++u)
                        if ((s_bits[q[u].x >> 5] >> (q[u].x & 31u)) & 1u) a = __fadd_rn(a, __uint_as_float(q[u].y));
                    if (more) {
#pragma unroll
                        for (int u = 0; u < kPullSmemUnroll; ++u) q[u] = qn[u];
                    }
                    k = kn;
                    have = more;
                }
                for (; k < width; ++k) {
                    const uint2 q1 = sp[k * 32u];
                    if ((s_bits[q1.x >> 5] >> (q1.x & 31u)) & 1u) a = __fadd_rn(a, __uint_as_float(q1.y));
                }
                acc[j] = a;
            }
        }
#pragma unroll
        for (int j = 0; j < kPullBlocksPerWarp; ++j) {
            const uint64_t b = sb + (uint64_t)j * kWarps + warp;
            const uint64_t t = b * 32u + lane;
            if (b < c_hi && t < n_local) next[t] = acc[j];
        }
    }
    // Event statistics: out-degree (towards this rank) of every spiking row.
    const uint64_t gthread = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nthreads = (uint64_t)gridDim.x * blockDim.x;
    unsigned long long events = 0;
    for (uint64_t s = gthread; s < count; s += nthreads) events += out_degree[(uint64_t)list[s]];
    block_add_u64(events, &ctr->events);
    block_add_u64(events, &ctr->pull_events);
    if (blockIdx.x == 0 && threadIdx.x == 0) ctr->pull_runs += 1ull;
    step_epilogue(ctr, parity, count_spikes, count, 1);
}

// ----------------------------------------------------------- streaming ----
// One chunk of rows whose CSR slice was just copied in: warp per 32 rows,
// ballot over the rows' spike bits, then the warp strides each spiking row.
__global__ void __launch_bounds__(256) propagate_chunk_kernel(uint64_t row0, uint64_t rows, uint64_t edge_base,
                                                              const uint32_t *__restrict__ bitmap,
                                                              const uint64_t *__restrict__ row_ptr,
                                                              const uint64_t *__restrict__ col,
                                                              const float *__restrict__ w, float *__restrict__ next,
                                                              DevCounters *ctr, int parity, int first_chunk,
                                                              int count_spikes) {
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    unsigned long long events = 0;
    for (uint64_t base = gwarp * 32u; base < rows; base += nwarps * 32u) {
        const uint64_t r = base + lane;
        uint32_t bit = 0;
        if (r < rows) {
            const uint64_t g = row0 + r;
            bit = (bitmap[g >> 5] >> (g & 31u)) & 1u;
        }
        uint32_t m = __ballot_sync(kFull, bit);
        while (m) {
            const int j = __ffs(m) - 1;
            m &= m - 1u;
            const uint64_t lr = base + (uint64_t)j;
            const uint64_t b = row_ptr[lr] - edge_base;
            const uint64_t e = row_ptr[lr + 1] - edge_base;
            events += e - b;
            push_row<uint64_t>(b, e, col, w, next, lane);
        }
    }
    block_add_u64(lane == 0 ? events : 0ull, &ctr->events);
    if (first_chunk) {
        const uint32_t count = *(volatile uint32_t *)&ctr->list_count[parity];
        step_epilogue(ctr, parity, count_spikes, count);
    }
}

__global__ void step_epilogue_kernel(DevCounters *ctr, int parity, int count_spikes) {
    const uint32_t count = ctr->list_count[parity];
    step_epilogue(ctr, parity, count_spikes, count);
}

// ------------------------------------------------------------- inject ----
// Equal values: one value for every index (any order gives the same bits).
__global__ void inject_uniform_kernel(uint64_t count, const uint64_t *__restrict__ idx, float value, float scale,
                                      float *__restrict__ cur, uint64_t lo, uint64_t hi) {
    const float add = __fmul_rn(value, scale);
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const uint64_t i = idx[k];
        if (i >= lo && i < hi) red_add(cur + (i - lo), add);
    }
}

// The thread at the head of each run of equal (stably sorted) indices folds
// the run sequentially: c = (c + v0*s) + v1*s ... exactly as the CPU's
// in-order loop does (src/snn.c:737-739).
__global__ void inject_ordered_kernel(uint64_t count, const uint64_t *__restrict__ idx,
                                      const float *__restrict__ val, float scale, float *__restrict__ cur,
                                      uint64_t lo, uint64_t hi) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const uint64_t i = idx[k];
        if ((k != 0 && idx[k - 1] == i) || i < lo || i >= hi) continue;
        float c = cur[i - lo];
        for (uint64_t q = k; q < count && idx[q] == i; ++q) c = __fadd_rn(c, __fmul_rn(val[q], scale));
        cur[i - lo] = c;
    }
}

__global__ void inject_stream_kernel(uint64_t seed, uint64_t first_draw, uint64_t count, uint64_t n, float addend,
                                     float *__restrict__ cur, uint64_t lo, uint64_t hi,
                                     const unsigned long long *__restrict__ step_dev) {
    if (step_dev != nullptr) first_draw = (uint64_t)*step_dev * count;
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride) {
        const uint64_t i = draw_at(seed, first_draw + k + 1u) % n;
        if (i >= lo && i < hi) red_add(cur + (i - lo), addend);
    }
}

// ------------------------------------------------------------ topology ----
template <typename TCol>
__global__ void convert_cols_kernel(const uint64_t *__restrict__ src, TCol *__restrict__ dst, uint64_t count,
                                    uint64_t lo) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < count; k += stride)
        dst[k] = (TCol)(src[k] - lo);
}

__global__ void row_degrees_kernel(const uint64_t *__restrict__ row_ptr, uint64_t rows, uint32_t *__restrict__ deg) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += stride)
        deg[i] = (uint32_t)(row_ptr[i + 1] - row_ptr[i]);
}

// Target range of presynaptic row `pre`: random pool -> all n neurons;
// layered and feed-forward -> the next layer (the last layer has no edges).
// Also the row's edges: [first, first + edges), and for a sparse
// feed-forward layer the draw index of the row's first edge.
struct TargetRange {
    uint64_t base;
    uint64_t count;
    bool has_edges;
    uint64_t first;
    uint64_t edges;
    uint64_t draw0;  // feed-forward: ~0 for a dense layer
};

__device__ __forceinline__ uint64_t rows_with_edges(const GenParams &g) {
    return g.recurrent ? g.n : g.off[g.layers - 1];
}

__device__ __forceinline__ TargetRange target_range(const GenParams &g, uint64_t pre) {
    TargetRange t{0, g.n, true, 0, g.fanout, ~0ull};
    if (!g.recurrent) {
        int l = 0;
        while (l + 1 < g.layers && pre >= g.off[l + 1]) ++l;
        if (l + 1 >= g.layers) {
            t.has_edges = false;
            t.count = 0;
            t.edges = 0;
            t.first = g.feedforward ? g.ledge[g.layers - 1] : rows_with_edges(g) * g.fanout;
            return t;
        }
        t.base = g.off[l + 1];
        t.count = g.off[l + 2] - g.off[l + 1];
        if (g.feedforward) {
            t.edges = g.lfan[l];
            t.first = g.ledge[l] + (pre - g.off[l]) * t.edges;
            t.draw0 = g.ldraw[l] == ~0ull ? ~0ull : g.ldraw[l] + (pre - g.off[l]) * t.edges;
            return t;
        }
    }
    t.first = pre * g.fanout;
    return t;
}

__device__ __forceinline__ uint64_t total_edges(const GenParams &g) {
    return g.feedforward ? g.ledge[g.layers - 1] : rows_with_edges(g) * g.fanout;
}

// The presynaptic row that owns edge e.
__device__ __forceinline__ uint64_t edge_row(const GenParams &g, uint64_t e) {
    if (!g.feedforward) return e / g.fanout;
    int l = 0;
    while (l + 2 < g.layers && e >= g.ledge[l + 1]) ++l;
    return g.off[l] + (e - g.ledge[l]) / g.lfan[l];
}

// Edge e of row `pre` (t = target_range(g, pre)).
__device__ __forceinline__ uint64_t gen_target(const GenParams &g, uint64_t pre, uint64_t e, const TargetRange &t) {
    if (g.feedforward) {
        const uint64_t j = e - t.first;  // src/snn.c:507: j when dense, else the next draw % post
        return t.draw0 == ~0ull ? t.base + j : t.base + draw_at(g.seed, t.draw0 + j + 1u) % t.count;
    }
    uint64_t post = t.base + draw_at(g.seed, 2u * e + 1u) % t.count;
    if (g.recurrent && !g.allow_self && post == pre) post = (post + 1u) % g.n;  // src/snn.c:563-565
    return post;
}

__device__ __forceinline__ float gen_weight(const GenParams &g, uint64_t e) {
    if (g.feedforward) return g.wconst;
    return lerp_weight(g.wmin, g.wmax, unit_float(draw_at(g.seed, 2u * e + 2u)));
}

__global__ void gen_row_ptr_dense_kernel(GenParams g, uint64_t *__restrict__ row_ptr) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= g.n; i += stride)
        row_ptr[i] = i < g.n ? target_range(g, i).first : total_edges(g);
}

template <typename TCol>
__global__ void __launch_bounds__(256) gen_edges_dense_kernel(GenParams g, uint64_t e0, uint64_t e1,
                                                              TCol *__restrict__ col, float *__restrict__ w) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t e = e0 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < e1; e += stride) {
        const uint64_t pre = edge_row(g, e);
        const TargetRange t = target_range(g, pre);
        col[e] = (TCol)gen_target(g, pre, e, t);
        w[e] = gen_weight(g, e);
    }
}

// Warp per row: count the row's edges that target [lo, hi).
template <typename TCount>
__global__ void __launch_bounds__(256) gen_count_shard_kernel(GenParams g, uint64_t lo, uint64_t hi,
                                                              TCount *__restrict__ counts) {
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t pre = gwarp; pre < g.n; pre += nwarps) {
        const TargetRange t = target_range(g, pre);
        uint32_t c = 0;
        if (t.has_edges) {
            for (uint64_t j = lane; j < t.edges; j += 32u) {
                const uint64_t post = gen_target(g, pre, t.first + j, t);
                c += (post >= lo && post < hi);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) c += __shfl_xor_sync(kFull, c, d);
        if (lane == 0) counts[pre] = c;
    }
}

// Warp per row: write the kept edges in edge order (ballot compaction).
template <typename TCol>
__global__ void __launch_bounds__(256) gen_fill_shard_kernel(GenParams g, uint64_t lo, uint64_t hi,
                                                             const uint64_t *__restrict__ row_ptr,
                                                             TCol *__restrict__ col, float *__restrict__ w) {
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t pre = gwarp; pre < g.n; pre += nwarps) {
        const TargetRange t = target_range(g, pre);
        if (!t.has_edges) continue;
        uint64_t pos = row_ptr[pre];
        for (uint64_t j0 = 0; j0 < t.edges; j0 += 32u) {
            const uint64_t j = j0 + lane;
            bool keep = false;
            uint64_t post = 0;
            const uint64_t e = t.first + j;
            if (j < t.edges) {
                post = gen_target(g, pre, e, t);
                keep = post >= lo && post < hi;
            }
            const uint32_t m = __ballot_sync(kFull, keep);
            if (keep) {
                const uint64_t q = pos + __popc(m & ((1u << lane) - 1u));
                col[q] = (TCol)(post - lo);
                w[q] = gen_weight(g, e);
            }
            pos += __popc(m);
        }
    }
}

// --------------------------------------------------------- device CSC ----
// In-degree of the targets in [lo, hi): one relaxed atomic per kept edge.
__global__ void __launch_bounds__(256) gen_indegree_kernel(GenParams g, uint64_t lo, uint64_t hi,
                                                           unsigned long long *__restrict__ indeg) {
    const uint64_t total = total_edges(g);
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const uint64_t pre = edge_row(g, e);
        const uint64_t post = gen_target(g, pre, e, target_range(g, pre));
        if (post >= lo && post < hi) atomicAdd(indeg + (post - lo), 1ull);
    }
}

// Per local target and presynaptic chunk (pre / chunk_neurons): how many of
// the target's in-edges come from that chunk (chunked sliced-ELL layout).
__global__ void __launch_bounds__(256) gen_chunk_counts_kernel(GenParams g, uint64_t lo, uint64_t hi, uint32_t chunks,
                                                               uint64_t chunk_neurons, uint32_t *__restrict__ cnt) {
    const uint64_t total = total_edges(g);
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const uint64_t pre = edge_row(g, e);
        const uint64_t post = gen_target(g, pre, e, target_range(g, pre));
        if (post >= lo && post < hi) atomicAdd(cnt + (post - lo) * chunks + pre / chunk_neurons, 1u);
    }
}

// slots[b * chunks + c] = 32 x the largest count of block b's targets in chunk c.
__global__ void sell_slots_kernel(const uint32_t *__restrict__ cnt, uint64_t n_local, uint32_t chunks,
                                  uint64_t *__restrict__ slots) {
    const uint64_t blocks = (n_local + 31) / 32;
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < blocks * chunks; i += stride) {
        const uint64_t b = i / chunks, c = i % chunks;
        uint32_t m = 0;
        for (uint64_t t = b * 32; t < b * 32 + 32 && t < n_local; ++t) m = max(m, cnt[t * chunks + c]);
        slots[i] = 32ull * m;
    }
}

// Warp per row: (post - lo, global edge id) of the row's edges into
// [lo, hi), in edge order, at row_off[pre] (ballot compaction).
__global__ void __launch_bounds__(256) gen_fill_keys_kernel(GenParams g, uint64_t lo, uint64_t hi,
                                                            const uint64_t *__restrict__ row_off,
                                                            uint32_t *__restrict__ keys,
                                                            uint64_t *__restrict__ eids) {
    const unsigned lane = lane_id();
    const uint64_t gwarp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t pre = gwarp; pre < g.n; pre += nwarps) {
        const TargetRange t = target_range(g, pre);
        if (!t.has_edges) continue;
        uint64_t pos = row_off[pre];
        for (uint64_t j0 = 0; j0 < t.edges; j0 += 32u) {
            const uint64_t j = j0 + lane;
            const uint64_t e = t.first + j;
            uint64_t post = 0;
            bool keep = false;
            if (j < t.edges) {
                post = gen_target(g, pre, e, t);
                keep = post >= lo && post < hi;
            }
            const uint32_t m = __ballot_sync(kFull, keep);
            if (keep) {
                const uint64_t q = pos + __popc(m & ((1u << lane) - 1u));
                keys[q] = (uint32_t)(post - lo);
                eids[q] = e;
            }
            pos += __popc(m);
        }
    }
}

// Sorted pass position q holds the pass-local target keys[q] and the global
// edge id eids[q]; its rank in the target's CSR-ordered in-edge list is
// k = q0 + q - col_ptr[t]. In the chunked sliced-ELL layout it goes to the
// slots of (block t / 32, chunk c = pre / chunk_neurons) at rank k minus the
// target's in-edges from earlier chunks.
__global__ void gather_generated_sell_kernel(GenParams g, const uint32_t *__restrict__ keys,
                                             const uint64_t *__restrict__ eids, uint64_t e, uint64_t t0, uint64_t q0,
                                             const uint64_t *__restrict__ col_ptr, const uint32_t *__restrict__ cnt,
                                             uint32_t chunks, uint64_t chunk_neurons, int relative,
                                             const uint64_t *__restrict__ sell_off, uint2 *__restrict__ slots) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < e; q += stride) {
        const uint64_t ed = eids[q];
        const uint64_t t = t0 + keys[q];
        const uint64_t p = edge_row(g, ed);
        const uint32_t c = (uint32_t)(p / chunk_neurons);
        uint64_t k = q0 + q - col_ptr[t];
        for (uint32_t c2 = 0; c2 < c; ++c2) k -= cnt[t * chunks + c2];
        const uint64_t dst = sell_off[(t >> 5) * chunks + c] + k * 32u + (t & 31u);
        const uint32_t id = (uint32_t)(relative ? p - (uint64_t)c * chunk_neurons : p);
        slots[dst] = make_uint2(id, __float_as_uint(gen_weight(g, ed)));
    }
}

struct WidenU32 {
    __host__ __device__ unsigned long long operator()(uint32_t x) const { return x; }
};

int grid_for(int device, int blocks_per_sm, uint64_t work, uint64_t per_block) {
    const uint64_t need = (work + per_block - 1) / per_block;
    const uint64_t cap = (uint64_t)sm_count(device) * (uint64_t)blocks_per_sm;
    uint64_t g = need < cap ? need : cap;
    return g == 0 ? 1 : (int)g;
}

}  // namespace

int sm_count(int device) {
    static std::mutex mu;
    static std::vector<int> cache;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0) device = 0;
    if ((int)cache.size() <= device) cache.resize(device + 1, 0);
    if (cache[device] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0) v = 148;
        cache[device] = v;
    }
    return cache[device];
}

void launch_init_state(cudaStream_t s, uint64_t n, float v_rest, float *v, float *cur0, float *cur1, float *ext,
                       uint32_t *refr, uint8_t *spikes, uint64_t words, uint32_t *bitmap, DevCounters *ctr,
                       uint8_t *kind_log) {
    const uint64_t work = n > words ? n : words;
    uint64_t blocks = (work + 255) / 256;
    if (blocks > 65535) blocks = 65535;
    if (blocks == 0) blocks = 1;
    init_state_kernel<<<(unsigned)blocks, 256, 0, s>>>(n, v_rest, v, cur0, cur1, ext, refr, spikes, words, bitmap, ctr,
                                                       kind_log);
}

template <bool EXT, typename TIdx, int ITERS>
static void lif_dispatch(cudaStream_t s, int device, uint64_t n, const LifArgs &p, float *v, float *cur,
                         const float *ext, uint32_t *refr, uint8_t *spikes, uint32_t *bitmap, void *list,
                         uint64_t off, DevCounters *ctr, int parity) {
    constexpr uint64_t tile = (uint64_t)ITERS * kLifThreads * 4u;
    const int grid = grid_for(device, 6, n, tile);
    if (list != nullptr)
        lif_kernel<EXT, true, TIdx, ITERS><<<grid, kLifThreads, 0, s>>>(n, p, v, cur, ext, refr, spikes, bitmap,
                                                                        (TIdx *)list, off, ctr, parity);
    else
        lif_kernel<EXT, false, TIdx, ITERS><<<grid, kLifThreads, 0, s>>>(n, p, v, cur, ext, refr, spikes, bitmap,
                                                                         (TIdx *)list, off, ctr, parity);
}

void launch_lif(cudaStream_t s, int device, uint64_t n, const LifArgs &p, float *v, float *cur, const float *ext,
                uint32_t *refr, uint8_t *spikes, uint32_t *bitmap, void *list, int idx_bits, uint64_t off,
                DevCounters *ctr, int parity) {
    if (n == 0) return;
    // Small populations: 1024-neuron tiles, so the grid still covers the SMs.
    const bool small = n < (uint64_t)sm_count(device) * 2u * kLifThreads * 4u * 8u;
    if (idx_bits == 32 && small) {
        if (ext) lif_dispatch<true, uint32_t, 1>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
        else lif_dispatch<false, uint32_t, 1>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
    } else if (idx_bits == 32) {
        if (ext) lif_dispatch<true, uint32_t, 8>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
        else lif_dispatch<false, uint32_t, 8>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
    } else {
        if (ext) lif_dispatch<true, uint64_t, 4>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
        else lif_dispatch<false, uint64_t, 4>(s, device, n, p, v, cur, ext, refr, spikes, bitmap, list, off, ctr, parity);
    }
}

void launch_compact(cudaStream_t s, int device, uint32_t *bitmap, uint64_t words, void *list, int idx_bits,
                    DevCounters *ctr, int parity, uint64_t own_begin, uint64_t own_end, const PeerWait *wait) {
    PeerWait pw{};
    if (wait) pw = *wait;
    const int grid = grid_for(device, 8, words / 4, 256);
    if (idx_bits == 32)
        compact_kernel<uint32_t><<<grid, 256, 0, s>>>(bitmap, words, (uint32_t *)list, ctr, parity, own_begin, own_end, pw);
    else
        compact_kernel<uint64_t><<<grid, 256, 0, s>>>(bitmap, words, (uint64_t *)list, ctr, parity, own_begin, own_end, pw);
}

template <typename TIdx, typename TCol, int LANES>
static int push_grid(int device) {
    static int blocks_per_sm = 0;
    if (blocks_per_sm == 0) {
        int v = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, propagate_push_kernel<TIdx, TCol, LANES>, 256, 0) !=
                cudaSuccess ||
            v <= 0)
            v = 4;
        blocks_per_sm = v;
    }
    return sm_count(device) * blocks_per_sm;
}

template <typename TI, typename TC>
static void push_dispatch(cudaStream_t s, int device, const void *list, const uint64_t *row_ptr, const void *col,
                          const float *w, float *next, DevCounters *ctr, int parity, int count_spikes,
                          uint64_t batch_rows, uint32_t pull_above, uint32_t lanes) {
#define B200_PUSH(L)                                                                                            \
    propagate_push_kernel<TI, TC, L><<<push_grid<TI, TC, L>(device), 256, 0, s>>>(                              \
        (const TI *)list, row_ptr, (const TC *)col, w, next, ctr, parity, count_spikes, batch_rows, pull_above)
    if (lanes <= 8) B200_PUSH(8);
    else if (lanes <= 16) B200_PUSH(16);
    else B200_PUSH(32);
#undef B200_PUSH
}

void launch_propagate_push(cudaStream_t s, int device, const void *list, int idx_bits, const uint64_t *row_ptr,
                           const void *col, int col_bits, const float *w, float *next, DevCounters *ctr, int parity,
                           int count_spikes, uint64_t batch_rows, uint32_t pull_above, uint32_t lanes) {
    if (idx_bits == 32 && col_bits == 32)
        push_dispatch<uint32_t, uint32_t>(s, device, list, row_ptr, col, w, next, ctr, parity, count_spikes,
                                          batch_rows, pull_above, lanes);
    else if (idx_bits == 32)
        push_dispatch<uint32_t, uint64_t>(s, device, list, row_ptr, col, w, next, ctr, parity, count_spikes,
                                          batch_rows, pull_above, lanes);
    else if (col_bits == 32)
        push_dispatch<uint64_t, uint32_t>(s, device, list, row_ptr, col, w, next, ctr, parity, count_spikes,
                                          batch_rows, pull_above, lanes);
    else
        push_dispatch<uint64_t, uint64_t>(s, device, list, row_ptr, col, w, next, ctr, parity, count_spikes,
                                          batch_rows, pull_above, lanes);
}

uint32_t push_lanes(uint64_t synapses, uint64_t rows) {
    // About two 16-byte vectors per lane per row: rows of up to ~256 edges
    // share a warp between several rows.
    const uint64_t avg = rows ? synapses / rows : 0;
    return avg >= 512 ? 32u : avg >= 160 ? 16u : 8u;
}

// SNN_B200_PULL_CHUNK_WORDS (environment, read when a layout is built)
// shrinks the chunks, so tests reach several chunks with small networks.
uint64_t pull_chunk_words() {
    const char *env = std::getenv("SNN_B200_PULL_CHUNK_WORDS");
    const uint64_t v = env ? std::strtoull(env, nullptr, 10) : 0;
    return v ? std::min<uint64_t>(v, kPullChunkWords) : (uint64_t)kPullChunkWords;
}

uint32_t pull_chunks(uint64_t words) { return (uint32_t)((words + pull_chunk_words() - 1) / pull_chunk_words()); }

uint64_t pull_chunk_neurons() { return pull_chunk_words() * 32u; }

void launch_propagate_pull(cudaStream_t s, int device, uint64_t n_local, uint32_t chunks, uint64_t chunk_words,
                           const uint64_t *sell_off, const uint2 *slots, const uint32_t *bitmap, uint64_t words,
                           float *next, const void *list, int idx_bits, const uint32_t *out_degree, DevCounters *ctr,
                           int parity, int count_spikes, uint32_t pull_above, int events_gate,
                           unsigned long long events_above) {
    if ((uint64_t)chunks * chunk_words >= words) {
        // Chunked layout: shared-memory spike bits.
        const uint64_t blocks = (n_local + 31) / 32;
        const uint64_t sweeps = (blocks + (kPullSmemThreads / 32) * kPullBlocksPerWarp - 1) /
                                ((kPullSmemThreads / 32) * kPullBlocksPerWarp);
        // One CTA per SM (a chunk of spike bits fills its shared memory);
        // fewer when there are fewer sweeps than SMs.
        const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>(sweeps, (uint64_t)sm_count(device)));
        const size_t smem = (size_t)(chunk_words + 1) * 4;
#define B200_PULLS(TI)                                                                                          \
    do {                                                                                                        \
        static bool attr[64] = {};                                                                              \
        if (device >= 0 && device < 64 && !attr[device]) {                                                      \
            cudaFuncSetAttribute(propagate_pull_smem_kernel<TI>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                 (int)((kPullChunkWords + 1) * 4));                                             \
            attr[device] = true;                                                                                \
        }                                                                                                       \
        propagate_pull_smem_kernel<TI><<<grid, kPullSmemThreads, smem, s>>>(                                    \
            n_local, chunks, chunk_words, sell_off, slots, bitmap, words, next, (const TI *)list, out_degree,   \
            ctr, parity, count_spikes, pull_above, events_gate, events_above);                                  \
    } while (0)
        if (idx_bits == 32) B200_PULLS(uint32_t);
        else B200_PULLS(uint64_t);
#undef B200_PULLS
        return;
    }
    // One chunk over a bitmap larger than shared memory: lookups through L1/L2.
    const int grid = sm_count(device) * 8;
    if (idx_bits == 32)
        propagate_pull_kernel<uint32_t><<<grid, 256, 0, s>>>(n_local, sell_off, slots, bitmap, next,
                                                             (const uint32_t *)list, out_degree, ctr, parity,
                                                             count_spikes, pull_above, events_gate, events_above);
    else
        propagate_pull_kernel<uint64_t><<<grid, 256, 0, s>>>(n_local, sell_off, slots, bitmap, next,
                                                             (const uint64_t *)list, out_degree, ctr, parity,
                                                             count_spikes, pull_above, events_gate, events_above);
}

__global__ void gather_u64_kernel(const unsigned long long *src, const uint64_t *idx, uint64_t count,
                                  unsigned long long *dst) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) dst[i] = src[idx[i]];
}

void launch_publish_flags(cudaStream_t s, const PeerWait &pw) { publish_flags_kernel<<<1, 32, 0, s>>>(pw); }

void launch_gather_u64(cudaStream_t s, const unsigned long long *src, const uint64_t *idx, uint64_t count,
                       unsigned long long *dst) {
    if (count) gather_u64_kernel<<<(unsigned)((count + 255) / 256), 256, 0, s>>>(src, idx, count, dst);
}

__global__ void set_u64_kernel(unsigned long long *p, unsigned long long v) { *p = v; }

void launch_set_u64(cudaStream_t s, unsigned long long *p, unsigned long long v) { set_u64_kernel<<<1, 1, 0, s>>>(p, v); }

__global__ void fill_u2_kernel(uint2 *__restrict__ p, uint64_t n, uint2 v) {
    const uint64_t stride = (uint64_t)blockDim.x * gridDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) p[i] = v;
}

void launch_fill_u2(cudaStream_t s, int device, uint2 *p, uint64_t n, uint32_t x, uint32_t y) {
    fill_u2_kernel<<<grid_for(device, 8, n, 256), 256, 0, s>>>(p, n, make_uint2(x, y));
}

void launch_propagate_chunk(cudaStream_t s, int device, uint64_t row0, uint64_t rows, uint64_t edge_base,
                            const uint32_t *bitmap, const uint64_t *row_ptr, const uint64_t *col, const float *w,
                            float *next, DevCounters *ctr, int parity, int first_chunk, int count_spikes) {
    const int grid = grid_for(device, 8, rows, 256);
    propagate_chunk_kernel<<<grid, 256, 0, s>>>(row0, rows, edge_base, bitmap, row_ptr, col, w, next, ctr, parity,
                                                first_chunk, count_spikes);
}

void launch_step_epilogue(cudaStream_t s, DevCounters *ctr, int parity, int count_spikes) {
    step_epilogue_kernel<<<1, 32, 0, s>>>(ctr, parity, count_spikes);
}

void launch_inject_uniform(cudaStream_t s, int device, uint64_t count, const uint64_t *idx, float value,
                           float scale, float *cur, uint64_t lo, uint64_t hi) {
    inject_uniform_kernel<<<grid_for(device, 8, count, 256), 256, 0, s>>>(count, idx, value, scale, cur, lo, hi);
}

void launch_inject_ordered(cudaStream_t s, int device, uint64_t count, const uint64_t *idx, const float *val,
                           float scale, float *cur, uint64_t lo, uint64_t hi) {
    inject_ordered_kernel<<<grid_for(device, 8, count, 256), 256, 0, s>>>(count, idx, val, scale, cur, lo, hi);
}

void launch_inject_stream(cudaStream_t s, int device, uint64_t seed, uint64_t step, uint64_t count, uint64_t n,
                          float addend, float *cur, uint64_t lo, uint64_t hi, const unsigned long long *step_dev) {
    inject_stream_kernel<<<grid_for(device, 8, count, 256), 256, 0, s>>>(seed, step * count, count, n, addend, cur,
                                                                        lo, hi, step_dev);
}

void launch_convert_cols(cudaStream_t s, int device, const uint64_t *src, void *dst, int col_bits, uint64_t count,
                         uint64_t lo) {
    const int grid = grid_for(device, 8, count, 256);
    if (col_bits == 32) convert_cols_kernel<uint32_t><<<grid, 256, 0, s>>>(src, (uint32_t *)dst, count, lo);
    else convert_cols_kernel<uint64_t><<<grid, 256, 0, s>>>(src, (uint64_t *)dst, count, lo);
}

void launch_gen_row_ptr_dense(cudaStream_t s, int device, const GenParams &g, uint64_t *row_ptr) {
    gen_row_ptr_dense_kernel<<<grid_for(device, 8, g.n + 1, 256), 256, 0, s>>>(g, row_ptr);
}

void launch_gen_edges_dense(cudaStream_t s, int device, const GenParams &g, uint64_t e0, uint64_t e1, void *col,
                            int col_bits, float *w) {
    if (e1 <= e0) return;
    const int grid = grid_for(device, 8, e1 - e0, 256);
    if (col_bits == 32) gen_edges_dense_kernel<uint32_t><<<grid, 256, 0, s>>>(g, e0, e1, (uint32_t *)col, w);
    else gen_edges_dense_kernel<uint64_t><<<grid, 256, 0, s>>>(g, e0, e1, (uint64_t *)col, w);
}

void launch_gen_count_shard(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                            uint64_t *counts) {
    gen_count_shard_kernel<uint64_t><<<grid_for(device, 8, g.n * 32u, 256), 256, 0, s>>>(g, lo, hi, counts);
}

void launch_gen_fill_shard(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                           const uint64_t *row_ptr, void *col, int col_bits, float *w) {
    const int grid = grid_for(device, 8, g.n * 32u, 256);
    if (col_bits == 32)
        gen_fill_shard_kernel<uint32_t><<<grid, 256, 0, s>>>(g, lo, hi, row_ptr, (uint32_t *)col, w);
    else
        gen_fill_shard_kernel<uint64_t><<<grid, 256, 0, s>>>(g, lo, hi, row_ptr, (uint64_t *)col, w);
}

cudaError_t exclusive_scan_u64(cudaStream_t s, const uint64_t *in, uint64_t *out, uint64_t n, void *temp,
                               size_t *temp_bytes) {
    return cub::DeviceScan::ExclusiveSum(temp, *temp_bytes, in, out, (int64_t)n, s);
}

void launch_gen_indegree(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                         unsigned long long *indeg) {
    gen_indegree_kernel<<<grid_for(device, 8, g.n * g.fanout, 256), 256, 0, s>>>(g, lo, hi, indeg);
}

void launch_gen_count_shard_u32(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                                uint32_t *counts) {
    gen_count_shard_kernel<uint32_t><<<grid_for(device, 8, g.n * 32u, 256), 256, 0, s>>>(g, lo, hi, counts);
}

void launch_gen_fill_keys(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                          const uint64_t *row_off, uint32_t *keys, uint64_t *eids) {
    gen_fill_keys_kernel<<<grid_for(device, 8, g.n * 32u, 256), 256, 0, s>>>(g, lo, hi, row_off, keys, eids);
}

cudaError_t sort_pairs_u32_u64(cudaStream_t s, uint32_t *keys, uint32_t *keys_alt, uint64_t *vals,
                               uint64_t *vals_alt, uint64_t n, int end_bit, void *temp, size_t *temp_bytes,
                               bool *result_in_alt) {
    cub::DoubleBuffer<uint32_t> k(keys, keys_alt);
    cub::DoubleBuffer<uint64_t> v(vals, vals_alt);
    const cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, *temp_bytes, k, v, (int64_t)n, 0, end_bit, s);
    if (temp != nullptr) *result_in_alt = k.Current() != keys;
    return e;
}

void launch_gather_generated_sell(cudaStream_t s, int device, const GenParams &g, const uint32_t *keys,
                                  const uint64_t *eids, uint64_t e, uint64_t t0, uint64_t q0, const uint64_t *col_ptr,
                                  const uint32_t *cnt, uint32_t chunks, uint64_t chunk_neurons, int relative,
                                  const uint64_t *sell_off, uint2 *slots) {
    gather_generated_sell_kernel<<<grid_for(device, 8, e, 256), 256, 0, s>>>(g, keys, eids, e, t0, q0, col_ptr, cnt,
                                                                              chunks, chunk_neurons, relative,
                                                                              sell_off, slots);
}

void launch_gen_chunk_counts(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                             uint32_t chunks, uint64_t chunk_neurons, uint32_t *cnt) {
    gen_chunk_counts_kernel<<<grid_for(device, 8, g.n * g.fanout, 256), 256, 0, s>>>(g, lo, hi, chunks,
                                                                                      chunk_neurons, cnt);
}

void launch_sell_slots(cudaStream_t s, int device, const uint32_t *cnt, uint64_t n_local, uint32_t chunks,
                       uint64_t *slots) {
    const uint64_t items = (n_local + 31) / 32 * chunks;
    sell_slots_kernel<<<grid_for(device, 8, items, 256), 256, 0, s>>>(cnt, n_local, chunks, slots);
}

void launch_ordered_sdeg(cudaStream_t s, int device, const void *list, int idx_bits, DevCounters *ctr, int parity,
                         uint64_t max_rows, const uint64_t *row_ptr, uint32_t *sdeg, int clear,
                         uint64_t batch_rows) {
    const int grid = grid_for(device, 4, max_rows, 256);
    if (idx_bits == 32)
        ordered_sdeg_kernel<uint32_t><<<grid, 256, 0, s>>>((const uint32_t *)list, ctr, parity, row_ptr, sdeg, clear,
                                                           batch_rows);
    else
        ordered_sdeg_kernel<uint64_t><<<grid, 256, 0, s>>>((const uint64_t *)list, ctr, parity, row_ptr, sdeg, clear,
                                                           batch_rows);
}

void launch_ordered_gen(cudaStream_t s, int device, const void *list, int idx_bits, DevCounters *ctr, int parity,
                        uint64_t row_lo, uint64_t row_hi, const uint64_t *row_ptr, const void *col, int col_bits,
                        const float *w, const unsigned long long *eoff, uint64_t rows, uint64_t id_base,
                        uint32_t *sdeg, uint32_t *keys, float *vals, int epilogue, int count_spikes,
                        uint64_t batch_rows) {
    const int grid = sm_count(device) * 8;
#define B200_OG(TI, TC)                                                                                        \
    ordered_gen_kernel<TI, TC><<<grid, 256, 0, s>>>((const TI *)list, ctr, parity, row_lo, row_hi, row_ptr,     \
                                                    (const TC *)col, w, eoff, rows, id_base, sdeg, keys, vals,  \
                                                    epilogue, count_spikes, batch_rows)
    if (idx_bits == 32 && col_bits == 32) B200_OG(uint32_t, uint32_t);
    else if (idx_bits == 32) B200_OG(uint32_t, uint64_t);
    else if (col_bits == 32) B200_OG(uint64_t, uint32_t);
    else B200_OG(uint64_t, uint64_t);
#undef B200_OG
}

cudaError_t sort_pairs_u32_f32(cudaStream_t s, uint32_t *keys, uint32_t *keys_alt, float *vals, float *vals_alt,
                               uint64_t n, int begin_bit, int end_bit, void *temp, size_t *temp_bytes,
                               bool *result_in_alt) {
    cub::DoubleBuffer<uint32_t> k(keys, keys_alt);
    cub::DoubleBuffer<float> v(vals, vals_alt);
    const cudaError_t e =
        cub::DeviceRadixSort::SortPairs(temp, *temp_bytes, k, v, (int64_t)n, begin_bit, end_bit, s);
    if (temp != nullptr) *result_in_alt = k.Current() != keys;
    return e;
}

cudaError_t sort_pairs_u64_f32(cudaStream_t s, uint64_t *keys, uint64_t *keys_alt, float *vals, float *vals_alt,
                               uint64_t n, int end_bit, void *temp, size_t *temp_bytes, bool *result_in_alt) {
    cub::DoubleBuffer<uint64_t> k(keys, keys_alt);
    cub::DoubleBuffer<float> v(vals, vals_alt);
    const cudaError_t e = cub::DeviceRadixSort::SortPairs(temp, *temp_bytes, k, v, (int64_t)n, 0, end_bit, s);
    if (temp != nullptr) *result_in_alt = k.Current() != keys;
    return e;
}

void launch_ordered_fold(cudaStream_t s, int device, uint64_t events, const uint32_t *keys, const float *vals,
                         float *next) {
    ordered_fold_kernel<<<grid_for(device, 8, events, 256), 256, 0, s>>>(events, keys, vals, next);
}

void launch_ordered_group_fold(cudaStream_t s, int device, uint64_t events, const uint32_t *keys, const float *vals,
                               float *next, uint64_t n_targets) {
    const uint64_t groups = (n_targets + (1ull << kFoldGroupBits) - 1) >> kFoldGroupBits;
    ordered_group_fold_kernel<kFoldGroupBits><<<grid_for(device, 8, groups * 32u, 256), 256, 0, s>>>(
        events, keys, vals, next, n_targets);
}

cudaError_t scan_degrees_u64(cudaStream_t s, const uint32_t *in, unsigned long long *out, uint64_t n, void *temp,
                             size_t *temp_bytes) {
    // u32 degrees summed in 64 bits.
    thrust::transform_iterator<WidenU32, const uint32_t *, unsigned long long> it(in, WidenU32());
    return cub::DeviceScan::ExclusiveSum(temp, *temp_bytes, it, out, (int64_t)n, s);
}

void launch_row_degrees(cudaStream_t s, int device, const uint64_t *row_ptr, uint64_t rows, uint32_t *deg) {
    row_degrees_kernel<<<grid_for(device, 8, rows, 256), 256, 0, s>>>(row_ptr, rows, deg);
}

}  // namespace b200
