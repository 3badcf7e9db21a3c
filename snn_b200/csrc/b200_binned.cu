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

constexpr int kThreads = 512;
constexpr uint32_t kStage = 24;  // staged entries per destination tile

__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
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

// ---------------------------------------------------------------------------
// Warp roles (16 warps, one CTA per SM):
//   warp 0        router producer: streams spiking-row segments with TMA bulk
//                 copies (cp.async.bulk) into the router ring;
//   warps 1-7     router consumers: route the ring's edges into staging (a
//                 warp per row piece of <= 256 edges) and flush staging into
//                 this CTA's sub-bins;
//   warp 8        drain producer: streams this CTA's sub-bins of a finished
//                 round into the drain ring (cp.async.bulk);
//   warps 9-15    drain consumers: fold drain-ring entries into the tile.
// Sub-bins are padded to an even length with (0, +0.0f) entries, so the drain
// ring holds whole 16-byte entry pairs with no gaps.
// Rings are flow-controlled by mbarriers (full: TMA bytes landed; empty:
// consumers done), so no warp waits on memory latency.
constexpr int kRConsWarps = 7;  // warps 1..7
constexpr int kDConsWarps = 7;  // warps 9..15
constexpr int kRConsThreads = 32 * kRConsWarps;
constexpr int kDConsThreads = 32 * kDConsWarps;
constexpr int kDProdWarp = 1 + kRConsWarps;
constexpr uint32_t kPieceEdges = 256;  // longest row piece (one consumer warp routes a piece)
constexpr uint32_t kRSlots = 2;
constexpr uint32_t kRSlotEdges = 1536;                         // edges per router slot (one staging flush)
constexpr uint32_t kRMaxPieces = 32;                           // row segments per router slot
constexpr uint32_t kRSlotCap = kRSlotEdges + 8 * kRMaxPieces;  // + alignment slack of the copies
constexpr uint32_t kDSlots = 2;
constexpr uint32_t kDSlotEntries = 1536;  // sub-bin entries per drain slot
constexpr uint32_t kDMaxPieces = 64;      // sub-bins per drain slot
constexpr uint32_t kDSlotCap = kDSlotEntries + 2 * kDMaxPieces;
constexpr uint32_t kRoundEnd = 1u;

template <uint32_t MAXP>
struct SlotHdr {
    uint32_t npieces;
    uint32_t total;  // valid elements in the slot
    uint32_t flags;  // kRoundEnd: last slot of a round
    uint32_t pad;
    uint32_t start[MAXP];       // data index of each piece's first valid element
    uint32_t prefix[MAXP + 1];  // valid elements before each piece
};

struct Smem {
    float *tile;       // [tile]          the pass's targets owned by this CTA
    uint2 *stage;      // [grid][kStage]  staged events per destination
    uint32_t *scount;  // [grid]          staged entries per destination
    uint32_t *wcount;  // [grid]          entries written this round into my sub-bin of each destination
    uint32_t *sbase;   // [grid]          flush base per destination
    uint32_t *dcount;  // [grid]          drain producer: entries in each source's sub-bin
    uint32_t *rcol;    // [kRSlots][kRSlotCap]
    float *rw;         // [kRSlots][kRSlotCap]
    uint2 *dbuf;       // [kDSlots][kDSlotCap]
    SlotHdr<kRMaxPieces> *rhdr;  // [kRSlots]
    SlotHdr<kDMaxPieces> *dhdr;  // [kDSlots]
    uint64_t *bar;               // rfull[2], rempty[2], dfull[2], dempty[2]
};

__host__ __device__ constexpr size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

__host__ __device__ inline size_t smem_fixed_bytes(uint32_t grid) {
    return align16((size_t)grid * kStage * 8) + 4 * align16((size_t)grid * 4) +
           2 * align16((size_t)kRSlots * kRSlotCap * 4) + align16((size_t)kDSlots * kDSlotCap * 8) +
           align16(kRSlots * sizeof(SlotHdr<kRMaxPieces>)) + align16(kDSlots * sizeof(SlotHdr<kDMaxPieces>)) + 8 * 8;
}

__device__ __forceinline__ Smem smem_layout(const BinLayout &L) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem s;
    size_t o = 0;
    s.tile = reinterpret_cast<float *>(smem_raw + o);
    o += align16((size_t)L.tile * 4u);
    s.stage = reinterpret_cast<uint2 *>(smem_raw + o);
    o += align16((size_t)L.grid * kStage * 8u);
    s.scount = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += align16((size_t)L.grid * 4u);
    s.wcount = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += align16((size_t)L.grid * 4u);
    s.sbase = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += align16((size_t)L.grid * 4u);
    s.dcount = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += align16((size_t)L.grid * 4u);
    s.rcol = reinterpret_cast<uint32_t *>(smem_raw + o);
    o += align16((size_t)kRSlots * kRSlotCap * 4);
    s.rw = reinterpret_cast<float *>(smem_raw + o);
    o += align16((size_t)kRSlots * kRSlotCap * 4);
    s.dbuf = reinterpret_cast<uint2 *>(smem_raw + o);
    o += align16((size_t)kDSlots * kDSlotCap * 8);
    s.rhdr = reinterpret_cast<SlotHdr<kRMaxPieces> *>(smem_raw + o);
    o += align16(kRSlots * sizeof(SlotHdr<kRMaxPieces>));
    s.dhdr = reinterpret_cast<SlotHdr<kDMaxPieces> *>(smem_raw + o);
    o += align16(kDSlots * sizeof(SlotHdr<kDMaxPieces>));
    s.bar = reinterpret_cast<uint64_t *>(smem_raw + o);
    return s;
}

// ------------------------------------------------------------ mbarrier ----
__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(saddr(b))
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0u;
}
// Bounded wait for the phase with `parity` to complete; raises the error
// word on expiry and gives up at once if another CTA raised it.
__device__ bool mbar_wait(uint64_t *b, uint32_t parity, uint32_t limit, uint32_t *err) {
    for (uint32_t it = 0; !mbar_try_wait(b, parity); ++it) {
        if (*(volatile uint32_t *)err != 0u) return false;
        if (it >= limit) {
            atomicExch(err, 2u);
            return false;
        }
    }
    return true;
}
// 1-D TMA bulk copy global -> this CTA's shared memory (no multicast),
// completing `bytes` on the mbarrier. Addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(saddr(dst)),
        "l"(src), "r"(bytes), "r"(saddr(bar))
        : "memory");
}

// Optional per-CTA cycle accounting (BinLayout::prof), for diagnosing where
// a round's time goes. Slots: 0 rprod wait-empty, 1 rprod total, 2 rcons
// wait-drained, 3 rcons wait-full, 4 rcons route, 5 rcons flush, 6 dprod
// wait-routed, 7 dprod issue, 8 dcons wait-full, 9 dcons fold, 10 kernel.
__device__ __forceinline__ void prof_add(const BinLayout &L, int slot, long long dt) {
    if (L.prof) atomicAdd(L.prof + blockIdx.x * 16 + slot, (unsigned long long)dt);
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
    uint64_t *rfull = S.bar, *rempty = S.bar + 2, *dfull = S.bar + 4, *dempty = S.bar + 6;
    uint32_t *err = &ctr->error;
    const uint32_t lim = L.spin_limit;

    if (threadIdx.x == 0) {
        s_abort = 0u;
        for (int i = 0; i < 2; ++i) {
            mbar_init(rfull + i, 1);
            mbar_init(rempty + i, 1);
            mbar_init(dfull + i, 1);
            mbar_init(dempty + i, 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (uint32_t j = threadIdx.x; j < G; j += kThreads) S.scount[j] = 0u;
    unsigned long long events = 0;
    uint32_t rfill = 0, dfill = 0;
    const long long t_kernel = clock64();  // ring fills so far (slot = fill % 2, use = fill / 2)

    for (uint32_t pass = 0; pass < L.passes; ++pass) {
        const uint64_t *__restrict__ row_ptr = L.row_ptr[pass];
        const uint32_t *__restrict__ col = L.col[pass];
        const float *__restrict__ w = L.w[pass];
        float *next_pass = next + L.pass_lo[pass];
        for (uint32_t j = threadIdx.x; j < L.tile; j += kThreads) S.tile[j] = 0.0f;
        __syncthreads();
        if (warp == 0) {
            // ------------------------------------------- router producer --
            const long long t_rp = clock64();
            for (uint32_t k = 0; k < rounds && !s_abort; ++k) {
                const uint32_t r0 = k * rows_round + c * L.rows_per_cta;
                const uint32_t r1 = min(r0 + L.rows_per_cta, S_rows);
                uint32_t s = rfill & 1u, np = 0, total = 0, used = 0;
                bool ok = true;
                if (lane == 0 && rfill >= 2) ok = mbar_wait(rempty + s, ((rfill >> 1) - 1) & 1u, lim, err);
                for (uint32_t rb = r0; rb < r1 && __shfl_sync(kFull, ok, 0); rb += 32) {
                    uint64_t b = 0, e = 0;
                    if (rb + lane < r1) {
                        const uint64_t row = (uint64_t)list[rb + lane];
                        b = row_ptr[row];
                        e = row_ptr[row + 1];
                        events += e - b;
                    }
                    const uint32_t nrow = min(32u, r1 - rb);
                    for (uint32_t jr = 0; jr < nrow; ++jr) {
                        const uint64_t bj = __shfl_sync(kFull, b, jr), ej = __shfl_sync(kFull, e, jr);
                        if (lane == 0) {
                            uint64_t pos = bj;
                            while (ok && pos < ej) {
                                if (np == kRMaxPieces || total == kRSlotEdges) {
                                    SlotHdr<kRMaxPieces> &h = S.rhdr[s];
                                    h.npieces = np;
                                    h.total = total;
                                    h.prefix[np] = total;
                                    h.flags = 0u;
                                    mbar_arrive(rfull + s);
                                    ++rfill;
                                    s = rfill & 1u;
                                    np = total = used = 0;
                                    const long long tw = clock64();
                                    if (rfill >= 2) ok = mbar_wait(rempty + s, ((rfill >> 1) - 1) & 1u, lim, err);
                                    prof_add(L, 0, clock64() - tw);
                                    if (!ok) break;
                                }
                                const uint64_t take =
                                    min(min(ej - pos, (uint64_t)(kRSlotEdges - total)), (uint64_t)kPieceEdges);
                                const uint64_t ab = pos & ~(uint64_t)3;
                                const uint64_t ae = (pos + take + 3) & ~(uint64_t)3;
                                const uint32_t nal = (uint32_t)(ae - ab);
                                SlotHdr<kRMaxPieces> &h = S.rhdr[s];
                                h.start[np] = used + (uint32_t)(pos - ab);
                                h.prefix[np] = total;
                                ++np;
                                total += (uint32_t)take;
                                mbar_expect_tx(rfull + s, nal * 8u);
                                bulk_g2s(S.rcol + s * kRSlotCap + used, col + ab, nal * 4u, rfull + s);
                                bulk_g2s(S.rw + s * kRSlotCap + used, w + ab, nal * 4u, rfull + s);
                                used += nal;
                                pos += take;
                            }
                        }
                        ok = __shfl_sync(kFull, ok, 0);
                    }
                }
                if (lane == 0) {
                    if (ok) {
                        SlotHdr<kRMaxPieces> &h = S.rhdr[s];
                        h.npieces = np;
                        h.total = total;
                        h.prefix[np] = total;
                        h.flags = kRoundEnd;
                        mbar_arrive(rfull + s);
                        ++rfill;
                    } else {
                        s_abort = 1u;
                    }
                }
                if (!__shfl_sync(kFull, ok, 0)) break;
            }
            if (lane == 0) prof_add(L, 1, clock64() - t_rp);
        } else if (warp <= (unsigned)kRConsWarps) {
            // ------------------------------------------ router consumers --
            const unsigned rt = threadIdx.x - 32;
            const unsigned rw = warp - 1;
            for (uint32_t k = 0; k < rounds; ++k) {
                const uint32_t g = pass * rounds + k;
                const uint32_t b = g % L.nb;
                const RouteCtx R{L.bins + b * buf_stride + (size_t)c * L.cap, q_stride, next_pass};
                const long long t_wd = clock64();
                if (rt == 0 && g >= L.nb && !wait_geq(drained, (unsigned long long)G * (g - L.nb + 1), lim, err))
                    s_abort = 1u;
                if (rt == 0) prof_add(L, 2, clock64() - t_wd);
                for (uint32_t j = rt; j < G; j += kRConsThreads) S.wcount[j] = 0u;
                named_sync(1, kRConsThreads);
                if (s_abort) break;
                bool round_end = false;
                while (!round_end) {
                    const uint32_t s = rfill & 1u;
                    const long long t_wf = clock64();
                    const bool ok = mbar_wait(rfull + s, (rfill >> 1) & 1u, lim, err);
                    const long long t_rt = clock64();
                    if (rt == 0) prof_add(L, 3, t_rt - t_wf);
                    if (!ok) s_abort = 1u;
                    const SlotHdr<kRMaxPieces> &h = S.rhdr[s];
                    const uint32_t total = ok ? h.total : 0u;
                    round_end = !ok || (h.flags & kRoundEnd);
                    const uint32_t *scol = S.rcol + s * kRSlotCap;
                    const float *sw = S.rw + s * kRSlotCap;
                    const uint32_t np = ok ? h.npieces : 0u;
                    for (uint32_t p = rw; p < np; p += kRConsWarps) {
                        const uint32_t n = h.prefix[p + 1] - h.prefix[p];
                        const uint32_t base = h.start[p];
                        for (uint32_t j = lane; j < n; j += 32) route(scol[base + j], sw[base + j], L, S, R);
                    }
                    (void)total;
                    named_sync(1, kRConsThreads);
                    const long long t_fl = clock64();
                    if (rt == 0) prof_add(L, 4, t_fl - t_rt);
                    if (rt == 0 && ok) mbar_arrive(rempty + s);  // ring slot consumed
                    ++rfill;
                    // Flush: reserve per destination in shared memory, then
                    // copy each destination's staged run with one warp.
                    for (uint32_t q = rt; q < G; q += kRConsThreads) {
                        const uint32_t cnt = min(S.scount[q], kStage);
                        S.sbase[q] = S.wcount[q];
                        S.wcount[q] += cnt;
                    }
                    named_sync(1, kRConsThreads);
                    // Copy: one thread per staging slot (destination-major), so a
                    // destination's run is stored by consecutive threads.
                    for (uint32_t i = rt; i < G * kStage; i += kRConsThreads) {
                        const uint32_t q = i / kStage, k = i - q * kStage;
                        if (k < min(S.scount[q], kStage)) {
                            const uint2 ent = S.stage[i];
                            const uint32_t p = S.sbase[q] + k;
                            if (p < L.cap) R.sub[q * q_stride + p] = ent;
                            else red_add(next_pass + (size_t)q * L.tile + ent.x, __uint_as_float(ent.y));
                        }
                    }
                    named_sync(1, kRConsThreads);
                    for (uint32_t q = rt; q < G; q += kRConsThreads) S.scount[q] = 0u;
                    named_sync(1, kRConsThreads);
                    if (rt == 0) prof_add(L, 5, clock64() - t_fl);
                    if (s_abort) break;
                }
                if (s_abort) break;
                // Publish my sub-bin sizes for this round, then the round.
                uint32_t *counts = L.counts + (size_t)b * G * G;
                for (uint32_t q = rt; q < G; q += kRConsThreads) {
                    uint32_t cnt = min(S.wcount[q], L.cap);
                    if (cnt & 1u) R.sub[q * q_stride + cnt++] = make_uint2(0u, 0u);  // pad: adds +0.0f to entry 0
                    counts[(size_t)q * G + c] = cnt;
                }
                named_sync(1, kRConsThreads);
                if (rt == 0) {
                    __threadfence();
                    red_release_add(routed, 1ull);
                }
            }
        } else if (warp == (unsigned)kDProdWarp) {
            // -------------------------------------------- drain producer --
            for (uint32_t k = 0; k < rounds && !s_abort; ++k) {
                const uint32_t g = pass * rounds + k;
                const uint32_t b = g % L.nb;
                const long long t_wr = clock64();
                const bool ready = wait_geq(routed, (unsigned long long)G * (g + 1), lim, err);
                if (lane == 0) prof_add(L, 6, clock64() - t_wr);
                const long long t_is = clock64();
                if (!__all_sync(kFull, ready)) {
                    if (lane == 0) s_abort = 1u;
                    break;
                }
                const uint32_t *counts = L.counts + (size_t)b * G * G + (size_t)c * G;
                for (uint32_t src = lane; src < G; src += 32) S.dcount[src] = __ldcg(counts + src);
                __syncwarp();
                if (lane == 0) {
                    const uint2 *mine = L.bins + b * buf_stride + (size_t)c * q_stride;
                    uint32_t s = dfill & 1u, np = 0, total = 0, used = 0;
                    bool ok = dfill < 2 || mbar_wait(dempty + s, ((dfill >> 1) - 1) & 1u, lim, err);
                    for (uint32_t src = 0; src < G && ok; ++src) {
                        const uint32_t cnt = S.dcount[src];
                        if (cnt == 0) continue;
                        const uint32_t nal = cnt;  // even: sub-bins are padded to entry pairs
                        if (np == kDMaxPieces || used + nal > kDSlotCap) {
                            SlotHdr<kDMaxPieces> &h = S.dhdr[s];
                            h.npieces = np;
                            h.total = total;
                            h.prefix[np] = total;
                            h.flags = 0u;
                            mbar_arrive(dfull + s);
                            ++dfill;
                            s = dfill & 1u;
                            np = total = used = 0;
                            if (dfill >= 2) ok = mbar_wait(dempty + s, ((dfill >> 1) - 1) & 1u, lim, err);
                            if (!ok) break;
                        }
                        SlotHdr<kDMaxPieces> &h = S.dhdr[s];
                        h.start[np] = used;
                        h.prefix[np] = total;
                        ++np;
                        total += cnt;
                        mbar_expect_tx(dfull + s, nal * 8u);
                        bulk_g2s(S.dbuf + s * kDSlotCap + used, mine + (size_t)src * L.cap, nal * 8u, dfull + s);
                        used += nal;
                    }
                    if (ok) {
                        SlotHdr<kDMaxPieces> &h = S.dhdr[s];
                        h.npieces = np;
                        h.total = total;
                        h.prefix[np] = total;
                        h.flags = kRoundEnd;
                        mbar_arrive(dfull + s);
                        ++dfill;
                    } else {
                        s_abort = 1u;
                    }
                }
                dfill = __shfl_sync(kFull, dfill, 0);
                __syncwarp();
                if (lane == 0) prof_add(L, 7, clock64() - t_is);
            }
        } else {
            // ------------------------------------------- drain consumers --
            const unsigned dt = threadIdx.x - (kDProdWarp + 1) * 32;
            for (uint32_t k = 0; k < rounds; ++k) {
                bool round_end = false;
                while (!round_end) {
                    const uint32_t s = dfill & 1u;
                    const long long t_df = clock64();
                    const bool ok = mbar_wait(dfull + s, (dfill >> 1) & 1u, lim, err);
                    const long long t_fo = clock64();
                    if (dt == 0) prof_add(L, 8, t_fo - t_df);
                    if (!ok) s_abort = 1u;
                    const SlotHdr<kDMaxPieces> &h = S.dhdr[s];
                    const uint32_t total = ok ? h.total : 0u;
                    round_end = !ok || (h.flags & kRoundEnd);
                    // Dense entry pairs: one 16-byte load per thread and pair.
                    const uint4 *buf = reinterpret_cast<const uint4 *>(S.dbuf + s * kDSlotCap);
                    for (uint32_t j = dt; 2 * j < total; j += kDConsThreads) {
                        const uint4 e = buf[j];
                        atomicAdd(&S.tile[e.x], __uint_as_float(e.y));
                        atomicAdd(&S.tile[e.z], __uint_as_float(e.w));
                    }
                    named_sync(2, kDConsThreads);
                    if (dt == 0) prof_add(L, 9, clock64() - t_fo);
                    if (dt == 0 && ok) mbar_arrive(dempty + s);
                    ++dfill;
                }
                if (s_abort) break;
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
    if (threadIdx.x == 0) prof_add(L, 10, clock64() - t_kernel);
    block_add_u64(events, &ctr->events);
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
    const size_t fixed = smem_fixed_bytes(G) + 1024;  // + static smem and slack
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
    const double per_tile = 16384.0;
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
    L->smem_bytes = (uint32_t)(align16(tile * 4) + smem_fixed_bytes(G));
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
