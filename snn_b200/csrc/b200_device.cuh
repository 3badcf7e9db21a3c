// Device helpers shared by the snn_b200 kernel translation units.
#pragma once

#include "b200_kernels.h"

namespace b200 {
namespace dev {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// Fire-and-forget fp32 add into L2 (red.global.add.f32). The PTX f32 atomic
// flushes subnormal inputs/results to zero, as the reference's atomicAdd does.
__device__ __forceinline__ void red_add(float *p, float v) { atomicAdd(p, v); }

// Block-level sum of per-thread u64 values, added once into *dst. Every
// thread of the block must call it.
__device__ __forceinline__ void block_add_u64(unsigned long long v, unsigned long long *dst) {
    __shared__ unsigned long long s_acc;
    if (threadIdx.x == 0) s_acc = 0ull;
    __syncthreads();
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(kFull, v, d);
    if (lane_id() == 0 && v) atomicAdd(&s_acc, v);
    __syncthreads();
    if (threadIdx.x == 0 && s_acc) atomicAdd(dst, s_acc);
}

// Per step bookkeeping done by block 0 of the (last) propagation kernel:
// zero the list slot the next step appends to, and count this step's spikes.
// pulled: this step's propagation was a pull kernel (recorded in the step
// kind log and the pull statistics).
__device__ __forceinline__ void step_epilogue(DevCounters *ctr, int parity, int count_spikes, uint32_t count,
                                              int pulled = 0) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        ctr->list_count[parity ^ 1] = 0u;
        ctr->step_events[parity ^ 1] = 0ull;
        if (count_spikes) ctr->spikes += count;
        if (pulled) ctr->pull_spikes += count;
        if (ctr->kind_log) ctr->kind_log[ctr->step_seq % kStepLog] = (uint8_t)(pulled != 0);
        ctr->step_seq += 1ull;
    }
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// The peer exchange's wait, by every thread of a CTA: thread r < nflags
// waits (bounded) for rank r's flag. False when a wait expired or another
// wait already failed (ctr->error is set). Block 0 adds its wait to
// ctr->wait_ns / wait_max_ns.
__device__ __forceinline__ bool block_peer_sync(const PeerWait &pw, DevCounters *ctr) {
    __shared__ uint32_t s_fail;
    __shared__ unsigned long long s_t0;
    if (threadIdx.x == 0) {
        s_fail = 0u;
        s_t0 = global_ns();
    }
    __syncthreads();
    if (threadIdx.x < pw.nflags) {
        const uint32_t r = threadIdx.x;
        for (uint32_t it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(pw.flags + r) : "memory");
            if (v >= pw.tag) break;
            if (*(volatile uint32_t *)&ctr->error != 0u || it >= pw.spin_limit) {
                atomicExch(&ctr->error, 3u);
                s_fail = 1u;
                break;
            }
            __nanosleep(64);
        }
    }
    __syncthreads();
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const unsigned long long dt = global_ns() - s_t0;
        ctr->wait_ns += dt;
        if (dt > ctr->wait_max_ns) ctr->wait_max_ns = dt;
    }
    return s_fail == 0u;
}

// Word wi of the global bitmap after the peer wait: this rank's words from
// the local buffer, the others read from their owner over NVLink (relaxed,
// system scope: ordered after the flag acquire by the CTA barrier) and
// stored into the local buffer.
__device__ __forceinline__ uint32_t gather_word(const PeerWait &pw, uint32_t *local, uint64_t wi) {
    const uint32_t r = (uint32_t)(wi / pw.slot_words);
    if (r == pw.rank) return __ldcg(local + wi);
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(pw.src[r] + wi) : "memory");
    local[wi] = v;
    return v;
}

// Four words [wi, wi + 4) (wi a multiple of 4, inside one rank's slice),
// gathered like gather_word with one 16-byte load.
__device__ __forceinline__ uint4 gather_vec(const PeerWait &pw, uint32_t *local, uint64_t wi) {
    const uint32_t r = (uint32_t)(wi / pw.slot_words);
    uint4 *dst = reinterpret_cast<uint4 *>(local + wi);
    if (r == pw.rank) return __ldcg(dst);
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(pw.src[r] + wi)
                 : "memory");
    *dst = v;
    return v;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
    uint32_t m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// Lanes of `active` whose `key` (its low `nbits` bits) equals this lane's:
// one ballot per key bit. Cheaper than __match_any_sync when most lanes hold
// distinct keys (its cost grows with the number of distinct values).
template <int NB>
__device__ __forceinline__ uint32_t match_bits_n(uint32_t key, uint32_t active) {
    uint32_t peers = active;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const uint32_t bit = (key >> b) & 1u;
        peers &= ~(__ballot_sync(kFull, bit) ^ (0u - bit));  // equal bit b
    }
    return peers;
}

// Groups the active lanes by key through a scratch array over the key range
// (this warp's): every active lane writes its lane id into tag[key] and reads
// back one writer per key, the group's id (5 bits). Returns the lanes of this
// lane's group, in lane order: rank = popc(peers & lanemask_lt). When no two
// lanes share a key (the common case) no ballot beyond the first is needed.
// Stale scratch entries are harmless: each active lane writes before it reads.
__device__ __forceinline__ uint32_t group_by_key(uint8_t *tag, uint32_t key, bool act, unsigned lane) {
    if (act) tag[key] = (uint8_t)lane;
    __syncwarp();
    const uint32_t g = act ? tag[key] : lane;
    const uint32_t active = __ballot_sync(kFull, act);
    uint32_t peers;
    if (__ballot_sync(kFull, g != lane) == 0u)
        peers = 1u << lane;  // all keys distinct
    else
        peers = match_bits_n<5>(g, active);
    __syncwarp();
    return act ? peers : (1u << lane);
}

}  // namespace dev
}  // namespace b200
