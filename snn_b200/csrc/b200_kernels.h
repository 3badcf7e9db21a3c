// Host-side launch interface of the snn_b200 kernels (b200_kernels.cu).
// Everything here is C++ with no torch types; the C ABI lives in snn_cuda_b200.cu.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

// LIF constants captured at create time (src/snn_cuda.cu:456-460): the host's
// decay = expf(-dt/tau) is used as is, never recomputed on the device.
struct LifArgs {
    float decay;
    float v_rest;
    float v_reset;
    float v_threshold;
    float input_scale;
    uint32_t refractory_steps;
    // When set (graph-replayed runs), block 0 of the LIF kernel advances this
    // device-side injection-stream step index once per step.
    unsigned long long *stream_step;
};

// Small device-side bookkeeping block, one per context.
//  list_count[p]  number of entries of the spike list of a step with parity p
//                 (ping-pong: the propagation of step t zeroes slot (t+1)&1).
//  spikes/events  cumulative statistics (this rank's neurons / targets).
//  error          first error code raised by a bounded device wait (0 = none).
//  step_seq       steps completed since the context was created (never reset).
//  kind_log       optional ring of kStepLog bytes: entry step_seq % kStepLog
//                 is 1 when that step's propagation ran a pull kernel.
//  wait_ns        nanoseconds the peer-exchange compaction spent waiting for
//                 the other ranks' flags (summed over steps), wait_max_ns the
//                 longest single wait.
constexpr uint32_t kStepLog = 8192;
struct DevCounters {
    uint32_t list_count[2];
    uint32_t error;
    uint32_t pad;
    unsigned long long spikes;
    unsigned long long events;
    unsigned long long stream_step;  // injection-stream step of graph-replayed runs
    unsigned long long pull_runs;    // steps whose propagation ran a pull kernel
    unsigned long long pull_events;  // synaptic events of those steps
    unsigned long long pull_spikes;  // spiking rows of those steps
    unsigned long long step_seq;
    unsigned long long wait_ns;
    unsigned long long wait_max_ns;
    uint8_t *kind_log;
    unsigned long long step_events[2];  // ordered compaction: events of the step of each parity
};
static_assert(sizeof(DevCounters) <= 256, "DevCounters must fit its 256-byte block");

// Peer (NVLink, CUDA IPC) spike-bitmap exchange, pull style: the LIF kernel
// writes this rank's bitmap words into its own exchange buffer (passed as
// its bitmap); launch_publish_flags then releases this rank's flag and the
// compaction waits and gathers (PeerWait).
constexpr uint32_t kMaxPeers = 8;
// A one-CTA kernel behind LIF releases `tag` into this rank's flag slot at
// every rank (publish[r]). The compaction then waits (bounded, one thread
// per flag) until all `nflags` flags (in the local buffer) reach `tag`;
// then
// the words of every other rank r are read from src[r] (that rank's exchange
// buffer of this parity, over NVLink) and stored into the local buffer, so
// the local buffer holds the whole global bitmap afterwards. Rank r owns
// words [r * slot_words, (r + 1) * slot_words).
struct PeerWait {
    unsigned long long *publish[kMaxPeers];  // this rank's flag slot at each rank (publication kernel)
    const unsigned long long *flags;
    unsigned long long tag;
    uint32_t nflags;
    uint32_t spin_limit;
    const uint32_t *src[kMaxPeers];
    uint64_t slot_words;
    uint32_t rank;
};

// Network generator description shared by the random-pool and the layered
// generators. Edge e (CSR order) uses draws 2e+1 (target) and 2e+2 (weight)
// of the splitmix64 stream seeded `seed` (src/snn.c:94-105, 553-568).
struct GenParams {
    uint64_t n;           // global neuron count
    uint64_t fanout;      // edges per non-last-layer neuron
    uint64_t seed;
    float wmin;
    float wmax;
    int allow_self;       // recurrent pool only
    int recurrent;        // 1: random pool (targets in [0,n)), 0: layered
    int layers;           // layered: number of layers (<= 16)
    uint64_t off[17];     // layered: prefix offsets of the layers
    // Feed-forward (snn_build_feedforward, src/snn.c:463-521): per layer, the
    // edges of each row (0 for the last layer), the first edge of the layer,
    // and the first splitmix64 draw of its edges (~0: a dense layer, which
    // draws nothing); every weight is wconst. fanout then holds the largest
    // per-row edge count (an upper bound for grid sizing).
    int feedforward;
    float wconst;
    uint64_t lfan[16];
    uint64_t ledge[17];
    uint64_t ldraw[16];
};

// Number of SMs of the current device (cached per device).
int sm_count(int device);

// ctr != nullptr: the counters are zeroed and ctr->kind_log set to kind_log.
void launch_init_state(cudaStream_t s, uint64_t n, float v_rest, float *v, float *cur0, float *cur1, float *ext,
                       uint32_t *refr, uint8_t *spikes, uint64_t bitmap_words, uint32_t *bitmap,
                       DevCounters *ctr, uint8_t *kind_log = nullptr);

// LIF update of n local neurons; writes spikes (u8), the local bitmap words
// and, when list != nullptr, appends the spiking ids (+ global_offset) to the
// spike list of parity `parity`. idx_bits selects a 32- or 64-bit list.
void launch_lif(cudaStream_t s, int device, uint64_t n, const LifArgs &p, float *v, float *cur, const float *ext,
                uint32_t *refr, uint8_t *spikes, uint32_t *bitmap, void *list, int idx_bits, uint64_t global_offset,
                DevCounters *ctr, int parity);

// The flag release of the peer exchange (behind the LIF kernel).
void launch_publish_flags(cudaStream_t s, const PeerWait &pw);

// Global bitmap -> spike list (sharded contexts, after the all-gather; with a
// peer wait, the other ranks' words are first gathered into `bitmap`).
// Also adds the popcount of words [own_begin, own_end) to ctr->spikes.
void launch_compact(cudaStream_t s, int device, uint32_t *bitmap, uint64_t words, void *list, int idx_bits,
                    DevCounters *ctr, int parity, uint64_t own_begin, uint64_t own_end, const PeerWait *wait = nullptr);

// Push propagation from the spike list over a resident CSR.
// col_bits = 32 or 64 (local target ids), idx_bits = spike list width.
// batch_rows != 0: batched states; list id g is row g % batch_rows of the
// topology adding into the current slice starting at g - g % batch_rows.
// lanes: 32, 16 or 8 lanes per spiking row (push_lanes picks it from the
// average row length).
void launch_propagate_push(cudaStream_t s, int device, const void *list, int idx_bits, const uint64_t *row_ptr,
                           const void *col, int col_bits, const float *w, float *next, DevCounters *ctr,
                           int parity, int count_spikes, uint64_t batch_rows = 0, uint32_t pull_above = 0,
                           uint32_t lanes = 32);
uint32_t push_lanes(uint64_t synapses, uint64_t rows);

// Ordered pull over a sliced-ELL CSC: local targets in blocks of 32,
// presynaptic ids cut into `chunks` chunks of chunk_words * 32 ids; the slots
// of (block b, chunk c) start at sell_off[b * chunks + c] (32 per rank: slot
// k of target t at + 32k + t%32), each a (presynaptic id, weight bits) pair;
// each target's slots in a chunk keep CSR order. For every local target,
// folds the weights of its spiking presynaptic rows in (row, edge) order
// from 0.0f. chunks * chunk_words >= words: ids are chunk-relative, padding
// id chunk_words * 32, spike bits staged in shared memory; otherwise (one
// chunk over a larger bitmap) ids are global, padding id all ones, lookups
// through L1/L2. pull_above != 0: a push kernel launched with the same gate
// handles steps of at most pull_above spikes; the pull runs only above it.
// events_gate != 0: the kernel runs only if ctr->step_events[parity] (the
// ordered compaction's event total) exceeds events_above.
// The layout's chunk size is fixed when it is built: pull_chunk_words() then.
uint64_t pull_chunk_words();
uint32_t pull_chunks(uint64_t words);
uint64_t pull_chunk_neurons();
void launch_propagate_pull(cudaStream_t s, int device, uint64_t n_local, uint32_t chunks, uint64_t chunk_words,
                           const uint64_t *sell_off, const uint2 *slots, const uint32_t *bitmap, uint64_t words,
                           float *next, const void *list, int idx_bits, const uint32_t *out_degree, DevCounters *ctr,
                           int parity, int count_spikes, uint32_t pull_above = 0, int events_gate = 0,
                           unsigned long long events_above = 0);
void launch_fill_u2(cudaStream_t s, int device, uint2 *p, uint64_t n, uint32_t x, uint32_t y);
// dst[i] = src[idx[i]] for i < count.
void launch_gather_u64(cudaStream_t s, const unsigned long long *src, const uint64_t *idx, uint64_t count,
                       unsigned long long *dst);
// *p = v, in stream order.
void launch_set_u64(cudaStream_t s, unsigned long long *p, unsigned long long v);

// STREAMING: one chunk of `rows` rows starting at row0, with the chunk's raw
// row_ptr slice (rows+1 entries, absolute edge offsets) and its edges starting
// at edge_base; col holds 64-bit global target ids.
void launch_propagate_chunk(cudaStream_t s, int device, uint64_t row0, uint64_t rows, uint64_t edge_base,
                            const uint32_t *bitmap, const uint64_t *row_ptr, const uint64_t *col, const float *w,
                            float *next, DevCounters *ctr, int parity, int first_chunk, int count_spikes = 1);

// Step epilogue for STREAMING contexts with no chunk (never happens) or for
// steps without a propagation launch: zeroes the next list slot, adds stats.
void launch_step_epilogue(cudaStream_t s, DevCounters *ctr, int parity, int count_spikes);

// Sparse injection. Indices outside [lo, hi) are skipped (other shards).
// Every index receives value * scale (equal values: order-free).
void launch_inject_uniform(cudaStream_t s, int device, uint64_t count, const uint64_t *idx, float value,
                           float scale, float *cur, uint64_t lo, uint64_t hi);
// Stable radix sort of injection (index, value) pairs by index (low end_bit bits).
cudaError_t sort_pairs_u64_f32(cudaStream_t s, uint64_t *keys, uint64_t *keys_alt, float *vals, float *vals_alt,
                               uint64_t n, int end_bit, void *temp, size_t *temp_bytes, bool *result_in_alt);
// Indices sorted ascending with a stable sort: every run of equal indices is
// folded sequentially in its (original k) order.
void launch_inject_ordered(cudaStream_t s, int device, uint64_t count, const uint64_t *idx, const float *val,
                           float scale, float *cur, uint64_t lo, uint64_t hi);
// The seeded injection stream (see snn_b200_inject_stream_async).
// step_dev != nullptr: the step index is read on the device from *step_dev
// (graph-replayed runs; `step` is then ignored).
void launch_inject_stream(cudaStream_t s, int device, uint64_t seed, uint64_t step, uint64_t count, uint64_t n,
                          float addend, float *cur, uint64_t lo, uint64_t hi,
                          const unsigned long long *step_dev = nullptr);

// u64 global column ids -> local ids of the chosen width (subtracting lo).
void launch_convert_cols(cudaStream_t s, int device, const uint64_t *src, void *dst, int col_bits, uint64_t count,
                         uint64_t lo);

// Device network generation.
// Unsharded: row_ptr[i] = edges before row i, col/w of every edge.
void launch_gen_row_ptr_dense(cudaStream_t s, int device, const GenParams &g, uint64_t *row_ptr);
void launch_gen_edges_dense(cudaStream_t s, int device, const GenParams &g, uint64_t edge_begin, uint64_t edge_end,
                            void *col, int col_bits, float *w);
// Sharded: per-row counts of edges targeting [lo, hi), then the fill.
void launch_gen_count_shard(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                            uint64_t *counts);
void launch_gen_fill_shard(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                           const uint64_t *row_ptr, void *col, int col_bits, float *w);

// Exclusive prefix sum of n u64 values (temp storage allocated by the caller
// through the returned size when temp == nullptr).
cudaError_t exclusive_scan_u64(cudaStream_t s, const uint64_t *in, uint64_t *out, uint64_t n, void *temp,
                               size_t *temp_bytes);

// Device CSC construction (ORDERED propagation of generated networks), one
// pass per local target range [a, b) (global [lo+a, lo+b)):
//  * gen_indegree: in-degree of every local target (col_ptr = its scan);
//  * gen_count_shard (u32 variant): per-row edge counts into a range;
//  * gen_fill_keys: (target - range_lo, global edge id) pairs in CSR order;
//  * sort_pairs_u32_u64: stable radix sort by target, so each target's
//    in-edges stay in ascending edge id = CSR order;
//  * gather_generated_sell: presynaptic row = id / fanout (every row with
//    edges owns [row*F, row*F+F)) and the weight recomputed from the id.
void launch_gen_indegree(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                         unsigned long long *indeg);
void launch_gen_count_shard_u32(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                                uint32_t *counts);
void launch_gen_fill_keys(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                          const uint64_t *row_off, uint32_t *keys, uint64_t *eids);
cudaError_t sort_pairs_u32_u64(cudaStream_t s, uint32_t *keys, uint32_t *keys_alt, uint64_t *vals,
                               uint64_t *vals_alt, uint64_t n, int end_bit, void *temp, size_t *temp_bytes,
                               bool *result_in_alt);
void launch_gather_generated_sell(cudaStream_t s, int device, const GenParams &g, const uint32_t *keys,
                                  const uint64_t *eids, uint64_t e, uint64_t t0, uint64_t q0, const uint64_t *col_ptr,
                                  const uint32_t *cnt, uint32_t chunks, uint64_t chunk_neurons, int relative,
                                  const uint64_t *sell_off, uint2 *slots);
// cnt[t * chunks + c]: in-edges of local target t from presynaptic chunk c.
void launch_gen_chunk_counts(cudaStream_t s, int device, const GenParams &g, uint64_t lo, uint64_t hi,
                             uint32_t chunks, uint64_t chunk_neurons, uint32_t *cnt);
// slots[b * chunks + c] = 32 x the largest cnt of block b's targets in chunk c.
void launch_sell_slots(cudaStream_t s, int device, const uint32_t *cnt, uint64_t n_local, uint32_t chunks,
                       uint64_t *slots);

// Ordered push (bit-exact, event-driven), in step order: sdeg of the
// spiking rows -> scan_degrees_u64 (eoff, rows+1 entries) -> per row range:
// gen (events in CSR order) -> sort_pairs_u32_f32 (stable, by target, or by
// target group) -> fold (or group fold).
void launch_ordered_sdeg(cudaStream_t s, int device, const void *list, int idx_bits, DevCounters *ctr, int parity,
                         uint64_t max_rows, const uint64_t *row_ptr, uint32_t *sdeg, int clear,
                         uint64_t batch_rows);
cudaError_t scan_degrees_u64(cudaStream_t s, const uint32_t *in, unsigned long long *out, uint64_t n, void *temp,
                             size_t *temp_bytes);
void launch_ordered_gen(cudaStream_t s, int device, const void *list, int idx_bits, DevCounters *ctr, int parity,
                        uint64_t row_lo, uint64_t row_hi, const uint64_t *row_ptr, const void *col, int col_bits,
                        const float *w, const unsigned long long *eoff, uint64_t rows, uint64_t id_base,
                        uint32_t *sdeg, uint32_t *keys, float *vals, int epilogue, int count_spikes,
                        uint64_t batch_rows);
// Sorts by key bits [begin_bit, end_bit), stably.
cudaError_t sort_pairs_u32_f32(cudaStream_t s, uint32_t *keys, uint32_t *keys_alt, float *vals, float *vals_alt,
                               uint64_t n, int begin_bit, int end_bit, void *temp, size_t *temp_bytes,
                               bool *result_in_alt);
// Fold of events sorted fully by target (begin_bit 0).
void launch_ordered_fold(cudaStream_t s, int device, uint64_t events, const uint32_t *keys, const float *vals,
                         float *next);
// Fold of events sorted by target >> kFoldGroupBits (the sort's begin_bit);
// keys below n_targets. (512-target groups measured the same as 256.)
constexpr int kFoldGroupBits = 9;
void launch_ordered_group_fold(cudaStream_t s, int device, uint64_t events, const uint32_t *keys, const float *vals,
                               float *next, uint64_t n_targets);

// Per-row out-degrees (u32) from a row_ptr, for event statistics in ordered mode.
void launch_row_degrees(cudaStream_t s, int device, const uint64_t *row_ptr, uint64_t rows, uint32_t *deg);

}  // namespace b200
