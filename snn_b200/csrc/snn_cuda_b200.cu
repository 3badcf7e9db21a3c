// snn_b200: the C ABI (include/snn_b200.h) over the sm_100a kernels.
//
// Drop-in replacement for the reference's src/snn_cuda.cu: same eight
// snn_cuda_* entry points, same status codes, same fault-seam numbering
// (so the reference's own tests/test_snn.c links and passes against it),
// plus the snn_b200_* extensions. Differences in how the work is done:
//  * each context owns a non-blocking stream (and a copy stream for
//    STREAMING); every public reference call is still synchronous on return;
//  * the LIF kernel emits a spike bitmap and a compacted spike list, and
//    propagation is driven by the list instead of a scan of all n rows;
//  * device col_idx is 32-bit when the target ids fit (the host CSR stays 64-bit);
//  * STREAMING double-buffers the CSR chunks on a copy stream so the copy of
//    chunk i+1 overlaps the propagation of chunk i;
//  * ORDERED propagation (extension) folds every target's events in CSR
//    order (a stable sort of each step's events by target, or a pull over a
//    CSC on dense steps) and is bit-identical to the reference's serial CPU
//    step for any weights;
//  * sharded contexts (extension) own a contiguous range of postsynaptic
//    neurons and all-gather the spike bitmap with NCCL every step.
#include "snn_b200.h"
#include "b200_binfold.h"
#include "b200_kernels.h"
#include "b200_network.h"

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <array>
#include <utility>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <numeric>
#include <vector>

namespace {

// ------------------------------------------------------------------ seams --
// Deterministic fault injection with the reference's semantics
// (src/snn_cuda.cu:46-125): the k-th seam call after set_fail_after(k) fails.
int64_t g_fail_after = -1;
int g_force_unavailable = 0;
int g_force_meminfo_fail = 0;

int seam_fail() {
    if (g_fail_after < 0) return 0;
    if (g_fail_after == 0) return 1;
    --g_fail_after;
    return 0;
}

thread_local char g_last_error[512] = "";
// Set while snn_b200_create_sharded creates its member contexts: their NCCL
// communicator is made afterwards for all of them at once (ncclCommInitAll).
thread_local bool t_group_member = false;

void set_error(const char *what, const char *detail) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, detail ? detail : "");
}

snn_status_t cuda_status_at(cudaError_t e, const char *where) {
    if (e == cudaSuccess) return SNN_OK;
    set_error(where, cudaGetErrorString(e));
    return SNN_ERR_CUDA;
}

#define cuda_status(e) cuda_status_at((e), __func__)

struct StreamChunk {
    uint64_t row_begin;
    uint64_t rows;
    uint64_t edge_begin;
    uint64_t edge_count;
};

struct TimingGroup {
    cudaEvent_t ev[4];  // start, after LIF, after exchange, after propagation
    uint64_t seq = 0;   // the step's index since create (DevCounters::step_seq)
};

// What the three phases of one step (LIF, exchange, propagation) share.
struct StepState {
    int parity = 0;
    float *next = nullptr;
    TimingGroup *tg = nullptr;
    bool sharded = false, peer = false, ordered_list = false;
    uint32_t *own_bitmap = nullptr;
    uint32_t *xbitmap = nullptr;
    b200::PeerWait pw{};
    uint64_t brows = 0;
};

}  // namespace

struct snn_cuda_context {
    const snn_network_t *network = nullptr;
    snn_cuda_mode_t mode = SNN_CUDA_MODE_NONE;
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t copy_stream = nullptr;
    int propagation = SNN_B200_PROPAGATE_PUSH;
    int col_bits = 32;
    int idx_bits = 32;
    uint32_t rank = 0;
    uint32_t world = 1;
    uint64_t n_global = 0;  // neurons of the state: batch x n_rows
    uint64_t n_rows = 0;    // rows of the topology (the network's n)
    uint64_t batch = 1;     // independent states sharing the topology
    uint64_t slot = 0;  // neurons per shard slot (multiple of 32)
    uint64_t lo = 0, hi = 0, n_local = 0;
    uint64_t e_local = 0;
    snn_lif_params_t lif{};
    b200::LifArgs args{};

    float *d_v = nullptr;
    float *d_cur_pair = nullptr;
    float *d_cur[2] = {nullptr, nullptr};
    int cur = 0;
    float *d_ext = nullptr;
    bool ext_held = false;  // snn_b200_set_external: d_ext applies to every step without its own
    uint64_t inject_range = 0;  // snn_b200_set_stream_range: stream indices drawn in [0, range); 0 = all
    // run_stream_async on unsharded push and bin-fold contexts replays a captured CUDA
    // graph of two steps (one per parity); the injection step index then
    // lives on the device (DevCounters::stream_step, advanced by LIF).
    bool dev_stream_step = false;
    cudaGraphExec_t graph = nullptr;
    uint64_t graph_seed = 0, graph_count = 0, graph_launches = 0, graph_range = 0;
    float graph_value = 0.0f;
    bool graph_ext = false;
    uint32_t *d_refr = nullptr;
    uint8_t *d_spikes = nullptr;
    void *d_ws = nullptr;
    uint32_t *d_bitmap = nullptr;  // global (padded) bitmap
    uint64_t bitmap_words = 0;
    void *d_list = nullptr;
    b200::DevCounters *d_ctr = nullptr;

    uint64_t *d_row_ptr = nullptr;
    void *d_col = nullptr;
    float *d_w = nullptr;

    uint32_t *h_err = nullptr;  // pinned copy of DevCounters::error

    uint64_t *d_col_ptr = nullptr;
    void *d_pre = nullptr;
    float *d_cw = nullptr;
    uint32_t *d_deg = nullptr;
    // Ordered push (bit-exact, event-driven; the default ORDERED kernel):
    // per-row spiking degrees and event offsets over all rows, and the
    // double-buffered (target, weight) event arrays of ocap entries.
    bool opull = false;    // SNN_B200_ORDERED_PULL: always the pull over a CSC (no CSR)
    bool has_csc = false;  // a SELL CSC beside the CSR: dense steps pull
    uint64_t *d_sell_off = nullptr;  // SELL-32 block offsets (blocks + 1); d_pre / d_cw are the slot arrays
    uint64_t sell_slots = 0;
    uint32_t sell_chunks = 1;  // presynaptic chunks of the SELL layout (b200::pull_chunks: shared-memory bits)
    uint64_t sell_chunk_words = 0;  // bitmap words per chunk, fixed when the layout is built
    uint32_t pull_above = 0;  // PUSH with a SELL CSC: steps with more spikes than this pull
    uint64_t pull_div = 10;  // pull when a step's events exceed local synapses / pull_div
    uint32_t *d_sdeg = nullptr;
    unsigned long long *d_eoff = nullptr;
    uint32_t *d_okeys[2] = {nullptr, nullptr};
    float *d_ovals[2] = {nullptr, nullptr};
    uint64_t ocap = 0;
    void *d_otemp = nullptr;
    size_t otemp_bytes = 0;
    unsigned long long *h_ototal = nullptr;
    // ORDERED through the bin-fold (the default ORDERED propagation): ordered
    // compaction, per-tile counts, stable scatter and shared-memory fold, all
    // gated on the device against the pull for steps above bf_gate events.
    bool binfold = false;
    bool want_binfold = false;
    uint32_t push_lanes = 0;  // lanes per spiking row of the push kernel (0: not chosen yet)  // SNN_B200_PROPAGATE_PUSH_BINNED: the bin-fold rather than the event sort
    b200::BinFoldPlan bf{};
    b200::BinFoldBuffers bfb{};
    uint64_t bf_cap = 0;
    unsigned long long bf_gate = 0;

    std::vector<StreamChunk> chunks;
    // Sharded STREAMING: the rank's slice of the host CSR (local target ids),
    // viewed as a network by the streaming code.
    snn_network_t slice_net{};
    uint64_t *h_slice_rp = nullptr, *h_slice_col = nullptr;
    float *h_slice_w = nullptr;
    uint64_t slot_rows = 0, slot_edges = 0, slot_stride = 0;
    uint64_t *d_chunk_row = nullptr;
    // ORDERED over chunked STREAMING: each chunk's first row (device), and
    // the step's event offsets at the chunk boundaries (pinned host).
    uint64_t *d_chunk_rb = nullptr;
    unsigned long long *d_bounds = nullptr, *h_bounds = nullptr;
    uint64_t *d_chunk_col = nullptr;
    float *d_chunk_w = nullptr;
    cudaEvent_t ev_copied[2] = {nullptr, nullptr};
    cudaEvent_t ev_free[2] = {nullptr, nullptr};
    const void *registered[3] = {nullptr, nullptr, nullptr};

    uint64_t *d_inj_idx = nullptr;
    float *d_inj_val = nullptr;
    uint64_t inj_cap = 0;
    // Injections copy the caller's arrays straight to the device on their own
    // stream (the host waits for that copy only); ev_inj_used marks the last
    // injection kernel, after which the buffers are free. d_inj_idx holds the
    // indices and their sort's alternate buffer (2 x inj_cap); d_inj_val the
    // values, their alternate and the sort's scratch (inj_tmp_bytes).
    size_t inj_tmp_bytes = 0;
    cudaStream_t inj_stream = nullptr;
    cudaEvent_t ev_inj_copy = nullptr, ev_inj_used = nullptr;
    // snn_cuda_step on FULL contexts: the spike download runs on its own
    // stream as soon as the LIF kernel is done, overlapping propagation.
    cudaStream_t spk_stream = nullptr;
    cudaEvent_t ev_lif = nullptr, ev_spk = nullptr;
    uint8_t *spk_dst = nullptr;  // set for the duration of one snn_cuda_step

    ncclComm_t comm = nullptr;
    // Peer exchange (SNN_B200_EXCHANGE_PEER): [2 parities][bitmap_words] u32,
    // then world u64 flags (slot r: rank r's step tag); peers' buffers mapped by IPC.
    int exchange = SNN_B200_EXCHANGE_NCCL;
    int streaming = SNN_B200_STREAMING_CHUNKED;
    // Sparse streaming: device pointers of the page-locked, mapped host CSR.
    const uint64_t *h_col_dev = nullptr;
    const float *h_w_dev = nullptr;
    void *d_xbuf = nullptr;
    uint32_t *peer_x[b200::kMaxPeers] = {};
    bool peer_ipc[b200::kMaxPeers] = {};  // mapping opened with cudaIpcOpenMemHandle
    bool peers_connected = false;
    unsigned long long xstep = 0;  // monotonic exchange counter (never reset)
    uint32_t peer_spin_limit = 1u << 24;

    uint64_t step = 0;
    uint64_t launches = 0;
    int timing = 0;
    uint64_t seq = 0;  // steps enqueued since create (mirrors DevCounters::step_seq)
    uint8_t *d_kind_log = nullptr;  // inside d_ws: b200::kStepLog bytes
    std::vector<TimingGroup> pending, pool;
    double t_step = 0, t_lif = 0, t_exchange = 0, t_prop = 0, t_prop_pull = 0;
    StepState ps;  // the step in progress between its phases
    // A context made by snn_cuda_create_sharded drives one member context per
    // device (ranks 0..G-1 of the postsynaptic sharding); the public calls on
    // it act on every member.
    std::vector<snn_cuda_context *> group;
};

namespace {

snn_status_t dmalloc(void **ptr, uint64_t count, uint64_t elem) {
    *ptr = nullptr;
    if (count == 0) return SNN_OK;
    if (seam_fail()) {
        set_error("cudaMalloc", "fault injected by snn_test_cuda_set_fail_after");
        return SNN_ERR_CUDA;
    }
    return cuda_status(cudaMalloc(ptr, (size_t)(count * elem)));
}

snn_status_t h2d(snn_cuda_context_t *c, void *dst, const void *src, uint64_t bytes) {
    if (bytes == 0) return SNN_OK;
    if (seam_fail()) return SNN_ERR_CUDA;
    return cuda_status(cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyHostToDevice, c->stream));
}

snn_status_t check_launch(snn_cuda_context_t *c) {
    c->launches++;
    if (seam_fail()) return SNN_ERR_CUDA;
    return cuda_status(cudaGetLastError());
}

snn_status_t set_device(const snn_cuda_context_t *c) { return cuda_status(cudaSetDevice(c->device)); }

uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

using b200host::lif_valid;
using b200host::validate_csr;

void free_context(snn_cuda_context_t *c) {
    if (c == nullptr) return;
    if (!c->group.empty()) {
        for (snn_cuda_context_t *m : c->group) free_context(m);
        delete c;
        return;
    }
    if (c->device >= 0) cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    if (c->spk_stream) cudaStreamSynchronize(c->spk_stream);
    if (c->comm) ncclCommDestroy(c->comm);
    for (uint32_t r = 0; r < b200::kMaxPeers; ++r)
        if (c->peer_ipc[r]) cudaIpcCloseMemHandle(c->peer_x[r]);
    if (c->d_xbuf) cudaFree(c->d_xbuf);
    void *dev[] = {c->d_v, c->d_cur_pair, c->d_ext, c->d_refr, c->d_spikes, c->d_ws, c->d_row_ptr, c->d_col,
                   c->d_w, c->d_col_ptr, c->d_pre, c->d_cw, c->d_deg, c->d_sell_off, c->d_sdeg, c->d_eoff, c->d_okeys[0], c->d_okeys[1], c->d_ovals[0], c->d_ovals[1], c->d_otemp,
                   c->d_chunk_row, c->d_chunk_col, c->d_chunk_rb, c->d_bounds,
                   c->d_chunk_w, c->d_inj_idx, c->d_inj_val, c->bfb.hist, c->bfb.offs,
                   c->bfb.bins, c->bfb.ccnt, c->bfb.scan_temp};
    for (void *p : dev)
        if (p) cudaFree(p);
    if (c->h_err) cudaFreeHost(c->h_err);
    if (c->h_ototal) cudaFreeHost(c->h_ototal);
    if (c->h_bounds) cudaFreeHost(c->h_bounds);
    for (const void *p : c->registered)
        if (p) cudaHostUnregister(const_cast<void *>(p));
    std::free(c->h_slice_rp);
    std::free(c->h_slice_col);
    std::free(c->h_slice_w);
    for (int i = 0; i < 2; ++i) {
        if (c->ev_copied[i]) cudaEventDestroy(c->ev_copied[i]);
        if (c->ev_free[i]) cudaEventDestroy(c->ev_free[i]);
    }
    if (c->ev_inj_copy) cudaEventDestroy(c->ev_inj_copy);
    if (c->ev_inj_used) cudaEventDestroy(c->ev_inj_used);
    if (c->inj_stream) cudaStreamDestroy(c->inj_stream);
    if (c->ev_lif) cudaEventDestroy(c->ev_lif);
    if (c->ev_spk) cudaEventDestroy(c->ev_spk);
    if (c->spk_stream) cudaStreamDestroy(c->spk_stream);
    if (c->graph) cudaGraphExecDestroy(c->graph);
    for (auto *v : {&c->pending, &c->pool})
        for (auto &g : *v)
            for (auto e : g.ev) cudaEventDestroy(e);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    cudaGetLastError();  // leave no non-sticky error behind for the next launch check
}

// Rank r owns [r*S, min((r+1)*S, n)) with S = ceil(n / world / 128) * 128:
// equal 128-aligned slots keep every rank's bitmap slice whole 16-byte
// vectors of words, all of equal size (the in-place all-gather needs equal
// counts; the compaction reads the bitmap 4 words at a time).
void shard_geometry(uint64_t n, uint32_t world, uint32_t rank, uint64_t *slot, uint64_t *lo, uint64_t *hi) {
    *slot = ceil_div(ceil_div(n, world), 128) * 128;
    *lo = std::min<uint64_t>(n, (uint64_t)rank * *slot);
    *hi = std::min<uint64_t>(n, *lo + *slot);
}

// Resolves options, validates them and fills the shard geometry.
snn_status_t apply_options(snn_cuda_context_t *c, uint64_t n, const snn_b200_options_t &o) {
    if (o.world_size == 0 || o.rank >= o.world_size) return SNN_ERR_INVALID_ARGUMENT;
    if (o.propagation != SNN_B200_PROPAGATE_PUSH && o.propagation != SNN_B200_PROPAGATE_ORDERED &&
        o.propagation != SNN_B200_PROPAGATE_PUSH_ATOMIC && o.propagation != SNN_B200_PROPAGATE_PUSH_BINNED)
        return SNN_ERR_INVALID_ARGUMENT;
    if (o.index_width != 0 && o.index_width != 32 && o.index_width != 64) return SNN_ERR_INVALID_ARGUMENT;
    if (o.exchange != SNN_B200_EXCHANGE_NCCL && o.exchange != SNN_B200_EXCHANGE_PEER) return SNN_ERR_INVALID_ARGUMENT;
    if (o.world_size > 1 && o.exchange == SNN_B200_EXCHANGE_NCCL && o.nccl_id == nullptr && !t_group_member)
        return SNN_ERR_INVALID_ARGUMENT;
    if (o.exchange == SNN_B200_EXCHANGE_PEER && o.world_size > b200::kMaxPeers) return SNN_ERR_UNSUPPORTED;
    c->exchange = o.exchange;
    if (o.streaming != SNN_B200_STREAMING_CHUNKED && o.streaming != SNN_B200_STREAMING_SPARSE)
        return SNN_ERR_INVALID_ARGUMENT;
    c->streaming = o.streaming;
    // The binned push is the bin-fold, which keeps CSR order: ORDERED.
    c->propagation = o.propagation == SNN_B200_PROPAGATE_PUSH_BINNED ? SNN_B200_PROPAGATE_ORDERED : o.propagation;
    c->want_binfold = o.propagation == SNN_B200_PROPAGATE_PUSH_BINNED;
    c->opull = o.propagation == SNN_B200_PROPAGATE_ORDERED && std::getenv("SNN_B200_ORDERED_PULL") != nullptr;
    c->world = o.world_size;
    c->rank = o.rank;
    c->timing = o.timing;
    // Batched states: B copies of the n-neuron state over one topology, seen
    // by every per-neuron kernel as one B*n-neuron network whose spike list
    // ids g map to topology row g % n and target offset g - g % n.
    const uint64_t batch = o.batch ? o.batch : 1;
    if (batch > 1) {
        if (o.world_size != 1 || o.streaming != SNN_B200_STREAMING_CHUNKED ||
            (c->propagation != SNN_B200_PROPAGATE_PUSH && c->propagation != SNN_B200_PROPAGATE_PUSH_ATOMIC &&
             c->propagation != SNN_B200_PROPAGATE_ORDERED) ||
            (c->propagation == SNN_B200_PROPAGATE_ORDERED && c->opull))
            return SNN_ERR_UNSUPPORTED;
        if (n > UINT64_MAX / batch) return SNN_ERR_OVERFLOW;
    }
    c->batch = batch;
    c->n_rows = n;
    const uint64_t ns = n * batch;
    c->n_global = ns;
    shard_geometry(ns, o.world_size, o.rank, &c->slot, &c->lo, &c->hi);
    c->n_local = c->hi - c->lo;
    c->bitmap_words = c->slot / 32 * o.world_size;
    const bool fits32 = n <= 0xffffffffull;
    c->idx_bits = ns <= 0xffffffffull ? 32 : 64;
    c->col_bits = (o.index_width == 64 || !fits32) ? 64 : 32;
    if (o.index_width == 32 && !fits32) return SNN_ERR_INVALID_ARGUMENT;
    if (c->n_local >= 0xffffffffull) return SNN_ERR_UNSUPPORTED;
    return SNN_OK;
}

uint64_t state_bytes(const snn_cuda_context_t *c) {
    return c->n_local * (4u + 8u + 4u + 4u + 1u) + c->bitmap_words * 4u + c->n_global * (c->idx_bits / 8) + 256u +
           b200::kStepLog;
}

// Device state: seams #1-#6 (six allocations) and #7 (init launch), matching
// the reference's allocate_device_state (src/snn_cuda.cu:264-289).
snn_status_t allocate_state(snn_cuda_context_t *c) {
    snn_status_t st;
    const uint64_t n = c->n_local;
    if ((st = dmalloc((void **)&c->d_v, n, 4)) != SNN_OK) return st;
    // Both current buffers start on a 256-byte boundary (16-byte vector loads).
    const uint64_t cur_stride = (n + 63) / 64 * 64;
    if ((st = dmalloc((void **)&c->d_cur_pair, 2 * cur_stride, 4)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_ext, n, 4)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_refr, n, 4)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_spikes, n, 1)) != SNN_OK) return st;
    // Workspace: [counters | step kind log | bitmap (global, padded) | spike list (global)].
    const uint64_t list_bytes = c->n_global * (c->idx_bits / 8);
    const uint64_t head = 256 + b200::kStepLog;
    const uint64_t ws = head + ((c->bitmap_words * 4 + 255) / 256) * 256 + list_bytes;
    if ((st = dmalloc(&c->d_ws, ws, 1)) != SNN_OK) return st;
    c->d_ctr = (b200::DevCounters *)c->d_ws;
    c->d_kind_log = (uint8_t *)c->d_ws + 256;
    c->d_bitmap = (uint32_t *)((char *)c->d_ws + head);
    c->d_list = (char *)c->d_ws + head + ((c->bitmap_words * 4 + 255) / 256) * 256;
    c->d_cur[0] = c->d_cur_pair;
    c->d_cur[1] = c->d_cur_pair ? c->d_cur_pair + cur_stride : nullptr;
    b200::launch_init_state(c->stream, n, c->lif.v_rest, c->d_v, c->d_cur[0], c->d_cur[1], c->d_ext, c->d_refr,
                            c->d_spikes, c->bitmap_words, c->d_bitmap, c->d_ctr, c->d_kind_log);
    return check_launch(c);
}

snn_status_t create_streams(snn_cuda_context_t *c) {
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return SNN_ERR_CUDA;
    if (cudaStreamCreateWithFlags(&c->inj_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_inj_copy, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_inj_used, cudaEventDisableTiming) != cudaSuccess)
        return SNN_ERR_CUDA;
    if (cudaMallocHost(&c->h_err, sizeof(uint32_t)) != cudaSuccess) return SNN_ERR_OUT_OF_MEMORY;
    *c->h_err = 0;
    return SNN_OK;
}

// Offsets inside the peer exchange buffer.
uint64_t xflags_offset(const snn_cuda_context_t *c) { return ((2 * c->bitmap_words * 4 + 255) / 256) * 256; }

snn_status_t init_peer_exchange(snn_cuda_context_t *c) {
    if (c->world <= 1 || c->exchange != SNN_B200_EXCHANGE_PEER) return SNN_OK;
    const uint64_t bytes = xflags_offset(c) + c->world * 8 + 256;
    // Plain cudaMalloc (not the seam wrapper): IPC export needs its own allocation.
    if (cudaMalloc(&c->d_xbuf, bytes) != cudaSuccess) return SNN_ERR_CUDA;
    return cuda_status(cudaMemset(c->d_xbuf, 0, bytes));
}

snn_status_t init_nccl(snn_cuda_context_t *c, const void *id) {
    if (c->world <= 1 || c->exchange != SNN_B200_EXCHANGE_NCCL || t_group_member) return SNN_OK;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = ncclCommInitRank(&c->comm, (int)c->world, uid, (int)c->rank);
    if (r != ncclSuccess) {
        set_error("ncclCommInitRank", ncclGetErrorString(r));
        c->comm = nullptr;
        return SNN_ERR_CUDA;
    }
    return SNN_OK;
}

// Uploads a host u64 column array as local ids of c->col_bits, through a
// bounded device staging buffer when narrowing. One fault seam.
snn_status_t upload_cols(snn_cuda_context_t *c, void *dst, const uint64_t *src, uint64_t count, uint64_t lo,
                         int bits) {
    if (count == 0) return SNN_OK;
    if (seam_fail()) return SNN_ERR_CUDA;
    if (bits == 64 && lo == 0)
        return cuda_status(cudaMemcpyAsync(dst, src, count * 8, cudaMemcpyHostToDevice, c->stream));
    const uint64_t chunk = std::min<uint64_t>(count, 1ull << 26);
    uint64_t *tmp = nullptr;
    if (cudaMalloc(&tmp, chunk * 8) != cudaSuccess) return SNN_ERR_CUDA;
    snn_status_t st = SNN_OK;
    for (uint64_t k = 0; k < count && st == SNN_OK; k += chunk) {
        const uint64_t m = std::min(chunk, count - k);
        st = cuda_status(cudaMemcpyAsync(tmp, src + k, m * 8, cudaMemcpyHostToDevice, c->stream));
        if (st == SNN_OK) {
            b200::launch_convert_cols(c->stream, c->device, tmp, (char *)dst + k * (bits / 8), bits, m, lo);
            st = cuda_status(cudaGetLastError());
        }
        if (st == SNN_OK) st = cuda_status(cudaStreamSynchronize(c->stream));
    }
    cudaFree(tmp);
    return st;
}

// Push CSR of the edges that target [rlo, rhi) (global ids), columns stored
// relative to rlo; all presynaptic rows kept. The whole-network case uploads
// the host arrays directly. Seams: three allocations then three uploads, as
// the reference's allocate_full_topology (src/snn_cuda.cu:291-314).
snn_status_t upload_push_range(snn_cuda_context_t *c, const snn_network_t *net, uint64_t rlo, uint64_t rhi,
                               uint64_t **d_row, void **d_col, float **d_w, uint64_t *edges) {
    const uint64_t n = net->neuron_count;
    std::vector<uint64_t> rp, cl;
    std::vector<float> wl;
    const uint64_t *row_ptr = net->row_ptr, *col = net->col_idx;
    const float *w = net->weights;
    uint64_t e = net->synapse_count;
    if (rlo != 0 || rhi != n) {
        try {
            rp.assign(n + 1, 0);
            for (uint64_t i = 0; i < n; ++i) {
                uint64_t k = 0;
                for (uint64_t q = net->row_ptr[i]; q < net->row_ptr[i + 1]; ++q)
                    k += (net->col_idx[q] >= rlo && net->col_idx[q] < rhi);
                rp[i + 1] = rp[i] + k;
            }
            cl.resize(rp[n]);
            wl.resize(rp[n]);
            uint64_t pos = 0;
            for (uint64_t q = 0; q < net->synapse_count; ++q) {
                if (net->col_idx[q] >= rlo && net->col_idx[q] < rhi) {
                    cl[pos] = net->col_idx[q];
                    wl[pos] = net->weights[q];
                    ++pos;
                }
            }
        } catch (const std::bad_alloc &) {
            return SNN_ERR_OUT_OF_MEMORY;
        }
        row_ptr = rp.data();
        col = cl.data();
        w = wl.data();
        e = rp[n];
    }
    *edges = e;
    snn_status_t st;
    if ((st = dmalloc((void **)d_row, n + 1, 8)) != SNN_OK) return st;
    // +16 bytes of tail so no vector load can run past the allocation.
    if ((st = dmalloc(d_col, e ? e + 16 / (c->col_bits / 8) : 0, c->col_bits / 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)d_w, e ? e + 4 : 0, 4)) != SNN_OK) return st;
    if ((st = h2d(c, *d_row, row_ptr, (n + 1) * 8)) != SNN_OK) return st;
    if ((st = upload_cols(c, *d_col, col, e, rlo, c->col_bits)) != SNN_OK) return st;
    if ((st = h2d(c, *d_w, w, e * 4)) != SNN_OK) return st;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

// FULL push topology from a host network: the edges into the rank's range.
snn_status_t upload_full_push(snn_cuda_context_t *c, const snn_network_t *net) {
    uint64_t e = 0;
    const snn_status_t st =
        upload_push_range(c, net, c->lo, std::min(c->hi, c->n_rows), &c->d_row_ptr, &c->d_col, &c->d_w, &e);
    c->e_local = e;
    return st;
}

// Radix bits that cover the local target ids.
int target_bits(const snn_cuda_context_t *c) {
    int bits = 1;
    while (bits < 32 && (1ull << bits) < c->n_local) ++bits;
    return bits;
}

// Ordered push buffers, after the push CSR exists. The event capacity (events
// per sort) is bounded by half of the free device memory at 16 B per event
// (keys and weights, double-buffered) and by the local synapse count.
snn_status_t setup_ordered_push(snn_cuda_context_t *c, uint64_t cap_limit = UINT64_MAX) {
    const uint64_t n = c->n_global, nl = c->n_local;
    auto fail = [&](const char *what) {
        set_error("ordered push setup", what);
        return SNN_ERR_OUT_OF_MEMORY;
    };
    if (nl > 0xffffffffull) return SNN_ERR_UNSUPPORTED;  // 32-bit sort keys
    if (cudaMalloc(&c->d_sdeg, (n + 1) * 4) != cudaSuccess || cudaMalloc(&c->d_eoff, (n + 1) * 8) != cudaSuccess)
        return fail("out of device memory for the per-row arrays");
    if (cudaMallocHost(&c->h_ototal, 8) != cudaSuccess) return fail("out of pinned memory");
    cudaMemsetAsync(c->d_sdeg, 0, (n + 1) * 4, c->stream);
    // Largest row: one row's events must fit one sort.
    const uint64_t rows = c->n_rows;
    std::vector<uint64_t> rp;
    try {
        rp.resize(rows + 1);
    } catch (const std::bad_alloc &) {
        return SNN_ERR_OUT_OF_MEMORY;
    }
    if (cudaMemcpy(rp.data(), c->d_row_ptr, (rows + 1) * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
        return SNN_ERR_CUDA;
    uint64_t max_deg = 0;
    for (uint64_t i = 0; i < rows; ++i) max_deg = std::max(max_deg, rp[i + 1] - rp[i]);
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return SNN_ERR_CUDA;
    uint64_t cap = std::min<uint64_t>({c->e_local * c->batch, (uint64_t)(free_b / 2) / 16, cap_limit});
    if (const char *env = std::getenv("SNN_B200_ORDERED_CAP")) {  // tests: force the multi-range path
        const uint64_t v = std::strtoull(env, nullptr, 10);
        if (v) cap = std::min(cap, v);
    }
    if (c->e_local && cap < std::max<uint64_t>(max_deg, 1)) return fail("a row's events exceed the event capacity");
    c->ocap = c->e_local ? cap : 0;
    if (c->ocap) {
        for (int i = 0; i < 2; ++i)
            if (cudaMalloc(&c->d_okeys[i], c->ocap * 4) != cudaSuccess ||
                cudaMalloc(&c->d_ovals[i], c->ocap * 4) != cudaSuccess)
                return fail("out of device memory for the event arrays");
    }
    size_t a = 0, b = 0;
    bool alt = false;
    b200::scan_degrees_u64(c->stream, nullptr, nullptr, n + 1, nullptr, &a);
    if (c->ocap)
        b200::sort_pairs_u32_f32(c->stream, nullptr, nullptr, nullptr, nullptr, c->ocap, 0, target_bits(c), nullptr,
                                 &b, &alt);
    c->otemp_bytes = std::max({a, b, (size_t)256});
    if (cudaMalloc(&c->d_otemp, c->otemp_bytes) != cudaSuccess) return fail("out of device memory for sort scratch");
    return cuda_status(cudaStreamSynchronize(c->stream));
}

// Bin-fold buffers (b200_binfold.cu). Returns false (nothing allocated)
// when the bin-fold cannot serve this context: too many local targets for its
// tiles, or, without a pull topology for dense steps, too little memory for
// an event array as large as the local synapses.
bool setup_binfold(snn_cuda_context_t *c) {
    b200::BinFoldPlan plan{};
    if (!b200::binfold_plan(c->device, c->n_local, &plan)) return false;
    plan.chunks = b200::binfold_chunks(c->bitmap_words);
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return false;
    const uint64_t fixed = plan.hist_entries * 8 + (uint64_t)plan.chunks * 4 + (64ull << 20);
    const uint64_t margin = 512ull << 20;
    if (free_b < fixed + margin) return false;
    const uint64_t all = c->e_local * c->batch;
    uint64_t cap = std::min<uint64_t>(all, (free_b - fixed - margin) / 8);
    cap = std::min<uint64_t>(cap, 0xffffffffull);  // 32-bit slot offsets
    if (const char *env = std::getenv("SNN_B200_ORDERED_CAP")) {  // tests: dense steps at a low count
        const uint64_t v = std::strtoull(env, nullptr, 10);
        if (v) cap = std::min(cap, v);
    }
    if (!c->has_csc && cap < all) return false;
    uint64_t gate = cap;
    if (c->has_csc && c->pull_div) gate = std::min<uint64_t>(cap, all / c->pull_div);
    b200::BinFoldBuffers b{};
    size_t scan_bytes = 0;
    b200::binfold_scan(c->stream, nullptr, nullptr, plan.hist_entries, nullptr, &scan_bytes);
    if (cudaMalloc(&b.hist, plan.hist_entries * 4) != cudaSuccess ||
        cudaMalloc(&b.offs, plan.hist_entries * 4) != cudaSuccess ||
        cudaMalloc(&b.ccnt, (uint64_t)plan.chunks * 4 + 4) != cudaSuccess ||
        cudaMalloc(&b.scan_temp, std::max<size_t>(scan_bytes, 256)) != cudaSuccess ||
        (cap && cudaMalloc(&b.bins, cap * 8) != cudaSuccess)) {
        cudaGetLastError();
        for (void *p : {(void *)b.hist, (void *)b.offs, (void *)b.ccnt, b.scan_temp, (void *)b.bins})
            if (p) cudaFree(p);
        return false;
    }
    b.scan_bytes = std::max<size_t>(scan_bytes, 256);
    // The last hist entry is never written: the scan's total lands in offs.
    cudaMemsetAsync(b.hist, 0, plan.hist_entries * 4, c->stream);
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return false;
    c->bf = plan;
    c->bfb = b;
    c->bf_cap = cap;
    c->bf_gate = gate;
    c->binfold = true;
    return true;
}

// Sorts a range's events (in CSR order in d_okeys[0] / d_ovals[0]) and folds
// them onto next. By default the sort orders only the target-group bits and
// the group fold finishes (one radix pass fewer); SNN_B200_ORDERED_FOLD=full
// sorts by the whole target and folds runs. With one group, no sort at all.
snn_status_t sort_and_fold(snn_cuda_context_t *c, uint64_t events, float *next) {
    const char *fold_env = std::getenv("SNN_B200_ORDERED_FOLD");
    const bool full = fold_env != nullptr && std::strcmp(fold_env, "full") == 0;
    const int end_bit = target_bits(c);
    const int begin_bit = full ? 0 : b200::kFoldGroupBits;
    bool alt = false;
    if (end_bit > begin_bit) {
        size_t tb = c->otemp_bytes;
        const snn_status_t st = cuda_status(b200::sort_pairs_u32_f32(c->stream, c->d_okeys[0], c->d_okeys[1],
                                                                     c->d_ovals[0], c->d_ovals[1], events, begin_bit,
                                                                     end_bit, c->d_otemp, &tb, &alt));
        if (st != SNN_OK) return st;
    }
    const uint32_t *keys = c->d_okeys[alt ? 1 : 0];
    const float *vals = c->d_ovals[alt ? 1 : 0];
    if (full)
        b200::launch_ordered_fold(c->stream, c->device, events, keys, vals, next);
    else
        b200::launch_ordered_group_fold(c->stream, c->device, events, keys, vals, next, c->n_local);
    return SNN_OK;
}

// ORDERED propagation set-up after the push CSR (and the pull topology, when
// there is room) exist. The event sort by default: per event it costs less
// than the bin-fold on B200 (the same config 2 quiet steps: 2.35 ms with a
// full sort by target, less with the group sort, against 8.2 ms), at the
// price of one host read per step. PUSH_BINNED asks
// for the bin-fold (no host round trip, graph-replayable); it falls back to
// the event sort when it cannot be set up.
snn_status_t setup_ordered(snn_cuda_context_t *c) {
    if (c->want_binfold && setup_binfold(c)) return SNN_OK;
    // The event sort costs more per event: its dense-step bound is lower.
    if (std::getenv("SNN_B200_ORDERED_PULL_DIV") == nullptr && c->pull_div) c->pull_div = 10;
    return setup_ordered_push(c);
}

// One ordered push propagation (b200_kernels.cu describes the steps); one
// host round trip reads the step's event count to size the sort.
// The CSR comes in explicitly: the resident one (FULL) or the mapped host
// CSR (sparse STREAMING; col is then 64-bit).
snn_status_t ordered_push_step(snn_cuda_context_t *c, int parity, float *next, bool sharded,
                               const uint32_t *bitmap, const uint64_t *row_ptr, const void *col, int col_bits,
                               const float *w) {
    const uint64_t n = c->n_global;
    snn_status_t st;
    const uint64_t brows = c->batch > 1 ? c->n_rows : 0;
    b200::launch_ordered_sdeg(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, n, row_ptr,
                              c->d_sdeg, 0, brows);
    size_t tb = c->otemp_bytes;
    if ((st = cuda_status(b200::scan_degrees_u64(c->stream, c->d_sdeg, c->d_eoff, n + 1, c->d_otemp, &tb))) != SNN_OK)
        return st;
    if ((st = cuda_status(cudaMemcpyAsync(c->h_ototal, c->d_eoff + n, 8, cudaMemcpyDeviceToHost, c->stream))) !=
        SNN_OK)
        return st;
    if ((st = cuda_status(cudaStreamSynchronize(c->stream))) != SNN_OK) return st;
    const uint64_t total = *c->h_ototal;
    if (c->has_csc && c->pull_div && total > c->e_local / c->pull_div) {
        // Most rows spike: the pull over the CSC reads every synapse once,
        // cheaper than sorting this many events.
        b200::launch_ordered_sdeg(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, n, row_ptr,
                                  c->d_sdeg, 1, brows);
        b200::launch_propagate_pull(c->stream, c->device, c->n_local, c->sell_chunks, c->sell_chunk_words,
                                    c->d_sell_off, (const uint2 *)c->d_pre, 
                                    bitmap, c->bitmap_words, next, c->d_list, c->idx_bits, c->d_deg, c->d_ctr, parity,
                                    !sharded);
        c->launches += 2;
        return SNN_OK;
    }
    // Row ranges of at most ocap events each (one range unless the step is huge).
    std::vector<std::array<uint64_t, 3>> ranges;  // row_lo, row_hi, first event id
    if (total <= c->ocap) {
        ranges.push_back({0, n, 0});
    } else {
        std::vector<unsigned long long> eo(n + 1);
        if ((st = cuda_status(cudaMemcpy(eo.data(), c->d_eoff, (n + 1) * 8, cudaMemcpyDeviceToHost))) != SNN_OK)
            return st;
        uint64_t r0 = 0;
        while (r0 < n) {
            uint64_t r1 = (uint64_t)(std::upper_bound(eo.begin() + r0, eo.end(), eo[r0] + c->ocap) - eo.begin()) - 1;
            if (r1 <= r0) r1 = r0 + 1;  // cannot happen: ocap >= the largest row
            ranges.push_back({r0, r1, eo[r0]});
            r0 = r1;
        }
    }
    for (size_t i = 0; i < ranges.size(); ++i) {
        const uint64_t r0 = ranges[i][0], r1 = ranges[i][1], base = ranges[i][2];
        const uint64_t events = (i + 1 < ranges.size() ? ranges[i + 1][2] : total) - base;
        b200::launch_ordered_gen(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, r0, r1, row_ptr,
                                 col, col_bits, w, c->d_eoff, n, base, c->d_sdeg, c->d_okeys[0],
                                 c->d_ovals[0], i + 1 == ranges.size(), !sharded, brows);
        c->launches++;
        if (!events) continue;
        if ((st = sort_and_fold(c, events, next)) != SNN_OK) return st;
        c->launches++;
    }
    return SNN_OK;
}

// ORDERED over chunked STREAMING. The step's events are numbered in CSR
// order once (spiking degrees over the resident row_ptr, scanned); one host
// read fetches the event offsets at the chunk boundaries. Then each chunk, as
// its copy lands, copies its spiking rows' events, sorts them stably by
// target and folds them onto the currents the earlier chunks left. Chunks are
// in ascending row order, so every target's fold is the serial CPU order
// (src/snn.c:898-906): bit-identical for any weights.
snn_status_t ordered_stream_chunked(snn_cuda_context_t *c, int parity, float *next, bool sharded) {
    const uint64_t n = c->n_global;
    const snn_network_t *net = c->network;
    snn_status_t st;
    b200::launch_ordered_sdeg(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, n, c->d_row_ptr,
                              c->d_sdeg, 0, 0);
    size_t tb = c->otemp_bytes;
    if ((st = cuda_status(b200::scan_degrees_u64(c->stream, c->d_sdeg, c->d_eoff, n + 1, c->d_otemp, &tb))) != SNN_OK)
        return st;
    const uint64_t K = c->chunks.size();
    b200::launch_gather_u64(c->stream, c->d_eoff, c->d_chunk_rb, K + 1, c->d_bounds);
    if ((st = cuda_status(cudaMemcpyAsync(c->h_bounds, c->d_bounds, (K + 1) * 8, cudaMemcpyDeviceToHost,
                                          c->stream))) != SNN_OK)
        return st;
    if ((st = cuda_status(cudaStreamSynchronize(c->stream))) != SNN_OK) return st;
    c->launches += 3;
    for (size_t i = 0; i < K; ++i) {
        const StreamChunk &ch = c->chunks[i];
        const uint64_t events = c->h_bounds[i + 1] - c->h_bounds[i];
        if (events == 0) continue;  // no spiking row in this chunk: nothing to copy
        const int s = (int)(i & 1u);
        uint64_t *drow = c->d_chunk_row + (uint64_t)s * (c->slot_rows + 1);
        uint64_t *dcol = c->d_chunk_col + (uint64_t)s * c->slot_stride;
        float *dw = c->d_chunk_w + (uint64_t)s * c->slot_stride;
        cudaStreamWaitEvent(c->copy_stream, c->ev_free[s], 0);
        if (cudaMemcpyAsync(drow, net->row_ptr + ch.row_begin, (ch.rows + 1) * 8, cudaMemcpyHostToDevice,
                            c->copy_stream) != cudaSuccess ||
            cudaMemcpyAsync(dcol, net->col_idx + ch.edge_begin, ch.edge_count * 8, cudaMemcpyHostToDevice,
                            c->copy_stream) != cudaSuccess ||
            cudaMemcpyAsync(dw, net->weights + ch.edge_begin, ch.edge_count * 4, cudaMemcpyHostToDevice,
                            c->copy_stream) != cudaSuccess)
            return SNN_ERR_CUDA;
        cudaEventRecord(c->ev_copied[s], c->copy_stream);
        cudaStreamWaitEvent(c->stream, c->ev_copied[s], 0);
        // The chunk arrays hold rows [row_begin, row_begin + rows) and edges
        // from edge_begin: index them with absolute row and edge numbers.
        b200::launch_ordered_gen(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, ch.row_begin,
                                 ch.row_begin + ch.rows, drow - ch.row_begin, dcol - ch.edge_begin, 64,
                                 dw - ch.edge_begin, c->d_eoff, n, c->h_bounds[i], c->d_sdeg, c->d_okeys[0],
                                 c->d_ovals[0], 0, 0, 0);
        if ((st = sort_and_fold(c, events, next)) != SNN_OK) return st;
        cudaEventRecord(c->ev_free[s], c->stream);
        c->launches += 3;
    }
    // Statistics and the step epilogue (an empty row range).
    b200::launch_ordered_gen(c->stream, c->device, c->d_list, c->idx_bits, c->d_ctr, parity, 0, 0, c->d_row_ptr,
                             nullptr, 64, nullptr, c->d_eoff, n, 0, c->d_sdeg, c->d_okeys[0], c->d_ovals[0], 1,
                             !sharded, 0);
    c->launches++;
    return cuda_status(cudaGetLastError());
}

// ORDERED set-up of a STREAMING context: row_ptr resident (8 B per row), the
// event sort's buffers (chunked: as large as a chunk's synapses), and the
// chunk boundary tables.
snn_status_t setup_ordered_streaming(snn_cuda_context_t *c) {
    const snn_network_t *net = c->network;
    const uint64_t n = net->neuron_count;
    snn_status_t st;
    if (c->d_row_ptr == nullptr) {
        if (cudaMalloc(&c->d_row_ptr, (n + 1) * 8) != cudaSuccess) return SNN_ERR_OUT_OF_MEMORY;
        if ((st = cuda_status(cudaMemcpy(c->d_row_ptr, net->row_ptr, (n + 1) * 8, cudaMemcpyHostToDevice))) !=
            SNN_OK)
            return st;
    }
    const bool chunked = c->streaming == SNN_B200_STREAMING_CHUNKED;
    if ((st = setup_ordered_push(c, chunked ? std::max<uint64_t>(c->slot_edges, 1) : UINT64_MAX)) != SNN_OK)
        return st;
    if (chunked) {
        const uint64_t K = c->chunks.size();
        std::vector<uint64_t> rb(K + 1);
        for (uint64_t i = 0; i < K; ++i) rb[i] = c->chunks[i].row_begin;
        rb[K] = n;
        if (cudaMalloc(&c->d_chunk_rb, (K + 1) * 8) != cudaSuccess ||
            cudaMalloc(&c->d_bounds, (K + 1) * 8) != cudaSuccess ||
            cudaMallocHost(&c->h_bounds, (K + 1) * 8) != cudaSuccess)
            return SNN_ERR_OUT_OF_MEMORY;
        if ((st = cuda_status(cudaMemcpy(c->d_chunk_rb, rb.data(), (K + 1) * 8, cudaMemcpyHostToDevice))) != SNN_OK)
            return st;
    }
    return SNN_OK;
}

// Chunked sliced-ELL layout from per-(target, chunk) counts cnt[t * C + c]:
// the slots of (block b, chunk c) start at off[b * C + c], 32 x the block's
// largest count in that chunk.
std::vector<uint64_t> sell_offsets(const std::vector<uint32_t> &cnt, uint64_t nl, uint32_t chunks) {
    const uint64_t blocks = (nl + 31) / 32;
    std::vector<uint64_t> off(blocks * chunks + 1, 0);
    for (uint64_t b = 0; b < blocks; ++b)
        for (uint32_t c = 0; c < chunks; ++c) {
            uint32_t m = 0;
            for (uint64_t t = b * 32; t < std::min(nl, b * 32 + 32); ++t) m = std::max(m, cnt[t * chunks + c]);
            off[b * chunks + c + 1] = off[b * chunks + c] + 32ull * m;
        }
    return off;
}

// Presynaptic chunks for the shared-memory pull (the builders fall back to
// one chunk when that layout's padding would not fit the free memory).
uint32_t choose_chunks(snn_cuda_context_t *c) {
    c->sell_chunk_words = b200::pull_chunk_words();
    return b200::pull_chunks(c->bitmap_words);
}

// Allocates the SELL slot arrays (padding: all-ones ids, zero weights) and
// uploads the block offsets.
// Chunk-relative ids (shared-memory bits) when the chunks cover the bitmap.
bool sell_relative(const snn_cuda_context_t *c) {
    return (uint64_t)c->sell_chunks * c->sell_chunk_words >= c->bitmap_words;
}

uint32_t sell_pad_id(const snn_cuda_context_t *c) {
    return sell_relative(c) ? (uint32_t)(c->sell_chunk_words * 32u) : 0xffffffffu;
}

// The slot array: (id, weight bits) pairs, d_pre as uint2[slots].
snn_status_t alloc_sell_slots(snn_cuda_context_t *c, uint64_t slots) {
    c->sell_slots = slots;
    if (slots && cudaMalloc(&c->d_pre, slots * 8) != cudaSuccess) {
        cudaGetLastError();
        set_error("pull topology", "out of device memory for the sliced-ELL CSC");
        return SNN_ERR_OUT_OF_MEMORY;
    }
    // Padding slots: an id whose spike bit is always zero, weight 0.
    if (slots) b200::launch_fill_u2(c->stream, c->device, (uint2 *)c->d_pre, slots, sell_pad_id(c), 0u);
    snn_status_t st = cuda_status(cudaGetLastError());
    if (st == SNN_OK) st = cuda_status(cudaStreamSynchronize(c->stream));
    return st;
}

snn_status_t alloc_sell(snn_cuda_context_t *c, const std::vector<uint64_t> &off) {
    if (cudaMalloc(&c->d_sell_off, off.size() * 8) != cudaSuccess) {
        cudaGetLastError();
        set_error("pull topology", "out of device memory for the sliced-ELL CSC");
        return SNN_ERR_OUT_OF_MEMORY;
    }
    snn_status_t st = cuda_status(cudaMemcpyAsync(c->d_sell_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice,
                                                  c->stream));
    if (st == SNN_OK) st = alloc_sell_slots(c, off.back());
    return st;
}

// Releases a pull topology (a hybrid context that could not finish one goes on without it).
void free_sell(snn_cuda_context_t *c) {
    cudaStreamSynchronize(c->stream);
    for (void **p : {(void **)&c->d_sell_off, &c->d_pre, (void **)&c->d_cw, (void **)&c->d_col_ptr,
                     (void **)&c->d_deg}) {
        if (*p) cudaFree(*p);
        *p = nullptr;
    }
    cudaGetLastError();
    c->sell_slots = 0;
}

// FULL pull topology from a host network: the CSC of the rank's targets built
// with a stable counting sort (every target's in-edges keep CSR order:
// ascending presynaptic row, ascending edge index), stored sliced-ELL; plus
// the out-degree table for event statistics.
snn_status_t upload_full_ordered(snn_cuda_context_t *c, const snn_network_t *net) {
    const uint64_t n = net->neuron_count;
    const uint64_t nl = c->n_local;
    const uint32_t first_choice = choose_chunks(c);
    const uint64_t chunk_neurons = c->sell_chunk_words * 32u;
    std::vector<uint64_t> off, slot;  // slot: weight bits << 32 | id (a little-endian uint2)
    std::vector<uint32_t> deg, cnt;
    uint64_t e = 0;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return SNN_ERR_CUDA;
    if (c->idx_bits != 32) return SNN_ERR_UNSUPPORTED;  // 32-bit slot ids
    try {
        deg.assign(n, 0);
        for (uint32_t chunks : {first_choice, 1u}) {
            c->sell_chunks = chunks;
            cnt.assign(nl * chunks, 0);
            e = 0;
            for (uint64_t i = 0; i < n; ++i) {
                for (uint64_t q = net->row_ptr[i]; q < net->row_ptr[i + 1]; ++q) {
                    const uint64_t t = net->col_idx[q];
                    if (t >= c->lo && t < c->hi) {
                        cnt[(t - c->lo) * chunks + (chunks > 1 ? i / chunk_neurons : 0)]++;
                        ++e;
                    }
                }
            }
            off = sell_offsets(cnt, nl, chunks);
            if (chunks == 1 || off.back() * 8 + (1ull << 30) < free_b) break;
        }
        for (uint64_t i = 0; i < n; ++i)
            for (uint64_t q = net->row_ptr[i]; q < net->row_ptr[i + 1]; ++q)
                deg[i] += (net->col_idx[q] >= c->lo && net->col_idx[q] < c->hi);
        const uint32_t chunks = c->sell_chunks;
        const bool relative = sell_relative(c);
        slot.assign(off.back(), (uint64_t)sell_pad_id(c));
        std::vector<uint32_t> fill(nl * chunks, 0);
        for (uint64_t i = 0; i < n; ++i) {
            const uint32_t ch = chunks > 1 ? (uint32_t)(i / chunk_neurons) : 0u;
            for (uint64_t q = net->row_ptr[i]; q < net->row_ptr[i + 1]; ++q) {
                const uint64_t t = net->col_idx[q];
                if (t >= c->lo && t < c->hi) {
                    const uint64_t tl = t - c->lo;
                    const uint64_t dst = off[(tl >> 5) * chunks + ch] + (uint64_t)fill[tl * chunks + ch]++ * 32 + (tl & 31);
                    uint32_t wb;
                    std::memcpy(&wb, &net->weights[q], 4);
                    slot[dst] = (uint64_t)wb << 32 | (uint32_t)(relative ? i - (uint64_t)ch * chunk_neurons : i);
                }
            }
        }
    } catch (const std::bad_alloc &) {
        return SNN_ERR_OUT_OF_MEMORY;
    }
    c->e_local = e;
    snn_status_t st;
    if ((st = alloc_sell(c, off)) != SNN_OK) return st;
    if ((st = h2d(c, c->d_pre, slot.data(), off.back() * 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_deg, n, 4)) != SNN_OK) return st;
    if ((st = h2d(c, c->d_deg, deg.data(), n * 4)) != SNN_OK) return st;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

uint64_t max_degree(const snn_network_t *net) {
    uint64_t m = 0;
    for (uint64_t i = 0; i < net->neuron_count; ++i) m = std::max<uint64_t>(m, net->row_ptr[i + 1] - net->row_ptr[i]);
    return m;
}

// Sharded STREAMING: copies the edges into [lo, hi) to host buffers (every
// row kept, CSR order, targets relative to lo) that the streaming code reads
// in place of the borrowed network.
snn_status_t make_stream_slice(snn_cuda_context_t *c, const snn_network_t *net) {
    const uint64_t n = net->neuron_count;
    uint64_t e = 0;
    for (uint64_t q = 0; q < net->synapse_count; ++q) e += (net->col_idx[q] >= c->lo && net->col_idx[q] < c->hi);
    auto alloc = [](uint64_t bytes) { return std::aligned_alloc(64, (bytes + 63) / 64 * 64 + 64); };
    c->h_slice_rp = (uint64_t *)alloc((n + 1) * 8);
    c->h_slice_col = (uint64_t *)alloc(e * 8);
    c->h_slice_w = (float *)alloc(e * 4);
    if (!c->h_slice_rp || !c->h_slice_col || !c->h_slice_w) return SNN_ERR_OUT_OF_MEMORY;
    uint64_t pos = 0;
    for (uint64_t i = 0; i < n; ++i) {
        c->h_slice_rp[i] = pos;
        for (uint64_t q = net->row_ptr[i]; q < net->row_ptr[i + 1]; ++q) {
            const uint64_t t = net->col_idx[q];
            if (t >= c->lo && t < c->hi) {
                c->h_slice_col[pos] = t - c->lo;
                c->h_slice_w[pos] = net->weights[q];
                ++pos;
            }
        }
    }
    c->h_slice_rp[n] = pos;
    c->slice_net = *net;
    c->slice_net.synapse_count = e;
    c->slice_net.row_ptr = c->h_slice_rp;
    c->slice_net.col_idx = c->h_slice_col;
    c->slice_net.weights = c->h_slice_w;
    c->network = &c->slice_net;
    c->e_local = e;
    return SNN_OK;
}

// STREAMING: chunk sizing follows the reference's rules
// (src/snn_cuda.cu:327-401): rows <= 65536 and <= n; auto rows take at most
// half of the budget left after the resident state; an explicit synapse cap
// below the densest row is INVALID_ARGUMENT; auto synapses fill the rest,
// clamped up to the densest row and down to the synapse count, minimum 1.
// Two copy slots are allocated (double buffering), so auto sizes are halved.
// Seams: #8 host chunk table (OUT_OF_MEMORY), #9-#11 chunk buffers.
snn_status_t allocate_streaming(snn_cuda_context_t *c, const snn_cuda_config_t &cfg, uint64_t budget) {
    const snn_network_t *net = c->network;
    const uint64_t n = net->neuron_count, e = net->synapse_count;
    const uint64_t maxdeg = max_degree(net);
    const uint64_t sb = state_bytes(c);
    const uint64_t avail = budget > sb ? budget - sb : 0;
    uint64_t rows = cfg.max_stream_rows ? cfg.max_stream_rows : n;
    rows = std::min<uint64_t>(std::min<uint64_t>(rows, 65536), n);
    if (cfg.max_stream_rows == 0) {
        const uint64_t max_rows = avail / 2 / 2 / 8;
        if (rows + 1 > max_rows) rows = max_rows > 1 ? max_rows - 1 : 1;
    }
    const uint64_t row_bytes = (rows + 1) * 8;
    uint64_t syn;
    if (cfg.max_stream_synapses != 0) {
        if (cfg.max_stream_synapses < maxdeg) return SNN_ERR_INVALID_ARGUMENT;
        syn = cfg.max_stream_synapses;
    } else {
        syn = avail > 2 * (row_bytes + 12) ? (avail - 2 * row_bytes) / (2 * 12) : 0;
        if (syn < maxdeg) syn = maxdeg;
    }
    if (syn > e) syn = e;
    if (syn == 0) syn = 1;
    if (seam_fail()) return SNN_ERR_OUT_OF_MEMORY;
    try {
        // Greedy row admission, as the reference's per-step loop does
        // (src/snn_cuda.cu:586-601); the schedule is fixed, so it is built once.
        uint64_t r = 0;
        while (r < n) {
            StreamChunk ch{r, 0, net->row_ptr[r], 0};
            uint64_t end = r;
            while (end < n && ch.rows < rows) {
                const uint64_t d = net->row_ptr[end + 1] - net->row_ptr[end];
                if (ch.rows != 0 && ch.edge_count + d > syn) break;
                ch.edge_count += d;
                ++end;
                ++ch.rows;
                if (ch.edge_count == syn) break;
            }
            c->chunks.push_back(ch);
            r = end;
        }
    } catch (const std::bad_alloc &) {
        return SNN_ERR_OUT_OF_MEMORY;
    }
    c->slot_rows = rows;
    c->slot_edges = syn;
    // Slot strides are multiples of 4 elements so every slot base keeps the
    // 16-byte alignment the vectorised edge loads rely on.
    c->slot_stride = (syn + 3) / 4 * 4;
    snn_status_t st;
    if ((st = dmalloc((void **)&c->d_chunk_row, 2 * (rows + 1), 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_chunk_col, 2 * c->slot_stride + 4, 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_chunk_w, 2 * c->slot_stride + 4, 4)) != SNN_OK) return st;
    if (cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess) return SNN_ERR_CUDA;
    for (int i = 0; i < 2; ++i) {
        if (cudaEventCreateWithFlags(&c->ev_copied[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_free[i], cudaEventDisableTiming) != cudaSuccess)
            return SNN_ERR_CUDA;
        cudaEventRecord(c->ev_free[i], c->stream);
    }
    // Page-lock the borrowed host CSR in place (best effort) so chunk copies
    // run asynchronously at full host-link speed; unregistered on free.
    const void *arrays[3] = {net->row_ptr, net->col_idx, net->weights};
    const uint64_t sizes[3] = {(n + 1) * 8, e * 8, e * 4};
    for (int i = 0; i < 3; ++i) {
        if (arrays[i] == nullptr || sizes[i] == 0) continue;
        // Read-only first: the device only reads the CSR, and a read-only
        // file mapping (snn_b200_network_map) can only be locked that way.
        if (cudaHostRegister(const_cast<void *>(arrays[i]), sizes[i], cudaHostRegisterReadOnly) == cudaSuccess ||
            (cudaGetLastError(),
             cudaHostRegister(const_cast<void *>(arrays[i]), sizes[i], cudaHostRegisterDefault) == cudaSuccess))
            c->registered[i] = arrays[i];
        else
            cudaGetLastError();
    }
    return SNN_OK;
}

// Sparse STREAMING: the host CSR's col_idx and weights are page-locked in
// place and mapped into the device address space; only row_ptr is resident.
// Each step the push kernel reads the spiking rows' edges straight from host
// memory over the host link (no chunk copies, no per-step work for silent
// rows). Falls back to chunked streaming if the arrays cannot be mapped.
snn_status_t allocate_sparse_streaming(snn_cuda_context_t *c, bool *fallback) {
    const snn_network_t *net = c->network;
    const uint64_t n = net->neuron_count, e = net->synapse_count;
    *fallback = false;
    const void *arrays[2] = {net->col_idx, net->weights};
    const uint64_t sizes[2] = {e * 8, e * 4};
    void *dev[2] = {nullptr, nullptr};
    for (int i = 0; i < 2 && e; ++i) {
        if ((uintptr_t)arrays[i] % 16 != 0 ||
            (cudaHostRegister(const_cast<void *>(arrays[i]), sizes[i],
                              cudaHostRegisterMapped | cudaHostRegisterPortable | cudaHostRegisterReadOnly) !=
                 cudaSuccess &&
             (cudaGetLastError(), cudaHostRegister(const_cast<void *>(arrays[i]), sizes[i],
                                                   cudaHostRegisterMapped | cudaHostRegisterPortable) !=
                                      cudaSuccess)) ||
            cudaHostGetDevicePointer(&dev[i], const_cast<void *>(arrays[i]), 0) != cudaSuccess) {
            cudaGetLastError();
            for (int k = 0; k < 2; ++k)
                if (c->registered[k + 1]) {
                    cudaHostUnregister(const_cast<void *>(c->registered[k + 1]));
                    c->registered[k + 1] = nullptr;
                }
            *fallback = true;
            return SNN_OK;
        }
        c->registered[i + 1] = arrays[i];
    }
    c->h_col_dev = (const uint64_t *)dev[0];
    c->h_w_dev = (const float *)dev[1];
    snn_status_t st;
    if ((st = dmalloc((void **)&c->d_row_ptr, n + 1, 8)) != SNN_OK) return st;
    if ((st = h2d(c, c->d_row_ptr, net->row_ptr, (n + 1) * 8)) != SNN_OK) return st;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

uint64_t full_push_bytes(const snn_cuda_context_t *c, uint64_t e) {
    return state_bytes(c) + (c->n_rows + 1) * 8 + e * (c->col_bits / 8 + 4);
}

struct CreateEnv {
    uint64_t budget = 0;
};

// Shared prologue: availability, device, memory info, context allocation
// (seam #0), streams, NCCL, device state (seams #1-#7).
snn_status_t begin_create(uint64_t n, const snn_lif_params_t &lif, float decay, const snn_cuda_config_t *config,
                          const snn_b200_options_t *options, snn_cuda_context_t **out, CreateEnv *env) {
    if (!snn_cuda_available()) return SNN_ERR_CUDA;
    const snn_b200_options_t o = options ? *options : snn_b200_default_options();
    const snn_cuda_config_t cfg = config ? *config : snn_cuda_default_config();
    int dev = o.device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) return SNN_ERR_CUDA;
    if (cudaSetDevice(dev) != cudaSuccess) return SNN_ERR_CUDA;
    size_t free_b = 0, total_b = 0;
    if (g_force_meminfo_fail || cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return SNN_ERR_CUDA;
    env->budget = (cfg.max_vram_bytes == 0 || cfg.max_vram_bytes > free_b) ? (uint64_t)free_b : cfg.max_vram_bytes;
    if (seam_fail()) return SNN_ERR_OUT_OF_MEMORY;
    snn_cuda_context_t *c = new (std::nothrow) snn_cuda_context();
    if (c == nullptr) return SNN_ERR_OUT_OF_MEMORY;
    c->device = dev;
    c->lif = lif;
    c->args = b200::LifArgs{decay, lif.v_rest, lif.v_reset, lif.v_threshold, lif.input_scale, lif.refractory_steps};
    snn_status_t st = apply_options(c, n, o);
    if (st == SNN_OK) st = create_streams(c);
    if (st == SNN_OK) st = init_nccl(c, o.nccl_id);
    if (st == SNN_OK) st = init_peer_exchange(c);
    if (st == SNN_OK) st = allocate_state(c);
    if (st != SNN_OK) {
        free_context(c);
        return st;
    }
    *out = c;
    return SNN_OK;
}

// Queues a copy of the device error word (raised by a bounded device wait
// that expired) behind the work already on the stream.
void queue_error_check(snn_cuda_context_t *c) {
    cudaMemcpyAsync(c->h_err, &c->d_ctr->error, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream);
}

snn_status_t error_after_sync(snn_cuda_context_t *c, snn_status_t st) {
    if (st == SNN_OK && c->h_err && *c->h_err) {
        set_error("device", *c->h_err == 3u ? "a peer's spike exchange flag did not arrive in time (bounded wait expired)"
                                            : "a bounded cross-CTA wait expired (propagation aborted)");
        return SNN_ERR_CUDA;
    }
    return st;
}

// --------------------------------------------------------------- timing --
TimingGroup *timing_begin(snn_cuda_context_t *c) {
    if (!c->timing) return nullptr;
    if (c->pool.empty()) {
        TimingGroup g;
        for (auto &e : g.ev) cudaEventCreate(&e);
        c->pool.push_back(g);
    }
    c->pending.push_back(c->pool.back());
    c->pool.pop_back();
    TimingGroup *g = &c->pending.back();
    g->seq = c->seq;
    cudaEventRecord(g->ev[0], c->stream);
    return g;
}

void timing_mark(snn_cuda_context_t *c, TimingGroup *g, int k) {
    if (g) cudaEventRecord(g->ev[k], c->stream);
}

void timing_fold(snn_cuda_context_t *c) {
    // Which steps ran a pull kernel (device-chosen): the step kind log, for
    // the steps still inside its ring.
    std::vector<uint8_t> kinds;
    if (!c->pending.empty() && c->d_kind_log) {
        kinds.resize(b200::kStepLog);
        if (cudaMemcpy(kinds.data(), c->d_kind_log, b200::kStepLog, cudaMemcpyDeviceToHost) != cudaSuccess)
            kinds.clear();
    }
    for (auto &g : c->pending) {
        float a = 0, b = 0, d = 0, t = 0;
        if (cudaEventElapsedTime(&a, g.ev[0], g.ev[1]) == cudaSuccess &&
            cudaEventElapsedTime(&b, g.ev[1], g.ev[2]) == cudaSuccess &&
            cudaEventElapsedTime(&d, g.ev[2], g.ev[3]) == cudaSuccess &&
            cudaEventElapsedTime(&t, g.ev[0], g.ev[3]) == cudaSuccess) {
            c->t_lif += a;
            c->t_exchange += b;
            c->t_prop += d;
            c->t_step += t;
            if (!kinds.empty() && c->seq - g.seq <= b200::kStepLog && kinds[g.seq % b200::kStepLog]) c->t_prop_pull += d;
        }
        c->pool.push_back(g);
    }
    c->pending.clear();
    cudaGetLastError();
}

// --------------------------------------------------------------- step ----
// Phase 1 of a step: LIF (writing this rank's bitmap words; with the peer
// exchange, followed by the flag publication) and the early spike download.
snn_status_t step_lif(snn_cuda_context_t *c, bool has_ext) {
    StepState &ps = c->ps;
    ps = StepState{};
    ps.parity = (int)(c->step & 1u);
    const int parity = ps.parity;
    float *cur = c->d_cur[c->cur];
    ps.next = c->d_cur[c->cur ^ 1];
    ps.tg = timing_begin(c);
    TimingGroup *tg = ps.tg;
    const bool sharded = ps.sharded = c->world > 1;
    ps.own_bitmap = c->d_bitmap + (uint64_t)c->rank * (c->slot / 32);
    const bool peer = ps.peer = sharded && c->exchange == SNN_B200_EXCHANGE_PEER;
    if (peer && !c->peers_connected) {
        set_error("snn_b200", "peer exchange used before snn_b200_ipc_connect");
        return SNN_ERR_INVALID_ARGUMENT;
    }
    b200::PeerWait &pw = ps.pw;
    if (peer) {
        // Pull exchange: LIF writes this rank's words into its own buffer of
        // this parity, a one-CTA kernel behind it releases this rank's flag
        // at every rank; the compaction waits for every flag and reads the
        // other ranks' words over NVLink.
        ++c->xstep;
        const uint64_t par = c->xstep & 1u;
        for (uint32_t r = 0; r < c->world; ++r) {
            pw.publish[r] = (unsigned long long *)((char *)c->peer_x[r] + xflags_offset(c)) + c->rank;
            pw.src[r] = c->peer_x[r] + par * c->bitmap_words;
        }
        ps.xbitmap = (uint32_t *)c->d_xbuf + par * c->bitmap_words;
        ps.own_bitmap = ps.xbitmap + (uint64_t)c->rank * (c->slot / 32);
        pw.flags = (const unsigned long long *)((char *)c->d_xbuf + xflags_offset(c));
        pw.tag = c->xstep;
        pw.nflags = c->world;
        pw.spin_limit = c->peer_spin_limit;
        pw.slot_words = c->slot / 32;
        pw.rank = c->rank;
    }
    b200::LifArgs lif_args = c->args;
    if (c->dev_stream_step) lif_args.stream_step = &c->d_ctr->stream_step;
    // The bin-fold needs an ascending spike list: the ordered compaction
    // below builds it from the bitmap, so LIF writes no list then.
    const bool ordered_list = ps.ordered_list = c->binfold && c->mode == SNN_CUDA_MODE_FULL;
    b200::launch_lif(c->stream, c->device, c->n_local, lif_args, c->d_v, cur, has_ext ? c->d_ext : nullptr, c->d_refr,
                     c->d_spikes, ps.own_bitmap, (sharded || ordered_list) ? nullptr : c->d_list, c->idx_bits, c->lo,
                     c->d_ctr, parity);
    snn_status_t st = check_launch(c);
    if (st != SNN_OK) return st;
    if (peer) {
        b200::launch_publish_flags(c->stream, pw);
        c->launches++;
    }
    timing_mark(c, tg, 1);
    if (c->spk_dst != nullptr) {
        // The spikes are final once LIF is done; download them while the
        // propagation runs. The main stream waits for the copy at the end of
        // the step (the next LIF overwrites d_spikes).
        cudaEventRecord(c->ev_lif, c->stream);
        cudaStreamWaitEvent(c->spk_stream, c->ev_lif, 0);
        if (cudaMemcpyAsync(c->spk_dst, c->d_spikes, c->n_local, cudaMemcpyDeviceToHost, c->spk_stream) !=
            cudaSuccess)
            return SNN_ERR_CUDA;
        cudaEventRecord(c->ev_spk, c->spk_stream);
    }
    ps.brows = c->batch > 1 ? c->n_rows : 0;
    return SNN_OK;
}

// Phase 2: the NCCL all-gather of the bitmap (NCCL exchange only). Several
// ranks driven from one thread issue theirs inside one NCCL group.
snn_status_t step_exchange(snn_cuda_context_t *c) {
    const StepState &ps = c->ps;
    if (!ps.sharded || ps.peer) return SNN_OK;
    const ncclResult_t r = ncclAllGather(ps.own_bitmap, c->d_bitmap, c->slot / 32, ncclUint32, c->comm, c->stream);
    if (r != ncclSuccess) {
        set_error("ncclAllGather", ncclGetErrorString(r));
        return SNN_ERR_CUDA;
    }
    return SNN_OK;
}

// Phase 3: compaction (the global spike list; with the peer exchange after
// the flag waits and the NVLink gather). Ranks driven from one thread
// enqueue every compaction before any propagation: a propagation may wait on
// the host (ORDERED's event count).
snn_status_t step_compact(snn_cuda_context_t *c) {
    StepState &ps = c->ps;
    const int parity = ps.parity;
    TimingGroup *tg = ps.tg;
    const bool sharded = ps.sharded, peer = ps.peer, ordered_list = ps.ordered_list;
    uint32_t *xbitmap = ps.xbitmap;
    const b200::PeerWait &pw = ps.pw;
    const uint64_t brows = ps.brows;
    snn_status_t st = SNN_OK;
    if (ordered_list) {
        // Ascending spike list (and the step's event total) from the bitmap:
        // gathered from the peers (after the flag waits), assembled by the
        // NCCL all-gather, or this rank's own.
        b200::launch_compact_ordered(c->stream, c->device, peer ? xbitmap : c->d_bitmap, c->bitmap_words,
                                     c->bfb.ccnt, c->d_list, c->idx_bits, c->d_ctr, parity, c->lo / 32,
                                     ceil_div(c->hi, 32), c->d_row_ptr, brows, peer ? &pw : nullptr);
        c->launches += 2;
        if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
    } else if (peer) {
        // The compaction waits for all flags of this step and gathers the
        // other ranks' words into the local buffer as it compacts.
        b200::launch_compact(c->stream, c->device, xbitmap, c->bitmap_words, c->d_list, c->idx_bits, c->d_ctr,
                             parity, c->lo / 32, ceil_div(c->hi, 32), &pw);
        c->launches++;
        if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
    } else if (sharded) {
        b200::launch_compact(c->stream, c->device, c->d_bitmap, c->bitmap_words, c->d_list, c->idx_bits, c->d_ctr,
                             parity, c->lo / 32, ceil_div(c->hi, 32));
        c->launches++;
        if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
    }
    timing_mark(c, tg, 2);
    return SNN_OK;
}

// Phase 4: propagation and buffer swap.
snn_status_t step_propagate(snn_cuda_context_t *c) {
    StepState &ps = c->ps;
    const int parity = ps.parity;
    float *next = ps.next;
    TimingGroup *tg = ps.tg;
    const bool sharded = ps.sharded, peer = ps.peer;
    uint32_t *xbitmap = ps.xbitmap;
    const uint64_t brows = ps.brows;
    snn_status_t st = SNN_OK;
    if (c->mode == SNN_CUDA_MODE_FULL) {
        if (c->binfold) {
            const cudaError_t e = b200::launch_binfold(c->stream, c->device, c->bf, c->bfb, c->d_list, c->idx_bits,
                                                       c->d_row_ptr, c->d_col, c->col_bits, c->d_w, brows,
                                                       c->n_local, next, c->d_ctr, parity, c->bf_gate);
            c->launches += 5;  // count, scan (two), scatter, fold
            if (e != cudaSuccess) return cuda_status(e);
            if (c->has_csc) {
                // Dense steps (more than bf_gate events) take the pull instead.
                b200::launch_propagate_pull(c->stream, c->device, c->n_local, c->sell_chunks, c->sell_chunk_words,
                                            c->d_sell_off, (const uint2 *)c->d_pre, peer ? xbitmap : c->d_bitmap,
                                            c->bitmap_words, next, c->d_list, c->idx_bits, c->d_deg, c->d_ctr,
                                            parity, 0, 0, 1, c->bf_gate);
                c->launches++;
            }
        } else if (c->propagation == SNN_B200_PROPAGATE_ORDERED && !c->opull) {
            if ((st = ordered_push_step(c, parity, next, sharded, peer ? xbitmap : c->d_bitmap, c->d_row_ptr, c->d_col,
                                        c->col_bits, c->d_w)) != SNN_OK)
                return st;
        } else if (c->propagation == SNN_B200_PROPAGATE_ORDERED)
            b200::launch_propagate_pull(c->stream, c->device, c->n_local, c->sell_chunks, c->sell_chunk_words,
                                    c->d_sell_off, (const uint2 *)c->d_pre,
                                         peer ? xbitmap : c->d_bitmap, c->bitmap_words, next, c->d_list, c->idx_bits,
                                        c->d_deg, c->d_ctr, parity, !sharded);
        else {
            if (c->push_lanes == 0) {
                // From the average row length of this rank's topology;
                // SNN_B200_PUSH_LANES (environment: 8, 16 or 32) overrides it.
                c->push_lanes = b200::push_lanes(c->e_local, c->n_rows);
                if (const char *env = std::getenv("SNN_B200_PUSH_LANES")) c->push_lanes = (uint32_t)std::atoi(env);
            }
            // With a SELL CSC both kernels are launched behind the same
            // device-side gate on this step's spike count: one of them runs.
            b200::launch_propagate_push(c->stream, c->device, c->d_list, c->idx_bits, c->d_row_ptr, c->d_col,
                                        c->col_bits, c->d_w, next, c->d_ctr, parity, !sharded,
                                        c->batch > 1 ? c->n_rows : 0, c->has_csc ? c->pull_above : 0,
                                        c->push_lanes);
            if (c->has_csc) {
                b200::launch_propagate_pull(c->stream, c->device, c->n_local, c->sell_chunks, c->sell_chunk_words,
                                    c->d_sell_off, (const uint2 *)c->d_pre,
                                             peer ? xbitmap : c->d_bitmap, c->bitmap_words, next, c->d_list, c->idx_bits,
                                            c->d_deg, c->d_ctr, parity, !sharded, c->pull_above);
                c->launches++;
            }
        }
        if ((st = check_launch(c)) != SNN_OK) return st;
    } else if (c->propagation == SNN_B200_PROPAGATE_ORDERED && c->streaming == SNN_B200_STREAMING_SPARSE) {
        // Bit-exact sparse STREAMING: the event sort over the mapped host CSR.
        if ((st = ordered_push_step(c, parity, next, sharded, peer ? xbitmap : c->d_bitmap, c->d_row_ptr,
                                    c->h_col_dev, 64, c->h_w_dev)) != SNN_OK)
            return st;
    } else if (c->propagation == SNN_B200_PROPAGATE_ORDERED) {
        if ((st = ordered_stream_chunked(c, parity, next, sharded)) != SNN_OK) return st;
    } else if (c->streaming == SNN_B200_STREAMING_SPARSE) {
        // Sparse STREAMING: spiking rows read straight from mapped host memory.
        b200::launch_propagate_push(c->stream, c->device, c->d_list, c->idx_bits, c->d_row_ptr, c->h_col_dev, 64,
                                    c->h_w_dev, next, c->d_ctr, parity, !sharded);
        if ((st = check_launch(c)) != SNN_OK) return st;
    } else {
        // STREAMING: chunk i uses copy slot i&1; its copies wait until the
        // propagation that last used the slot is done, and its propagation
        // waits for its copies, so copy i+1 overlaps propagation i.
        const snn_network_t *net = c->network;
        for (size_t i = 0; i < c->chunks.size(); ++i) {
            const StreamChunk &ch = c->chunks[i];
            const int s = (int)(i & 1u);
            uint64_t *drow = c->d_chunk_row + (uint64_t)s * (c->slot_rows + 1);
            uint64_t *dcol = c->d_chunk_col + (uint64_t)s * c->slot_stride;
            float *dw = c->d_chunk_w + (uint64_t)s * c->slot_stride;
            cudaStreamWaitEvent(c->copy_stream, c->ev_free[s], 0);
            if (seam_fail()) return SNN_ERR_CUDA;
            if (cudaMemcpyAsync(drow, net->row_ptr + ch.row_begin, (ch.rows + 1) * 8, cudaMemcpyHostToDevice,
                                c->copy_stream) != cudaSuccess)
                return SNN_ERR_CUDA;
            if (ch.edge_count) {
                if (seam_fail()) return SNN_ERR_CUDA;
                if (cudaMemcpyAsync(dcol, net->col_idx + ch.edge_begin, ch.edge_count * 8, cudaMemcpyHostToDevice,
                                    c->copy_stream) != cudaSuccess)
                    return SNN_ERR_CUDA;
                if (seam_fail()) return SNN_ERR_CUDA;
                if (cudaMemcpyAsync(dw, net->weights + ch.edge_begin, ch.edge_count * 4, cudaMemcpyHostToDevice,
                                    c->copy_stream) != cudaSuccess)
                    return SNN_ERR_CUDA;
            }
            cudaEventRecord(c->ev_copied[s], c->copy_stream);
            cudaStreamWaitEvent(c->stream, c->ev_copied[s], 0);
            b200::launch_propagate_chunk(c->stream, c->device, ch.row_begin, ch.rows, ch.edge_begin,
                                         peer ? xbitmap : c->d_bitmap, drow, dcol, dw, next, c->d_ctr, parity,
                                         i == 0, !sharded);
            if ((st = check_launch(c)) != SNN_OK) return st;
            cudaEventRecord(c->ev_free[s], c->stream);
        }
    }
    if (c->spk_dst != nullptr) cudaStreamWaitEvent(c->stream, c->ev_spk, 0);
    timing_mark(c, tg, 3);
    c->cur ^= 1;
    c->step++;
    c->seq++;
    return SNN_OK;
}

// The device part of one step (the three phases in a row), enqueued on
// c->stream. Seams: #1 integrate launch, #2 propagate launch (or the
// per-chunk copies and launches in STREAMING).
snn_status_t enqueue_step(snn_cuda_context_t *c, bool has_ext) {
    snn_status_t st = step_lif(c, has_ext);
    if (st == SNN_OK) st = step_exchange(c);
    if (st == SNN_OK) st = step_compact(c);
    if (st == SNN_OK) st = step_propagate(c);
    return st;
}

// Bits that cover every global index (the injection sort's key width).
int inject_key_bits(const snn_cuda_context_t *c) {
    int bits = 1;
    while (bits < 64 && (1ull << bits) < c->n_global) ++bits;
    return bits;
}

snn_status_t ensure_inject_capacity(snn_cuda_context_t *c, uint64_t count) {
    if (count <= c->inj_cap) return SNN_OK;
    cudaStreamSynchronize(c->stream);
    cudaFree(c->d_inj_idx);
    cudaFree(c->d_inj_val);
    c->d_inj_idx = nullptr;
    c->d_inj_val = nullptr;
    c->inj_cap = 0;
    size_t tmp = 0;
    if (b200::sort_pairs_u64_f32(c->stream, nullptr, nullptr, nullptr, nullptr, count, inject_key_bits(c), nullptr,
                                 &tmp, nullptr) != cudaSuccess)
        return SNN_ERR_CUDA;
    // Values and their alternate (2 x count floats), the scratch from the
    // next 256-byte boundary.
    const uint64_t val_bytes = (count * 8 + 255) & ~255ull;
    snn_status_t st;
    if ((st = dmalloc((void **)&c->d_inj_idx, count * 2, 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_inj_val, val_bytes + tmp, 1)) != SNN_OK) return st;
    c->inj_tmp_bytes = tmp;
    c->inj_cap = count;
    return SNN_OK;
}

// Device generation of the edges that target [rlo, rhi) (global ids) into a
// push CSR with columns relative to rlo. The whole network takes the dense
// path (row_ptr is i * fanout); a sub-range counts per row, scans, and fills.
snn_status_t generate_range(snn_cuda_context_t *c, const b200::GenParams &g, uint64_t e_total, uint64_t rlo,
                            uint64_t rhi, uint64_t **d_row, void **d_col, float **d_w, uint64_t *edges) {
    snn_status_t st;
    const uint64_t n = g.n;
    if ((st = dmalloc((void **)d_row, n + 1, 8)) != SNN_OK) return st;
    uint64_t e = e_total;
    const bool whole = rlo == 0 && rhi == n;
    if (!whole) {
        uint64_t *counts = nullptr;
        if (cudaMalloc(&counts, (n + 1) * 8) != cudaSuccess) return SNN_ERR_CUDA;
        cudaMemsetAsync(counts, 0, (n + 1) * 8, c->stream);
        b200::launch_gen_count_shard(c->stream, c->device, g, rlo, rhi, counts);
        size_t tb = 0;
        b200::exclusive_scan_u64(c->stream, counts, *d_row, n + 1, nullptr, &tb);
        void *tmp = nullptr;
        if (cudaMalloc(&tmp, tb ? tb : 1) != cudaSuccess) {
            cudaFree(counts);
            return SNN_ERR_CUDA;
        }
        st = cuda_status(b200::exclusive_scan_u64(c->stream, counts, *d_row, n + 1, tmp, &tb));
        if (st == SNN_OK) st = cuda_status(cudaMemcpyAsync(&e, *d_row + n, 8, cudaMemcpyDeviceToHost, c->stream));
        if (st == SNN_OK) st = cuda_status(cudaStreamSynchronize(c->stream));
        cudaFree(tmp);
        cudaFree(counts);
        if (st != SNN_OK) return st;
    } else {
        b200::launch_gen_row_ptr_dense(c->stream, c->device, g, *d_row);
    }
    *edges = e;
    if ((st = dmalloc(d_col, e ? e + 16 / (c->col_bits / 8) : 0, c->col_bits / 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)d_w, e ? e + 4 : 0, 4)) != SNN_OK) return st;
    if (!whole) {
        b200::launch_gen_fill_shard(c->stream, c->device, g, rlo, rhi, *d_row, *d_col, c->col_bits, *d_w);
        if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
    } else {
        // Bounded launches (<= 2^30 edges each) keep every kernel short.
        const uint64_t step = 1ull << 30;
        for (uint64_t e0 = 0; e0 < e; e0 += step) {
            b200::launch_gen_edges_dense(c->stream, c->device, g, e0, std::min(e, e0 + step), *d_col, c->col_bits,
                                         *d_w);
            if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
        }
    }
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t generate_full(snn_cuda_context_t *c, const b200::GenParams &g, uint64_t e_total) {
    uint64_t e = 0;
    const snn_status_t st =
        generate_range(c, g, e_total, c->lo, std::min(c->hi, c->n_rows), &c->d_row_ptr, &c->d_col, &c->d_w, &e);
    c->e_local = e;
    return st;
}

// ORDERED for a device-generated network: build the CSC the ordered pull
// kernel folds over directly on the device, never materialising the CSR.
// col_ptr is the scan of the local targets' in-degrees. The edges are then
// produced in passes over local target ranges sized to the free memory: each
// pass generates (target - range start, global edge id) pairs in CSR order
// and stable-radix-sorts them by target, so every target's in-edges keep
// ascending edge id = CSR order = the serial CPU fold order
// (src/snn.c:898-906). The presynaptic row is id / fanout and the weight is
// recomputed from the id, bit-identical to snn_build_random_pool.
snn_status_t build_generated_csc(snn_cuda_context_t *c, const b200::GenParams &g) {
    const uint64_t n = g.n, nl = c->n_local, lo = c->lo;
    snn_status_t st;
    if (c->idx_bits != 32) return SNN_ERR_UNSUPPORTED;  // 32-bit slot ids
    if ((st = dmalloc((void **)&c->d_col_ptr, nl + 1, 8)) != SNN_OK) return st;
    if ((st = dmalloc((void **)&c->d_deg, n, 4)) != SNN_OK) return st;
    {
        unsigned long long *indeg = nullptr;
        void *tmp = nullptr;
        size_t tb = 0;
        if (cudaMalloc(&indeg, (nl + 1) * 8) != cudaSuccess) return SNN_ERR_OUT_OF_MEMORY;
        cudaMemsetAsync(indeg, 0, (nl + 1) * 8, c->stream);
        b200::launch_gen_indegree(c->stream, c->device, g, lo, lo + nl, indeg);
        b200::exclusive_scan_u64(c->stream, (const uint64_t *)indeg, c->d_col_ptr, nl + 1, nullptr, &tb);
        if (cudaMalloc(&tmp, tb ? tb : 1) != cudaSuccess) {
            cudaFree(indeg);
            return SNN_ERR_OUT_OF_MEMORY;
        }
        st = cuda_status(b200::exclusive_scan_u64(c->stream, (const uint64_t *)indeg, c->d_col_ptr, nl + 1, tmp, &tb));
        cudaStreamSynchronize(c->stream);
        cudaFree(tmp);
        cudaFree(indeg);
        if (st != SNN_OK) return st;
    }
    b200::launch_gen_count_shard_u32(c->stream, c->device, g, lo, lo + nl, c->d_deg);
    std::vector<uint64_t> col_ptr;
    try {
        col_ptr.resize(nl + 1);
    } catch (const std::bad_alloc &) {
        return SNN_ERR_OUT_OF_MEMORY;
    }
    if ((st = cuda_status(cudaMemcpy(col_ptr.data(), c->d_col_ptr, (nl + 1) * 8, cudaMemcpyDeviceToHost))) != SNN_OK)
        return st;
    const uint64_t e = col_ptr[nl];
    c->e_local = e;
    // Chunked layout when it fits with room left for fast build passes, else
    // one chunk (lookups through L1/L2).
    uint32_t *cnt = nullptr;
    const uint64_t blocks = (nl + 31) / 32;
    for (uint32_t chunks : {choose_chunks(c), 1u}) {
        c->sell_chunks = chunks;
        const uint64_t chunk_neurons = chunks > 1 ? c->sell_chunk_words * 32u : UINT64_MAX;
        uint64_t *slots = nullptr;
        void *tmp = nullptr;
        size_t tb = 0;
        if (cudaMalloc(&cnt, (nl ? nl : 1) * chunks * 4) != cudaSuccess ||
            cudaMalloc(&slots, (blocks * chunks + 1) * 8) != cudaSuccess ||
            cudaMalloc(&c->d_sell_off, (blocks * chunks + 1) * 8) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(cnt);
            cudaFree(slots);
            return SNN_ERR_OUT_OF_MEMORY;
        }
        cudaMemsetAsync(cnt, 0, (nl ? nl : 1) * chunks * 4, c->stream);
        cudaMemsetAsync(slots, 0, (blocks * chunks + 1) * 8, c->stream);
        b200::launch_gen_chunk_counts(c->stream, c->device, g, lo, lo + nl, chunks, chunk_neurons, cnt);
        b200::launch_sell_slots(c->stream, c->device, cnt, nl, chunks, slots);
        b200::exclusive_scan_u64(c->stream, slots, c->d_sell_off, blocks * chunks + 1, nullptr, &tb);
        if (cudaMalloc(&tmp, tb ? tb : 1) == cudaSuccess)
            st = cuda_status(b200::exclusive_scan_u64(c->stream, slots, c->d_sell_off, blocks * chunks + 1, tmp, &tb));
        else
            st = SNN_ERR_OUT_OF_MEMORY;
        uint64_t total = 0;
        if (st == SNN_OK)
            st = cuda_status(cudaMemcpyAsync(&total, c->d_sell_off + blocks * chunks, 8, cudaMemcpyDeviceToHost,
                                             c->stream));
        if (st == SNN_OK) st = cuda_status(cudaStreamSynchronize(c->stream));
        cudaFree(tmp);
        cudaFree(slots);
        size_t free_b = 0, total_b = 0;
        if (st == SNN_OK) st = cuda_status(cudaMemGetInfo(&free_b, &total_b));
        const bool fits = total * 8 + (8ull << 30) < free_b;
        if (st == SNN_OK && (fits || chunks == 1)) {
            st = alloc_sell_slots(c, total);
            break;
        }
        cudaFree(cnt);
        cudaFree(c->d_sell_off);
        cnt = nullptr;
        c->d_sell_off = nullptr;
        if (st != SNN_OK) return st;
    }
    if (st != SNN_OK || e == 0) {
        cudaFree(cnt);
        return st != SNN_OK ? st : cuda_status(cudaStreamSynchronize(c->stream));
    }

    // Pass size: what fits in the free memory at 24 B per edge (keys and ids,
    // double-buffered) plus the per-pass row offsets and sort workspace.
    size_t free_b = 0, total_b = 0;
    if ((st = cuda_status(cudaMemGetInfo(&free_b, &total_b))) != SNN_OK) return st;
    const uint64_t fixed = 2 * (n + 1) * 8 + (512ull << 20);
    if (free_b <= fixed) {
        set_error("ordered CSC build", "no device memory left for the sort passes");
        return SNN_ERR_OUT_OF_MEMORY;
    }
    uint64_t cap = (free_b - fixed) / 26;
    // SNN_B200_CSC_PASS_EDGES (environment) caps the pass size, for tests.
    if (const char *env = std::getenv("SNN_B200_CSC_PASS_EDGES")) {
        const uint64_t v = std::strtoull(env, nullptr, 10);
        if (v) cap = std::min(cap, v);
    }
    uint64_t max_in = 0;
    for (uint64_t t = 0; t < nl; ++t) max_in = std::max(max_in, col_ptr[t + 1] - col_ptr[t]);
    if (cap < max_in) {
        set_error("ordered CSC build", "one target's in-edges exceed the sort pass memory");
        return SNN_ERR_OUT_OF_MEMORY;
    }
    std::vector<uint64_t> cuts{0};  // pass boundaries in local targets
    uint64_t pass_max = 0;
    while (cuts.back() < nl) {
        const uint64_t a = cuts.back();
        // Largest b with col_ptr[b] - col_ptr[a] <= cap.
        const uint64_t b = (uint64_t)(std::upper_bound(col_ptr.begin() + a, col_ptr.end(), col_ptr[a] + cap) -
                                      col_ptr.begin()) - 1;
        cuts.push_back(std::max(b, a + 1));
        pass_max = std::max(pass_max, col_ptr[cuts.back()] - col_ptr[a]);
    }
    uint32_t *keys = nullptr, *keys_alt = nullptr;
    uint64_t *ids = nullptr, *ids_alt = nullptr, *counts = nullptr, *row_off = nullptr;
    void *temp = nullptr;
    size_t temp_bytes = 0, scan_bytes = 0;
    bool alt = false;
    b200::sort_pairs_u32_u64(c->stream, nullptr, nullptr, nullptr, nullptr, pass_max, 32, nullptr, &temp_bytes,
                             &alt);
    b200::exclusive_scan_u64(c->stream, nullptr, nullptr, n + 1, nullptr, &scan_bytes);
    temp_bytes = std::max(temp_bytes, scan_bytes);
    if (cudaMalloc(&keys, pass_max * 4) != cudaSuccess || cudaMalloc(&keys_alt, pass_max * 4) != cudaSuccess ||
        cudaMalloc(&ids, pass_max * 8) != cudaSuccess || cudaMalloc(&ids_alt, pass_max * 8) != cudaSuccess ||
        cudaMalloc(&counts, (n + 1) * 8) != cudaSuccess || cudaMalloc(&row_off, (n + 1) * 8) != cudaSuccess ||
        cudaMalloc(&temp, temp_bytes ? temp_bytes : 1) != cudaSuccess) {
        set_error("ordered CSC build", "out of device memory for the sort passes");
        st = SNN_ERR_OUT_OF_MEMORY;
    }
    for (size_t p = 0; p + 1 < cuts.size() && st == SNN_OK; ++p) {
        const uint64_t a = cuts[p], b = cuts[p + 1];
        const uint64_t ep = col_ptr[b] - col_ptr[a];
        if (ep == 0) continue;
        cudaMemsetAsync(counts, 0, (n + 1) * 8, c->stream);
        b200::launch_gen_count_shard(c->stream, c->device, g, lo + a, lo + b, counts);
        size_t tb = temp_bytes;
        if ((st = cuda_status(b200::exclusive_scan_u64(c->stream, counts, row_off, n + 1, temp, &tb))) != SNN_OK)
            break;
        b200::launch_gen_fill_keys(c->stream, c->device, g, lo + a, lo + b, row_off, keys, ids);
        int end_bit = 1;
        while (end_bit < 32 && (1ull << end_bit) < b - a) ++end_bit;
        tb = temp_bytes;
        if ((st = cuda_status(b200::sort_pairs_u32_u64(c->stream, keys, keys_alt, ids, ids_alt, ep, end_bit, temp,
                                                       &tb, &alt))) != SNN_OK)
            break;
        b200::launch_gather_generated_sell(c->stream, c->device, g, alt ? keys_alt : keys, alt ? ids_alt : ids, ep,
                                           a, col_ptr[a], c->d_col_ptr, cnt, c->sell_chunks,
                                           c->sell_chunks > 1 ? c->sell_chunk_words * 32u : UINT64_MAX,
                                           sell_relative(c) ? 1 : 0, c->d_sell_off, (uint2 *)c->d_pre);
        st = cuda_status(cudaGetLastError());
    }
    if (st == SNN_OK) st = cuda_status(cudaStreamSynchronize(c->stream));
    cudaFree(keys);
    cudaFree(keys_alt);
    cudaFree(ids);
    cudaFree(ids_alt);
    cudaFree(counts);
    cudaFree(row_off);
    cudaFree(temp);
    cudaFree(cnt);
    return st;
}

// FULL contexts keep a sliced-ELL CSC beside the push CSR when the device
// has room for it (and for a working margin): dense steps then take the pull,
// which reads every local synapse once instead of one atomic (PUSH) or one
// sorted event (ORDERED) per event. ORDERED decides per step from the exact
// event count (events > local synapses / SNN_B200_ORDERED_PULL_DIV, default
// 10); PUSH decides on the device from the spike count (spikes > rows /
// SNN_B200_PUSH_PULL_DIV, default 4), launching both kernels behind the same
// gate so no host round trip is added. A divisor of 0 disables the pull.
snn_status_t add_pull_topology(snn_cuda_context_t *c, const snn_network_t *net, const b200::GenParams *g) {
    const bool ordered = c->propagation == SNN_B200_PROPAGATE_ORDERED;
    if (!ordered && (c->propagation != SNN_B200_PROPAGATE_PUSH || c->mode != SNN_CUDA_MODE_FULL))
        return SNN_OK;
    // Measured at config 2 on B200: the pull takes ~16 ms whatever the
    // firing; the ordered push costs about as much at ~1e9 events, the
    // atomic push at ~2.5e9 (25% firing at fanout 1000).
    uint64_t div = ordered ? 3 : 4;
    if (const char *env = std::getenv(ordered ? "SNN_B200_ORDERED_PULL_DIV" : "SNN_B200_PUSH_PULL_DIV"))
        div = std::strtoull(env, nullptr, 10);
    c->pull_div = div;
    if (div == 0 || c->e_local == 0 || c->batch > 1 || c->idx_bits != 32) return SNN_OK;
    // PUSH launches the gated pull kernel every step (a few microseconds even
    // when it exits at once): small networks, where that is a visible share
    // of a step and a dense step is cheap anyway, keep the plain push.
    // SNN_B200_PUSH_PULL_MIN_SYNAPSES (environment) moves the bound (tests).
    uint64_t min_syn = 1ull << 26;
    if (const char *env = std::getenv("SNN_B200_PUSH_PULL_MIN_SYNAPSES")) min_syn = std::strtoull(env, nullptr, 10);
    if (!ordered && c->e_local < min_syn) return SNN_OK;
    if (!ordered && c->n_rows / div > 0xffffffffull) return SNN_OK;
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return SNN_ERR_CUDA;
    // Padding of the sliced ELL: about 1.07x at fan-in 1000; budget 1.15x.
    const uint64_t sell = (uint64_t)((double)c->e_local * 1.15) * 8 + (c->n_local + 1) * 8 +
                          c->n_global * 4;
    const uint64_t reserve = (2 * (c->n_rows + 1) * 8) + (4ull << 30);  // build scratch + working margin
    if (sell + reserve > free_b) return SNN_OK;  // no room: every step takes the push
    const uint64_t e_push = c->e_local;
    snn_status_t st = net ? upload_full_ordered(c, net) : build_generated_csc(c, *g);
    if (st == SNN_ERR_OUT_OF_MEMORY) {  // the estimate was short: go on without the pull
        free_sell(c);
        c->e_local = e_push;
        return SNN_OK;
    }
    if (st != SNN_OK) return st;
    if (c->e_local != e_push) {
        set_error("pull topology", "CSC and CSR synapse counts differ");
        return SNN_ERR_CUDA;
    }
    if (c->d_col_ptr) {  // only the build needs the column pointers
        cudaFree(c->d_col_ptr);
        c->d_col_ptr = nullptr;
    }
    c->has_csc = true;
    if (!ordered) c->pull_above = (uint32_t)std::max<uint64_t>(1, c->n_rows / div);
    return SNN_OK;
}

// STREAMING for a device-generated network (config prefer_streaming, or a
// topology larger than the VRAM budget): the rank's slice (targets relative
// to its first neuron, 64-bit) is generated on the device in scratch memory,
// copied into host memory owned by the context, released on the device, and
// then streamed every step like a host network's slice. Each rank of a
// sharded run thus holds and streams only its own slice.
snn_status_t generate_streaming(snn_cuda_context_t *c, const b200::GenParams &g, uint64_t e_total,
                                const snn_cuda_config_t &cfg, uint64_t budget) {
    const uint64_t n = g.n;
    c->col_bits = 64;
    uint64_t *d_row = nullptr;
    void *d_col = nullptr;
    float *d_w = nullptr;
    uint64_t e = 0;
    snn_status_t st = generate_range(c, g, e_total, c->lo, std::min(c->hi, c->n_rows), &d_row, &d_col, &d_w, &e);
    auto alloc = [](uint64_t bytes) { return std::aligned_alloc(64, (bytes + 63) / 64 * 64 + 64); };
    if (st == SNN_OK) {
        c->h_slice_rp = (uint64_t *)alloc((n + 1) * 8);
        c->h_slice_col = (uint64_t *)alloc(e * 8);
        c->h_slice_w = (float *)alloc(e * 4);
        if (!c->h_slice_rp || !c->h_slice_col || !c->h_slice_w) st = SNN_ERR_OUT_OF_MEMORY;
    }
    if (st == SNN_OK) st = cuda_status(cudaMemcpy(c->h_slice_rp, d_row, (n + 1) * 8, cudaMemcpyDeviceToHost));
    if (st == SNN_OK && e) st = cuda_status(cudaMemcpy(c->h_slice_col, d_col, e * 8, cudaMemcpyDeviceToHost));
    if (st == SNN_OK && e) st = cuda_status(cudaMemcpy(c->h_slice_w, d_w, e * 4, cudaMemcpyDeviceToHost));
    cudaFree(d_row);
    cudaFree(d_col);
    cudaFree(d_w);
    if (st != SNN_OK) return st;
    snn_network_t &sn = c->slice_net;
    sn.neuron_count = n;
    sn.synapse_count = e;
    sn.architecture = g.recurrent ? SNN_ARCH_RANDOM_POOL : SNN_ARCH_CUSTOM_CSR;
    sn.lif = c->lif;
    sn.decay = c->args.decay;
    sn.row_ptr = c->h_slice_rp;
    sn.col_idx = c->h_slice_col;
    sn.weights = c->h_slice_w;
    c->network = &sn;
    c->e_local = e;
    c->mode = SNN_CUDA_MODE_STREAMING;
    bool fallback = true;
    if (c->streaming == SNN_B200_STREAMING_SPARSE && (st = allocate_sparse_streaming(c, &fallback)) != SNN_OK)
        return st;
    if (fallback) {
        c->streaming = SNN_B200_STREAMING_CHUNKED;
        st = allocate_streaming(c, cfg, budget);
    }
    return st;
}

snn_status_t finish_generated(snn_cuda_context_t *c, const b200::GenParams &g, uint64_t e_total,
                              snn_cuda_context_t **out, const snn_cuda_config_t *config = nullptr,
                              uint64_t budget = 0) {
    snn_status_t st = SNN_OK;
    c->mode = SNN_CUDA_MODE_FULL;
    const snn_cuda_config_t cfg = config ? *config : snn_cuda_default_config();
    const uint64_t e_est = (uint64_t)((double)e_total * ((double)c->n_local / (double)c->n_global));
    const bool full_only = c->propagation == SNN_B200_PROPAGATE_ORDERED || c->batch > 1;
    if (!full_only && budget && (cfg.prefer_streaming || full_push_bytes(c, e_est) > budget)) {
        st = generate_streaming(c, g, e_total, cfg, budget);
    } else if (c->propagation != SNN_B200_PROPAGATE_ORDERED) {
        if ((st = generate_full(c, g, e_total)) == SNN_OK) st = add_pull_topology(c, nullptr, &g);
    }
    else if (!c->opull) {
        if ((st = generate_full(c, g, e_total)) == SNN_OK && (st = add_pull_topology(c, nullptr, &g)) == SNN_OK)
            st = setup_ordered(c);
    } else if (c->n_local > 0xffffffffull) st = SNN_ERR_UNSUPPORTED;  // 32-bit sort keys
    else st = build_generated_csc(c, g);
    if (st != SNN_OK) {
        free_context(c);
        return st;
    }
    *out = c;
    return SNN_OK;
}

uint64_t stream_range(const snn_cuda_context_t *c) { return c->inject_range ? c->inject_range : c->n_global; }

// Launch-bound loops (small networks, quiet steps) pay a launch gap per
// kernel; unsharded push and bin-fold contexts without device timing replay a captured
// graph of two steps instead. SNN_B200_NO_GRAPHS (environment) disables it.
bool graph_eligible(const snn_cuda_context_t *c) {
    return c->world == 1 && c->mode == SNN_CUDA_MODE_FULL &&
           (c->propagation != SNN_B200_PROPAGATE_ORDERED || c->binfold) && !c->timing &&
           std::getenv("SNN_B200_NO_GRAPHS") == nullptr;
}

// One step of the injection stream with the step index read on the device.
snn_status_t stream_step_dev(snn_cuda_context_t *c, uint64_t seed, snn_size_t count, float value) {
    if (count) {
        b200::launch_inject_stream(c->stream, c->device, seed, 0, count, stream_range(c), value * c->lif.input_scale,
                                   c->d_cur[c->cur], c->lo, c->hi, &c->d_ctr->stream_step);
        c->launches++;
    }
    return enqueue_step(c, c->ext_held);
}

snn_status_t run_stream_graph(snn_cuda_context_t *c, uint64_t seed, uint64_t first_step, uint64_t steps,
                              snn_size_t count, float value) {
    snn_status_t st = SNN_OK;
    b200::launch_set_u64(c->stream, &c->d_ctr->stream_step, first_step);
    c->launches++;
    c->dev_stream_step = true;
    uint64_t t = 0;
    // The graph starts on an even step (current buffer 0, list parity 0).
    if (c->step & 1u) {
        st = stream_step_dev(c, seed, count, value);
        ++t;
    }
    if (st == SNN_OK && (c->graph == nullptr || c->graph_seed != seed || c->graph_count != count ||
                         c->graph_value != value || c->graph_ext != c->ext_held ||
                         c->graph_range != stream_range(c))) {
        if (c->graph) cudaGraphExecDestroy(c->graph);
        c->graph = nullptr;
        const uint64_t step0 = c->step, launches0 = c->launches;
        const int cur0 = c->cur;
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeRelaxed) == cudaSuccess) {
            snn_status_t cs = stream_step_dev(c, seed, count, value);
            if (cs == SNN_OK) cs = stream_step_dev(c, seed, count, value);
            const cudaError_t ce = cudaStreamEndCapture(c->stream, &g);
            if (cs == SNN_OK && ce == cudaSuccess && g != nullptr &&
                cudaGraphInstantiate(&c->graph, g, 0) == cudaSuccess) {
                c->graph_seed = seed;
                c->graph_count = count;
                c->graph_value = value;
                c->graph_ext = c->ext_held;
                c->graph_range = stream_range(c);
                c->graph_launches = c->launches - launches0;
            } else {
                c->graph = nullptr;
            }
            if (g) cudaGraphDestroy(g);
        }
        cudaGetLastError();
        // Capture recorded the work without running it: undo its host state.
        c->step = step0;
        c->cur = cur0;
        c->launches = launches0;
    }
    while (st == SNN_OK && c->graph != nullptr && steps - t >= 2) {
        st = cuda_status(cudaGraphLaunch(c->graph, c->stream));
        c->step += 2;
        c->launches += c->graph_launches;
        t += 2;
    }
    while (st == SNN_OK && t < steps) {  // odd remainder, or no graph could be made
        st = stream_step_dev(c, seed, count, value);
        ++t;
    }
    c->dev_stream_step = false;
    return st == SNN_OK ? cuda_status(cudaGetLastError()) : st;
}

bool is_group(const snn_cuda_context_t *c) { return c != nullptr && !c->group.empty(); }

// The early spike download of snn_cuda_step (FULL contexts): a side stream
// copies the spikes as soon as the LIF kernel is done.
snn_status_t prepare_spike_stream(snn_cuda_context_t *c) {
    if (c->spk_stream != nullptr) return SNN_OK;
    if (cudaStreamCreateWithFlags(&c->spk_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_lif, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->ev_spk, cudaEventDisableTiming) != cudaSuccess)
        return SNN_ERR_CUDA;
    return SNN_OK;
}

// Runs one phase on every member, each with its device current.
template <typename F>
snn_status_t for_members(snn_cuda_context_t *g, F &&f) {
    snn_status_t st = SNN_OK;
    for (snn_cuda_context_t *m : g->group) {
        snn_status_t s2 = set_device(m);
        if (s2 == SNN_OK) s2 = f(m);
        if (st == SNN_OK) st = s2;
    }
    return st;
}

// The NCCL all-gathers of all members, issued from this thread as one group.
snn_status_t group_exchange(snn_cuda_context_t *g) {
    if (g->group[0]->exchange != SNN_B200_EXCHANGE_NCCL) return SNN_OK;
    if (ncclGroupStart() != ncclSuccess) return SNN_ERR_CUDA;
    const snn_status_t st = for_members(g, [](snn_cuda_context_t *m) { return step_exchange(m); });
    const ncclResult_t r = ncclGroupEnd();
    if (r != ncclSuccess) {
        set_error("ncclGroupEnd", ncclGetErrorString(r));
        return SNN_ERR_CUDA;
    }
    return st;
}

// One step of every member: all LIF phases first, the all-gathers as one
// NCCL group, all compactions (with the peer exchange each releases its
// member's flag and waits for every other's), then the propagations.
snn_status_t group_step_async(snn_cuda_context_t *g, const float *ext, uint8_t *spikes) {
    snn_status_t st = for_members(g, [&](snn_cuda_context_t *m) {
        if (ext != nullptr && m->n_local) {
            if (cudaMemcpyAsync(m->d_ext, ext + m->lo, m->n_local * 4, cudaMemcpyHostToDevice, m->stream) !=
                cudaSuccess)
                return SNN_ERR_CUDA;
            m->ext_held = false;
        }
        m->spk_dst = nullptr;
        if (spikes != nullptr && m->n_local && m->mode == SNN_CUDA_MODE_FULL) {
            const snn_status_t s2 = prepare_spike_stream(m);
            if (s2 != SNN_OK) return s2;
            m->spk_dst = spikes + m->lo;
        }
        return step_lif(m, ext != nullptr || m->ext_held);
    });
    if (st == SNN_OK) st = group_exchange(g);
    if (st == SNN_OK) st = for_members(g, [](snn_cuda_context_t *m) { return step_compact(m); });
    const snn_status_t s3 = for_members(g, [&](snn_cuda_context_t *m) {
        const snn_status_t s2 = st == SNN_OK ? step_propagate(m) : SNN_OK;
        m->spk_dst = nullptr;
        return s2;
    });
    return st == SNN_OK ? s3 : st;
}

snn_status_t group_synchronize(snn_cuda_context_t *g) {
    return for_members(g, [](snn_cuda_context_t *m) {
        if (m->exchange == SNN_B200_EXCHANGE_PEER) queue_error_check(m);
        return error_after_sync(m, cuda_status(cudaStreamSynchronize(m->stream)));
    });
}

snn_status_t group_step(snn_cuda_context_t *g, const float *ext, uint8_t *spikes) {
    snn_status_t st = group_step_async(g, ext, spikes);
    // STREAMING members download their spikes after the step.
    const snn_status_t s2 = for_members(g, [&](snn_cuda_context_t *m) {
        if (spikes == nullptr || m->n_local == 0 || m->mode == SNN_CUDA_MODE_FULL) return SNN_OK;
        return cudaMemcpyAsync(spikes + m->lo, m->d_spikes, m->n_local, cudaMemcpyDeviceToHost, m->stream) ==
                       cudaSuccess
                   ? SNN_OK
                   : SNN_ERR_CUDA;
    });
    const snn_status_t s3 = group_synchronize(g);
    if (st == SNN_OK) st = s2;
    return st == SNN_OK ? s3 : st;
}

}  // namespace

// ======================================================================
//                              C ABI
// ======================================================================
extern "C" {

snn_cuda_config_t snn_cuda_default_config(void) {
    snn_cuda_config_t c;
    c.max_vram_bytes = 0;
    c.max_stream_synapses = 0;
    c.max_stream_rows = 0;
    c.prefer_streaming = 0;
    return c;
}

int snn_cuda_available(void) {
    if (g_force_unavailable) return 0;
    int count = 0;
    return cudaGetDeviceCount(&count) == cudaSuccess && count > 0;
}

snn_b200_options_t snn_b200_default_options(void) {
    snn_b200_options_t o;
    o.propagation = SNN_B200_PROPAGATE_PUSH;
    o.device = -1;
    o.index_width = 0;
    o.rank = 0;
    o.world_size = 1;
    o.nccl_id = nullptr;
    o.timing = 0;
    o.exchange = SNN_B200_EXCHANGE_NCCL;
    o.streaming = SNN_B200_STREAMING_CHUNKED;
    o.batch = 1;
    return o;
}

snn_status_t snn_b200_create(const snn_network_t *network, const snn_cuda_config_t *config,
                             const snn_b200_options_t *options, snn_cuda_context_t **out_context) {
    if (out_context == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out_context = nullptr;
    if (network == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    const snn_cuda_config_t cfg = config ? *config : snn_cuda_default_config();
    const snn_b200_options_t o = options ? *options : snn_b200_default_options();
    if ((o.propagation == SNN_B200_PROPAGATE_PUSH_BINNED || o.batch > 1) && cfg.prefer_streaming)
        return SNN_ERR_UNSUPPORTED;
    snn_cuda_context_t *c = nullptr;
    CreateEnv env;
    snn_status_t st = begin_create(network->neuron_count, network->lif, network->decay, &cfg, &o, &c, &env);
    if (st != SNN_OK) return st;
    c->network = network;
    const bool full_only = c->want_binfold || c->batch > 1;
    if (full_only || (!cfg.prefer_streaming && full_push_bytes(c, network->synapse_count) <= env.budget)) {
        c->mode = SNN_CUDA_MODE_FULL;
        if (c->propagation != SNN_B200_PROPAGATE_ORDERED) {
            st = upload_full_push(c, network);
            // The reference entry point (no options) and explicit VRAM budgets
            // keep the plain push topology.
            if (st == SNN_OK && options != nullptr && cfg.max_vram_bytes == 0)
                st = add_pull_topology(c, network, nullptr);
        } else if (c->opull) st = upload_full_ordered(c, network);
        else if ((st = upload_full_push(c, network)) == SNN_OK && (st = add_pull_topology(c, network, nullptr)) == SNN_OK)
            st = setup_ordered(c);
    } else {
        c->mode = SNN_CUDA_MODE_STREAMING;
        c->e_local = network->synapse_count;
        // A shard streams only the edges into its own neurons: a host copy of
        // them, with local target ids, stands in for the network.
        if (c->world > 1) st = make_stream_slice(c, network);
        bool fallback = true;
        if (st == SNN_OK && c->streaming == SNN_B200_STREAMING_SPARSE) st = allocate_sparse_streaming(c, &fallback);
        if (st == SNN_OK && fallback) {
            c->streaming = SNN_B200_STREAMING_CHUNKED;
            st = allocate_streaming(c, cfg, env.budget);
        }
        if (st == SNN_OK && c->propagation == SNN_B200_PROPAGATE_ORDERED) st = setup_ordered_streaming(c);
    }
    if (st != SNN_OK) {
        free_context(c);
        return st;
    }
    *out_context = c;
    return SNN_OK;
}

snn_status_t snn_cuda_create(const snn_network_t *network, const snn_cuda_config_t *config,
                             snn_cuda_context_t **out_context) {
    return snn_b200_create(network, config, nullptr, out_context);
}

snn_status_t snn_b200_create_sharded(const snn_network_t *network, const snn_cuda_config_t *config,
                                     const snn_b200_options_t *options, int device_count, const int *devices,
                                     snn_cuda_context_t **out_context) {
    if (out_context == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out_context = nullptr;
    if (network == nullptr || devices == nullptr || device_count < 1 || device_count > (int)b200::kMaxPeers)
        return SNN_ERR_INVALID_ARGUMENT;
    if (!snn_cuda_available()) return SNN_ERR_CUDA;
    int have = 0;
    if (cudaGetDeviceCount(&have) != cudaSuccess) return SNN_ERR_CUDA;
    for (int r = 0; r < device_count; ++r) {
        if (devices[r] < 0 || devices[r] >= have) return SNN_ERR_INVALID_ARGUMENT;
        for (int q = 0; q < r; ++q)
            if (devices[q] == devices[r]) return SNN_ERR_INVALID_ARGUMENT;  // one rank per device
    }
    snn_b200_options_t o = options ? *options : snn_b200_default_options();
    if (o.batch > 1) return SNN_ERR_UNSUPPORTED;
    if (device_count == 1) {
        o.world_size = 1;
        o.rank = 0;
        o.device = devices[0];
        return snn_b200_create(network, config, &o, out_context);
    }
    // Peer exchange when every pair of devices can reach the other's memory
    // (without options: whenever it can), else NCCL.
    bool peer_ok = true;
    for (int a = 0; a < device_count && peer_ok; ++a)
        for (int b = 0; b < device_count && peer_ok; ++b) {
            int can = 0;
            if (a != b && (cudaDeviceCanAccessPeer(&can, devices[a], devices[b]) != cudaSuccess || !can))
                peer_ok = false;
        }
    cudaGetLastError();
    int exchange = options ? o.exchange : SNN_B200_EXCHANGE_PEER;
    if (exchange == SNN_B200_EXCHANGE_PEER && !peer_ok) exchange = SNN_B200_EXCHANGE_NCCL;
    if (exchange == SNN_B200_EXCHANGE_PEER) {
        for (int a = 0; a < device_count; ++a) {
            if (cudaSetDevice(devices[a]) != cudaSuccess) return SNN_ERR_CUDA;
            for (int b = 0; b < device_count; ++b) {
                if (a == b) continue;
                const cudaError_t e = cudaDeviceEnablePeerAccess(devices[b], 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_status(e);
                cudaGetLastError();
            }
        }
    }
    snn_cuda_context_t *g = new (std::nothrow) snn_cuda_context();
    if (g == nullptr) return SNN_ERR_OUT_OF_MEMORY;
    g->group.assign((size_t)device_count, nullptr);
    snn_status_t st = SNN_OK;
    t_group_member = true;
    for (int r = 0; r < device_count && st == SNN_OK; ++r) {
        snn_b200_options_t m = o;
        m.rank = (uint32_t)r;
        m.world_size = (uint32_t)device_count;
        m.device = devices[r];
        m.nccl_id = nullptr;
        m.exchange = exchange;
        st = snn_b200_create(network, config, &m, &g->group[r]);
    }
    t_group_member = false;
    if (st == SNN_OK && exchange == SNN_B200_EXCHANGE_NCCL) {
        std::vector<ncclComm_t> comms((size_t)device_count);
        const ncclResult_t r = ncclCommInitAll(comms.data(), device_count, devices);
        if (r != ncclSuccess) {
            set_error("ncclCommInitAll", ncclGetErrorString(r));
            st = SNN_ERR_CUDA;
        } else {
            for (int q = 0; q < device_count; ++q) g->group[q]->comm = comms[q];
        }
    }
    if (st == SNN_OK && exchange == SNN_B200_EXCHANGE_PEER) {
        // In-process peer mappings: every member reaches the others'
        // exchange buffers directly (unified addressing, peer access on).
        for (snn_cuda_context_t *m : g->group) {
            for (int q = 0; q < device_count; ++q) m->peer_x[q] = (uint32_t *)g->group[q]->d_xbuf;
            m->peers_connected = true;
        }
    }
    if (st != SNN_OK) {
        g->group.erase(std::remove(g->group.begin(), g->group.end(), nullptr), g->group.end());
        if (g->group.empty())
            delete g;
        else
            free_context(g);
        return st;
    }
    snn_cuda_context_t *m0 = g->group[0];
    g->network = network;
    g->mode = m0->mode;
    g->device = devices[0];
    g->propagation = m0->propagation;
    g->exchange = exchange;
    g->world = (uint32_t)device_count;
    g->n_global = g->n_rows = g->n_local = g->hi = network->neuron_count;
    g->col_bits = m0->col_bits;
    for (snn_cuda_context_t *m : g->group) g->e_local += m->e_local;
    *out_context = g;
    return SNN_OK;
}

snn_status_t snn_cuda_create_sharded(const snn_network_t *network, const snn_cuda_config_t *config,
                                     int device_count, const int *devices, snn_cuda_context_t **out_context) {
    return snn_b200_create_sharded(network, config, nullptr, device_count, devices, out_context);
}

void snn_cuda_free(snn_cuda_context_t *context) { free_context(context); }

snn_cuda_mode_t snn_cuda_context_mode(const snn_cuda_context_t *context) {
    return context == nullptr ? SNN_CUDA_MODE_NONE : context->mode;
}

snn_status_t snn_cuda_inject_current(snn_cuda_context_t *c, const snn_size_t *host_indices,
                                     const float *host_values, snn_size_t count) {
    if (c == nullptr || (count != 0 && (host_indices == nullptr || host_values == nullptr)))
        return SNN_ERR_INVALID_ARGUMENT;
    if (count == 0) return SNN_OK;
    if (is_group(c)) {
        // All-or-nothing validation first, then every member takes the
        // indices of its own range.
        for (uint64_t k = 0; k < count; ++k)
            if (host_indices[k] >= c->n_global) return SNN_ERR_INVALID_ARGUMENT;
        snn_status_t st = SNN_OK;
        for (snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_cuda_inject_current(m, host_indices, host_values, count);
        return st;
    }
    if (count > UINT64_MAX / sizeof(snn_size_t)) return SNN_ERR_INVALID_ARGUMENT;
    // One pass: every index in range, and whether all values are equal.
    uint32_t v0;
    std::memcpy(&v0, host_values, 4);
    uint64_t bad = 0;
    uint32_t differ = 0;
    for (uint64_t k = 0; k < count; ++k) {
        uint32_t vk;
        std::memcpy(&vk, host_values + k, 4);
        bad |= (uint64_t)(host_indices[k] >= c->n_global);
        differ |= vk ^ v0;
    }
    if (bad) return SNN_ERR_INVALID_ARGUMENT;
    const bool uniform = differ == 0;
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    if ((st = ensure_inject_capacity(c, count)) != SNN_OK) return st;
    // The arrays go straight from the caller's buffers; the call returns once
    // those copies are done (the caller may reuse them). Fault seams as the
    // reference's staging: index copy, value copy, launch.
    if (seam_fail()) return SNN_ERR_CUDA;
    cudaStreamWaitEvent(c->inj_stream, c->ev_inj_used, 0);  // the previous injection has read the buffers
    if (cudaMemcpyAsync(c->d_inj_idx, host_indices, count * 8, cudaMemcpyHostToDevice, c->inj_stream) != cudaSuccess)
        return cuda_status(cudaGetLastError());
    if (seam_fail()) return SNN_ERR_CUDA;
    if (!uniform &&
        cudaMemcpyAsync(c->d_inj_val, host_values, count * 4, cudaMemcpyHostToDevice, c->inj_stream) != cudaSuccess)
        return cuda_status(cudaGetLastError());
    cudaEventRecord(c->ev_inj_copy, c->inj_stream);
    cudaStreamWaitEvent(c->stream, c->ev_inj_copy, 0);
    if ((st = cuda_status(cudaEventSynchronize(c->ev_inj_copy))) != SNN_OK) return st;
    if (uniform) {
        // Equal values: any accumulation order gives the same bits, so a
        // plain atomic scatter is exact; the value is a kernel argument.
        float vf;
        std::memcpy(&vf, &v0, 4);
        b200::launch_inject_uniform(c->stream, c->device, count, c->d_inj_idx, vf, c->lif.input_scale,
                                    c->d_cur[c->cur], c->lo, c->hi);
    } else {
        // Unequal values: a stable radix sort by index, so each index's
        // values fold in their original order (src/snn.c:737-739).
        uint64_t *idx_alt = c->d_inj_idx + c->inj_cap;
        float *val_alt = c->d_inj_val + c->inj_cap;
        void *tmp = (char *)c->d_inj_val + ((c->inj_cap * 8 + 255) & ~255ull);
        size_t tmp_bytes = c->inj_tmp_bytes;
        bool in_alt = false;
        if ((st = cuda_status(b200::sort_pairs_u64_f32(c->stream, c->d_inj_idx, idx_alt, c->d_inj_val, val_alt, count,
                                                       inject_key_bits(c), tmp, &tmp_bytes, &in_alt))) != SNN_OK)
            return st;
        b200::launch_inject_ordered(c->stream, c->device, count, in_alt ? idx_alt : c->d_inj_idx,
                                    in_alt ? val_alt : c->d_inj_val, c->lif.input_scale, c->d_cur[c->cur], c->lo,
                                    c->hi);
    }
    st = check_launch(c);
    cudaEventRecord(c->ev_inj_used, c->stream);
    return st;
}

snn_status_t snn_cuda_step(snn_cuda_context_t *c, const float *host_external_current, uint8_t *host_out_spikes) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return group_step(c, host_external_current, host_out_spikes);
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    if (host_external_current != nullptr) {
        if (seam_fail()) return SNN_ERR_CUDA;
        if (cudaMemcpyAsync(c->d_ext, host_external_current, c->n_local * 4, cudaMemcpyHostToDevice, c->stream) !=
            cudaSuccess)
            return SNN_ERR_CUDA;
    }
    // FULL contexts download the spikes inside the step (overlapping the
    // propagation); the fault seam of that copy keeps its place below.
    const bool early = host_out_spikes != nullptr && c->n_local != 0 && c->mode == SNN_CUDA_MODE_FULL;
    if (early && c->spk_stream == nullptr) {
        if (cudaStreamCreateWithFlags(&c->spk_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_lif, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_spk, cudaEventDisableTiming) != cudaSuccess)
            return SNN_ERR_CUDA;
    }
    c->spk_dst = early ? host_out_spikes : nullptr;
    if (host_external_current != nullptr) c->ext_held = false;  // the held frame was overwritten
    st = enqueue_step(c, host_external_current != nullptr || c->ext_held);
    c->spk_dst = nullptr;
    if (st != SNN_OK) {
        if (early) cudaStreamSynchronize(c->spk_stream);  // no copy lands after the return
        return st;
    }
    if (c->exchange == SNN_B200_EXCHANGE_PEER) queue_error_check(c);
    if (host_out_spikes != nullptr && c->n_local != 0) {
        if (seam_fail()) {
            cudaStreamSynchronize(c->stream);
            return SNN_ERR_CUDA;
        }
        if (!early && cudaMemcpyAsync(host_out_spikes, c->d_spikes, c->n_local, cudaMemcpyDeviceToHost,
                                      c->stream) != cudaSuccess)
            return SNN_ERR_CUDA;
    }
    return error_after_sync(c, cuda_status(cudaStreamSynchronize(c->stream)));
}

snn_status_t snn_cuda_download_voltage(const snn_cuda_context_t *c, float *host_voltage, snn_size_t count) {
    if (c == nullptr || host_voltage == nullptr || count < c->n_local) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (const snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_cuda_download_voltage(m, host_voltage + m->lo, m->n_local);
        return st;
    }
    if (c->n_local == 0) return SNN_OK;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    if (seam_fail()) return SNN_ERR_CUDA;
    if (cudaMemcpyAsync(host_voltage, c->d_v, c->n_local * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

// ----------------------------------------------------------- test hooks --
snn_cuda_context_t *snn_test_nonnull_cuda_context(void) { return (snn_cuda_context_t *)(uintptr_t)1u; }
void snn_test_cuda_set_fail_after(int64_t calls_before_failure) { g_fail_after = calls_before_failure; }
void snn_test_cuda_disable_failure(void) {
    g_fail_after = -1;
    g_force_unavailable = 0;
    g_force_meminfo_fail = 0;
}
void snn_test_cuda_force_unavailable(int enable) { g_force_unavailable = enable; }
void snn_test_cuda_force_meminfo_fail(int enable) { g_force_meminfo_fail = enable; }

// ----------------------------------------------------------- extensions --
snn_status_t snn_b200_create_random_pool(const snn_random_pool_config_t *pool, const snn_lif_params_t *lif,
                                         const snn_cuda_config_t *config, const snn_b200_options_t *options,
                                         snn_cuda_context_t **out_context) {
    if (out_context == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out_context = nullptr;
    // src/snn.c:536-548
    if (pool == nullptr || pool->neuron_count == 0 ||
        (!pool->allow_self_connections && pool->neuron_count == 1u && pool->fanout_per_neuron != 0u) ||
        !std::isfinite(pool->weight_min) || !std::isfinite(pool->weight_max) || pool->weight_max < pool->weight_min ||
        !std::isfinite(pool->weight_max - pool->weight_min))
        return SNN_ERR_INVALID_ARGUMENT;
    const snn_lif_params_t p = lif ? *lif : snn_lif_params_t{1.0f, 20.0f, 0.0f, 0.0f, 1.0f, 1.0f, 1u};
    if (!lif_valid(&p)) return SNN_ERR_INVALID_ARGUMENT;
    const uint64_t n = pool->neuron_count, f = pool->fanout_per_neuron;
    if (f != 0 && n > UINT64_MAX / f) return SNN_ERR_OVERFLOW;
    b200::GenParams g{};
    g.n = n;
    g.fanout = f;
    g.seed = pool->seed;
    g.wmin = pool->weight_min;
    g.wmax = pool->weight_max;
    g.allow_self = pool->allow_self_connections;
    g.recurrent = 1;
    snn_cuda_context_t *c = nullptr;
    CreateEnv env;
    snn_status_t st = begin_create(n, p, expf(-p.dt_ms / p.membrane_tau_ms), config, options, &c, &env);
    if (st != SNN_OK) return st;
    return finish_generated(c, g, n * f, out_context, config, env.budget);
}

snn_status_t snn_b200_create_layered_random(const snn_size_t *layer_sizes, size_t layer_count, snn_size_t fanout,
                                            float weight_min, float weight_max, uint64_t seed,
                                            const snn_lif_params_t *lif, const snn_b200_options_t *options,
                                            snn_cuda_context_t **out_context) {
    if (out_context == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out_context = nullptr;
    if (layer_sizes == nullptr || layer_count < 2 || layer_count > 16 || fanout == 0 || !std::isfinite(weight_min) ||
        !std::isfinite(weight_max) || weight_max < weight_min || !std::isfinite(weight_max - weight_min))
        return SNN_ERR_INVALID_ARGUMENT;
    const snn_lif_params_t p = lif ? *lif : snn_lif_params_t{1.0f, 20.0f, 0.0f, 0.0f, 1.0f, 1.0f, 1u};
    if (!lif_valid(&p)) return SNN_ERR_INVALID_ARGUMENT;
    b200::GenParams g{};
    g.off[0] = 0;
    for (size_t l = 0; l < layer_count; ++l) {
        if (layer_sizes[l] == 0 || g.off[l] > UINT64_MAX - layer_sizes[l]) return SNN_ERR_INVALID_ARGUMENT;
        g.off[l + 1] = g.off[l] + layer_sizes[l];
    }
    g.n = g.off[layer_count];
    g.fanout = fanout;
    g.seed = seed;
    g.wmin = weight_min;
    g.wmax = weight_max;
    g.recurrent = 0;
    g.layers = (int)layer_count;
    const uint64_t rows = g.off[layer_count - 1];
    if (rows > UINT64_MAX / fanout) return SNN_ERR_OVERFLOW;
    snn_cuda_context_t *c = nullptr;
    CreateEnv env;
    snn_status_t st = begin_create(g.n, p, expf(-p.dt_ms / p.membrane_tau_ms), nullptr, options, &c, &env);
    if (st != SNN_OK) return st;
    return finish_generated(c, g, rows * fanout, out_context);
}

// Device build of snn_build_feedforward (src/snn.c:463-521), bit-identical:
// per layer, dense (fanout 0 or >= the next layer: every target in order,
// no draws) or fanout targets drawn from one splitmix64 stream seeded with
// `seed` and consumed in edge order across the sparse layers; every weight
// `weight`. Validation as src/snn.c:184-215 plus isfinite(weight).
snn_status_t snn_b200_create_feedforward(const snn_size_t *layer_sizes, size_t layer_count, snn_size_t fanout,
                                         float weight, uint64_t seed, const snn_lif_params_t *lif,
                                         const snn_b200_options_t *options, snn_cuda_context_t **out_context) {
    if (out_context == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out_context = nullptr;
    if (layer_sizes == nullptr || layer_count < 2 || layer_count > 16 || !std::isfinite(weight))
        return SNN_ERR_INVALID_ARGUMENT;
    const snn_lif_params_t p = lif ? *lif : snn_lif_params_t{1.0f, 20.0f, 0.0f, 0.0f, 1.0f, 1.0f, 1u};
    if (!lif_valid(&p)) return SNN_ERR_INVALID_ARGUMENT;
    b200::GenParams g{};
    g.off[0] = 0;
    for (size_t l = 0; l < layer_count; ++l) {
        if (layer_sizes[l] == 0) return SNN_ERR_INVALID_ARGUMENT;
        if (g.off[l] > UINT64_MAX - layer_sizes[l]) return SNN_ERR_OVERFLOW;
        g.off[l + 1] = g.off[l] + layer_sizes[l];
    }
    g.n = g.off[layer_count];
    g.seed = seed;
    g.wconst = weight;
    g.recurrent = 0;
    g.feedforward = 1;
    g.layers = (int)layer_count;
    uint64_t edges = 0, draws = 0, widest = 1;
    for (size_t l = 0; l + 1 < layer_count; ++l) {
        const uint64_t pre = layer_sizes[l], post = layer_sizes[l + 1];
        const bool dense = fanout == 0 || fanout >= post;
        const uint64_t f = dense ? post : fanout;
        if (f != 0 && pre > UINT64_MAX / f) return SNN_ERR_OVERFLOW;
        const uint64_t le = pre * f;
        if (edges > UINT64_MAX - le) return SNN_ERR_OVERFLOW;
        g.lfan[l] = f;
        g.ledge[l] = edges;
        g.ldraw[l] = dense ? ~0ull : draws;
        if (!dense) draws += le;
        edges += le;
        widest = std::max(widest, f);
    }
    g.ledge[layer_count - 1] = edges;
    g.fanout = widest;
    snn_cuda_context_t *c = nullptr;
    CreateEnv env;
    snn_status_t st = begin_create(g.n, p, expf(-p.dt_ms / p.membrane_tau_ms), nullptr, options, &c, &env);
    if (st != SNN_OK) return st;
    return finish_generated(c, g, edges, out_context);
}

const char *snn_b200_last_error(void) { return g_last_error; }

snn_status_t snn_test_b200_peer_loopback(snn_cuda_context_t *c, uint32_t spin_limit) {
    if (c == nullptr || c->d_xbuf == nullptr || c->peers_connected) return SNN_ERR_INVALID_ARGUMENT;
    for (uint32_t r = 0; r < c->world; ++r) c->peer_x[r] = (uint32_t *)c->d_xbuf;
    c->peer_spin_limit = spin_limit;
    c->peers_connected = true;
    return SNN_OK;
}

snn_status_t snn_b200_ipc_handle(const snn_cuda_context_t *c, void *out_handle64) {
    if (c == nullptr || out_handle64 == nullptr || c->d_xbuf == nullptr || is_group(c)) return SNN_ERR_INVALID_ARGUMENT;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    cudaIpcMemHandle_t h;
    const snn_status_t st = cuda_status(cudaIpcGetMemHandle(&h, c->d_xbuf));
    if (st == SNN_OK) std::memcpy(out_handle64, &h, sizeof(h));
    return st;
}

snn_status_t snn_b200_ipc_connect(snn_cuda_context_t *c, const void *handles) {
    if (c == nullptr || handles == nullptr || c->d_xbuf == nullptr || c->peers_connected)
        return SNN_ERR_INVALID_ARGUMENT;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    for (uint32_t r = 0; r < c->world; ++r) {
        if (r == c->rank) {
            c->peer_x[r] = (uint32_t *)c->d_xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const char *)handles + (size_t)r * sizeof(h), sizeof(h));
        void *p = nullptr;
        const snn_status_t st = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        if (st != SNN_OK) return st;
        c->peer_x[r] = (uint32_t *)p;
        c->peer_ipc[r] = true;
    }
    c->peers_connected = true;
    return SNN_OK;
}

snn_status_t snn_b200_shard_range(snn_size_t n, uint32_t world, uint32_t rank, snn_size_t *out_begin,
                                  snn_size_t *out_count) {
    if (out_begin == nullptr || out_count == nullptr || world == 0 || rank >= world || n == 0)
        return SNN_ERR_INVALID_ARGUMENT;
    uint64_t slot, lo, hi;
    shard_geometry(n, world, rank, &slot, &lo, &hi);
    *out_begin = lo;
    *out_count = hi - lo;
    return SNN_OK;
}

snn_status_t snn_b200_nccl_unique_id(void *out_id128) {
    if (out_id128 == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return SNN_ERR_CUDA;
    std::memcpy(out_id128, &id, sizeof(id));
    return SNN_OK;
}

snn_status_t snn_b200_reset(snn_cuda_context_t *c) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_b200_reset(m);
        return st;
    }
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    cudaStreamSynchronize(c->stream);
    // Keep the cumulative statistics across the reset.
    b200::DevCounters saved{};
    if (cudaMemcpy(&saved, c->d_ctr, sizeof(saved), cudaMemcpyDeviceToHost) != cudaSuccess) return SNN_ERR_CUDA;
    b200::launch_init_state(c->stream, c->n_local, c->lif.v_rest, c->d_v, c->d_cur[0], c->d_cur[1],
                            c->ext_held ? nullptr : c->d_ext, c->d_refr, c->d_spikes, c->bitmap_words, c->d_bitmap,
                            c->d_ctr, c->d_kind_log);
    c->launches++;
    if ((st = cuda_status(cudaGetLastError())) != SNN_OK) return st;
    saved.list_count[0] = saved.list_count[1] = 0;
    saved.step_events[0] = saved.step_events[1] = 0;
    if (cudaMemcpyAsync(c->d_ctr, &saved, sizeof(saved), cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    c->cur = 0;
    c->step = 0;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t snn_b200_inject_stream_async(snn_cuda_context_t *c, uint64_t seed, uint64_t step, snn_size_t count,
                                          float value) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_b200_inject_stream_async(m, seed, step, count, value);
        return st;
    }
    if (count == 0) return SNN_OK;
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    // Uniform value: the atomic scatter is order-exact (see inject_current).
    b200::launch_inject_stream(c->stream, c->device, seed, step, count, stream_range(c),
                               value * c->lif.input_scale, c->d_cur[c->cur], c->lo, c->hi);
    c->launches++;
    return cuda_status(cudaGetLastError());
}

snn_status_t snn_b200_step_async(snn_cuda_context_t *c) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return group_step_async(c, nullptr, nullptr);
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    return enqueue_step(c, c->ext_held);
}

snn_status_t snn_b200_set_stream_range(snn_cuda_context_t *c, snn_size_t range) {
    if (c == nullptr || range > c->n_global) return SNN_ERR_INVALID_ARGUMENT;
    for (snn_cuda_context_t *m : c->group) m->inject_range = range;
    c->inject_range = range;
    return SNN_OK;
}

snn_status_t snn_b200_set_external(snn_cuda_context_t *c, const float *host_external_current) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_b200_set_external(m, host_external_current ? host_external_current + m->lo : nullptr);
        return st;
    }
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    if (host_external_current == nullptr) {
        c->ext_held = false;
        return SNN_OK;
    }
    if (c->n_local &&
        (st = cuda_status(cudaMemcpyAsync(c->d_ext, host_external_current, c->n_local * 4, cudaMemcpyHostToDevice,
                                          c->stream))) != SNN_OK)
        return st;
    if ((st = cuda_status(cudaStreamSynchronize(c->stream))) != SNN_OK) return st;
    c->ext_held = true;
    return SNN_OK;
}

snn_status_t snn_b200_run_stream_async(snn_cuda_context_t *c, uint64_t seed, uint64_t first_step, uint64_t steps,
                                       snn_size_t count, float value) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (uint64_t t = 0; t < steps && st == SNN_OK; ++t) {
            st = snn_b200_inject_stream_async(c, seed, first_step + t, count, value);
            if (st == SNN_OK) st = group_step_async(c, nullptr, nullptr);
        }
        return st;
    }
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    if (graph_eligible(c) && steps >= 8) return run_stream_graph(c, seed, first_step, steps, count, value);
    for (uint64_t t = 0; t < steps; ++t) {
        if (count) {
            b200::launch_inject_stream(c->stream, c->device, seed, first_step + t, count, stream_range(c),
                                       value * c->lif.input_scale, c->d_cur[c->cur], c->lo, c->hi);
            c->launches++;
        }
        if ((st = enqueue_step(c, c->ext_held)) != SNN_OK) return st;
    }
    return cuda_status(cudaGetLastError());
}

snn_status_t snn_b200_synchronize(snn_cuda_context_t *c) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        const snn_status_t st = group_synchronize(c);
        for (snn_cuda_context_t *m : c->group) timing_fold(m);
        return st;
    }
    snn_status_t st = set_device(c);
    if (st != SNN_OK) return st;
    queue_error_check(c);
    st = error_after_sync(c, cuda_status(cudaStreamSynchronize(c->stream)));
    timing_fold(c);
    return st;
}

snn_status_t snn_b200_get_stats(snn_cuda_context_t *c, snn_b200_stats_t *out) {
    if (c == nullptr || out == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        // Counts summed over the members (events are per target, spikes per
        // own neuron), device times the slowest member's.
        snn_b200_stats_t acc{};
        for (snn_cuda_context_t *m : c->group) {
            snn_b200_stats_t s1{};
            const snn_status_t st = snn_b200_get_stats(m, &s1);
            if (st != SNN_OK) return st;
            acc.steps = s1.steps;
            acc.spikes += s1.spikes;
            acc.events += s1.events;
            acc.kernel_launches += s1.kernel_launches;
            acc.step_ms = std::max(acc.step_ms, s1.step_ms);
            acc.propagate_ms = std::max(acc.propagate_ms, s1.propagate_ms);
            acc.lif_ms = std::max(acc.lif_ms, s1.lif_ms);
            acc.exchange_ms = std::max(acc.exchange_ms, s1.exchange_ms);
            acc.pull_steps = std::max(acc.pull_steps, s1.pull_steps);
            acc.pull_events += s1.pull_events;
            acc.pull_spikes = std::max(acc.pull_spikes, s1.pull_spikes);
            acc.propagate_pull_ms = std::max(acc.propagate_pull_ms, s1.propagate_pull_ms);
            acc.exchange_wait_ms = std::max(acc.exchange_wait_ms, s1.exchange_wait_ms);
            acc.exchange_wait_max_ms = std::max(acc.exchange_wait_max_ms, s1.exchange_wait_max_ms);
        }
        *out = acc;
        return SNN_OK;
    }
    snn_status_t st = snn_b200_synchronize(c);
    if (st != SNN_OK) return st;
    b200::DevCounters d{};
    if (cudaMemcpy(&d, c->d_ctr, sizeof(d), cudaMemcpyDeviceToHost) != cudaSuccess) return SNN_ERR_CUDA;
    out->steps = c->step;
    out->spikes = d.spikes;
    out->events = d.events;
    out->kernel_launches = c->launches;
    out->step_ms = c->t_step;
    out->propagate_ms = c->t_prop;
    out->lif_ms = c->t_lif;
    out->exchange_ms = c->t_exchange;
    out->pull_steps = d.pull_runs;
    out->pull_events = d.pull_events;
    out->pull_spikes = d.pull_spikes;
    out->propagate_pull_ms = c->t_prop_pull;
    out->exchange_wait_ms = (double)d.wait_ns * 1e-6;
    out->exchange_wait_max_ms = (double)d.wait_max_ns * 1e-6;
    return SNN_OK;
}

snn_status_t snn_b200_reset_stats(snn_cuda_context_t *c) {
    if (c == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        snn_status_t st = SNN_OK;
        for (snn_cuda_context_t *m : c->group)
            if (st == SNN_OK) st = snn_b200_reset_stats(m);
        return st;
    }
    snn_status_t st = snn_b200_synchronize(c);
    if (st != SNN_OK) return st;
    b200::DevCounters d{};
    if (cudaMemcpy(&d, c->d_ctr, sizeof(d), cudaMemcpyDeviceToHost) != cudaSuccess) return SNN_ERR_CUDA;
    d.spikes = 0;
    d.events = 0;
    d.pull_runs = 0;
    d.pull_events = 0;
    d.pull_spikes = 0;
    d.wait_ns = 0;
    d.wait_max_ns = 0;
    if (cudaMemcpy(c->d_ctr, &d, sizeof(d), cudaMemcpyHostToDevice) != cudaSuccess) return SNN_ERR_CUDA;
    c->launches = 0;
    c->t_step = c->t_lif = c->t_exchange = c->t_prop = c->t_prop_pull = 0;
    return SNN_OK;
}

snn_status_t snn_b200_get_layout(const snn_cuda_context_t *c, snn_b200_layout_t *out) {
    if (c == nullptr || out == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) {
        // The whole network over all members (device bytes summed).
        snn_status_t st = snn_b200_get_layout(c->group[0], out);
        if (st != SNN_OK) return st;
        out->local_begin = 0;
        out->local_count = c->n_global;
        out->local_synapses = c->e_local;
        for (size_t r = 1; r < c->group.size(); ++r) {
            snn_b200_layout_t l{};
            if ((st = snn_b200_get_layout(c->group[r], &l)) != SNN_OK) return st;
            out->device_state_bytes += l.device_state_bytes;
            out->device_topology_bytes += l.device_topology_bytes;
            out->pull_slots += l.pull_slots;
        }
        return SNN_OK;
    }
    out->neuron_count = c->n_global;
    out->local_begin = c->lo;
    out->local_count = c->n_local;
    out->local_synapses = c->e_local;
    out->index_bits = (uint32_t)c->col_bits;
    out->propagation = c->propagation;
    out->device_state_bytes = state_bytes(c);
    if (c->mode == SNN_CUDA_MODE_STREAMING && c->streaming == SNN_B200_STREAMING_SPARSE)
        out->device_topology_bytes = (c->n_rows + 1) * 8;
    else if (c->mode == SNN_CUDA_MODE_STREAMING)
        out->device_topology_bytes = 2 * ((c->slot_rows + 1) * 8 + c->slot_edges * 12);
    else if (c->opull || c->has_csc)
        out->device_topology_bytes = (c->has_csc ? (c->n_rows + 1) * 8 + c->e_local * (c->col_bits / 8 + 4) : 0) +
                                     ((c->n_local + 31) / 32 * c->sell_chunks + 1) * 8 + c->sell_slots * 8 +
                                     c->n_rows * 4;
    else
        out->device_topology_bytes = (c->n_rows + 1) * 8 + c->e_local * (c->col_bits / 8 + 4);
    out->binned = c->binfold ? 1u : 0u;
    out->binned_passes = c->binfold ? c->bf.tiles : 0u;
    out->ordered_csc = (c->opull || c->has_csc) ? 1u : 0u;
    out->pull_slots = c->sell_slots;
    out->batch = (uint32_t)c->batch;
    out->topology_rows = c->n_rows;
    return SNN_OK;
}

void *snn_b200_stream(const snn_cuda_context_t *c) {
    if (is_group(c)) return (void *)c->group[0]->stream;  // the first member's (device devices[0])
    return c ? (void *)c->stream : nullptr;
}

snn_status_t snn_b200_download_spikes(const snn_cuda_context_t *c, uint8_t *host, snn_size_t count) {
    if (c == nullptr || host == nullptr || count < c->n_local) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return SNN_ERR_UNSUPPORTED;  // per member state: use one context per device
    if (c->n_local == 0) return SNN_OK;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    if (cudaMemcpyAsync(host, c->d_spikes, c->n_local, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t snn_b200_download_current(const snn_cuda_context_t *c, float *host, snn_size_t count) {
    if (c == nullptr || host == nullptr || count < c->n_local) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return SNN_ERR_UNSUPPORTED;  // per member state: use one context per device
    if (c->n_local == 0) return SNN_OK;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    if (cudaMemcpyAsync(host, c->d_cur[c->cur], c->n_local * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t snn_b200_upload_state(snn_cuda_context_t *c, const float *v, const float *cur, const uint32_t *refr,
                                   snn_size_t count) {
    if (c == nullptr || count < c->n_local) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return SNN_ERR_UNSUPPORTED;  // per member state: use one context per device
    if (c->n_local == 0) return SNN_OK;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    const uint64_t n = c->n_local;
    if (v && cudaMemcpyAsync(c->d_v, v, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return SNN_ERR_CUDA;
    if (cur && cudaMemcpyAsync(c->d_cur[c->cur], cur, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    if (refr && cudaMemcpyAsync(c->d_refr, refr, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t snn_b200_download_state(const snn_cuda_context_t *c, float *v, float *cur, uint32_t *refr,
                                     snn_size_t count) {
    if (c == nullptr || count < c->n_local) return SNN_ERR_INVALID_ARGUMENT;
    if (is_group(c)) return SNN_ERR_UNSUPPORTED;  // per member state: use one context per device
    if (c->n_local == 0) return SNN_OK;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    const uint64_t n = c->n_local;
    if (v && cudaMemcpyAsync(v, c->d_v, n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return SNN_ERR_CUDA;
    if (cur && cudaMemcpyAsync(cur, c->d_cur[c->cur], n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    if (refr && cudaMemcpyAsync(refr, c->d_refr, n * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        return SNN_ERR_CUDA;
    return cuda_status(cudaStreamSynchronize(c->stream));
}

snn_status_t snn_b200_download_topology(const snn_cuda_context_t *c, snn_size_t *row_ptr, snn_size_t row_capacity,
                                        snn_size_t *col_idx, float *weights, snn_size_t edge_capacity) {
    if (c == nullptr || is_group(c) || c->mode != SNN_CUDA_MODE_FULL || c->propagation == SNN_B200_PROPAGATE_ORDERED)
        return SNN_ERR_INVALID_ARGUMENT;
    if ((row_ptr && row_capacity < c->n_rows + 1) || ((col_idx || weights) && edge_capacity < c->e_local))
        return SNN_ERR_INVALID_ARGUMENT;
    if (set_device(c) != SNN_OK) return SNN_ERR_CUDA;
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return SNN_ERR_CUDA;
    if (row_ptr && cudaMemcpy(row_ptr, c->d_row_ptr, (c->n_rows + 1) * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
        return SNN_ERR_CUDA;
    if (weights && c->e_local &&
        cudaMemcpy(weights, c->d_w, c->e_local * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return SNN_ERR_CUDA;
    if (col_idx && c->e_local) {
        if (c->col_bits == 64) {
            if (cudaMemcpy(col_idx, c->d_col, c->e_local * 8, cudaMemcpyDeviceToHost) != cudaSuccess)
                return SNN_ERR_CUDA;
        } else {
            std::vector<uint32_t> tmp(c->e_local);
            if (cudaMemcpy(tmp.data(), c->d_col, c->e_local * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                return SNN_ERR_CUDA;
            for (uint64_t k = 0; k < c->e_local; ++k) col_idx[k] = tmp[k];
        }
        for (uint64_t k = 0; k < c->e_local; ++k) col_idx[k] += c->lo;
    }
    return SNN_OK;
}

snn_status_t snn_b200_network_wrap(snn_size_t n, snn_size_t e, const snn_size_t *row_ptr, const snn_size_t *col_idx,
                                   const float *weights, const snn_lif_params_t *lif, snn_network_t **out) {
    if (out == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    snn_status_t st = validate_csr(n, e, row_ptr, col_idx, weights);
    if (st != SNN_OK) return st;
    const snn_lif_params_t p = lif ? *lif : snn_lif_params_t{1.0f, 20.0f, 0.0f, 0.0f, 1.0f, 1.0f, 1u};
    if (!lif_valid(&p)) return SNN_ERR_INVALID_ARGUMENT;
    snn_network_t *net = new (std::nothrow) snn_network_t();
    if (net == nullptr) return SNN_ERR_OUT_OF_MEMORY;
    net->neuron_count = n;
    net->synapse_count = e;
    net->architecture = SNN_ARCH_CUSTOM_CSR;
    net->lif = p;
    net->decay = expf(-p.dt_ms / p.membrane_tau_ms);  // src/snn.c:111-113
    net->row_ptr = const_cast<snn_size_t *>(row_ptr);
    net->col_idx = const_cast<snn_size_t *>(col_idx);
    net->weights = const_cast<float *>(weights);
    *out = net;
    return SNN_OK;
}

void snn_b200_network_unwrap(snn_network_t *network) {
    if (network != nullptr && !b200host::release_mapping(network)) delete network;
}

}  // extern "C"
