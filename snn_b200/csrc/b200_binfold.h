// Bin-fold propagation (b200_binfold.cu): bit-exact CSR-order propagation
// driven by an ordered spike list, device-gated against the pull on dense steps.
#pragma once

#include "b200_kernels.h"

namespace b200 {

constexpr uint32_t kBinFoldMaxTiles = 2048;

struct BinFoldPlan {
    uint32_t tile_bits;     // targets per tile = 2^tile_bits (1024 .. 32768)
    uint32_t tiles;         // ceil(n_local / 2^tile_bits) <= kBinFoldMaxTiles
    uint32_t grid;          // CTAs of the count and scatter kernels (spike-list slices)
    uint64_t hist_entries;  // tiles * grid + 1 (the last entry stays 0: the scan's total)
    uint32_t chunks;        // compaction chunks of the bitmap
};

struct BinFoldBuffers {
    uint32_t *hist = nullptr;   // [hist_entries], tile-major
    uint32_t *offs = nullptr;   // [hist_entries], exclusive scan of hist
    uint2 *bins = nullptr;      // [cap] (target within tile, weight bits)
    uint32_t *ccnt = nullptr;   // [chunks] per-chunk spike counts
    void *scan_temp = nullptr;
    size_t scan_bytes = 0;
};

// false when n_local needs more than kBinFoldMaxTiles tiles of 32768.
bool binfold_plan(int device, uint64_t n_local, BinFoldPlan *plan);
uint32_t binfold_chunks(uint64_t words);
// Scan of n hist entries (temp == nullptr: query the temp size).
cudaError_t binfold_scan(cudaStream_t s, const uint32_t *hist, uint32_t *offs, uint64_t n, void *temp,
                         size_t *temp_bytes);

// Ordered compaction of the global bitmap (words of 32 neurons) into the
// ascending spike list of parity `parity`; adds the own-range popcount to
// ctr->spikes and the spiking rows' degrees to ctr->step_events[parity].
// With a peer wait, first waits (bounded) for every rank's flag.
void launch_compact_ordered(cudaStream_t s, int device, uint32_t *bitmap, uint64_t words, uint32_t *ccnt,
                            void *list, int idx_bits, DevCounters *ctr, int parity, uint64_t own_begin,
                            uint64_t own_end, const uint64_t *row_ptr, uint64_t batch_rows,
                            const PeerWait *wait = nullptr);

// Count, scan, scatter and fold of one step (skipped on the device when
// step_events[parity] > gate). The fold runs the step epilogue.
cudaError_t launch_binfold(cudaStream_t s, int device, const BinFoldPlan &plan, const BinFoldBuffers &buf,
                           const void *list, int idx_bits, const uint64_t *row_ptr, const void *col, int col_bits,
                           const float *w, uint64_t batch_rows, uint64_t n_local, float *next, DevCounters *ctr,
                           int parity, unsigned long long gate);

}  // namespace b200
