// Host-side network view shared by the C ABI translation units.
#pragma once

#include "snn_b200.h"

// Same field layout as the reference's struct snn_network (src/snn_internal.h:15-24):
// the backend reads a network built by the reference's host library directly.
struct snn_network {
    snn_size_t neuron_count;
    snn_size_t synapse_count;
    snn_architecture_t architecture;
    snn_lif_params_t lif;
    float decay;
    snn_size_t *row_ptr;
    snn_size_t *col_idx;
    float *weights;
};

namespace b200host {

// src/snn.c:308-316
bool lif_valid(const snn_lif_params_t *p);
// src/snn.c:158-180 (custom CSR validation).
snn_status_t validate_csr(uint64_t n, uint64_t e, const uint64_t *row_ptr, const uint64_t *col, const float *w);
// Networks mapped from a CSR file (b200_csr_file.cu) own their mapping:
// unmaps and frees such a network and returns true, else returns false.
bool release_mapping(snn_network_t *network);

}  // namespace b200host
