/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the snn_b200 parity tests.
 *
 * A plain-C restatement of the reference simulator's CPU path
 * (Ichigo-Labs/snn src/snn.c): LIF parameters, the deterministic network
 * builders, the memory dry-run, the simulation state, sparse injection and the
 * serial CSR-order step. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it, and only as the checker or the timed CPU
 * baseline; the shipped library (snn_b200/) never links or calls it.
 *
 * Parity pin: tests/test_oracle_pin.py checks every function here against the
 * reference's own known-answer tests (tests/test_snn.c) and, where the
 * reference compiles in this container, against the reference library itself
 * (oracle/_ref, built by oracle/Makefile); tests/golden/ holds the committed
 * fixtures generated from oracle/_ref by tests/golden/make_golden.py.
 *
 * The network struct has the reference's exact field layout
 * (src/snn_internal.h:15-24) so that a network built here can be handed to the
 * snn_b200 backend exactly like one built by the reference's src/snn.c.
 */
#ifndef SNN_ORACLE_H
#define SNN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t orc_size_t;

/* Status codes: same values as the reference's snn_status_t (include/snn/snn.h:17-24). */
enum {
    ORC_OK = 0,
    ORC_ERR_INVALID_ARGUMENT = -1,
    ORC_ERR_OUT_OF_MEMORY = -2,
    ORC_ERR_OVERFLOW = -3
};

/* include/snn/snn.h:32-40 */
typedef struct orc_lif_params {
    float dt_ms;
    float membrane_tau_ms;
    float v_rest;
    float v_reset;
    float v_threshold;
    float input_scale;
    uint32_t refractory_steps;
} orc_lif_params_t;

/* Same layout as the reference's struct snn_network (src/snn_internal.h:15-24). */
typedef struct orc_network {
    orc_size_t neuron_count;
    orc_size_t synapse_count;
    int architecture; /* 0 custom CSR, 1 feed-forward, 2 random pool */
    orc_lif_params_t lif;
    float decay;
    orc_size_t *row_ptr;
    orc_size_t *col_idx;
    float *weights;
} orc_network_t;

typedef struct orc_state {
    orc_size_t neuron_count;
    float *voltage;
    float *current;
    float *next_current;
    uint32_t *refractory;
    uint8_t *spikes;
    orc_size_t *spike_indices;
    orc_size_t spike_count;
} orc_state_t;

/* Mirrors snn_memory_plan_t (include/snn/snn.h:71-85). */
typedef struct orc_memory_plan {
    orc_size_t neuron_count;
    orc_size_t synapse_count;
    uint64_t row_ptr_bytes;
    uint64_t col_index_bytes;
    uint64_t weight_bytes;
    uint64_t host_topology_bytes;
    uint64_t host_state_bytes;
    uint64_t host_total_bytes;
    uint64_t device_topology_bytes;
    uint64_t device_state_bytes;
    uint64_t device_total_full_bytes;
    uint64_t device_streaming_min_bytes;
    int overflowed;
} orc_memory_plan_t;

/* ---- random numbers (src/snn.c:94-105) ---- */
uint64_t orc_splitmix64_next(uint64_t *state);
float orc_uniform_float(uint64_t *state);

/* ---- parameters (src/snn.c:290-316) ---- */
orc_lif_params_t orc_default_lif_params(void);
int orc_lif_params_validate(const orc_lif_params_t *params);
float orc_lif_decay(const orc_lif_params_t *params);

/* ---- builders (src/snn.c:427-574) ---- */
int orc_build_custom_csr(orc_size_t neuron_count, orc_size_t synapse_count, const orc_size_t *row_ptr,
                         const orc_size_t *col_idx, const float *weights, const orc_lif_params_t *params,
                         orc_network_t **out);
int orc_build_feedforward(const orc_size_t *layer_sizes, size_t layer_count, orc_size_t fanout, float weight,
                          uint64_t seed, const orc_lif_params_t *params, orc_network_t **out);
int orc_build_random_pool(orc_size_t neuron_count, orc_size_t fanout, float weight_min, float weight_max,
                          uint64_t seed, int allow_self, const orc_lif_params_t *params, orc_network_t **out);
/* orc_build_random_pool filled by all host threads (OpenMP), bit-identical. */
int orc_build_random_pool_parallel(orc_size_t neuron_count, orc_size_t fanout, float weight_min,
                                   float weight_max, uint64_t seed, int allow_self,
                                   const orc_lif_params_t *params, orc_network_t **out);
/* Deep fixed-fanout layered net: every neuron of layer l < L-1
 * sends `fanout` edges to uniform targets (with replacement) in layer l+1, weights
 * U[wmin, wmax] with the random-pool interpolation; the last layer has no edges. */
int orc_build_layered_random(const orc_size_t *layer_sizes, size_t layer_count, orc_size_t fanout,
                             float weight_min, float weight_max, uint64_t seed, const orc_lif_params_t *params,
                             orc_network_t **out);
/* Dense layered net with N(0, 1/sqrt(fan_in)) weights. */
int orc_build_dense_gaussian(const orc_size_t *layer_sizes, size_t layer_count, uint64_t seed,
                             const orc_lif_params_t *params, orc_network_t **out);
void orc_network_free(orc_network_t *network);
int orc_network_set_lif_params(orc_network_t *network, const orc_lif_params_t *params);

/* ---- memory dry-run (src/snn.c:339-425) ---- */
int orc_estimate_memory_for_counts(orc_size_t neuron_count, orc_size_t synapse_count, orc_memory_plan_t *out);
int orc_network_memory_plan(const orc_network_t *network, orc_memory_plan_t *out);

/* ---- state, injection, step (src/snn.c:623-937) ---- */
int orc_state_create(const orc_network_t *network, orc_state_t **out);
void orc_state_free(orc_state_t *state);
int orc_state_reset(const orc_network_t *network, orc_state_t *state);
int orc_state_inject_current(const orc_network_t *network, orc_state_t *state, const orc_size_t *indices,
                             const float *values, orc_size_t count);
int orc_step(const orc_network_t *network, orc_state_t *state, const float *external_current,
             uint8_t *out_spikes);
/* Synaptic events of the last step: sum of out-degrees of the spiking rows. */
uint64_t orc_last_step_events(const orc_network_t *network, const orc_state_t *state);

/* ---- seeded per-step input streams shared with the GPU benchmark ---- */
/* Indices of step `step`: draws step*count+1 .. step*count+count of the
 * splitmix64 stream seeded `seed`, each reduced modulo neuron_count. */
void orc_inject_stream_indices(uint64_t seed, uint64_t step, orc_size_t count, orc_size_t neuron_count,
                               orc_size_t *out_indices);
/* Run `steps` steps, each injecting `count` stream indices of value `value`
 * (NULL external). Writes the per-step spike count and event count when the
 * output arrays are non-NULL, and an FNV-1a hash of every step's spike vector. */
int orc_run_inject_stream(const orc_network_t *network, orc_state_t *state, uint64_t seed,
                          uint64_t first_step, uint64_t steps, orc_size_t count, float value,
                          uint64_t *out_spike_counts, uint64_t *out_events, uint64_t *out_hashes,
                          uint8_t *out_raster);
/* Config-1 style static frame: layer-0 pixels U[0,1] from the stream, each
 * zeroed when a second draw falls below zero_prob; zeros beyond `pixels`. */
void orc_sparse_frame(uint64_t seed, uint64_t sample, orc_size_t pixels, float zero_prob,
                      orc_size_t neuron_count, float *out_frame);

uint64_t orc_fnv1a(const void *data, size_t bytes, uint64_t h);

#ifdef __cplusplus
}
#endif

#endif /* SNN_ORACLE_H */
