/*
 * snn_b200 -- B200 (sm_100a) CUDA backend for the Ichigo-Labs/snn LIF simulator.
 *
 * Part 1 declares the reference's CUDA entry points with identical names,
 * argument types, meaning and status codes, so the library links behind the
 * reference's host code (src/snn.c) in place of src/snn_cuda.cu. When the
 * reference header <snn/snn.h> is included first, its declarations are used;
 * otherwise this header declares the same types itself (identical layouts).
 *
 * Part 2 declares the test hooks of include/snn/snn_test.h:19-25 that the
 * reference's unit tests call (deterministic fault injection).
 *
 * Part 3 declares extensions with no counterpart in the reference's CUDA API:
 * postsynaptic sharding over several GPUs (one process per GPU, NCCL spike
 * all-gather), on-device network generation, device-resident input streams,
 * state reset, ordered (CSR-order bit-exact) propagation and device timing.
 *
 * Every call is synchronous on return unless its name ends in _async.
 */
#ifndef SNN_B200_H
#define SNN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================== Part 1: reference CUDA API ====================== */
#ifndef SNN_SNN_H
/* Types of include/snn/snn.h, same names, values and layouts. */
typedef uint64_t snn_size_t; /* include/snn/snn.h:15 */

typedef enum snn_status { /* include/snn/snn.h:17-24 */
    SNN_OK = 0,
    SNN_ERR_INVALID_ARGUMENT = -1,
    SNN_ERR_OUT_OF_MEMORY = -2,
    SNN_ERR_OVERFLOW = -3,
    SNN_ERR_CUDA = -4,
    SNN_ERR_UNSUPPORTED = -5
} snn_status_t;

typedef enum snn_architecture { /* include/snn/snn.h:26-30 */
    SNN_ARCH_CUSTOM_CSR = 0,
    SNN_ARCH_FEED_FORWARD = 1,
    SNN_ARCH_RANDOM_POOL = 2
} snn_architecture_t;

typedef struct snn_lif_params { /* include/snn/snn.h:32-40 */
    float dt_ms;
    float membrane_tau_ms;
    float v_rest;
    float v_reset;
    float v_threshold;
    float input_scale;
    uint32_t refractory_steps;
} snn_lif_params_t;

typedef struct snn_random_pool_config { /* include/snn/snn.h:50-57 */
    snn_size_t neuron_count;
    snn_size_t fanout_per_neuron;
    float weight_min;
    float weight_max;
    uint64_t seed;
    int allow_self_connections;
} snn_random_pool_config_t;

typedef struct snn_network snn_network_t; /* include/snn/snn.h:87 */

typedef enum snn_cuda_mode { /* include/snn/snn.h:90-94 */
    SNN_CUDA_MODE_NONE = 0,
    SNN_CUDA_MODE_FULL = 1,
    SNN_CUDA_MODE_STREAMING = 2
} snn_cuda_mode_t;

typedef struct snn_cuda_config { /* include/snn/snn.h:96-108 */
    uint64_t max_vram_bytes;
    snn_size_t max_stream_synapses;
    snn_size_t max_stream_rows;
    int prefer_streaming;
} snn_cuda_config_t;

typedef struct snn_cuda_context snn_cuda_context_t; /* include/snn/snn.h:110 */

/* Replaces include/snn/snn.h:182 (src/snn_cuda.cu:403-410): all-zero config. */
snn_cuda_config_t snn_cuda_default_config(void);
/* Replaces include/snn/snn.h:183 (src/snn_cuda.cu:412-418): 1 if a CUDA device is usable. */
int snn_cuda_available(void);
/* Replaces include/snn/snn.h:189-191 (src/snn_cuda.cu:420-483). Chooses FULL
 * (topology resident) when the device layout fits the budget and streaming is
 * not preferred, else STREAMING (topology copied in bounded chunks each step).
 * The network must outlive the context. Propagation is the atomic push. */
snn_status_t snn_cuda_create(const snn_network_t *network, const snn_cuda_config_t *config,
                             snn_cuda_context_t **out_context);
/* Replaces include/snn/snn.h:192 (src/snn_cuda.cu:485-503). NULL-safe. */
void snn_cuda_free(snn_cuda_context_t *context);
/* Replaces include/snn/snn.h:193 (src/snn_cuda.cu:505-508). */
snn_cuda_mode_t snn_cuda_context_mode(const snn_cuda_context_t *context);
/* Replaces include/snn/snn.h:197-200 (src/snn_cuda.cu:510-563). Adds
 * values[k]*input_scale into the current the next step consumes; all indices
 * are validated before anything is applied; duplicates accumulate. Unlike the
 * reference, duplicate indices with unequal values fold in k order, matching
 * snn_state_inject_current bit for bit. */
snn_status_t snn_cuda_inject_current(snn_cuda_context_t *context, const snn_size_t *host_indices,
                                     const float *host_values, snn_size_t count);
/* Replaces include/snn/snn.h:204-206 (src/snn_cuda.cu:635-682). One LIF step
 * plus propagation; host_external_current (n floats) and host_out_spikes
 * (n bytes) are optional. On a sharded context both cover the rank's own
 * neurons only (see snn_b200_get_layout). */
snn_status_t snn_cuda_step(snn_cuda_context_t *context, const float *host_external_current,
                           uint8_t *host_out_spikes);
/* Replaces include/snn/snn.h:207-209 (src/snn_cuda.cu:684-691). count is a
 * capacity; exactly n (or the rank's local count) voltages are written. */
snn_status_t snn_cuda_download_voltage(const snn_cuda_context_t *context, float *host_voltage,
                                       snn_size_t count);
#endif /* SNN_SNN_H */

/* ===================== Part 2: reference test hooks ===================== */
#ifndef SNN_SNN_TEST_H
/* include/snn/snn_test.h:19-25 (src/snn_cuda.cu:51-67,694-698). The fault
 * seams are numbered exactly like the reference's: create #0 context calloc,
 * #1-#6 device state, #7 init launch, then FULL #8-#10 topology allocations
 * and #11-#13 uploads, or STREAMING #8 host chunk table and #9-#11 chunk
 * buffers; step #0 external upload, #1 integrate launch, #2 propagate launch
 * (STREAMING: per chunk row_ptr, col_idx, weights copy then launch), #3 spike
 * download; inject #0-#1 device buffer growth, then the index and value
 * copies and the launch. */
snn_cuda_context_t *snn_test_nonnull_cuda_context(void);
void snn_test_cuda_set_fail_after(int64_t calls_before_failure);
void snn_test_cuda_disable_failure(void);
void snn_test_cuda_force_unavailable(int enable);
void snn_test_cuda_force_meminfo_fail(int enable);
#endif

/* ===================== Part 3: snn_b200 extensions ====================== */

typedef enum snn_b200_propagation {
    /* Push from the compacted spike list with L2-resident fp32 red.add
     * (the reference's accumulation semantics; order not deterministic).
     * Contexts made with options or by the device generators also keep a
     * pull topology (chunked sliced-ELL CSC) when the device has room and
     * the network has 2^26+ synapses; steps where more than a quarter of the
     * rows fire then take the pull instead (chosen on the device), which
     * folds in CSR order. snn_cuda_create keeps the plain push. */
    SNN_B200_PROPAGATE_PUSH = 0,
    /* Every target folds its contributions in CSR order (ascending
     * presynaptic row, ascending edge): bit-identical to the reference's
     * serial CPU step (src/snn.c:898-906) for any weights. FULL and STREAMING
     * (STREAMING: each streamed chunk sorts and folds its own events, in row order).
     * Each step either sorts its events by target (a stable radix sort of
     * the spiking rows' CSR slices, then an in-order fold; cost ~ events;
     * one host read of the event count per step), or, on dense steps when a
     * CSC fits beside the CSR, pulls over the CSC (cost ~ synapses). */
    SNN_B200_PROPAGATE_ORDERED = 1,
    /* The plain push kernel: one red.global.add.f32 per event. */
    SNN_B200_PROPAGATE_PUSH_ATOMIC = 2,
    /* ORDERED through the bin-fold: each step's events are binned by target
     * tile in CSR order and every tile is folded in shared memory, gated on
     * the device against the pull for dense steps: no host round trip, so
     * multi-step runs replay as CUDA graphs. Bit-identical to ORDERED (the
     * context reports ORDERED and layout.binned = 1). */
    SNN_B200_PROPAGATE_PUSH_BINNED = 3
} snn_b200_propagation_t;

typedef enum snn_b200_exchange {
    /* ncclAllGather of the spike bitmap after the LIF kernel (needs nccl_id). */
    SNN_B200_EXCHANGE_NCCL = 0,
    /* The LIF kernel itself stores its bitmap words into every rank's buffer
     * over NVLink (CUDA IPC mappings, one node) and raises a per-step flag
     * that the other ranks wait on (bounded) before compacting. Needs
     * snn_b200_ipc_handle / snn_b200_ipc_connect after create; <= 8 ranks. */
    SNN_B200_EXCHANGE_PEER = 1
} snn_b200_exchange_t;

typedef enum snn_b200_streaming {
    /* The reference's scheme: every step copies the whole host CSR to the
     * device in bounded chunks (double-buffered: copy overlaps propagation). */
    SNN_B200_STREAMING_CHUNKED = 0,
    /* The host col_idx/weights are page-locked and mapped; each step the push
     * kernel reads only the spiking rows' edges over the host link (row_ptr
     * resident). Arrays must be 16-byte aligned; otherwise CHUNKED is used. */
    SNN_B200_STREAMING_SPARSE = 1
} snn_b200_streaming_t;

typedef struct snn_b200_options {
    int propagation;        /* snn_b200_propagation_t */
    int device;             /* CUDA device ordinal; -1 = the calling thread's current device */
    int index_width;        /* device col_idx width: 0 auto (32 bits when n <= 2^32), 32 or 64 */
    uint32_t rank;          /* shard index in [0, world_size) */
    uint32_t world_size;    /* number of postsynaptic shards (1 = unsharded) */
    const void *nccl_id;    /* 128-byte NCCL unique id (snn_b200_nccl_unique_id), world_size > 1 */
    int timing;             /* 1: record per-step device timings (snn_b200_stats) */
    int exchange;           /* snn_b200_exchange_t: how sharded ranks share spikes */
    int streaming;          /* snn_b200_streaming_t: how a STREAMING context reads the host CSR */
    uint32_t batch;         /* independent network states sharing the topology (0 or 1 = one).
                             * With batch B every per-neuron argument covers B x n neurons,
                             * sample b owning [b*n, (b+1)*n): inject indices, external
                             * current, spikes and voltages. FULL, world_size 1, PUSH /
                             * PUSH_ATOMIC / ORDERED (event-driven) only. */
} snn_b200_options_t;

typedef struct snn_b200_stats {
    uint64_t steps;            /* steps completed since create / reset_stats */
    uint64_t spikes;           /* spikes of this rank's neurons */
    uint64_t events;           /* synaptic events delivered to this rank's targets */
    uint64_t kernel_launches;  /* kernels launched by the library */
    double step_ms;            /* device time of the whole steps (timing = 1) */
    double propagate_ms;       /* device time of the propagation kernels (timing = 1) */
    double lif_ms;             /* device time of the LIF kernels (timing = 1) */
    double exchange_ms;        /* device time of the spike all-gather + compaction (timing = 1) */
    uint64_t pull_steps;       /* steps whose propagation ran the pull kernel (dense steps) */
    uint64_t pull_events;      /* synaptic events of those steps */
    uint64_t pull_spikes;      /* spiking rows of those steps */
    double propagate_pull_ms;  /* share of propagate_ms spent in those steps (timing = 1) */
    double exchange_wait_ms;   /* peer exchange: device time this rank waited for the other
                                * ranks' spike slices (flag waits, summed over steps) */
    double exchange_wait_max_ms;  /* the longest single flag wait */
} snn_b200_stats_t;

typedef struct snn_b200_layout {
    snn_size_t neuron_count;        /* global n */
    snn_size_t local_begin;         /* first neuron owned by this rank */
    snn_size_t local_count;         /* neurons owned by this rank */
    snn_size_t local_synapses;      /* edges targeting this rank's neurons */
    uint32_t index_bits;            /* 32 or 64 */
    int propagation;                /* snn_b200_propagation_t */
    uint64_t device_state_bytes;    /* resident per-neuron state + spike workspace */
    uint64_t device_topology_bytes; /* resident topology (FULL) or chunk buffers (STREAMING) */
    uint32_t binned;                /* 1: ORDERED runs the bin-fold (events binned per target tile) */
    uint32_t binned_passes;         /* bin-fold: number of target tiles */
    uint32_t ordered_csc;           /* ORDERED: 1 when a CSC is resident (pull for dense steps) */
    uint32_t batch;                 /* states sharing the topology (neuron_count = batch x rows) */
    snn_size_t topology_rows;       /* rows of the shared topology (n of the network) */
    uint64_t pull_slots;            /* slots (8-byte id/weight pairs) of the pull topology, 0 without */
} snn_b200_layout_t;

snn_b200_options_t snn_b200_default_options(void);

/* snn_cuda_create with options: propagation mode, device, index width and
 * postsynaptic sharding. With world_size > 1 every rank passes the same
 * host network and the same NCCL id; rank r owns neurons
 * [r*S, min((r+1)*S, n)) with S = ceil(n / world_size / 128) * 128. */
snn_status_t snn_b200_create(const snn_network_t *network, const snn_cuda_config_t *config,
                             const snn_b200_options_t *options, snn_cuda_context_t **out_context);

/* One context driving device_count GPUs of this process (no counterpart in
 * the reference, whose CUDA backend uses one device): the network is sharded
 * by postsynaptic neuron, rank r on devices[r] (distinct devices), and the
 * spike bitmap is exchanged every step over NVLink peer memory when every
 * pair of devices can reach the other's, else with NCCL (ncclCommInitAll).
 * The returned context works with the reference's snn_cuda_inject_current,
 * snn_cuda_step (external current and spikes cover all n neurons),
 * snn_cuda_download_voltage, snn_cuda_context_mode and snn_cuda_free, and
 * with snn_b200_reset, _get_stats, _get_layout, _run_stream_async,
 * _step_async, _inject_stream_async, _set_external, _set_stream_range and
 * _synchronize; the per-member state calls return SNN_ERR_UNSUPPORTED. With
 * ORDERED propagation the result is bit-identical to the serial CPU step at
 * any device count. device_count 1 returns a plain context on devices[0]. */
snn_status_t snn_cuda_create_sharded(const snn_network_t *network, const snn_cuda_config_t *config,
                                     int device_count, const int *devices, snn_cuda_context_t **out_context);
/* The same with options (propagation, index width, streaming mode, timing;
 * exchange: SNN_B200_EXCHANGE_PEER falls back to NCCL when a pair of devices
 * has no peer access). rank, world_size, device and nccl_id are ignored. */
snn_status_t snn_b200_create_sharded(const snn_network_t *network, const snn_cuda_config_t *config,
                                     const snn_b200_options_t *options, int device_count, const int *devices,
                                     snn_cuda_context_t **out_context);

/* Generates the network of snn_build_random_pool (src/snn.c:523-574) directly
 * on the device, bit-identical to the host builder, without a host copy:
 * edge e takes draws 2e+1 (target) and 2e+2 (weight) of the seeded splitmix64
 * stream. Each shard generates only the edges that target its neurons.
 * The context is FULL; config may be NULL. */
snn_status_t snn_b200_create_random_pool(const snn_random_pool_config_t *pool, const snn_lif_params_t *lif,
                                         const snn_cuda_config_t *config, const snn_b200_options_t *options,
                                         snn_cuda_context_t **out_context);

/* Deep layered net generated on the device: every neuron of layer l < L-1
 * sends `fanout` edges to uniform targets (with replacement) in layer l+1,
 * weights weight_min + (weight_max - weight_min) * u clamped to weight_max,
 * draws as in snn_b200_create_random_pool. At most 16 layers. */
snn_status_t snn_b200_create_layered_random(const snn_size_t *layer_sizes, size_t layer_count,
                                            snn_size_t fanout, float weight_min, float weight_max,
                                            uint64_t seed, const snn_lif_params_t *lif,
                                            const snn_b200_options_t *options,
                                            snn_cuda_context_t **out_context);

/* Device build of the reference's snn_build_feedforward (src/snn.c:463-521),
 * bit-identical: layer l's rows connect to every neuron of layer l+1 in order
 * when fanout is 0 or >= its size, else to `fanout` targets drawn from one
 * splitmix64 stream seeded with `seed` (edge order, sparse layers only);
 * every weight is `weight`. At most 16 layers. */
snn_status_t snn_b200_create_feedforward(const snn_size_t *layer_sizes, size_t layer_count, snn_size_t fanout,
                                         float weight, uint64_t seed, const snn_lif_params_t *lif,
                                         const snn_b200_options_t *options, snn_cuda_context_t **out_context);

/* Human-readable detail of the calling thread's most recent CUDA/NCCL
 * failure inside the library ("" if none); valid until the next failure. */
const char *snn_b200_last_error(void);

/* Postsynaptic shard geometry (pure host computation, no device needed):
 * rank r of world_size owns neurons [*out_begin, *out_begin + *out_count),
 * slots of S = ceil(n / world_size / 32) * 32 neurons. */
snn_status_t snn_b200_shard_range(snn_size_t neuron_count, uint32_t world_size, uint32_t rank,
                                  snn_size_t *out_begin, snn_size_t *out_count);

/* Peer exchange set-up: every rank exports the 64-byte CUDA IPC handle of its
 * exchange buffer, the caller gathers all ranks' handles in rank order
 * (world_size * 64 bytes) and hands them to every rank's context. */
snn_status_t snn_b200_ipc_handle(const snn_cuda_context_t *context, void *out_handle64);
snn_status_t snn_b200_ipc_connect(snn_cuda_context_t *context, const void *handles);

/* Test hook for failure detection: maps every peer of a sharded
 * SNN_B200_EXCHANGE_PEER context onto its own exchange buffer and sets the
 * poll budget of the exchange wait, so the other ranks' step flags never
 * arrive: the next step's bounded wait expires and the step returns
 * SNN_ERR_CUDA (no device fault, the GPU stays usable). */
snn_status_t snn_test_b200_peer_loopback(snn_cuda_context_t *context, uint32_t spin_limit);

/* Writes a fresh 128-byte NCCL unique id (rank 0 calls it and shares the bytes). */
snn_status_t snn_b200_nccl_unique_id(void *out_id128);

/* Voltages back to v_rest, currents, refractory counters and spikes to zero;
 * the topology stays resident (no re-upload). */
snn_status_t snn_b200_reset(snn_cuda_context_t *context);

/* Device-resident input: the seeded injection stream. Step t injects `count`
 * events of `value` at indices mix64(seed + (t*count + k + 1) * 0x9e3779b97f4a7c15) % n,
 * k = 0..count-1, generated on the device (each shard applies its own). */
snn_status_t snn_b200_inject_stream_async(snn_cuda_context_t *context, uint64_t seed, uint64_t step,
                                          snn_size_t count, float value);

/* `steps` steps, each after injecting step t of the seeded stream (t from
 * first_step), with no host synchronisation between steps and no host
 * copies. count = 0 runs without input. */
snn_status_t snn_b200_run_stream_async(snn_cuda_context_t *context, uint64_t seed, uint64_t first_step,
                                       uint64_t steps, snn_size_t count, float value);

/* One step without host input or output and without a final synchronisation. */
snn_status_t snn_b200_step_async(snn_cuda_context_t *context);

/* Restricts the seeded injection stream's indices to [0, range) (mix64(...)
 * % range instead of % n; range 0 restores all neurons), e.g. to drive only
 * the input layer of a layered network. */
snn_status_t snn_b200_set_stream_range(snn_cuda_context_t *context, snn_size_t range);

/* Holds an external current frame on the device (local-count floats, scaled
 * by input_scale like snn_cuda_step's): every later step that does not pass
 * its own external current adds it (snn_cuda_step with NULL, step_async,
 * run_stream_async), across snn_b200_reset, until NULL clears it or a
 * snn_cuda_step call passes its own frame (which replaces it for that step
 * and ends the hold). For static per-sample inputs (one upload, many steps). */
snn_status_t snn_b200_set_external(snn_cuda_context_t *context, const float *host_external_current);

/* Waits for all work of the context; folds pending timings into the stats. */
snn_status_t snn_b200_synchronize(snn_cuda_context_t *context);

snn_status_t snn_b200_get_stats(snn_cuda_context_t *context, snn_b200_stats_t *out_stats);
snn_status_t snn_b200_reset_stats(snn_cuda_context_t *context);
snn_status_t snn_b200_get_layout(const snn_cuda_context_t *context, snn_b200_layout_t *out_layout);

/* The context's CUDA stream (a cudaStream_t), for callers that order their
 * own work or events against the library's. */
void *snn_b200_stream(const snn_cuda_context_t *context);

/* Checkpoint / resume of this rank's neuron state: voltages, the current the
 * next step consumes (propagated + injected so far) and refractory counters,
 * `count` >= local neuron count (exactly the local count is read/written).
 * Any pointer may be NULL to skip that array. */
snn_status_t snn_b200_upload_state(snn_cuda_context_t *context, const float *voltage, const float *current,
                                   const uint32_t *refractory, snn_size_t count);
snn_status_t snn_b200_download_state(const snn_cuda_context_t *context, float *voltage, float *current,
                                     uint32_t *refractory, snn_size_t count);

/* Diagnostics for parity tests: copy this rank's spike bytes (last step),
 * the current the next step will consume, or the device topology. */
snn_status_t snn_b200_download_spikes(const snn_cuda_context_t *context, uint8_t *host_spikes, snn_size_t count);
snn_status_t snn_b200_download_current(const snn_cuda_context_t *context, float *host_current, snn_size_t count);
/* Device CSR of a FULL push context (row_ptr over all n presynaptic rows,
 * col_idx as global neuron ids, weights); pass NULL to skip an array. */
snn_status_t snn_b200_download_topology(const snn_cuda_context_t *context, snn_size_t *row_ptr,
                                        snn_size_t row_capacity, snn_size_t *col_idx, float *weights,
                                        snn_size_t edge_capacity);

/* A network view over caller-owned CSR arrays (no copy; the arrays must
 * outlive the view and every context made from it), for callers that do not
 * link the reference's host library. Validates like snn_build_custom_csr
 * (src/snn.c:158-180, 427-461). */
snn_status_t snn_b200_network_wrap(snn_size_t neuron_count, snn_size_t synapse_count, const snn_size_t *row_ptr,
                                   const snn_size_t *col_idx, const float *weights, const snn_lif_params_t *lif,
                                   snn_network_t **out_network);
void snn_b200_network_unwrap(snn_network_t *network);

/* The snn_b200 CSR file: header (4096 bytes: magic "SNNCSR01", version 1,
 * n, e, architecture, LIF parameters, decay, section offsets, file size),
 * then u64 row_ptr[n+1], u64 col_idx[e], f32 weights[e], each section
 * 4096-byte aligned. snn_b200_network_save writes any network (written under
 * "<path>.partial", then renamed). snn_b200_network_map maps a file read-only
 * (no copy), validates it like snn_build_custom_csr and returns a network
 * view that works with every create call; release it with
 * snn_b200_network_unwrap (which unmaps it) after its contexts are freed.
 * STREAMING contexts over a mapped network copy their chunks straight from
 * the page cache (the library tries to lock the mapping read-only; where the
 * OS refuses to lock file pages, SPARSE streaming falls back to chunks). */
snn_status_t snn_b200_network_save(const snn_network_t *network, const char *path);
snn_status_t snn_b200_network_map(const char *path, snn_network_t **out_network);

/* Diagnostic, no counterpart in the reference: the rate (per second) at which
 * this device's L2 serves red.global.add.f32 to uniformly random slots of a
 * `targets`-float array (the push propagation's access pattern), measured
 * over `repeats` launches of `events` reductions. Allocates its own buffers. */
snn_status_t snn_b200_probe_red_rate(int device, uint64_t targets, uint64_t events, uint32_t repeats,
                                     double *out_reds_per_s);

/* Largest network snn_b200_step_noalloc accepts: its scratch is a fixed
 * array of this many spike-list entries (plus bitmap and counters, ~4.2 MB)
 * compiled into the library and resident on every GPU that loads it. */
#define SNN_B200_NOALLOC_MAX_NEURONS 1048576u

/* No counterpart in the reference: it has no allocation-free call.
 *
 * One push-mode step (LIF update, spike compaction, propagation) over device
 * arrays the caller owns, for callers that cannot allocate device memory
 * while they run -- memory owned by an outer framework's pool or arena, or
 * loops where allocation after start-up is forbidden. It calls no cudaMalloc,
 * cudaFree or other allocating routine; its only scratch is the fixed
 * library array above. Same arithmetic as snn_cuda_step on a FULL push
 * context: `current` (the input this step consumes) is zeroed, `next_current`
 * must be all zero on entry and receives the propagated input; swap the two
 * before the next call. `external` may be NULL (every other array is
 * required; a network without edges still passes aligned col_idx and weights
 * buffers); row_ptr holds n+1 edge offsets, col_idx 32-bit target ids. Neuron, external, col_idx and weight
 * arrays must be 16-byte aligned, spikes 4-byte aligned.
 *
 * Work is enqueued on `stream` (a cudaStream_t, NULL = legacy default) of
 * `device`; the call does not synchronise. neuron_count of 0 or above
 * SNN_B200_NOALLOC_MAX_NEURONS, NULL or misaligned arrays return
 * SNN_ERR_INVALID_ARGUMENT. The first call on a device looks up the scratch
 * array's device address (make it before any stream capture) and keeps it for
 * the lifetime of the device's primary context: do not call it again on a
 * device after cudaDeviceReset. All calls on a device share the scratch:
 * calls that overlap on the GPU race. */
snn_status_t snn_b200_step_noalloc(int device, void *stream, snn_size_t neuron_count, const snn_lif_params_t *lif,
                                   float decay, float *voltage, float *current, const float *external,
                                   uint32_t *refractory, uint8_t *spikes, const snn_size_t *row_ptr,
                                   const uint32_t *col_idx, const float *weights, float *next_current);

#ifdef __cplusplus
}
#endif

#endif /* SNN_B200_H */
