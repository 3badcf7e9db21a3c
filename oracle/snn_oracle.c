/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the snn_b200 parity tests.
 * See snn_oracle.h for what may use it. Every function states the reference
 * lines (Ichigo-Labs/snn) whose behaviour it restates.
 *
 * Compile with -ffp-contract=off (oracle/Makefile does): the reference's
 * bit-exactness contract assumes no fused multiply-add on the host
 * (CMakeLists.txt:57-60, README.md:51-52).
 */
#include "snn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORC_GAMMA UINT64_C(0x9e3779b97f4a7c15)

static int add_u64(uint64_t a, uint64_t b, uint64_t *out) {
    if (UINT64_MAX - a < b) {
        return 0;
    }
    *out = a + b;
    return 1;
}

static int mul_u64(uint64_t a, uint64_t b, uint64_t *out) {
    if (a != 0 && b > UINT64_MAX / a) {
        return 0;
    }
    *out = a * b;
    return 1;
}

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}

/* src/snn.c:94-99: the state advances by the golden gamma, then is mixed. */
uint64_t orc_splitmix64_next(uint64_t *state) {
    *state += ORC_GAMMA;
    return mix64(*state);
}

/* Draw number d (1-based) of the stream seeded `seed`, without iterating. */
static uint64_t draw_at(uint64_t seed, uint64_t d) {
    return mix64(seed + d * ORC_GAMMA);
}

static float unit_from_bits(uint64_t r) {
    const double unit = (double)(r >> 11) * (1.0 / 9007199254740992.0);
    return (float)unit;
}

/* src/snn.c:101-105: top 53 bits as a double in [0,1), rounded to float. */
float orc_uniform_float(uint64_t *state) {
    return unit_from_bits(orc_splitmix64_next(state));
}

/* src/snn.c:290-300 */
orc_lif_params_t orc_default_lif_params(void) {
    orc_lif_params_t p;
    p.dt_ms = 1.0f;
    p.membrane_tau_ms = 20.0f;
    p.v_rest = 0.0f;
    p.v_reset = 0.0f;
    p.v_threshold = 1.0f;
    p.input_scale = 1.0f;
    p.refractory_steps = 1u;
    return p;
}

/* src/snn.c:308-316 */
int orc_lif_params_validate(const orc_lif_params_t *p) {
    if (p == NULL || !isfinite(p->dt_ms) || !isfinite(p->membrane_tau_ms) || !isfinite(p->v_rest) ||
        !isfinite(p->v_reset) || !isfinite(p->v_threshold) || !isfinite(p->input_scale) || p->dt_ms <= 0.0f ||
        p->membrane_tau_ms <= 0.0f || p->v_threshold <= p->v_reset) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    return ORC_OK;
}

/* src/snn.c:111-113: decay = expf(-dt/tau), computed once on the host. */
float orc_lif_decay(const orc_lif_params_t *p) {
    return expf(-p->dt_ms / p->membrane_tau_ms);
}

/* src/snn.c:115-156 */
static int alloc_network(orc_size_t n, orc_size_t e, int arch, const orc_lif_params_t *params,
                         orc_network_t **out) {
    orc_lif_params_t lif = params != NULL ? *params : orc_default_lif_params();
    uint64_t rows = 0, tmp = 0;
    orc_network_t *net = NULL;
    *out = NULL;
    if (orc_lif_params_validate(&lif) != ORC_OK) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    if (!add_u64(n, 1u, &rows) || !mul_u64(rows, 8u, &tmp) || !mul_u64(e, 8u, &tmp)) {
        return ORC_ERR_OVERFLOW;
    }
    net = (orc_network_t *)calloc(1u, sizeof(*net));
    if (net == NULL) {
        return ORC_ERR_OUT_OF_MEMORY;
    }
    net->row_ptr = (orc_size_t *)calloc((size_t)rows, sizeof(orc_size_t));
    net->col_idx = e == 0 ? NULL : (orc_size_t *)malloc((size_t)e * sizeof(orc_size_t));
    net->weights = e == 0 ? NULL : (float *)malloc((size_t)e * sizeof(float));
    if (net->row_ptr == NULL || (e != 0 && (net->col_idx == NULL || net->weights == NULL))) {
        orc_network_free(net);
        return ORC_ERR_OUT_OF_MEMORY;
    }
    net->neuron_count = n;
    net->synapse_count = e;
    net->architecture = arch;
    net->lif = lif;
    net->decay = orc_lif_decay(&lif);
    *out = net;
    return ORC_OK;
}

void orc_network_free(orc_network_t *net) {
    if (net != NULL) {
        free(net->row_ptr);
        free(net->col_idx);
        free(net->weights);
        free(net);
    }
}

/* src/snn.c:613-621 */
int orc_network_set_lif_params(orc_network_t *net, const orc_lif_params_t *params) {
    orc_lif_params_t lif = params != NULL ? *params : orc_default_lif_params();
    if (net == NULL || orc_lif_params_validate(&lif) != ORC_OK) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    net->lif = lif;
    net->decay = orc_lif_decay(&lif);
    return ORC_OK;
}

/* src/snn.c:158-180 (validate_csr) and :427-461 (snn_build_custom_csr). */
int orc_build_custom_csr(orc_size_t n, orc_size_t e, const orc_size_t *row_ptr, const orc_size_t *col_idx,
                         const float *weights, const orc_lif_params_t *params, orc_network_t **out) {
    orc_size_t i;
    int st;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    if (n == 0 || row_ptr == NULL || (e != 0 && (col_idx == NULL || weights == NULL))) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    if (row_ptr[0] != 0 || row_ptr[n] != e) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    for (i = 0; i < n; ++i) {
        if (row_ptr[i] > row_ptr[i + 1u] || row_ptr[i + 1u] > e) {
            return ORC_ERR_INVALID_ARGUMENT;
        }
    }
    for (i = 0; i < e; ++i) {
        if (col_idx[i] >= n || !isfinite(weights[i])) {
            return ORC_ERR_INVALID_ARGUMENT;
        }
    }
    st = alloc_network(n, e, 0, params, out);
    if (st != ORC_OK) {
        return st;
    }
    memcpy((*out)->row_ptr, row_ptr, (size_t)(n + 1u) * sizeof(orc_size_t));
    if (e != 0) {
        memcpy((*out)->col_idx, col_idx, (size_t)e * sizeof(orc_size_t));
        memcpy((*out)->weights, weights, (size_t)e * sizeof(float));
    }
    return ORC_OK;
}

/* Layer totals of a layered build; fanout 0 or >= post means dense
 * (src/snn.c:182-212, count_feedforward_synapses). */
static int layered_counts(const orc_size_t *sizes, size_t layers, orc_size_t fanout, orc_size_t *out_n,
                          orc_size_t *out_e) {
    uint64_t n = 0, e = 0;
    size_t l;
    if (sizes == NULL || layers < 2u) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    for (l = 0; l < layers; ++l) {
        if (sizes[l] == 0) {
            return ORC_ERR_INVALID_ARGUMENT;
        }
        if (!add_u64(n, sizes[l], &n)) {
            return ORC_ERR_OVERFLOW;
        }
    }
    for (l = 0; l + 1u < layers; ++l) {
        const orc_size_t post = sizes[l + 1u];
        const orc_size_t f = (fanout == 0 || fanout >= post) ? post : fanout;
        uint64_t le = 0;
        if (!mul_u64(sizes[l], f, &le) || !add_u64(e, le, &e)) {
            return ORC_ERR_OVERFLOW;
        }
    }
    *out_n = n;
    *out_e = e;
    return ORC_OK;
}

/* src/snn.c:463-521: one sequential splitmix64 stream over the whole build; a
 * draw is consumed only for sampled (non-dense) layers. */
int orc_build_feedforward(const orc_size_t *sizes, size_t layers, orc_size_t fanout, float weight, uint64_t seed,
                          const orc_lif_params_t *params, orc_network_t **out) {
    orc_size_t n = 0, e = 0, edge = 0, pre = 0, offset = 0;
    orc_network_t *net = NULL;
    uint64_t rng = seed;
    size_t l;
    int st;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    st = layered_counts(sizes, layers, fanout, &n, &e);
    if (st != ORC_OK) {
        return st;
    }
    if (!isfinite(weight)) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    st = alloc_network(n, e, 1, params, &net);
    if (st != ORC_OK) {
        return st;
    }
    for (l = 0; l + 1u < layers; ++l) {
        const orc_size_t pre_count = sizes[l];
        const orc_size_t post_count = sizes[l + 1u];
        const orc_size_t post_base = offset + pre_count;
        const orc_size_t f = (fanout == 0 || fanout >= post_count) ? post_count : fanout;
        orc_size_t i, j;
        for (i = 0; i < pre_count; ++i, ++pre) {
            net->row_ptr[pre] = edge;
            for (j = 0; j < f; ++j) {
                const orc_size_t post_local = (f == post_count) ? j : orc_splitmix64_next(&rng) % post_count;
                net->col_idx[edge] = post_base + post_local;
                net->weights[edge] = weight;
                ++edge;
            }
        }
        offset += pre_count;
    }
    while (pre <= n) {
        net->row_ptr[pre++] = edge;
    }
    *out = net;
    return ORC_OK;
}

/* src/snn.c:559-567: min + span*u in float (no FMA), clamped to max. */
static float lerp_weight(float wmin, float wmax, float u) {
    const float w = wmin + (wmax - wmin) * u;
    return w < wmax ? w : wmax;
}

/* src/snn.c:523-574 */
int orc_build_random_pool(orc_size_t n, orc_size_t fanout, float wmin, float wmax, uint64_t seed, int allow_self,
                          const orc_lif_params_t *params, orc_network_t **out) {
    uint64_t e = 0;
    orc_network_t *net = NULL;
    uint64_t rng = seed;
    orc_size_t pre, edge = 0;
    int st;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    if (n == 0 || (!allow_self && n == 1u && fanout != 0u) || !isfinite(wmin) || !isfinite(wmax) || wmax < wmin ||
        !isfinite(wmax - wmin)) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    if (!mul_u64(n, fanout, &e)) {
        return ORC_ERR_OVERFLOW;
    }
    st = alloc_network(n, e, 2, params, &net);
    if (st != ORC_OK) {
        return st;
    }
    for (pre = 0; pre < n; ++pre) {
        orc_size_t j;
        net->row_ptr[pre] = edge;
        for (j = 0; j < fanout; ++j) {
            orc_size_t post = orc_splitmix64_next(&rng) % n;
            const float u = orc_uniform_float(&rng);
            if (!allow_self && post == pre) {
                post = (post + 1u) % n;
            }
            net->col_idx[edge] = post;
            net->weights[edge] = lerp_weight(wmin, wmax, u);
            ++edge;
        }
    }
    net->row_ptr[n] = edge;
    *out = net;
    return ORC_OK;
}

/* The same network as orc_build_random_pool, built by all host threads.
 * Draw d of the stream is mix64(seed + d * gamma) (src/snn.c:94-99), so edge
 * e = pre * fanout + j reads draws 2e+1 (target) and 2e+2 (weight) in any
 * order: the rows are filled in parallel and the result is bit-identical to
 * the serial builder (src/snn.c:523-574). Used to give the reference's own
 * CPU step a full-size (10M x 1000) pool in seconds instead of minutes. */
int orc_build_random_pool_parallel(orc_size_t n, orc_size_t fanout, float wmin, float wmax, uint64_t seed,
                                   int allow_self, const orc_lif_params_t *params, orc_network_t **out) {
    uint64_t e = 0;
    orc_network_t *net = NULL;
    int64_t pre;
    int st;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    if (n == 0 || (!allow_self && n == 1u && fanout != 0u) || !isfinite(wmin) || !isfinite(wmax) || wmax < wmin ||
        !isfinite(wmax - wmin)) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    if (!mul_u64(n, fanout, &e) || n > (orc_size_t)INT64_MAX) {
        return ORC_ERR_OVERFLOW;
    }
    st = alloc_network(n, e, 2, params, &net);
    if (st != ORC_OK) {
        return st;
    }
#pragma omp parallel for schedule(static)
    for (pre = 0; pre < (int64_t)n; ++pre) {
        orc_size_t j;
        orc_size_t edge = (orc_size_t)pre * fanout;
        net->row_ptr[pre] = edge;
        for (j = 0; j < fanout; ++j, ++edge) {
            orc_size_t post = mix64(seed + (2u * edge + 1u) * ORC_GAMMA) % n;
            const float u = unit_from_bits(mix64(seed + (2u * edge + 2u) * ORC_GAMMA));
            if (!allow_self && post == (orc_size_t)pre) {
                post = (post + 1u) % n;
            }
            net->col_idx[edge] = post;
            net->weights[edge] = lerp_weight(wmin, wmax, u);
        }
    }
    net->row_ptr[n] = e;
    *out = net;
    return ORC_OK;
}

/* BASELINE config 4 generator (no reference builder exists for it): edge e in
 * CSR order takes draws 2e+1 (target) and 2e+2 (weight) of the stream seeded
 * `seed`, exactly like the random-pool builder's per-edge pair. */
int orc_build_layered_random(const orc_size_t *sizes, size_t layers, orc_size_t fanout, float wmin, float wmax,
                             uint64_t seed, const orc_lif_params_t *params, orc_network_t **out) {
    orc_size_t n = 0, e = 0, pre = 0, edge = 0, offset = 0;
    orc_network_t *net = NULL;
    size_t l;
    int st;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    if (fanout == 0 || !isfinite(wmin) || !isfinite(wmax) || wmax < wmin || !isfinite(wmax - wmin)) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    st = layered_counts(sizes, layers, 0, &n, &e);
    if (st != ORC_OK) {
        return st;
    }
    e = 0;
    for (l = 0; l + 1u < layers; ++l) {
        e += sizes[l] * fanout;
    }
    st = alloc_network(n, e, 0, params, &net);
    if (st != ORC_OK) {
        return st;
    }
    for (l = 0; l < layers; ++l) {
        const orc_size_t count = sizes[l];
        const int last = (l + 1u == layers);
        const orc_size_t post_base = offset + count;
        const orc_size_t post_count = last ? 0 : sizes[l + 1u];
        orc_size_t i, j;
        for (i = 0; i < count; ++i, ++pre) {
            net->row_ptr[pre] = edge;
            if (last) {
                continue;
            }
            for (j = 0; j < fanout; ++j) {
                const uint64_t r_post = draw_at(seed, 2u * edge + 1u);
                const uint64_t r_w = draw_at(seed, 2u * edge + 2u);
                net->col_idx[edge] = post_base + r_post % post_count;
                net->weights[edge] = lerp_weight(wmin, wmax, unit_from_bits(r_w));
                ++edge;
            }
        }
        offset += count;
    }
    net->row_ptr[n] = edge;
    *out = net;
    return ORC_OK;
}

/* BASELINE config 1 generator: dense all-to-all between consecutive layers,
 * weight of edge e = sigma * z with z from the Box-Muller transform
 * (Box & Muller 1958) of draws 2e+1, 2e+2, sigma = 1/sqrt(pre-layer size).
 * Computed in double, rounded once to float. */
int orc_build_dense_gaussian(const orc_size_t *sizes, size_t layers, uint64_t seed, const orc_lif_params_t *params,
                             orc_network_t **out) {
    orc_size_t n = 0, e = 0, pre = 0, edge = 0, offset = 0;
    orc_network_t *net = NULL;
    size_t l;
    int st;
    const double two_pi = 6.283185307179586476925286766559;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    st = layered_counts(sizes, layers, 0, &n, &e);
    if (st != ORC_OK) {
        return st;
    }
    st = alloc_network(n, e, 1, params, &net);
    if (st != ORC_OK) {
        return st;
    }
    for (l = 0; l < layers; ++l) {
        const orc_size_t count = sizes[l];
        const int last = (l + 1u == layers);
        const orc_size_t post_base = offset + count;
        const orc_size_t post_count = last ? 0 : sizes[l + 1u];
        const double sigma = 1.0 / sqrt((double)count);
        orc_size_t i, j;
        for (i = 0; i < count; ++i, ++pre) {
            net->row_ptr[pre] = edge;
            for (j = 0; j < post_count; ++j) {
                const double u1 = (double)(draw_at(seed, 2u * edge + 1u) >> 11) * (1.0 / 9007199254740992.0);
                const double u2 = (double)(draw_at(seed, 2u * edge + 2u) >> 11) * (1.0 / 9007199254740992.0);
                const double z = sqrt(-2.0 * log(1.0 - u1)) * cos(two_pi * u2);
                net->col_idx[edge] = post_base + j;
                net->weights[edge] = (float)(sigma * z);
                ++edge;
            }
        }
        offset += count;
    }
    net->row_ptr[n] = edge;
    *out = net;
    return ORC_OK;
}

/* src/snn.c:339-396 */
int orc_estimate_memory_for_counts(orc_size_t n, orc_size_t e, orc_memory_plan_t *out) {
    uint64_t np1, row, col, w, topo, fl, refr, spk, sidx, dev, host, smin;
    if (out == NULL || n == 0) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    memset(out, 0, sizeof(*out));
    out->neuron_count = n;
    out->synapse_count = e;
    if (!add_u64(n, 1u, &np1) || !mul_u64(np1, 8u, &row) || !mul_u64(e, 8u, &col) || !mul_u64(e, 4u, &w) ||
        !add_u64(row, col, &topo) || !add_u64(topo, w, &topo) || !mul_u64(n, 16u, &fl) || !mul_u64(n, 4u, &refr) ||
        !mul_u64(n, 1u, &spk) || !mul_u64(n, 8u, &sidx) || !add_u64(fl, refr, &dev) || !add_u64(dev, spk, &dev) ||
        !add_u64(dev, 8u * 2u + 8u + 4u, &smin)) {
        out->overflowed = 1;
        return ORC_ERR_OVERFLOW;
    }
    host = dev - n * 4u;
    if (!add_u64(host, sidx, &host) || !add_u64(topo, host, &out->host_total_bytes)) {
        out->overflowed = 1;
        return ORC_ERR_OVERFLOW;
    }
    out->row_ptr_bytes = row;
    out->col_index_bytes = col;
    out->weight_bytes = w;
    out->host_topology_bytes = topo;
    out->host_state_bytes = host;
    out->device_topology_bytes = topo;
    out->device_state_bytes = dev;
    out->device_streaming_min_bytes = smin;
    out->device_total_full_bytes = topo + dev;
    return ORC_OK;
}

/* src/snn.c:398-425 */
int orc_network_memory_plan(const orc_network_t *net, orc_memory_plan_t *out) {
    orc_size_t i, maxdeg = 0, chunk;
    int st;
    if (net == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    st = orc_estimate_memory_for_counts(net->neuron_count, net->synapse_count, out);
    if (st != ORC_OK) {
        return st;
    }
    for (i = 0; i < net->neuron_count; ++i) {
        const orc_size_t d = net->row_ptr[i + 1u] - net->row_ptr[i];
        maxdeg = d > maxdeg ? d : maxdeg;
    }
    chunk = maxdeg > 1u ? maxdeg : 1u;
    out->device_streaming_min_bytes += (chunk - 1u) * 12u;
    return ORC_OK;
}

/* src/snn.c:623-696 */
int orc_state_create(const orc_network_t *net, orc_state_t **out) {
    orc_state_t *s;
    size_t n;
    if (out == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    *out = NULL;
    if (net == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    n = (size_t)net->neuron_count;
    s = (orc_state_t *)calloc(1u, sizeof(*s));
    if (s == NULL) {
        return ORC_ERR_OUT_OF_MEMORY;
    }
    s->neuron_count = net->neuron_count;
    s->voltage = (float *)malloc(n * sizeof(float));
    s->current = (float *)calloc(n, sizeof(float));
    s->next_current = (float *)calloc(n, sizeof(float));
    s->refractory = (uint32_t *)calloc(n, sizeof(uint32_t));
    s->spikes = (uint8_t *)calloc(n, 1u);
    s->spike_indices = (orc_size_t *)malloc(n * sizeof(orc_size_t));
    if (!s->voltage || !s->current || !s->next_current || !s->refractory || !s->spikes || !s->spike_indices) {
        orc_state_free(s);
        return ORC_ERR_OUT_OF_MEMORY;
    }
    *out = s;
    return orc_state_reset(net, s);
}

void orc_state_free(orc_state_t *s) {
    if (s != NULL) {
        free(s->voltage);
        free(s->current);
        free(s->next_current);
        free(s->refractory);
        free(s->spikes);
        free(s->spike_indices);
        free(s);
    }
}

/* src/snn.c:681-696 */
int orc_state_reset(const orc_network_t *net, orc_state_t *s) {
    orc_size_t i;
    if (net == NULL || s == NULL || s->neuron_count != net->neuron_count) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    s->spike_count = 0;
    for (i = 0; i < s->neuron_count; ++i) {
        s->voltage[i] = net->lif.v_rest;
        s->current[i] = 0.0f;
        s->next_current[i] = 0.0f;
        s->refractory[i] = 0u;
        s->spikes[i] = 0u;
    }
    return ORC_OK;
}

/* src/snn.c:718-742: all-or-nothing validation, then a sequential fold in k order. */
int orc_state_inject_current(const orc_network_t *net, orc_state_t *s, const orc_size_t *idx, const float *val,
                             orc_size_t count) {
    orc_size_t k;
    if (net == NULL || s == NULL || s->neuron_count != net->neuron_count ||
        (count != 0 && (idx == NULL || val == NULL))) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    for (k = 0; k < count; ++k) {
        if (idx[k] >= s->neuron_count) {
            return ORC_ERR_INVALID_ARGUMENT;
        }
    }
    for (k = 0; k < count; ++k) {
        s->current[idx[k]] += val[k] * net->lif.input_scale;
    }
    return ORC_OK;
}

/* src/snn.c:744-914, serial build: LIF update in the exact term order
 * ((v_rest + (v - v_rest)*decay) + current) + input, with the +0.0f literal
 * for a NULL external; then the ascending spike list; then the scatter in CSR
 * order (ascending spiking row, ascending edge) into next_current; then the
 * current/next_current swap. */
int orc_step(const orc_network_t *net, orc_state_t *s, const float *ext, uint8_t *out_spikes) {
    orc_size_t i, n, count = 0;
    if (net == NULL || s == NULL || s->neuron_count != net->neuron_count) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    n = net->neuron_count;
    {
        const float decay = net->decay;
        const float v_rest = net->lif.v_rest;
        const float v_reset = net->lif.v_reset;
        const float thr = net->lif.v_threshold;
        const float scale = net->lif.input_scale;
        const uint32_t refr_steps = net->lif.refractory_steps;
        for (i = 0; i < n; ++i) {
            const uint32_t r = s->refractory[i];
            const float in = ext != NULL ? ext[i] * scale : 0.0f;
            const float v_int = v_rest + (s->voltage[i] - v_rest) * decay + s->current[i] + in;
            const int active = r == 0u;
            const int fired = active & (v_int >= thr);
            s->current[i] = 0.0f;
            s->voltage[i] = (active & (fired ^ 1)) ? v_int : v_reset;
            s->refractory[i] = fired ? refr_steps : r - (uint32_t)(r != 0u);
            s->spikes[i] = (uint8_t)fired;
        }
    }
    if (out_spikes != NULL) {
        memcpy(out_spikes, s->spikes, (size_t)n);
    }
    for (i = 0; i < n; ++i) {
        s->spike_indices[count] = i;
        count += s->spikes[i];
    }
    s->spike_count = count;
    for (i = 0; i < count; ++i) {
        const orc_size_t pre = s->spike_indices[i];
        orc_size_t e;
        for (e = net->row_ptr[pre]; e < net->row_ptr[pre + 1u]; ++e) {
            s->next_current[net->col_idx[e]] += net->weights[e];
        }
    }
    {
        float *t = s->current;
        s->current = s->next_current;
        s->next_current = t;
    }
    return ORC_OK;
}

uint64_t orc_last_step_events(const orc_network_t *net, const orc_state_t *s) {
    uint64_t ev = 0;
    orc_size_t i;
    for (i = 0; i < s->spike_count; ++i) {
        const orc_size_t pre = s->spike_indices[i];
        ev += net->row_ptr[pre + 1u] - net->row_ptr[pre];
    }
    return ev;
}

void orc_inject_stream_indices(uint64_t seed, uint64_t step, orc_size_t count, orc_size_t n, orc_size_t *out) {
    orc_size_t k;
    for (k = 0; k < count; ++k) {
        out[k] = draw_at(seed, step * count + k + 1u) % n;
    }
}

uint64_t orc_fnv1a(const void *data, size_t bytes, uint64_t h) {
    const uint8_t *p = (const uint8_t *)data;
    size_t i;
    for (i = 0; i < bytes; ++i) {
        h ^= p[i];
        h *= UINT64_C(0x100000001b3);
    }
    return h;
}

int orc_run_inject_stream(const orc_network_t *net, orc_state_t *s, uint64_t seed, uint64_t first_step,
                          uint64_t steps, orc_size_t count, float value, uint64_t *spike_counts,
                          uint64_t *events, uint64_t *hashes, uint8_t *raster) {
    orc_size_t *idx = NULL;
    float *val = NULL;
    uint64_t t;
    orc_size_t k;
    int st = ORC_OK;
    if (net == NULL || s == NULL) {
        return ORC_ERR_INVALID_ARGUMENT;
    }
    if (count != 0) {
        idx = (orc_size_t *)malloc((size_t)count * sizeof(orc_size_t));
        val = (float *)malloc((size_t)count * sizeof(float));
        if (idx == NULL || val == NULL) {
            free(idx);
            free(val);
            return ORC_ERR_OUT_OF_MEMORY;
        }
        for (k = 0; k < count; ++k) {
            val[k] = value;
        }
    }
    for (t = 0; t < steps && st == ORC_OK; ++t) {
        if (count != 0) {
            orc_inject_stream_indices(seed, first_step + t, count, net->neuron_count, idx);
            st = orc_state_inject_current(net, s, idx, val, count);
        }
        if (st == ORC_OK) {
            st = orc_step(net, s, NULL, raster != NULL ? raster + t * net->neuron_count : NULL);
        }
        if (spike_counts != NULL) {
            spike_counts[t] = s->spike_count;
        }
        if (events != NULL) {
            events[t] = orc_last_step_events(net, s);
        }
        if (hashes != NULL) {
            hashes[t] = orc_fnv1a(s->spikes, (size_t)net->neuron_count, UINT64_C(0xcbf29ce484222325));
        }
    }
    free(idx);
    free(val);
    return st;
}

void orc_sparse_frame(uint64_t seed, uint64_t sample, orc_size_t pixels, float zero_prob, orc_size_t n,
                      float *frame) {
    orc_size_t p;
    for (p = 0; p < n; ++p) {
        frame[p] = 0.0f;
    }
    for (p = 0; p < pixels && p < n; ++p) {
        const uint64_t d = (sample * pixels + p) * 2u;
        const float u = unit_from_bits(draw_at(seed, d + 1u));
        const float z = unit_from_bits(draw_at(seed, d + 2u));
        frame[p] = z < zero_prob ? 0.0f : u;
    }
}
