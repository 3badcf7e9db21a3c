/*
 * snn_cuda_create_sharded against the reference's own serial CPU step.
 *
 * Linked with the reference's unchanged src/snn.c (builders, state, serial
 * step) and libsnn_b200 (oracle/Makefile target sharded-test). A random pool
 * with general (non-dyadic) weights runs for a number of steps with seeded
 * sparse injection, once through snn_step_cpu and once through one context
 * sharded over the given devices (ORDERED propagation, peer and NCCL
 * exchange): every step's spike vector and the final voltages must be
 * bit-identical. Usage: test_sharded_create <device_count>.
 */
#include <snn/snn.h>

#include "snn_b200.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * UINT64_C(0xbf58476d1ce4e5b9);
    z = (z ^ (z >> 27)) * UINT64_C(0x94d049bb133111eb);
    return z ^ (z >> 31);
}

static int run(int devices_n, int exchange, snn_size_t n, snn_size_t fanout, int steps) {
    snn_random_pool_config_t pool = {n, fanout, -0.2f, 0.5f, 11, 0};
    snn_lif_params_t lif = {1.0f, 20.0f, -65.0f, -65.0f, -50.0f, 1.0f, 2u};
    snn_network_t *net = NULL;
    snn_state_t *cpu = NULL;
    snn_cuda_context_t *ctx = NULL;
    int devices[8];
    int ok = 1, d, t;
    const snn_size_t count = n / 100;
    snn_size_t *idx = malloc(count * sizeof(snn_size_t));
    float *val = malloc(count * sizeof(float));
    uint8_t *cs = malloc(n), *gs = malloc(n);
    float *cv = malloc(n * sizeof(float)), *gv = malloc(n * sizeof(float));
    snn_b200_options_t o = snn_b200_default_options();
    for (d = 0; d < devices_n; ++d) devices[d] = d;
    o.propagation = SNN_B200_PROPAGATE_ORDERED;
    o.exchange = exchange;
    if (snn_build_random_pool(&pool, &lif, &net) != SNN_OK || snn_state_create(net, &cpu) != SNN_OK) {
        printf("reference build failed\n");
        return 0;
    }
    if (snn_b200_create_sharded(net, NULL, &o, devices_n, devices, &ctx) != SNN_OK) {
        printf("snn_b200_create_sharded failed: %s\n", snn_b200_last_error());
        return 0;
    }
    for (t = 0; t < steps && ok; ++t) {
        snn_size_t k;
        for (k = 0; k < count; ++k) {
            idx[k] = mix64(5 + (uint64_t)(t * count + k + 1) * UINT64_C(0x9e3779b97f4a7c15)) % n;
            val[k] = 25.0f;
        }
        ok = snn_state_inject_current(net, cpu, idx, val, count) == SNN_OK &&
             snn_cuda_inject_current(ctx, idx, val, count) == SNN_OK &&
             snn_step_cpu(net, cpu, NULL, cs) == SNN_OK && snn_cuda_step(ctx, NULL, gs) == SNN_OK;
        if (ok && memcmp(cs, gs, n) != 0) {
            printf("exchange %d: spikes differ at step %d\n", exchange, t);
            ok = 0;
        }
    }
    if (ok) {
        ok = snn_state_copy_voltage(cpu, cv, n) == SNN_OK && snn_cuda_download_voltage(ctx, gv, n) == SNN_OK &&
             memcmp(cv, gv, n * sizeof(float)) == 0;
        if (!ok) printf("exchange %d: voltages differ\n", exchange);
    }
    if (ok) {
        snn_b200_stats_t s;
        ok = snn_b200_get_stats(ctx, &s) == SNN_OK && s.spikes > 0;
        printf("exchange %d over %d devices: %d steps bit-identical, %llu spikes, %llu events\n", exchange,
               devices_n, steps, (unsigned long long)s.spikes, (unsigned long long)s.events);
    }
    snn_cuda_free(ctx);
    snn_state_free(cpu);
    snn_network_free(net);
    free(idx);
    free(val);
    free(cs);
    free(gs);
    free(cv);
    free(gv);
    return ok;
}

int main(int argc, char **argv) {
    const int devices_n = argc > 1 ? atoi(argv[1]) : 2;
    int ok = 1;
    if (devices_n < 2) {
        printf("needs 2 or more devices\n");
        return 2;
    }
    ok &= run(devices_n, SNN_B200_EXCHANGE_PEER, 30011, 200, 60);
    ok &= run(devices_n, SNN_B200_EXCHANGE_NCCL, 30011, 200, 60);
    printf(ok ? "SHARDED CREATE OK\n" : "SHARDED CREATE FAILED\n");
    return ok ? 0 : 1;
}
