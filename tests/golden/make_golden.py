"""Generates the golden fixtures in tests/golden/ from the REFERENCE itself:
oracle/_ref/libsnn_ref.so is the reference's src/snn.c compiled unchanged
(serial build, oracle/Makefile). Run in a container that has the reference
tree:

    make -C oracle && python tests/golden/make_golden.py

The fixtures pin the CPU oracle (oracle/snn_oracle.c) on machines where the
reference is absent (tests/test_oracle_pin.py) and give the GPU parity tests
reference-produced expectations.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import Oracle, State, baseline_lif, default_lif, fnv1a, ref_available  # noqa: E402


def frames(n, steps, seed, frac, amp):
    rng = np.random.default_rng(seed)
    return (rng.random((steps, n)) < frac).astype(np.float32) * np.float32(amp)


def main():
    assert ref_available("ref"), "build oracle/_ref first (make -C oracle)"
    ref = Oracle("ref")
    out = {}
    # Builder known answers (tests/test_snn.c:299-415 shapes).
    net = ref.random_pool(4, 3, 0.1, 0.3, 44)
    out["pool_4x3_row_ptr"], out["pool_4x3_col"], out["pool_4x3_w"] = net.row_ptr(), net.col_idx(), net.weights()
    net = ref.random_pool(1, 1, -8.0, 0.3, 13629332, allow_self=True)
    out["pool_clamp_w"] = net.weights()
    net = ref.random_pool(1000, 8, 0.0, 0.6, 7)
    out["pool_1000x8_col"], out["pool_1000x8_w"] = net.col_idx(), net.weights()
    net = ref.feedforward([2, 3, 1], 0, 0.75, 0)
    out["ff_dense_row_ptr"], out["ff_dense_col"] = net.row_ptr(), net.col_idx()
    net = ref.feedforward([2, 3, 1], 1, 0.75, 123)
    out["ff_fan1_row_ptr"], out["ff_fan1_col"] = net.row_ptr(), net.col_idx()
    net = ref.feedforward([300, 400, 50], 17, 0.5, 99)
    out["ff_300_400_50_col"] = net.col_idx()

    # BASELINE config 0 scaled to 10k neurons: injection stream, 60 steps.
    lif = baseline_lif()
    net = ref.random_pool(10000, 100, 0.0, 0.6, 0, lif=lif)
    st = State(net)
    sc, ev, hs, ras = ref.run_inject_stream(net, st, 0, 0, 60, 100, 20.0, raster=True)
    out["cfg0s_spikes"], out["cfg0s_events"], out["cfg0s_hash"] = sc, ev, hs
    out["cfg0s_raster_bits"] = np.packbits(ras, axis=1)
    out["cfg0s_voltage"] = st.voltage()

    # Mixed-sign weights (config 2 range) with a dense external input.
    lif2 = default_lif(v_rest=0.25, v_reset=-0.5, v_threshold=1.0, input_scale=0.7, refractory_steps=2)
    net = ref.random_pool(3000, 200, -0.2, 0.5, 77, lif=lif2)
    st = State(net)
    fr = frames(3000, 30, 5, 0.05, 1.3)
    r = np.array([st.step(fr[t]) for t in range(30)])
    out["mixed_raster_bits"] = np.packbits(r, axis=1)
    out["mixed_voltage"] = st.voltage()

    # Feed-forward 1024-2048-512 fanout 32 with a non-dyadic weight.
    net = ref.feedforward([1024, 2048, 512], 32, 0.1, 5, lif=default_lif(refractory_steps=1))
    st = State(net)
    fr = frames(net.neuron_count, 15, 2, 0.08, 1.5)
    r = np.array([st.step(fr[t]) for t in range(15)])
    out["ff_raster_bits"] = np.packbits(r, axis=1)
    out["ff_voltage"] = st.voltage()

    # Injection with duplicate indices and unequal values.
    net = ref.random_pool(500, 5, 0.1, 0.2, 3, lif=default_lif(v_threshold=100.0))
    st = State(net)
    rng = np.random.default_rng(0)
    idx = rng.integers(0, 50, 4000).astype(np.uint64)
    val = (rng.standard_normal(4000) * 1e-3).astype(np.float32)
    st.inject(idx, val)
    st.step()
    out["inject_dup_voltage"] = st.voltage()

    # Memory plans (src/snn.c:339-425).
    plans = []
    for n, e in [(1, 0), (100000, 10_000_000), (10_000_000, 10_000_000_000), (200_000_000, 200_000_000_000)]:
        stt, p = ref.plan_counts(n, e)
        plans.append([stt] + [getattr(p, f) for f, _ in p._fields_])
    out["plans_counts"] = np.array(plans, np.uint64)
    stt, p = ref.plan_network(ref.feedforward([2, 3, 1], 0, 0.75, 0))
    out["plan_ff"] = np.array([stt] + [getattr(p, f) for f, _ in p._fields_], np.uint64)
    out["meta_hash_check"] = np.array([fnv1a(np.arange(10, dtype=np.uint8))], np.uint64)
    np.savez_compressed(os.path.join(HERE, "reference_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_golden.npz"))


if __name__ == "__main__":
    main()
