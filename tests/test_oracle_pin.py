"""Pins the CPU oracle (oracle/snn_oracle.c) before anything trusts it.

1. The reference's own hand-computed known-answer tests (tests/test_snn.c),
   restated against the oracle port.
2. The committed golden fixtures produced by the reference library itself
   (tests/golden/make_golden.py over oracle/_ref/libsnn_ref.so).
3. When the compiled reference is present, randomized differential runs of
   port vs reference, bit for bit.
"""
import os

import numpy as np
import pytest

from oracle.oracle import Oracle, State, baseline_lif, default_lif, ref_available

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "reference_golden.npz"))
PORT = Oracle("port")


def frames(n, steps, seed, frac, amp):
    rng = np.random.default_rng(seed)
    return (rng.random((steps, n)) < frac).astype(np.float32) * np.float32(amp)


# ---------------------------------------------------------------- KATs ----
def test_kat_three_neuron_chain():
    """tests/test_snn.c:417-511"""
    lif = default_lif(refractory_steps=1)
    net = PORT.custom_csr([0, 1, 2, 2], [1, 2], [0.8, 1.1], lif=lif)
    st = State(net)
    assert st.voltage()[0] == 0.0
    assert st.step([1.2, 0.0, 0.0]).tolist() == [1, 0, 0]
    assert st.voltage()[0] == 0.0
    assert st.step([0.0, 0.0, 0.0]).tolist() == [0, 0, 0]
    assert st.step([0.0, 0.0, 0.0]).tolist() == [0, 0, 0]
    assert st.step([0.0, 0.3, 0.0]).tolist() == [0, 1, 0]


def test_kat_run_with_strides():
    """tests/test_snn.c:513-558: step 0 drives neuron 0; the propagated 1.0 fires neuron 1."""
    net = PORT.custom_csr([0, 1, 1], [1], [1.0])
    st = State(net)
    out = [st.step(x).tolist() for x in ([1.1, 0.0], [0.0, 0.0], [0.0, 0.0])]
    assert out == [[1, 0], [0, 1], [0, 0]]


@pytest.mark.parametrize("refr,expect", [(0, [1, 1]), (2, [1, 0, 0, 1])])
def test_kat_refractory(refr, expect):
    """tests/test_snn.c:676-711"""
    net = PORT.custom_csr([0, 0], [], [], lif=default_lif(refractory_steps=refr))
    st = State(net)
    assert [int(st.step([2.0])[0]) for _ in expect] == expect


def test_kat_inject_semantics():
    """tests/test_snn.c:713-735, 764-822"""
    net = PORT.custom_csr([0, 0], [], [])
    st = State(net)
    assert st.step([0.6])[0] == 0
    st.reset()
    assert st.inject([0], [0.6]) == 0
    assert st.step([0.6])[0] == 1
    net = PORT.custom_csr([0, 1, 2, 2], [1, 2], [0.8, 1.1])
    st = State(net)
    assert st.inject([0, 3], [0.7, 0.6]) == -1  # out of range: nothing applied
    assert st.step()[0] == 0
    assert st.inject([0, 0], [0.7, 0.6]) == 0  # duplicates accumulate
    assert st.step().tolist()[:2] == [1, 0]
    assert net.set_lif(default_lif(input_scale=2.0)) == 0
    st.reset()
    assert st.inject([2], [0.6]) == 0
    assert st.step()[2] == 1


def test_kat_null_external_equals_zero():
    """tests/test_snn.c:644-674"""
    net = PORT.custom_csr([0, 1, 2, 2], [1, 2], [0.8, 1.1])
    a, b = State(net), State(net)
    a.step([1.2, 0.4, 0.0])
    b.step([1.2, 0.4, 0.0])
    for _ in range(4):
        assert np.array_equal(a.step(), b.step([0.0, 0.0, 0.0]))
        assert np.array_equal(a.voltage().view(np.uint32), b.voltage().view(np.uint32))


def test_kat_builders():
    """tests/test_snn.c:299-415"""
    net = PORT.feedforward([2, 3, 1], 0, 0.75, 0)
    assert net.row_ptr().tolist() == [0, 3, 6, 7, 8, 9, 9]
    assert net.col_idx()[[0, 2, 8]].tolist() == [2, 4, 5]
    net = PORT.feedforward([2, 3, 1], 1, 0.75, 123)
    assert net.synapse_count == 5 and net.row_ptr()[2] == 2 and net.row_ptr()[5] == 5
    assert 2 <= net.col_idx()[0] < 5 and net.col_idx()[4] == 5
    net = PORT.random_pool(4, 3, 0.1, 0.3, 44)
    rp, ci, w = net.row_ptr(), net.col_idx(), net.weights()
    for i in range(4):
        assert rp[i] == 3 * i
        for e in range(rp[i], rp[i + 1]):
            assert ci[e] < 4 and ci[e] != i and 0.1 <= w[e] <= 0.3
    net = PORT.random_pool(1, 1, -8.0, 0.3, 13629332, allow_self=True)
    assert net.weights()[0] == np.float32(0.3)  # u rounds to 1.0f: clamp


def test_memory_plan_matches_reference_formula():
    """FULL device layout 29N+12E+8 (docs/gpu_capacity.md:30-34)."""
    st, p = PORT.plan_counts(10_000_000, 10_000_000_000)
    assert st == 0 and p.device_total_full_bytes == 29 * 10_000_000 + 12 * 10_000_000_000 + 8


# ------------------------------------------------------------- golden ----
def test_golden_builders():
    net = PORT.random_pool(4, 3, 0.1, 0.3, 44)
    assert np.array_equal(net.row_ptr(), G["pool_4x3_row_ptr"])
    assert np.array_equal(net.col_idx(), G["pool_4x3_col"])
    assert np.array_equal(net.weights().view(np.uint32), G["pool_4x3_w"].view(np.uint32))
    assert np.array_equal(PORT.random_pool(1, 1, -8.0, 0.3, 13629332, allow_self=True).weights(), G["pool_clamp_w"])
    net = PORT.random_pool(1000, 8, 0.0, 0.6, 7)
    assert np.array_equal(net.col_idx(), G["pool_1000x8_col"])
    assert np.array_equal(net.weights().view(np.uint32), G["pool_1000x8_w"].view(np.uint32))
    net = PORT.feedforward([2, 3, 1], 0, 0.75, 0)
    assert np.array_equal(net.row_ptr(), G["ff_dense_row_ptr"]) and np.array_equal(net.col_idx(), G["ff_dense_col"])
    net = PORT.feedforward([2, 3, 1], 1, 0.75, 123)
    assert np.array_equal(net.row_ptr(), G["ff_fan1_row_ptr"]) and np.array_equal(net.col_idx(), G["ff_fan1_col"])
    assert np.array_equal(PORT.feedforward([300, 400, 50], 17, 0.5, 99).col_idx(), G["ff_300_400_50_col"])


def test_golden_config0_scaled_run():
    net = PORT.random_pool(10000, 100, 0.0, 0.6, 0, lif=baseline_lif())
    st = State(net)
    sc, ev, hs, ras = PORT.run_inject_stream(net, st, 0, 0, 60, 100, 20.0, raster=True)
    assert np.array_equal(sc, G["cfg0s_spikes"]) and np.array_equal(ev, G["cfg0s_events"])
    assert np.array_equal(hs, G["cfg0s_hash"])
    assert np.array_equal(np.packbits(ras, axis=1), G["cfg0s_raster_bits"])
    assert np.array_equal(st.voltage().view(np.uint32), G["cfg0s_voltage"].view(np.uint32))


def test_golden_mixed_sign_dense_external():
    lif = default_lif(v_rest=0.25, v_reset=-0.5, v_threshold=1.0, input_scale=0.7, refractory_steps=2)
    net = PORT.random_pool(3000, 200, -0.2, 0.5, 77, lif=lif)
    st = State(net)
    fr = frames(3000, 30, 5, 0.05, 1.3)
    r = np.array([st.step(fr[t]) for t in range(30)])
    assert np.array_equal(np.packbits(r, axis=1), G["mixed_raster_bits"])
    assert np.array_equal(st.voltage().view(np.uint32), G["mixed_voltage"].view(np.uint32))


def test_golden_feedforward():
    net = PORT.feedforward([1024, 2048, 512], 32, 0.1, 5, lif=default_lif(refractory_steps=1))
    st = State(net)
    fr = frames(net.neuron_count, 15, 2, 0.08, 1.5)
    r = np.array([st.step(fr[t]) for t in range(15)])
    assert np.array_equal(np.packbits(r, axis=1), G["ff_raster_bits"])
    assert np.array_equal(st.voltage().view(np.uint32), G["ff_voltage"].view(np.uint32))


def test_golden_inject_duplicates_unequal_values():
    net = PORT.random_pool(500, 5, 0.1, 0.2, 3, lif=default_lif(v_threshold=100.0))
    st = State(net)
    rng = np.random.default_rng(0)
    idx = rng.integers(0, 50, 4000).astype(np.uint64)
    val = (rng.standard_normal(4000) * 1e-3).astype(np.float32)
    st.inject(idx, val)
    st.step()
    assert np.array_equal(st.voltage().view(np.uint32), G["inject_dup_voltage"].view(np.uint32))


def test_golden_memory_plans():
    for row in G["plans_counts"]:
        n, e = int(row[1]), int(row[2])
        st, p = PORT.plan_counts(n, e)
        got = [st & 0xFFFFFFFFFFFFFFFF] + [getattr(p, f) for f, _ in p._fields_]
        assert [int(x) for x in got] == [int(x) for x in row]
    st, p = PORT.plan_network(PORT.feedforward([2, 3, 1], 0, 0.75, 0))
    assert [int(x) for x in [st] + [getattr(p, f) for f, _ in p._fields_]] == [int(x) for x in G["plan_ff"]]


# ---------------------------------------------------------- differential ----
@pytest.mark.skipif(not ref_available("ref"), reason="compiled reference (oracle/_ref) absent")
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_port_equals_reference_randomized(seed):
    ref = Oracle("ref")
    rng = np.random.default_rng(seed)
    n = int(rng.integers(50, 3000))
    fan = int(rng.integers(1, 60))
    wmin = float(rng.uniform(-1, 0.5))
    wmax = wmin + float(rng.uniform(0, 1))
    lif = default_lif(v_rest=float(rng.uniform(-1, 0)), v_reset=float(rng.uniform(-1, 0)), v_threshold=1.0,
                      input_scale=float(rng.uniform(0.3, 2)), refractory_steps=int(rng.integers(0, 4)))
    nets = [L.random_pool(n, fan, wmin, wmax, seed, allow_self=bool(seed % 2), lif=lif) for L in (PORT, ref)]
    assert np.array_equal(nets[0].col_idx(), nets[1].col_idx())
    assert np.array_equal(nets[0].weights().view(np.uint32), nets[1].weights().view(np.uint32))
    sts = [State(x) for x in nets]
    for t in range(20):
        ext = (rng.random(n) < 0.2).astype(np.float32) * np.float32(rng.uniform(0.5, 2))
        idx = rng.integers(0, n, 30).astype(np.uint64)
        val = rng.standard_normal(30).astype(np.float32)
        for s in sts:
            assert s.inject(idx, val) == 0
        a, b = sts[0].step(ext if t % 2 else None), sts[1].step(ext if t % 2 else None)
        assert np.array_equal(a, b)
    assert np.array_equal(sts[0].voltage().view(np.uint32), sts[1].voltage().view(np.uint32))


@pytest.mark.parametrize("n,fanout,allow_self,seed", [(1, 0, False, 3), (2, 5, False, 0), (97, 13, False, 9),
                                                      (1000, 64, True, 123456789), (4096, 100, False, 0)])
def test_parallel_pool_builder_bit_identical(n, fanout, allow_self, seed):
    """The multi-threaded random-pool builder (used to give the reference's
    CPU step a full-size pool) equals the serial builder and, when present,
    the reference's own snn_build_random_pool bit for bit."""
    lif = baseline_lif()
    a = PORT.random_pool(n, fanout, -0.2, 0.5, seed, allow_self=allow_self, lif=lif)
    b = PORT.random_pool_parallel(n, fanout, -0.2, 0.5, seed, allow_self=allow_self, lif=lif)
    for x, y in ((a.row_ptr(), b.row_ptr()), (a.col_idx(), b.col_idx()),
                 (a.weights().view(np.uint32), b.weights().view(np.uint32))):
        np.testing.assert_array_equal(x, y)
    assert a.decay == b.decay
    if ref_available("ref"):
        r = Oracle("ref").random_pool(n, fanout, -0.2, 0.5, seed, allow_self=allow_self, lif=lif)
        np.testing.assert_array_equal(r.col_idx(), b.col_idx())
        np.testing.assert_array_equal(r.weights().view(np.uint32), b.weights().view(np.uint32))


@pytest.mark.skipif(not ref_available("ref"), reason="reference library not built")
def test_port_network_stepped_by_reference_library():
    """A port-built network has the reference's struct layout: the
    reference's own snn_step_cpu steps it exactly as it steps its own build."""
    lif = baseline_lif()
    ref = Oracle("ref")
    mine = PORT.random_pool_parallel(3000, 50, 0.0, 0.6, 7, lif=lif)
    theirs = ref.random_pool(3000, 50, 0.0, 0.6, 7, lif=lif)
    s1, s2 = State(mine, lib=ref), State(theirs)
    for t in range(30):
        idx = np.arange(t * 37, t * 37 + 60, dtype=np.uint64) % 3000
        val = np.full(60, 20.0, np.float32)
        assert s1.inject(idx, val) == 0 and s2.inject(idx, val) == 0
        np.testing.assert_array_equal(s1.step(), s2.step())
    np.testing.assert_array_equal(s1.voltage().view(np.uint32), s2.voltage().view(np.uint32))
