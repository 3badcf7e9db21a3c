"""GPU parity: the snn_b200 CUDA path against the CPU oracle on the same
seeded networks and inputs, through the C ABI.

Bars (the reference's parity contract, tests/test_snn.c:832-867, extended):
* ORDERED propagation: spike rasters AND voltages bit-identical to the
  serial CPU step for arbitrary (non-dyadic) weights;
* PUSH propagation: bit-identical for one shared dyadic weight (every sum is
  exact in any order, as the reference's own parity tests require); for
  general weights, from an identical state, voltages within 1e-5 relative
  and divergent spikes counted (fp32 atomics reassociate the sums).
"""
import os
import subprocess

import numpy as np
import pytest

import snn_b200 as sb
from oracle.oracle import Oracle, State, baseline_lif, default_lif, stream_indices_np
from tests._helpers import first_divergence, lif_to_sb, run_pair, stream_inject

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORC = Oracle("port")


def opts(**kw):
    return sb.default_options(**kw)


def ordered():
    return sb.default_options(propagation=sb.PROPAGATE_ORDERED)


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_reference_unit_suite_against_backend():
    """The reference's own tests/test_snn.c + test_bptt.c, unmodified, linked
    against libsnn_b200 instead of src/snn_cuda.cu (oracle/Makefile ref-tests):
    CPU/GPU parity runs, FULL/STREAMING policies, chunk clamps, inject
    staging, and the exact fault-seam numbering."""
    exe = os.path.join(ROOT, "oracle", "_ref", "test_snn_b200")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/test_snn_b200 not built (reference tree absent at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "all tests passed" in r.stdout


def test_ordered_config0_scaled_bit_exact():
    """BASELINE config 0 scaled to 20k neurons: random pool, fanout 100,
    w ~ U[0, 0.6], 1% injection of 20.0 per step, general weights."""
    lif = baseline_lif()
    net = ORC.random_pool(20000, 100, 0.0, 0.6, 0, lif=lif)
    ctx = sb.CudaContext.create(net, None, ordered())
    cr, gr, cv, gv = run_pair(net, ctx, 80, inject=stream_inject(0, 200, 20.0, 20000))
    assert first_divergence(cr, gr) is None
    assert cr.sum() > 1000
    np.testing.assert_array_equal(bits(cv), bits(gv))


def test_ordered_negative_weights_dense_external():
    """Mixed-sign weights (BASELINE config 2 range) driven by a dense external
    input, with nonzero rest/reset and a fractional input scale."""
    lif = default_lif(v_rest=0.25, v_reset=-0.5, v_threshold=1.0, input_scale=0.7, refractory_steps=2)
    net = ORC.random_pool(6000, 300, -0.2, 0.5, 77, lif=lif)
    ctx = sb.CudaContext.create(net, None, ordered())
    rng = np.random.default_rng(5)
    frames = [(rng.random(6000) < 0.05).astype(np.float32) * np.float32(1.3) for _ in range(4)]
    cr, gr, cv, gv = run_pair(net, ctx, 60, ext=lambda t: frames[t % 4])
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("prop", [sb.PROPAGATE_PUSH, sb.PROPAGATE_PUSH_BINNED, sb.PROPAGATE_PUSH_ATOMIC])
def test_push_dyadic_bit_exact(prop):
    lif = baseline_lif()
    net = ORC.random_pool(20000, 48, 0.046875, 0.046875, 4242, lif=lif)
    ctx = sb.CudaContext.create(net, None, opts(propagation=prop))
    assert ctx.mode == sb.MODE_FULL
    assert ctx.layout["binned"] == (1 if prop == sb.PROPAGATE_PUSH_BINNED else 0) or prop == sb.PROPAGATE_PUSH
    cr, gr, cv, gv = run_pair(net, ctx, 40, inject=stream_inject(3, 400, 20.0, 20000))
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("width,prop", [(32, sb.PROPAGATE_PUSH_ATOMIC), (64, sb.PROPAGATE_PUSH)])
def test_push_general_weights_tolerance(width, prop):
    """Push with fp32 atomics: from the SAME state each step (teacher forcing
    through snn_b200_upload_state), voltages agree within 1e-5 relative and
    the divergent spikes (threshold ties) are counted and must be rare."""
    lif = baseline_lif()
    n = 20000
    net = ORC.random_pool(n, 100, 0.0, 0.6, 0, lif=lif)
    ctx = sb.CudaContext.create(net, None, opts(index_width=width, propagation=prop))
    st = State(net)
    inj = stream_inject(1, 200, 20.0, n)
    divergent = 0
    max_rel = 0.0
    for t in range(40):
        v0, c0 = st.voltage(), st.current()
        r0 = st.refractory()
        ctx.upload_state(v0, c0, r0)
        idx, val = inj(t)
        st.inject(idx, val)
        ctx.inject_current(idx, val)
        cs = st.step()
        gs = ctx.step()
        divergent += int((cs != gs).sum())
        cv, gv = st.voltage(), ctx.download_voltage()
        same = cs == gs
        rel = np.abs(cv[same] - gv[same]) / np.maximum(np.abs(cv[same]), 1e-30)
        max_rel = max(max_rel, float(rel.max()))
        # The propagated currents (what the atomics produced) also agree.
        cc, gc = st.current(), ctx.download_current()
        assert np.allclose(cc, gc, rtol=1e-5, atol=1e-5)
    assert max_rel <= 1e-5, max_rel
    assert divergent <= 5, divergent


def test_feedforward_ordered_and_push():
    lif = default_lif(refractory_steps=1)
    net = ORC.feedforward([1024, 2048, 512], 32, 0.1, 5, lif=lif)
    rng = np.random.default_rng(2)
    frames = [(rng.random(net.neuron_count) < 0.08).astype(np.float32) * np.float32(1.5) for _ in range(15)]
    ctx = sb.CudaContext.create(net, None, ordered())
    cr, gr, cv, gv = run_pair(net, ctx, 15, ext=lambda t: frames[t])
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("rows,syn,budget", [(512, 24576, 0), (300, 0, 0), (0, 0, 2 << 20), (64, 3000, 0)])
def test_streaming_dyadic_bit_exact(rows, syn, budget):
    lif = default_lif(refractory_steps=2)
    net = ORC.random_pool(20000, 48, 0.046875, 0.046875, 4242, lif=lif)
    cfg = sb.default_config(prefer_streaming=1, max_stream_rows=rows, max_stream_synapses=syn,
                            max_vram_bytes=budget)
    ctx = sb.CudaContext.create(net, cfg)
    assert ctx.mode == sb.MODE_STREAMING
    rng = np.random.default_rng(11)
    frames = [(rng.random(20000) < 0.08).astype(np.float32) * np.float32(1.5) for _ in range(8)]
    cr, gr, cv, gv = run_pair(net, ctx, 8, ext=lambda t: frames[t])
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("allow_self", [0, 1])
@pytest.mark.parametrize("width", [32, 64])
def test_device_random_pool_matches_host_builder(allow_self, width):
    """snn_b200_create_random_pool reproduces snn_build_random_pool bit for bit."""
    n, f = 5003, 37
    net = ORC.random_pool(n, f, -0.2, 0.5, 9, allow_self=bool(allow_self))
    ctx = sb.CudaContext.random_pool(n, f, -0.2, 0.5, 9, allow_self=bool(allow_self),
                                     options=opts(index_width=width))
    rp, ci, w = ctx.download_topology()
    np.testing.assert_array_equal(rp, net.row_ptr())
    np.testing.assert_array_equal(ci, net.col_idx())
    np.testing.assert_array_equal(bits(w), bits(net.weights()))


def test_device_layered_matches_host_builder():
    layers = [300, 200, 157, 64]
    net = ORC.layered_random(layers, 17, 0.0, 1.0, 12345)
    ctx = sb.CudaContext.layered_random(layers, 17, 0.0, 1.0, 12345)
    rp, ci, w = ctx.download_topology()
    np.testing.assert_array_equal(rp, net.row_ptr())
    np.testing.assert_array_equal(ci, net.col_idx())
    np.testing.assert_array_equal(bits(w), bits(net.weights()))


def test_inject_unequal_duplicates_fold_in_order():
    """Duplicate indices with unequal values fold in k order like
    snn_state_inject_current (src/snn.c:737-739), bit for bit."""
    lif = default_lif(v_threshold=100.0)
    net = ORC.random_pool(1000, 5, 0.1, 0.2, 3, lif=lif)
    ctx = sb.CudaContext.create(net)
    st = State(net)
    rng = np.random.default_rng(0)
    for t in range(5):
        idx = rng.integers(0, 50, 4000).astype(np.uint64)
        val = rng.standard_normal(4000).astype(np.float32) * np.float32(1e-3)
        st.inject(idx, val)
        assert ctx.inject_current(idx, val) == 0
        np.testing.assert_array_equal(bits(st.current()), bits(ctx.download_current()))
        st.step()
        ctx.step()


def test_run_stream_async_matches_oracle():
    """The device-resident injection stream equals host injection of the same
    stream; stats count the same spikes and synaptic events."""
    lif = baseline_lif()
    n = 30000
    net = ORC.random_pool(n, 100, 0.0, 0.6, 0, lif=lif)
    st = State(net)
    sc, ev, hs, _ = ORC.run_inject_stream(net, st, 7, 0, 60, 300, 20.0)
    ctx = sb.CudaContext.create(net, None, ordered())
    ctx.run_stream_async(7, 0, 60, 300, 20.0)
    ctx.synchronize()
    s = ctx.stats()
    assert s["steps"] == 60
    assert s["spikes"] == int(sc.sum())
    assert s["events"] == int(ev.sum())
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))
    # Push mode counts the same spikes/events over the first steps (before
    # any reassociation-induced divergence can matter) -- at least step 0.
    ctxp = sb.CudaContext.create(net)
    ctxp.run_stream_async(7, 0, 1, 300, 20.0)
    sp = ctxp.stats()
    assert sp["spikes"] == int(sc[0]) and sp["events"] == int(ev[0])


def test_reset_replays_identically():
    lif = baseline_lif()
    net = ORC.random_pool(8000, 64, 0.0, 0.6, 1, lif=lif)
    ctx = sb.CudaContext.create(net, None, ordered())
    inj = stream_inject(2, 80, 20.0, 8000)
    runs = []
    for _ in range(2):
        r = []
        for t in range(20):
            ctx.inject_current(*inj(t))
            r.append(ctx.step())
        runs.append((np.array(r), ctx.download_voltage()))
        ctx.reset()
    np.testing.assert_array_equal(runs[0][0], runs[1][0])
    np.testing.assert_array_equal(bits(runs[0][1]), bits(runs[1][1]))


@pytest.mark.parametrize("n", [1, 2, 33, 129, 1027])
def test_small_and_ragged_sizes(n):
    lif = default_lif(refractory_steps=0)
    allow = n == 1
    net = ORC.random_pool(n, 3 if n > 1 else 2, 0.2, 0.9, n, allow_self=allow, lif=lif)
    for o in (None, ordered()):
        ctx = sb.CudaContext.create(net, None, o)
        rng = np.random.default_rng(n)
        frames = [(rng.random(n) < 0.3).astype(np.float32) * np.float32(1.2) for _ in range(10)]
        cr, gr, cv, gv = run_pair(net, ctx, 10, ext=lambda t: frames[t])
        assert first_divergence(cr, gr) is None
        if o is not None:
            np.testing.assert_array_equal(bits(cv), bits(gv))
        ctx.free()


def test_zero_synapses_and_hub_row():
    # Zero synapses.
    net = ORC.custom_csr(np.zeros(6, np.uint64), [], [])
    for o in (None, ordered()):
        ctx = sb.CudaContext.create(net, None, o)
        s = ctx.step(np.full(5, 2.0, np.float32))
        assert s.tolist() == [1] * 5
    # One hub row with 70k edges (wider than any per-warp vector loop).
    n = 70001
    rp = np.zeros(n + 1, np.uint64)
    rp[1:] = 70000
    col = (np.arange(70000, dtype=np.uint64) + 1)
    w = np.linspace(0.5, 1.5, 70000, dtype=np.float32)
    net = ORC.custom_csr(rp, col, w)
    ext = np.zeros(n, np.float32)
    ext[0] = 2.0
    for o in (None, ordered()):
        ctx = sb.CudaContext.create(net, None, o)
        cr, gr, cv, gv = run_pair(net, ctx, 3, ext=lambda t: ext if t == 0 else None)
        assert first_divergence(cr, gr) is None
        np.testing.assert_array_equal(bits(cv), bits(gv))


def test_layered_config4_scaled_bit_exact():
    """BASELINE config 4 scaled: 8 layers x 2000, fanout 500 to the next
    layer, w ~ U[0, 1], 5% of layer 0 injected with 30.0 per step."""
    lif = baseline_lif()
    layers = [2000] * 8
    net = ORC.layered_random(layers, 500, 0.0, 1.0, 4, lif=lif)
    ctx = sb.CudaContext.create(net, None, ordered())

    def inj(t):
        idx = stream_indices_np(44, t, 100, 2000)
        return idx, np.full(100, 30.0, np.float32)

    cr, gr, cv, gv = run_pair(net, ctx, 40, inject=inj)
    assert first_divergence(cr, gr) is None
    assert cr[:, 2000:].sum() > 0  # activity reaches deeper layers
    np.testing.assert_array_equal(bits(cv), bits(gv))


def test_dense_gaussian_config1_samples_with_reset():
    """BASELINE config 1 shape: 784-1000-10 dense N(0, 1/sqrt(fan_in)),
    25 steps per static sparse frame, state reset between samples."""
    lif = baseline_lif()
    net = ORC.dense_gaussian([784, 1000, 10], 21, lif=lif)
    n = net.neuron_count
    ctx = sb.CudaContext.create(net, None, ordered())
    st = State(net)
    for sample in range(3):
        frame = ORC.sparse_frame(99, sample, 784, 0.8, n) * np.float32(40.0)
        for t in range(25):
            cs = st.step(frame)
            gs = ctx.step(frame)
            np.testing.assert_array_equal(cs, gs)
        np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))
        st.reset()
        ctx.reset()


@pytest.mark.parametrize("prop", [sb.PROPAGATE_ORDERED, sb.PROPAGATE_PUSH_BINNED, sb.PROPAGATE_PUSH_ATOMIC])
def test_hub_row_collisions_exact(prop):
    """A hub row whose 70k edges hit 7 targets: in the bin-fold every round of
    32 events is all collisions (ten thousand events per target, applied in
    lane order). ORDERED with general weights, and the atomic push with one
    dyadic weight: bit-identical to the serial CPU fold."""
    n = 70001
    rp = np.zeros(n + 1, np.uint64)
    rp[1:] = 70000
    col = (np.arange(70000, dtype=np.uint64) % 7) + 1
    if prop != sb.PROPAGATE_PUSH_ATOMIC:
        w = np.random.default_rng(3).random(70000, dtype=np.float32)
    else:
        w = np.full(70000, 0.0625, np.float32)
    net = ORC.custom_csr(rp, col, w, lif=default_lif(v_threshold=1e6))
    ext = np.zeros(n, np.float32)
    ext[0] = 2e6
    ctx = sb.CudaContext.create(net, None, opts(propagation=prop))
    cr, gr, cv, gv = run_pair(net, ctx, 3, ext=lambda t: ext if t == 0 else None)
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))
    ctx.free()


@pytest.mark.parametrize("prop,env", [(sb.PROPAGATE_ORDERED, {}), (sb.PROPAGATE_PUSH_BINNED, {}),
                                      (sb.PROPAGATE_PUSH_BINNED, {"SNN_B200_ORDERED_CAP": "4000"})])
def test_generated_pool_binfold_exact(prop, env, monkeypatch):
    """Device-generated pool, general weights, ORDERED through the event sort
    and through the bin-fold (PUSH_BINNED), the latter also with an event
    capacity so small that busy steps go to the pull: spikes, events and
    voltages equal the serial CPU step's."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    lif = baseline_lif()
    n, f = 30011, 64
    net = ORC.random_pool(n, f, -0.1, 0.55, 21, lif=lif)
    st = State(net)
    sc, ev, hs, _ = ORC.run_inject_stream(net, st, 5, 0, 30, 600, 20.0)
    ctx = sb.CudaContext.random_pool(n, f, -0.1, 0.55, 21, lif=lif_to_sb(lif), options=opts(propagation=prop))
    lay = ctx.layout
    assert lay["propagation"] == sb.PROPAGATE_ORDERED
    assert lay["binned"] == (1 if prop == sb.PROPAGATE_PUSH_BINNED else 0)
    if lay["binned"]:
        assert lay["binned_passes"] == -(-n // 1024)  # tiles of 1024 targets
    ctx.run_stream_async(5, 0, 30, 600, 20.0)
    s = ctx.stats()
    assert s["spikes"] == int(sc.sum()) and s["events"] == int(ev.sum())
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))
    if "SNN_B200_ORDERED_CAP" in env:
        assert s["pull_steps"] > 0


def test_peer_exchange_wait_expires_without_fault():
    """Failure detection without a GPU fault: a 2-rank peer-exchange context
    whose peer mappings loop back to itself never receives rank 1's step
    flag. The compaction's bounded wait runs out, the step reports
    SNN_ERR_CUDA with a message, and the device stays usable."""
    import ctypes
    n = 4096
    net = ORC.random_pool(n, 16, 0.1, 0.2, 1)
    o = opts(world_size=2, rank=0, exchange=sb.EXCHANGE_PEER)
    ctx = sb.CudaContext.create(net, None, o)
    assert sb.lib().snn_test_b200_peer_loopback(ctx.handle, 2000) == sb.SNN_OK
    st = sb.lib().snn_cuda_step(ctx.handle, None, None)
    assert st == sb.SNN_ERR_CUDA
    assert "did not arrive" in sb.last_error()
    ctx.free()
    # The GPU and the library remain usable.
    ok = sb.CudaContext.create(net)
    ok.step(np.full(n, 2.0, np.float32))
    ok.free()
    del ctypes


def test_sparse_streaming_dyadic_bit_exact():
    """STREAMING with SNN_B200_STREAMING_SPARSE: only row_ptr is resident and
    the push kernel reads the spiking rows' edges from the page-locked host
    CSR. Dyadic weights: bit-exact with the CPU step."""
    lif = default_lif(refractory_steps=2)
    net = ORC.random_pool(20000, 48, 0.046875, 0.046875, 4242, lif=lif)
    cfg = sb.default_config(prefer_streaming=1)
    ctx = sb.CudaContext.create(net, cfg, opts(streaming=sb.STREAMING_SPARSE))
    assert ctx.mode == sb.MODE_STREAMING
    assert ctx.layout["device_topology_bytes"] == (20000 + 1) * 8  # row_ptr only
    rng = np.random.default_rng(11)
    frames = [(rng.random(20000) < 0.08).astype(np.float32) * np.float32(1.5) for _ in range(8)]
    cr, gr, cv, gv = run_pair(net, ctx, 8, ext=lambda t: frames[t])
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))
    s = ctx.stats()
    assert s["events"] == int(cr.sum()) * 48


@pytest.mark.parametrize("allow_self,env", [
    (0, {}),                                   # ordered push, one row range per step
    (0, {"SNN_B200_ORDERED_FOLD": "full"}),    # full sort by target + run fold
    (1, {"SNN_B200_ORDERED_CAP": "3000"}),     # ordered push, several row ranges per step
    (0, {"SNN_B200_ORDERED_PULL": "1"}),       # pull over a device-built CSC
    (1, {"SNN_B200_ORDERED_PULL": "1", "SNN_B200_CSC_PASS_EDGES": "150000"}),  # CSC built in several passes
    (0, {"SNN_B200_ORDERED_PULL": "1", "SNN_B200_PULL_CHUNK_WORDS": "100"}),  # 7 presynaptic chunks
])
def test_generated_pool_ordered_bit_exact(allow_self, env, monkeypatch):
    """snn_b200_create_random_pool with ORDERED propagation, through both
    bit-exact kernels: the event-driven ordered push (events copied in CSR
    order, sorted stably by target group, folded in order per group; or the
    full sort by target and a run fold) and the pull over a CSC built on the
    device. General weights: spikes, events and voltages bit-identical to the
    serial CPU step."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    lif = baseline_lif()
    n, f = 20011, 100
    net = ORC.random_pool(n, f, 0.0, 0.6, 31, allow_self=bool(allow_self), lif=lif)
    st = State(net)
    sc, ev, hs, _ = ORC.run_inject_stream(net, st, 7, 0, 50, 200, 20.0)
    ctx = sb.CudaContext.random_pool(n, f, 0.0, 0.6, 31, allow_self=bool(allow_self), lif=lif_to_sb(lif),
                                     options=ordered())
    lay = ctx.layout
    assert lay["propagation"] == sb.PROPAGATE_ORDERED and lay["local_synapses"] == n * f
    ctx.run_stream_async(7, 0, 50, 200, 20.0)
    s = ctx.stats()
    assert int(sc.sum()) > 1000
    assert s["spikes"] == int(sc.sum()) and s["events"] == int(ev.sum())
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))


def test_generated_layered_ordered_bit_exact():
    """snn_b200_create_layered_random with ORDERED propagation (the last
    layer owns no edges), stepped against the oracle with injection."""
    lif = baseline_lif()
    layers = [1500, 1200, 900, 64]
    net = ORC.layered_random(layers, 300, 0.0, 1.0, 8, lif=lif)
    ctx = sb.CudaContext.layered_random(layers, 300, 0.0, 1.0, 8, lif=lif_to_sb(lif), options=ordered())

    def inj(t):
        return stream_indices_np(9, t, 75, 1500), np.full(75, 30.0, np.float32)

    cr, gr, cv, gv = run_pair(net, ctx, 30, inject=inj)
    assert first_divergence(cr, gr) is None
    assert cr[:, 1500:].sum() > 0
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("cap,pull_div,chunk_words", [(None, "0", None), ("20000", "0", None), (None, None, None),
                                                      (None, None, "40")])
def test_ordered_dense_bursts_bit_exact(cap, pull_div, chunk_words, monkeypatch):
    """Dense recurrent pool (in-degree ~1500) with strong drive: most rows
    spike together, so every target's run of events is hundreds long (the
    warp-cooperative fold); with a small event capacity a step is split into
    many row ranges; with the default density threshold the dense steps take
    the pull over the CSC. Bit-identical to the serial CPU step."""
    if cap:
        monkeypatch.setenv("SNN_B200_ORDERED_CAP", cap)
    if pull_div:
        monkeypatch.setenv("SNN_B200_ORDERED_PULL_DIV", pull_div)
    if chunk_words:  # general weights over a 3-chunk pull layout
        monkeypatch.setenv("SNN_B200_PULL_CHUNK_WORDS", chunk_words)
    lif = default_lif(v_rest=0.0, v_reset=0.0, v_threshold=1.0, input_scale=1.0, refractory_steps=1)
    n = 3001
    net = ORC.random_pool(n, 1500, -0.05, 0.1, 12, allow_self=True, lif=lif)
    ctx = sb.CudaContext.create(net, None, ordered())
    rng = np.random.default_rng(8)
    frames = [(rng.random(n) < 0.6).astype(np.float32) * np.float32(1.5) for _ in range(3)]
    cr, gr, cv, gv = run_pair(net, ctx, 12, ext=lambda t: frames[t % 3])
    assert first_divergence(cr, gr) is None
    assert cr.sum(axis=1).max() > n // 2
    np.testing.assert_array_equal(bits(cv), bits(gv))
    assert ctx.layout["ordered_csc"] == (0 if pull_div == "0" else 1)
    pulls = ctx.stats()["pull_steps"]
    assert (pulls > 0) if pull_div is None else (pulls == 0)


@pytest.mark.parametrize("prop,weights", [(sb.PROPAGATE_ORDERED, "general"), (sb.PROPAGATE_PUSH, "dyadic")])
def test_batched_states_equal_independent_runs(prop, weights):
    """options.batch = B: B independent states over one shared topology.
    Sample b owns neurons [b*n, (b+1)*n) of every per-neuron argument. Each
    sample, driven by its own injection stream and external frames, must equal
    a separate serial CPU run of the network bit for bit (ORDERED for general
    weights; PUSH with one dyadic weight, where every sum is exact)."""
    lif = default_lif(v_rest=0.25, v_reset=-0.5, v_threshold=1.0, input_scale=0.7, refractory_steps=2)
    n, B, steps = 3001, 5, 25
    wmin, wmax = (-0.2, 0.5) if weights == "general" else (0.125, 0.125)
    net = ORC.random_pool(n, 64, wmin, wmax, 41, lif=lif)
    ctx = sb.CudaContext.create(net, None, sb.default_options(propagation=prop, batch=B))
    lay = ctx.layout
    assert (lay["batch"], lay["topology_rows"], lay["neuron_count"]) == (B, n, B * n)
    assert ctx.local_count == B * n
    rng = np.random.default_rng(2)
    inj = [[(rng.integers(0, n, 40).astype(np.uint64), np.full(40, 2.0, np.float32)) for _ in range(steps)]
           for _ in range(B)]
    ext = [[(rng.random(n) < 0.02 * (b + 1)).astype(np.float32) * np.float32(1.4) for _ in range(steps)]
           for b in range(B)]
    states = [State(net) for _ in range(B)]
    for t in range(steps):
        idx = np.concatenate([inj[b][t][0] + np.uint64(b * n) for b in range(B)])
        val = np.concatenate([inj[b][t][1] for b in range(B)])
        assert ctx.inject_current(idx, val) == 0
        got = ctx.step(np.concatenate([ext[b][t] for b in range(B)]))
        for b in range(B):
            assert states[b].inject(*inj[b][t]) == 0
            want = states[b].step(ext[b][t])
            assert np.array_equal(got[b * n:(b + 1) * n], want), (b, t)
    v = ctx.download_voltage()
    for b in range(B):
        np.testing.assert_array_equal(bits(v[b * n:(b + 1) * n]), bits(states[b].voltage()))
    assert sum(int(st.voltage().size) for st in states) == B * n
    assert ctx.stats()["spikes"] > 100
    # Batched contexts are FULL only.
    with pytest.raises(sb.SnnError):
        sb.CudaContext.create(net, sb.default_config(prefer_streaming=1), sb.default_options(batch=B))


def test_batched_config1_samples_with_held_frames():
    """BASELINE config 1 as batched samples: 784-1000-10 dense gaussian, B
    samples at once, each with its own static sparse frame held on the device
    (snn_b200_set_external, one upload for 25 steps), two rounds of samples
    with snn_b200_reset between them. Steps alternate between snn_cuda_step
    without an external (spikes checked) and snn_b200_step_async. Every sample
    equals its own serial CPU run bit for bit (ORDERED)."""
    lif = baseline_lif()
    net = ORC.dense_gaussian([784, 1000, 10], 21, lif=lif)
    n, B = net.neuron_count, 24
    ctx = sb.CudaContext.create(net, None, sb.default_options(propagation=sb.PROPAGATE_ORDERED, batch=B))
    for rnd in range(2):
        frames = [ORC.sparse_frame(99, rnd * B + b, 784, 0.8, n) * np.float32(40.0) for b in range(B)]
        ctx.set_external(np.concatenate(frames))
        ctx.reset()  # keeps the held frames
        states = [State(net) for _ in range(B)]
        for t in range(25):
            want = [states[b].step(frames[b]) for b in range(B)]
            if t % 2 == 0:
                got = ctx.step()
                for b in range(B):
                    assert np.array_equal(got[b * n:(b + 1) * n], want[b]), (rnd, t, b)
            else:
                ctx.step_async()
        ctx.synchronize()
        v = ctx.download_voltage()
        for b in range(B):
            np.testing.assert_array_equal(bits(v[b * n:(b + 1) * n]), bits(states[b].voltage()))
    # An explicit external replaces the held frame for that step and ends the hold.
    ctx.set_external(None)
    ctx.reset()
    st0 = State(net)
    zero_ext = np.zeros(B * n, np.float32)
    got = ctx.step(zero_ext)
    assert np.array_equal(got[:n], st0.step(np.zeros(n, np.float32)))


@pytest.mark.parametrize("mode", ["full", "chunked", "sparse", "ordered"])
def test_mapped_csr_file_contexts(mode, tmp_path):
    """A network saved as an snn_b200 CSR file and mapped back read-only
    (snn_b200_network_map, no copy) drives every policy: FULL push, STREAMING
    chunked and sparse-requested, and ORDERED. Bit-exact with the CPU step of
    the original."""
    lif = default_lif(refractory_steps=2)
    w = (0.046875, 0.046875) if mode != "ordered" else (-0.2, 0.5)
    net = ORC.random_pool(20000, 48, *w, 4242, lif=lif)
    path = str(tmp_path / "net.snncsr")
    sb.save_network(net, path)
    mapped = sb.Network.map(path)
    if mode == "full":
        ctx = sb.CudaContext.create(mapped, None)
    elif mode == "ordered":
        ctx = sb.CudaContext.create(mapped, None, ordered())
    else:
        ctx = sb.CudaContext.create(mapped, sb.default_config(prefer_streaming=1),
                                    opts(streaming=sb.STREAMING_SPARSE if mode == "sparse" else sb.STREAMING_CHUNKED))
        # Sparse streaming needs the mapping's pages locked; where the OS
        # refuses to lock file pages the context streams chunks instead.
        assert ctx.mode == sb.MODE_STREAMING
    rng = np.random.default_rng(11)
    frames = [(rng.random(20000) < 0.08).astype(np.float32) * np.float32(1.5) for _ in range(8)]
    cr, gr, cv, gv = run_pair(net, ctx, 8, ext=lambda t: frames[t])
    assert first_divergence(cr, gr) is None
    np.testing.assert_array_equal(bits(cv), bits(gv))
    ctx.free()
    mapped.free()


@pytest.mark.parametrize("generated,chunk_words", [(False, None), (True, None), (False, "32"), (True, "32")])
def test_push_with_pull_gate_dyadic_bit_exact(generated, chunk_words, monkeypatch):
    """PUSH contexts keep a sliced-ELL CSC beside the CSR when memory allows:
    steps with more spikes than rows / SNN_B200_PUSH_PULL_DIV take the pull
    kernel, the others the atomic push, chosen on the device. Frames alternate
    between sparse and dense drive so both kernels run; one shared dyadic
    weight makes every sum exact, so both equal the CPU step bit for bit.
    With SNN_B200_PULL_CHUNK_WORDS=32 the pull's layout is cut into 3
    presynaptic chunks (shared-memory spike bits staged chunk by chunk)."""
    monkeypatch.setenv("SNN_B200_PUSH_PULL_DIV", "4")
    monkeypatch.setenv("SNN_B200_PUSH_PULL_MIN_SYNAPSES", "0")
    if chunk_words:
        monkeypatch.setenv("SNN_B200_PULL_CHUNK_WORDS", chunk_words)
    lif = default_lif(v_rest=0.0, v_reset=0.0, v_threshold=1.0, input_scale=1.0, refractory_steps=1)
    n, f = 3001, 700
    net = ORC.random_pool(n, f, 0.0009765625, 0.0009765625, 12, lif=lif)
    if generated:
        ctx = sb.CudaContext.random_pool(n, f, 0.0009765625, 0.0009765625, 12, lif=lif, options=opts())
    else:
        ctx = sb.CudaContext.create(net, None, opts())
    assert ctx.layout["ordered_csc"] == 1
    rng = np.random.default_rng(8)
    frames = [(rng.random(n) < (0.6 if t % 3 == 0 else 0.02)).astype(np.float32) * np.float32(1.5)
              for t in range(12)]
    cr, gr, cv, gv = run_pair(net, ctx, 12, ext=lambda t: frames[t])
    assert first_divergence(cr, gr) is None
    dense = (cr.sum(axis=1) > n // 4).sum()
    assert 0 < dense < 12
    np.testing.assert_array_equal(bits(cv), bits(gv))
    s = ctx.stats()
    assert s["events"] == int(cr.sum()) * f
    assert s["pull_steps"] == dense  # the gate: more spikes than rows / 4
    assert s["pull_events"] == int(cr[cr.sum(axis=1) > n // 4].sum()) * f
    assert ctx.layout["pull_slots"] >= n * f


def test_push_pull_gate_disabled_keeps_plain_push(monkeypatch):
    net = ORC.random_pool(2000, 50, 0.1, 0.2, 3)
    # Below the synapse bound (2^26 by default) PUSH keeps the plain push.
    assert sb.CudaContext.create(net, None, opts()).layout["ordered_csc"] == 0
    monkeypatch.setenv("SNN_B200_PUSH_PULL_MIN_SYNAPSES", "0")
    monkeypatch.setenv("SNN_B200_PUSH_PULL_DIV", "0")
    ctx = sb.CudaContext.create(net, None, opts())
    assert ctx.layout["ordered_csc"] == 0
    ref = sb.CudaContext.create(net, None)  # the reference entry point never adds it
    assert ref.layout["ordered_csc"] == 0


def test_run_stream_graph_replay_dyadic_exact():
    """Unsharded push contexts replay run_stream_async as a captured CUDA
    graph of two steps (the injection step index kept on the device). Starting
    on an odd step, with an odd count of steps, then again with another seed
    (a new graph): spikes, events and voltages equal the CPU step (one shared
    dyadic weight makes every sum exact), and equal an eager run."""
    lif = baseline_lif()
    n, f = 30011, 64
    net = ORC.random_pool(n, f, 0.25, 0.25, 5, lif=lif)
    st = State(net)
    sc1, ev1, _, _ = ORC.run_inject_stream(net, st, 3, 0, 1, 600, 20.0)
    sc2, ev2, _, _ = ORC.run_inject_stream(net, st, 3, 1, 37, 600, 20.0)
    sc3, ev3, _, _ = ORC.run_inject_stream(net, st, 9, 38, 20, 600, 20.0)
    ctx = sb.CudaContext.create(net, None, opts())
    ctx.run_stream_async(3, 0, 1, 600, 20.0)   # step 0 (fewer than 8 steps: launched one by one)
    ctx.run_stream_async(3, 1, 37, 600, 20.0)  # starts on an odd step
    ctx.run_stream_async(9, 38, 20, 600, 20.0)  # another seed: a new graph
    ctx.synchronize()
    s = ctx.stats()
    assert s["steps"] == 58
    assert s["spikes"] == int(sc1.sum() + sc2.sum() + sc3.sum())
    assert s["events"] == int(ev1.sum() + ev2.sum() + ev3.sum())
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))


@pytest.mark.parametrize("layers,fanout,seed", [([2, 3, 1], 0, 0), ([2, 3, 1], 1, 123), ([300, 400, 50], 17, 99),
                                                ([400, 300, 600, 200], 25, 7)])
def test_device_feedforward_matches_host_builder(layers, fanout, seed):
    """snn_b200_create_feedforward reproduces snn_build_feedforward bit for
    bit (dense layers in order, sparse ones from one splitmix64 stream)."""
    net = ORC.feedforward(layers, fanout, 0.75, seed)
    ctx = sb.CudaContext.feedforward(layers, fanout, 0.75, seed)
    rp, ci, w = ctx.download_topology()
    np.testing.assert_array_equal(rp, net.row_ptr())
    np.testing.assert_array_equal(ci, net.col_idx())
    np.testing.assert_array_equal(bits(w), bits(net.weights()))


@pytest.mark.parametrize("mode", ["ordered", "binfold"])
def test_device_feedforward_steps_exact(mode):
    """A device-built feed-forward network (one dense and two sparse layers)
    stepped against the CPU step of the host-built one: ORDERED through the
    event sort and through the bin-fold (CSC built on the device from the
    generator for the dense steps)."""
    layers, fanout = [1500, 1200, 40, 900], 60
    weight = 0.75
    lif = default_lif(refractory_steps=1)
    net = ORC.feedforward(layers, fanout, weight, 11, lif=lif)
    o = ordered() if mode == "ordered" else opts(propagation=sb.PROPAGATE_PUSH_BINNED)
    ctx = sb.CudaContext.feedforward(layers, fanout, weight, 11, lif=lif_to_sb(lif), options=o)
    rng = np.random.default_rng(4)
    n = net.neuron_count
    frames = [np.concatenate([(rng.random(1500) < 0.2).astype(np.float32) * np.float32(1.5),
                              np.zeros(n - 1500, np.float32)]) for _ in range(6)]
    cr, gr, cv, gv = run_pair(net, ctx, 12, ext=lambda t: frames[t % 6])
    assert first_divergence(cr, gr) is None
    assert cr[:, 2700:].sum() > 0  # activity reaches the last layers
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("prop", [sb.PROPAGATE_ORDERED, sb.PROPAGATE_PUSH])
def test_stream_range_drives_input_layer(prop):
    """snn_b200_set_stream_range: the seeded injection stream drawn in
    [0, range) drives only the first layer of a layered network (BASELINE
    config 4 scaled). ORDERED with general weights, or PUSH (the two-step
    graph replay) with one dyadic weight: equal to host injection of the same
    indices into the CPU step, bit for bit."""
    lif = baseline_lif()
    layers, f = [2000, 2000, 2000, 2000], 100
    w = (0.0, 1.0) if prop == sb.PROPAGATE_ORDERED else (0.5, 0.5)
    net = ORC.layered_random(layers, f, *w, 4, lif=lif)
    ctx = sb.CudaContext.layered_random(layers, f, *w, 4, lif=lif_to_sb(lif), options=opts(propagation=prop))
    ctx.set_stream_range(2000)
    st = State(net)
    for t in range(24):
        assert st.inject(stream_indices_np(6, t, 100, 2000), np.full(100, 30.0, np.float32)) == 0
        st.step()
    ctx.run_stream_async(6, 0, 24, 100, 30.0)
    ctx.synchronize()
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))
    assert ctx.stats()["spikes"] > 0
    with pytest.raises(sb.SnnError):
        ctx.set_stream_range(8001)


@pytest.mark.parametrize("mode", [sb.STREAMING_CHUNKED, sb.STREAMING_SPARSE])
def test_generated_pool_streaming_exact(mode):
    """A device-generated pool under the STREAMING policy: the topology is
    generated on the device, moved to host memory and streamed from there
    every step (chunked, or sparse reads of the spiking rows). One dyadic
    weight (the atomic scatter is then exact): spikes, events and voltages
    equal the serial CPU step's on the host-built pool."""
    lif = baseline_lif()
    n, f = 20011, 80
    net = ORC.random_pool(n, f, 0.25, 0.25, 44, lif=lif)
    st = State(net)
    sc, ev, _, _ = ORC.run_inject_stream(net, st, 2, 0, 30, 300, 25.0)
    cfg = sb.default_config(prefer_streaming=1, max_vram_bytes=8 << 20)
    ctx = sb.CudaContext.random_pool(n, f, 0.25, 0.25, 44, lif=lif_to_sb(lif), config=cfg,
                                     options=opts(streaming=mode))
    assert ctx.mode == sb.MODE_STREAMING
    ctx.run_stream_async(2, 0, 30, 300, 25.0)
    s = ctx.stats()
    assert s["spikes"] == int(sc.sum()) and s["events"] == int(ev.sum())
    np.testing.assert_array_equal(bits(st.voltage()), bits(ctx.download_voltage()))


@pytest.mark.parametrize("mode,rows,syn", [(sb.STREAMING_CHUNKED, 700, 40000), (sb.STREAMING_CHUNKED, 0, 0),
                                           (sb.STREAMING_SPARSE, 0, 0)])
def test_streaming_ordered_general_weights_bit_exact(mode, rows, syn):
    """STREAMING with ORDERED propagation and general (non-dyadic, mixed-sign)
    weights: chunked (every chunk folds its own events onto the earlier
    chunks' sums; with small chunks a step spans dozens of them) and sparse
    (the event sort over the mapped host CSR). Rasters and voltages equal the
    serial CPU step bit for bit."""
    lif = baseline_lif()
    n = 20011
    net = ORC.random_pool(n, 100, -0.2, 0.5, 61, lif=lif)
    cfg = sb.default_config(prefer_streaming=1, max_stream_rows=rows, max_stream_synapses=syn)
    ctx = sb.CudaContext.create(net, cfg, opts(propagation=sb.PROPAGATE_ORDERED, streaming=mode))
    assert ctx.mode == sb.MODE_STREAMING
    cr, gr, cv, gv = run_pair(net, ctx, 40, inject=stream_inject(8, 200, 25.0, n))
    assert first_divergence(cr, gr) is None
    assert cr.sum() > 1000
    np.testing.assert_array_equal(bits(cv), bits(gv))


@pytest.mark.parametrize("mode", [sb.STREAMING_CHUNKED, sb.STREAMING_SPARSE])
def test_streaming_push_general_weights_tolerance(mode):
    """STREAMING with the atomic push and general weights: from the same state
    every step (teacher forcing), voltages and propagated currents within
    1e-5 relative of the serial CPU step, divergent spikes counted (rare)."""
    lif = baseline_lif()
    n = 20011
    net = ORC.random_pool(n, 100, -0.2, 0.5, 62, lif=lif)
    cfg = sb.default_config(prefer_streaming=1, max_stream_rows=900)
    ctx = sb.CudaContext.create(net, cfg, opts(streaming=mode))
    assert ctx.mode == sb.MODE_STREAMING
    st = State(net)
    inj = stream_inject(9, 200, 25.0, n)
    divergent, max_rel = 0, 0.0
    for t in range(40):
        ctx.upload_state(st.voltage(), st.current(), st.refractory())
        idx, val = inj(t)
        st.inject(idx, val)
        ctx.inject_current(idx, val)
        cs, gs = st.step(), ctx.step()
        divergent += int((cs != gs).sum())
        same = cs == gs
        cv, gv = st.voltage(), ctx.download_voltage()
        rel = np.abs(cv[same] - gv[same]) / np.maximum(np.abs(cv[same]), 1e-30)
        max_rel = max(max_rel, float(rel.max()))
        assert np.allclose(st.current(), ctx.download_current(), rtol=1e-5, atol=1e-5)
    assert max_rel <= 1e-5, max_rel
    assert divergent <= 5, divergent
