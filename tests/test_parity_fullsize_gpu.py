"""Full-size parity on the workloads the serial CPU step can run in seconds.

* Config 0 exactly as specified (random pool of 100,000 neurons, fanout 100,
  w ~ U[0, 0.6], 1% of the neurons injected with 20.0 per step, 1,000 steps):
  ORDERED must equal the reference's serial CPU step bit for bit (every
  step's spike vector and the final voltages). PUSH runs free (no state is
  re-uploaded) and the divergent spikes are counted per step and reported;
  its fp32 atomics reassociate, so a few threshold ties may flip.
* Config 1 at its real shape (784-1000-10 dense gaussian, 25 steps per static
  frame, state reset between samples) over 500 samples in ORDERED, batched
  500 at a time: every sample equals its own serial CPU run bit for bit.
"""
import json
import os

import numpy as np
import pytest

import snn_b200 as sb
from oracle.oracle import Oracle, State, baseline_lif, stream_indices_np
from tests._helpers import lif_to_sb

pytestmark = pytest.mark.gpu
ORC = Oracle("port")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _config0():
    n, fanout, steps, count = 100_000, 100, 1000, 1000
    lif = baseline_lif()
    net = ORC.random_pool(n, fanout, 0.0, 0.6, 0, lif=lif)
    return net, n, steps, count


def _cpu_raster(net, n, steps, count):
    st = State(net)
    raster = np.zeros((steps, n), np.uint8)
    val = np.full(count, 20.0, np.float32)
    for t in range(steps):
        assert st.inject(stream_indices_np(0, t, count, n), val) == 0
        raster[t] = st.step()
    return raster, st.voltage()


@pytest.fixture(scope="module")
def config0_cpu():
    net, n, steps, count = _config0()
    raster, v = _cpu_raster(net, n, steps, count)
    return net, n, steps, count, raster, v


def _gpu_run(net, n, steps, count, prop):
    ctx = sb.CudaContext.create(net, None, sb.default_options(propagation=prop))
    raster = np.zeros((steps, n), np.uint8)
    val = np.full(count, 20.0, np.float32)
    for t in range(steps):
        assert ctx.inject_current(stream_indices_np(0, t, count, n), val) == 0
        ctx.step(out=raster[t])
    v = ctx.download_voltage()
    lay = ctx.layout
    ctx.free()
    return raster, v, lay


@pytest.mark.parametrize("prop", [sb.PROPAGATE_ORDERED, sb.PROPAGATE_PUSH_BINNED])
def test_config0_full_ordered_bit_exact(config0_cpu, prop):
    """Both bit-exact propagations: the event sort and the bin-fold."""
    net, n, steps, count, cr, cv = config0_cpu
    gr, gv, lay = _gpu_run(net, n, steps, count, prop)
    assert lay["binned"] == (1 if prop == sb.PROPAGATE_PUSH_BINNED else 0)
    bad = np.nonzero((cr != gr).any(axis=1))[0]
    assert bad.size == 0, f"first divergent step {bad[0]}"
    np.testing.assert_array_equal(cv.view(np.uint32), gv.view(np.uint32))
    assert cr.sum() > 0.009 * n * steps  # ~0.98% firing, as the reference measures


def test_config0_full_push_free_running_divergence(config0_cpu):
    """PUSH free-running over the full 1,000 steps: divergent spikes counted
    per step against the serial CPU raster and reported (printed, and written
    to gpurun_out/ when that folder exists). The dynamics are input-driven,
    so reassociation flips at most a handful of threshold ties."""
    net, n, steps, count, cr, cv = config0_cpu
    gr, gv, _ = _gpu_run(net, n, steps, count, sb.PROPAGATE_PUSH)
    per_step = (cr != gr).sum(axis=1)
    total = int(per_step.sum())
    spikes = int(cr.sum())
    first = int(np.nonzero(per_step)[0][0]) if total else None
    same = (cr == gr).all(axis=0)
    rel = np.abs(cv[same] - gv[same]) / np.maximum(np.abs(cv[same]), 1e-30)
    report = {"workload": "config0 full (100k x 100, 1% x 20.0, 1000 steps)", "propagation": "PUSH (fp32 atomics)",
              "divergent_spikes": total, "spikes": spikes, "divergent_fraction": total / max(spikes, 1),
              "steps_with_divergence": int((per_step > 0).sum()), "first_divergent_step": first,
              "max_rel_voltage_diff_non_divergent": float(rel.max()) if rel.size else 0.0}
    print("PUSH divergence report:", json.dumps(report))
    out = os.path.join(ROOT, "gpurun_out")
    if os.path.isdir(out):
        with open(os.path.join(out, "push_divergence_config0.json"), "w") as f:
            json.dump(report, f)
    assert total <= 0.001 * spikes, report


@pytest.mark.parametrize("prop", [sb.PROPAGATE_ORDERED, sb.PROPAGATE_PUSH_BINNED])
def test_config1_real_shape_500_samples_ordered(prop):
    lif = baseline_lif()
    lif.input_scale = 20.0
    net = ORC.dense_gaussian([784, 1000, 10], 5, lif=lif)
    n, B, T = net.neuron_count, 500, 25
    frames = [ORC.sparse_frame(17, b, 784, 0.8, n) for b in range(B)]
    ctx = sb.CudaContext.create(net, None, sb.default_options(propagation=prop, batch=B))
    assert ctx.layout["binned"] == (1 if prop == sb.PROPAGATE_PUSH_BINNED else 0)
    ctx.set_external(np.concatenate(frames))
    ctx.reset()
    graster = np.zeros((T, B * n), np.uint8)
    for t in range(T):
        ctx.step(out=graster[t])
    gv = ctx.download_voltage()
    spikes = 0
    for b in range(B):
        st = State(net)
        for t in range(T):
            want = st.step(frames[b])
            assert np.array_equal(graster[t, b * n:(b + 1) * n], want), (b, t)
            spikes += int(want.sum())
        np.testing.assert_array_equal(gv[b * n:(b + 1) * n].view(np.uint32), st.voltage().view(np.uint32))
    assert spikes > 1000
    ctx.free()
