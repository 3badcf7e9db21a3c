"""Shared helpers of the parity tests: step the CPU oracle and the snn_b200
backend side by side on the same network and inputs."""
from __future__ import annotations

import numpy as np

import snn_b200 as sb
from oracle.oracle import Oracle, State, baseline_lif, default_lif, stream_indices_np  # noqa: F401


def lif_to_sb(lp) -> sb.LifParams:
    return sb.LifParams(lp.dt_ms, lp.membrane_tau_ms, lp.v_rest, lp.v_reset, lp.v_threshold, lp.input_scale,
                        lp.refractory_steps)


def run_pair(net, ctx, steps, *, inject=None, ext=None, check_voltage_each=False):
    """Steps the oracle state and the GPU context in lockstep.

    inject(step) -> (idx, val) or None; ext(step) -> float32[n] or None.
    Returns (cpu_raster, gpu_raster, cpu_v, gpu_v)."""
    st = State(net)
    n = net.neuron_count
    cr = np.zeros((steps, n), np.uint8)
    gr = np.zeros((steps, n), np.uint8)
    for t in range(steps):
        if inject is not None:
            iv = inject(t)
            if iv is not None:
                idx, val = iv
                assert st.inject(idx, val) == 0
                assert ctx.inject_current(idx, val) == 0
        e = ext(t) if ext is not None else None
        cr[t] = st.step(e)
        gr[t] = ctx.step(e)
        if check_voltage_each:
            np.testing.assert_array_equal(st.voltage().view(np.uint32), ctx.download_voltage().view(np.uint32))
    return cr, gr, st.voltage(), ctx.download_voltage()


def stream_inject(seed, count, value, n):
    def f(t):
        return stream_indices_np(seed, t, count, n), np.full(count, value, np.float32)
    return f


def first_divergence(cr, gr):
    bad = np.nonzero((cr != gr).any(axis=1))[0]
    return int(bad[0]) if bad.size else None
