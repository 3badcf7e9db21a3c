"""The allocation-free step (snn_b200_step_noalloc) against the regular one.

Callers whose device memory is all owned by someone else (a framework's pool
or arena) or who may not allocate once running cannot use a context, since
creating one allocates. snn_b200_step_noalloc serves them: they bring every
array, and the library's only scratch is a fixed array compiled into it.
This test owns its buffers (allocated here with torch), runs two allocation-
free steps in a row through the C ABI, and checks spikes, voltages and the
propagated current against two snn_cuda_step calls of a FULL push context
started from the same state: exactly for one shared dyadic weight (every sum
exact in any order), within 1e-5 relative for general weights (fp32 atomics
reassociate). It sits in its own file, collected last.
"""
import ctypes as C

import numpy as np
import pytest

import snn_b200 as sb
from oracle.oracle import Oracle, baseline_lif


def _ptr(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.gpu
@pytest.mark.parametrize("weights", ["dyadic", "general"])
def test_noalloc_step_matches_context_step(weights):
    import torch

    n, fanout = 50021, 48
    lif = baseline_lif()
    wmin, wmax = (0.046875, 0.046875) if weights == "dyadic" else (-0.2, 0.5)
    net = Oracle("port").random_pool(n, fanout, wmin, wmax, 17, lif=lif)
    rng = np.random.default_rng(3)
    v0 = (np.float32(-65.0) + rng.random(n, dtype=np.float32) * np.float32(20.0)).astype(np.float32)
    c0 = (rng.random(n, dtype=np.float32) * np.float32(4.0)).astype(np.float32)
    r0 = rng.integers(0, 3, n).astype(np.uint32)

    # Existing entry point: a FULL push context, two snn_cuda_step calls.
    ctx = sb.CudaContext.create(net, None, sb.default_options(device=0))
    assert ctx.mode == sb.MODE_FULL
    ctx.upload_state(v0, c0, r0)
    ref_spikes = [ctx.step(), ctx.step()]
    ref_v = ctx.download_voltage()
    ref_c = ctx.download_current()
    ctx.free()

    # Allocation-free entry point over buffers this test owns.
    dev = torch.device("cuda", 0)
    v = torch.from_numpy(v0).to(dev)
    cur = torch.from_numpy(c0).to(dev)
    nxt = torch.zeros(n, dtype=torch.float32, device=dev)
    refr = torch.from_numpy(r0.view(np.int32)).to(dev)
    spikes = torch.zeros(n, dtype=torch.uint8, device=dev)
    row_ptr = torch.from_numpy(net.row_ptr().view(np.int64)).to(dev)
    col = torch.from_numpy(net.col_idx().astype(np.uint32).view(np.int32)).to(dev)
    w = torch.from_numpy(net.weights()).to(dev)
    lp = sb.LifParams(lif.dt_ms, lif.membrane_tau_ms, lif.v_rest, lif.v_reset, lif.v_threshold, lif.input_scale,
                      lif.refractory_steps)
    stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    L = sb.lib()
    got = []
    for _ in range(2):
        st = L.snn_b200_step_noalloc(0, stream, n, C.byref(lp), net.decay, _ptr(v), _ptr(cur), None, _ptr(refr),
                                     _ptr(spikes), _ptr(row_ptr), _ptr(col), _ptr(w), _ptr(nxt))
        assert st == sb.SNN_OK
        torch.cuda.synchronize(dev)
        got.append(spikes.cpu().numpy().copy())
        cur, nxt = nxt, cur  # the consumed buffer was zeroed: it is the next target
    for a, b in zip(ref_spikes, got):
        assert np.array_equal(a, b)
    assert sum(int(s.sum()) for s in got) > 100
    gv, gc = v.cpu().numpy(), cur.cpu().numpy()
    if weights == "dyadic":
        assert np.array_equal(gv.view(np.uint32), ref_v.view(np.uint32))
        assert np.array_equal(gc.view(np.uint32), ref_c.view(np.uint32))
    else:
        np.testing.assert_allclose(gv, ref_v, rtol=1e-5, atol=0)
        np.testing.assert_allclose(gc, ref_c, rtol=1e-5, atol=1e-5)

    # The entry point allocates nothing: after the first call (which looks up
    # the scratch address), further calls leave the device's free memory and
    # torch's allocator exactly where they were.
    torch.cuda.synchronize(dev)
    free0, _ = torch.cuda.mem_get_info(dev)
    alloc0 = torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0)
    for _ in range(3):
        assert L.snn_b200_step_noalloc(0, stream, n, C.byref(lp), net.decay, _ptr(v), _ptr(cur), None, _ptr(refr),
                                       _ptr(spikes), _ptr(row_ptr), _ptr(col), _ptr(w), _ptr(nxt)) == sb.SNN_OK
        cur, nxt = nxt, cur
    torch.cuda.synchronize(dev)
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0
    assert torch.cuda.memory_stats(dev).get("allocation.all.allocated", 0) == alloc0

    # Limits: beyond the fixed scratch, misaligned or missing arrays are
    # rejected up front.
    assert L.snn_b200_step_noalloc(0, stream, n, C.byref(lp), net.decay, _ptr(v), _ptr(cur), None, _ptr(refr),
                                   _ptr(spikes), _ptr(row_ptr), None, _ptr(w),
                                   _ptr(nxt)) == sb.SNN_ERR_INVALID_ARGUMENT
    assert L.snn_b200_step_noalloc(0, stream, n, C.byref(lp), net.decay, _ptr(v), _ptr(cur), None, _ptr(refr),
                                   _ptr(spikes), _ptr(row_ptr), _ptr(col), None,
                                   _ptr(nxt)) == sb.SNN_ERR_INVALID_ARGUMENT
    too_big = sb.NOALLOC_MAX_NEURONS + 1
    assert L.snn_b200_step_noalloc(0, stream, too_big, C.byref(lp), net.decay, _ptr(v), _ptr(cur), None,
                                   _ptr(refr), _ptr(spikes), _ptr(row_ptr), _ptr(col), _ptr(w),
                                   _ptr(nxt)) == sb.SNN_ERR_INVALID_ARGUMENT
    assert L.snn_b200_step_noalloc(0, stream, n, C.byref(lp), net.decay, C.c_void_p(v.data_ptr() + 4), _ptr(cur),
                                   None, _ptr(refr), _ptr(spikes), _ptr(row_ptr), _ptr(col), _ptr(w),
                                   _ptr(nxt)) == sb.SNN_ERR_INVALID_ARGUMENT
