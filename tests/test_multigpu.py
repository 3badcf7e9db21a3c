"""Sharded multi-GPU parity (needs >= 2 GPUs): runs tests/mgpu_worker.py
under torch.distributed.run with one process per GPU."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_sharded_parity_two_gpus(gpu_count):
    if gpu_count < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29517",
                        os.path.join(ROOT, "tests", "mgpu_worker.py")],
                       capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "MGPU PARITY OK" in r.stdout


@pytest.mark.gpu
def test_single_process_sharded_create_c(gpu_count):
    """snn_cuda_create_sharded from plain C against the reference's serial CPU
    step (tests/c/test_sharded_create.c, linked with the reference's src/snn.c):
    ORDERED over 2+ devices of one process, peer and NCCL exchange, bit for bit."""
    if gpu_count < 2:
        pytest.skip("needs two GPUs")
    exe = os.path.join(ROOT, "oracle", "_ref", "test_sharded_create")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/test_sharded_create not built (reference tree absent at build time)")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([exe, str(min(gpu_count, 4))], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "SHARDED CREATE OK" in r.stdout


@pytest.mark.gpu
def test_single_process_sharded_python(gpu_count):
    """The same context from Python: ORDERED (general weights) and PUSH (one
    dyadic weight) over two devices through the multi-step stream and the
    reference entry points, FULL and STREAMING, against the CPU oracle."""
    if gpu_count < 2:
        pytest.skip("needs two GPUs")
    import numpy as np

    import snn_b200 as sb
    from oracle.oracle import Oracle, State, baseline_lif
    orc = Oracle("port")
    lif = baseline_lif()
    cases = [(sb.PROPAGATE_ORDERED, (-0.2, 0.5), None), (sb.PROPAGATE_PUSH, (0.25, 0.25), None),
             (sb.PROPAGATE_PUSH, (0.25, 0.25), sb.default_config(prefer_streaming=1))]
    for prop, (wmin, wmax), cfg in cases:
        net = orc.random_pool(20011, 120, wmin, wmax, 3, lif=lif)
        st = State(net)
        sc, ev, _, _ = orc.run_inject_stream(net, st, 9, 0, 40, 200, 25.0)
        ctx = sb.CudaContext.create_sharded(net, [0, 1], cfg, sb.default_options(propagation=prop))
        assert ctx.layout["local_count"] == 20011
        ctx.run_stream_async(9, 0, 40, 200, 25.0)
        ctx.synchronize()
        s = ctx.stats()
        assert s["spikes"] == int(sc.sum()) and s["events"] == int(ev.sum()), (prop, s)
        np.testing.assert_array_equal(st.voltage().view(np.uint32), ctx.download_voltage().view(np.uint32))
        ctx.free()
