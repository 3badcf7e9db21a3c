"""CPU checks of the C-ABI boundary: the library loads, exports every entry
point include/snn_b200.h declares, and behaves like the reference's backend
for every call that needs no device (argument validation, the no-device
create status, test hooks) -- tests/test_snn.c:869-925's unavailable branch."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import snn_b200 as sb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "snn_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(snn_(?:cuda|test|b200)_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_functions()
    assert len(names) >= 34
    out = subprocess.run(["nm", "-D", "--defined-only", sb.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    L = sb.lib()
    for n in names:
        assert hasattr(L, n)
    # The Python mirror binds every declared entry point.
    assert sorted(n for n, _, _ in sb.ENTRY_POINTS) == names


def test_library_is_sm100a_and_links_static_cudart():
    out = subprocess.run(["ldd", sb.LIB_PATH], capture_output=True, text=True, check=True).stdout
    assert "libcudart" not in out  # static runtime: no clash with the host process' cudart
    assert "libnccl" in out


def test_defaults_and_null_arguments():
    L = sb.lib()
    cfg = L.snn_cuda_default_config()
    assert (cfg.max_vram_bytes, cfg.max_stream_synapses, cfg.max_stream_rows, cfg.prefer_streaming) == (0, 0, 0, 0)
    o = L.snn_b200_default_options()
    assert (o.propagation, o.device, o.index_width, o.rank, o.world_size, o.timing, o.batch) == (0, -1, 0, 0, 1, 0, 1)
    assert L.snn_cuda_context_mode(None) == sb.MODE_NONE
    assert L.snn_cuda_step(None, None, None) == sb.SNN_ERR_INVALID_ARGUMENT
    assert L.snn_cuda_inject_current(None, None, None, 0) == sb.SNN_ERR_INVALID_ARGUMENT
    v = np.zeros(3, np.float32)
    assert L.snn_cuda_download_voltage(None, v.ctypes.data_as(C.c_void_p), 3) == sb.SNN_ERR_INVALID_ARGUMENT
    out = C.c_void_p(1)
    assert L.snn_cuda_create(None, None, C.byref(out)) == sb.SNN_ERR_INVALID_ARGUMENT
    assert out.value is None  # *out_context nulled before validation (src/snn_cuda.cu:433-436)
    L.snn_cuda_free(None)


def test_network_wrap_validates_like_build_custom_csr():
    rp = np.array([0, 1, 2, 2], np.uint64)
    ci = np.array([1, 2], np.uint64)
    w = np.array([0.75, 1.25], np.float32)
    net = sb.Network.from_csr(rp, ci, w)
    assert net.handle
    net.free()
    with pytest.raises(sb.SnnError):
        sb.Network.from_csr(rp, np.array([1, 3], np.uint64), w)  # column out of range
    with pytest.raises(sb.SnnError):
        sb.Network.from_csr(np.array([0, 2, 1, 2], np.uint64), ci, w)  # non-monotone
    with pytest.raises(sb.SnnError):
        sb.Network.from_csr(rp, ci, np.array([0.5, np.inf], np.float32))  # non-finite weight
    with pytest.raises(sb.SnnError):
        sb.Network.from_csr(rp, ci, w, sb.LifParams.default(v_threshold=-1.0))  # thr <= reset


def test_create_without_device_reports_cuda_error(gpu_count):
    if gpu_count:
        pytest.skip("a device is present")
    net = sb.Network.from_csr(np.array([0, 1, 2, 2], np.uint64), np.array([1, 2], np.uint64),
                              np.array([0.75, 1.25], np.float32))
    L = sb.lib()
    assert L.snn_cuda_available() == 0
    out = C.c_void_p(1)
    assert L.snn_cuda_create(net.handle, None, C.byref(out)) == sb.SNN_ERR_CUDA
    assert out.value is None
    # Fault-injection controls are pure setters.
    L.snn_test_cuda_set_fail_after(0)
    L.snn_test_cuda_force_unavailable(1)
    L.snn_test_cuda_force_meminfo_fail(1)
    L.snn_test_cuda_disable_failure()
    assert L.snn_test_nonnull_cuda_context()


def test_reference_unit_suite_links_and_passes_without_device(gpu_count):
    """The reference's tests/test_snn.c (unmodified) linked against
    libsnn_b200: on a machine without a GPU it takes the unavailable branch
    and every CPU test of the reference passes."""
    exe = os.path.join(ROOT, "oracle", "_ref", "test_snn_b200")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/test_snn_b200 not built (reference tree absent)")
    if gpu_count:
        pytest.skip("covered by the GPU test")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "all tests passed" in r.stdout
