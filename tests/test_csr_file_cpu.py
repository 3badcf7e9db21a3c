"""CPU checks of the snn_b200 CSR file (snn_b200_network_save / _map): a
saved network maps back bit for bit (topology, LIF parameters, decay), with
the sections 4096-byte aligned; damaged files (bad magic, truncation, a
column out of range, a non-finite weight) are rejected by the same validation
as snn_build_custom_csr (src/snn.c:158-180) instead of reaching a kernel."""
import ctypes as C
import os

import numpy as np
import pytest

import snn_b200 as sb
from oracle.oracle import NetworkStruct, Oracle, default_lif


def view(net):
    s = C.cast(net.handle, C.POINTER(NetworkStruct)).contents
    n, e = int(s.neuron_count), int(s.synapse_count)
    rp = np.ctypeslib.as_array(s.row_ptr, shape=(n + 1,)).copy()
    ci = np.ctypeslib.as_array(s.col_idx, shape=(e,)).copy() if e else np.zeros(0, np.uint64)
    w = np.ctypeslib.as_array(s.weights, shape=(e,)).copy() if e else np.zeros(0, np.float32)
    return s, rp, ci, w


def test_save_map_roundtrip(tmp_path):
    lif = default_lif(v_rest=0.25, v_reset=-0.5, v_threshold=1.0, input_scale=0.7, refractory_steps=2)
    src = Oracle("port").random_pool(5003, 37, -0.2, 0.5, 9, lif=lif)
    path = str(tmp_path / "pool.snncsr")
    sb.save_network(src, path)
    assert not os.path.exists(path + ".partial")
    assert open(path, "rb").read(8) == b"SNNCSR01"
    m = sb.Network.map(path)
    s, rp, ci, w = view(m)
    assert (s.neuron_count, s.synapse_count) == (5003, 5003 * 37)
    assert s.decay == np.float32(src.decay)
    assert (s.lif.v_rest, s.lif.v_reset, s.lif.refractory_steps) == (np.float32(0.25), np.float32(-0.5), 2)
    np.testing.assert_array_equal(rp, src.row_ptr())
    np.testing.assert_array_equal(ci, src.col_idx())
    np.testing.assert_array_equal(w.view(np.uint32), src.weights().view(np.uint32))
    for ptr in (C.cast(s.row_ptr, C.c_void_p).value, C.cast(s.col_idx, C.c_void_p).value,
                C.cast(s.weights, C.c_void_p).value):
        assert ptr % 4096 == 0
    # A mapped network saves again to the same bytes.
    sb.save_network(m, path + ".2")
    assert open(path, "rb").read() == open(path + ".2", "rb").read()
    m.free()


def test_empty_topology_roundtrip(tmp_path):
    net = sb.Network.from_csr(np.zeros(4, np.uint64), np.zeros(0, np.uint64), np.zeros(0, np.float32))
    path = str(tmp_path / "empty.snncsr")
    sb.save_network(net, path)
    m = sb.Network.map(path)
    s, rp, _, _ = view(m)
    assert (s.neuron_count, s.synapse_count) == (3, 0)
    np.testing.assert_array_equal(rp, np.zeros(4, np.uint64))
    m.free()


def test_damaged_files_are_rejected(tmp_path):
    rp = np.array([0, 2, 3, 3], np.uint64)
    ci = np.array([1, 2, 0], np.uint64)
    w = np.array([0.5, 0.25, 1.0], np.float32)
    path = str(tmp_path / "small.snncsr")
    sb.save_network(sb.Network.from_csr(rp, ci, w), path)
    good = bytearray(open(path, "rb").read())

    def rejected(data):
        bad = str(tmp_path / "bad.snncsr")
        open(bad, "wb").write(bytes(data))
        with pytest.raises(sb.SnnError):
            sb.Network.map(bad)

    rejected(b"NOTACSR!" + good[8:])  # magic
    rejected(good[:-4])               # truncated weights
    rejected(good[:100])              # shorter than the header
    # Header: magic 8, version 4, header_bytes 4, n 8, e 8, architecture 4,
    # lif 28, decay 4, padding 4, then the row_ptr / col_idx / weights offsets.
    col_off = int(np.frombuffer(bytes(good[80:88]), np.uint64)[0])
    w_off = int(np.frombuffer(bytes(good[88:96]), np.uint64)[0])
    assert col_off % 4096 == 0 and w_off % 4096 == 0
    bad = bytearray(good)
    bad[col_off:col_off + 8] = np.uint64(3).tobytes()  # column == n
    rejected(bad)
    bad = bytearray(good)
    bad[w_off:w_off + 4] = np.float32(np.inf).tobytes()  # non-finite weight
    rejected(bad)
    with pytest.raises(sb.SnnError):
        sb.Network.map(str(tmp_path / "missing.snncsr"))
