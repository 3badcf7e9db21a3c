"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU oracle.

Two interchangeable back ends share one Python surface:

* ``Oracle("port")``    -- oracle/liboracle.so, the C restatement in
  oracle/snn_oracle.c of the reference simulator's CPU path;
* ``Oracle("ref")``     -- oracle/_ref/libsnn_ref.so, the reference's own
  src/snn.c compiled here (serial build, CSR-order scatter, src/snn.c:898-906);
* ``Oracle("ref_omp")`` -- oracle/_ref/libsnn_ref_omp.so, the same source with
  OpenMP (the timed CPU baseline; not an exact oracle, src/snn.c:839-896).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module. A network built here is a pointer to a struct with the
reference's layout (src/snn_internal.h:15-24), so it can be passed straight to
the snn_b200 backend's ``snn_cuda_create``.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

u64 = C.c_uint64
f32 = C.c_float
P = C.c_void_p


class LifParams(C.Structure):
    """include/snn/snn.h:32-40"""
    _fields_ = [("dt_ms", f32), ("membrane_tau_ms", f32), ("v_rest", f32), ("v_reset", f32),
                ("v_threshold", f32), ("input_scale", f32), ("refractory_steps", C.c_uint32)]


class NetworkStruct(C.Structure):
    """src/snn_internal.h:15-24"""
    _fields_ = [("neuron_count", u64), ("synapse_count", u64), ("architecture", C.c_int),
                ("lif", LifParams), ("decay", f32), ("row_ptr", C.POINTER(u64)),
                ("col_idx", C.POINTER(u64)), ("weights", C.POINTER(f32))]


class RandomPoolConfig(C.Structure):
    """include/snn/snn.h:50-57"""
    _fields_ = [("neuron_count", u64), ("fanout_per_neuron", u64), ("weight_min", f32),
                ("weight_max", f32), ("seed", u64), ("allow_self_connections", C.c_int)]


class FeedforwardConfig(C.Structure):
    """include/snn/snn.h:42-48"""
    _fields_ = [("layer_sizes", C.POINTER(u64)), ("layer_count", C.c_size_t),
                ("fanout_per_neuron", u64), ("weight", f32), ("seed", u64)]


class MemoryPlan(C.Structure):
    """include/snn/snn.h:71-85"""
    _fields_ = [("neuron_count", u64), ("synapse_count", u64), ("row_ptr_bytes", u64),
                ("col_index_bytes", u64), ("weight_bytes", u64), ("host_topology_bytes", u64),
                ("host_state_bytes", u64), ("host_total_bytes", u64), ("device_topology_bytes", u64),
                ("device_state_bytes", u64), ("device_total_full_bytes", u64),
                ("device_streaming_min_bytes", u64), ("overflowed", C.c_int)]


def default_lif(**kw) -> LifParams:
    """src/snn.c:290-300 defaults, overridden by keyword."""
    p = LifParams(1.0, 20.0, 0.0, 0.0, 1.0, 1.0, 1)
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def baseline_lif() -> LifParams:
    """The LIF parameters every BASELINE config uses: dt 1 ms, tau 20 ms,
    rest = reset = -65 mV, threshold -50 mV, refractory 2 steps, scale 1."""
    return default_lif(v_rest=-65.0, v_reset=-65.0, v_threshold=-50.0, refractory_steps=2)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(P) if a is not None and a.size else None


class Network:
    """Owns a network built by one oracle back end."""

    def __init__(self, lib: "Oracle", handle: int):
        self.lib = lib
        self.handle = P(handle)
        self.s = C.cast(self.handle, C.POINTER(NetworkStruct)).contents

    @property
    def neuron_count(self) -> int:
        return int(self.s.neuron_count)

    @property
    def synapse_count(self) -> int:
        return int(self.s.synapse_count)

    @property
    def decay(self) -> float:
        return float(self.s.decay)

    def row_ptr(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.s.row_ptr, shape=(self.neuron_count + 1,)).copy()

    def col_idx(self) -> np.ndarray:
        if self.synapse_count == 0:
            return np.zeros(0, np.uint64)
        return np.ctypeslib.as_array(self.s.col_idx, shape=(self.synapse_count,)).copy()

    def weights(self) -> np.ndarray:
        if self.synapse_count == 0:
            return np.zeros(0, np.float32)
        return np.ctypeslib.as_array(self.s.weights, shape=(self.synapse_count,)).copy()

    def set_lif(self, p: LifParams) -> int:
        return self.lib._set_lif(self.handle, C.byref(p))

    def free(self):
        if self.handle:
            self.lib._net_free(self.handle)
            self.handle = P(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class State:
    """A simulation state. `lib` selects the back end that steps it (default:
    the one that built the network); networks of every back end share the
    reference's struct layout, so a port-built network can be stepped by the
    reference's own library."""

    def __init__(self, net: Network, lib: "Oracle | None" = None):
        self.net = net
        self.lib = lib if lib is not None else net.lib
        h = P()
        st = self.lib._state_create(net.handle, C.byref(h))
        if st != 0:
            raise RuntimeError(f"state_create failed: {st}")
        self.handle = h
        self.n = net.neuron_count

    def inject(self, idx, val) -> int:
        idx = np.ascontiguousarray(idx, np.uint64)
        val = np.ascontiguousarray(val, np.float32)
        return self.lib._inject(self.net.handle, self.handle, _ptr(idx), _ptr(val), u64(idx.size))

    def step(self, ext=None):
        """One step; returns the spike vector (uint8[n])."""
        spikes = np.zeros(self.n, np.uint8)
        e = None if ext is None else np.ascontiguousarray(ext, np.float32)
        st = self.lib._step(self.net.handle, self.handle, _ptr(e), _ptr(spikes))
        if st != 0:
            raise RuntimeError(f"step failed: {st}")
        return spikes

    def voltage(self) -> np.ndarray:
        out = np.zeros(self.n, np.float32)
        if self.lib.kind == "port":
            s = C.cast(self.handle, C.POINTER(_OrcState)).contents
            return np.ctypeslib.as_array(s.voltage, shape=(self.n,)).copy()
        st = self.lib._copy_voltage(self.handle, _ptr(out), u64(self.n))
        assert st == 0
        return out

    def current(self) -> np.ndarray:
        """The current the next step consumes (propagated + injected)."""
        if self.lib.kind != "port":
            raise NotImplementedError("current() is read from the oracle port only")
        s = C.cast(self.handle, C.POINTER(_OrcState)).contents
        return np.ctypeslib.as_array(s.current, shape=(self.n,)).copy()

    def refractory(self) -> np.ndarray:
        if self.lib.kind != "port":
            raise NotImplementedError("refractory() is read from the oracle port only")
        s = C.cast(self.handle, C.POINTER(_OrcState)).contents
        return np.ctypeslib.as_array(s.refractory, shape=(self.n,)).copy()

    def reset(self) -> int:
        return self.lib._reset(self.net.handle, self.handle)

    def free(self):
        if self.handle:
            self.lib._state_free(self.handle)
            self.handle = P(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class _OrcState(C.Structure):
    _fields_ = [("neuron_count", u64), ("voltage", C.POINTER(f32)), ("current", C.POINTER(f32)),
                ("next_current", C.POINTER(f32)), ("refractory", C.POINTER(C.c_uint32)),
                ("spikes", C.POINTER(C.c_uint8)), ("spike_indices", C.POINTER(u64)), ("spike_count", u64)]


def ref_available(kind: str = "ref") -> bool:
    name = {"ref": "libsnn_ref.so", "ref_omp": "libsnn_ref_omp.so"}[kind]
    return os.path.exists(os.path.join(HERE, "_ref", name))


class Oracle:
    def __init__(self, kind: str = "port"):
        self.kind = kind
        if kind == "port":
            path = os.path.join(HERE, "liboracle.so")
            pre = "orc_"
        elif kind in ("ref", "ref_omp"):
            path = os.path.join(HERE, "_ref", "libsnn_ref.so" if kind == "ref" else "libsnn_ref_omp.so")
            pre = "snn_"
        else:
            raise ValueError(kind)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        self.path = path
        L = C.CDLL(path)
        self.L = L

        def fn(name, res, *args):
            f = getattr(L, pre + name)
            f.restype = res
            f.argtypes = list(args)
            return f

        self._net_free = fn("network_free", None, P)
        self._set_lif = fn("network_set_lif_params", C.c_int, P, P)
        self._state_create = fn("state_create", C.c_int, P, P)
        self._state_free = fn("state_free", None, P)
        self._reset = fn("state_reset", C.c_int, P, P)
        self._inject = fn("state_inject_current", C.c_int, P, P, P, P, u64)
        self._step = fn("step" if kind == "port" else "step_cpu", C.c_int, P, P, P, P)
        self._custom = fn("build_custom_csr", C.c_int, u64, u64, P, P, P, P, P)
        self._plan_counts = fn("estimate_memory_for_counts", C.c_int, u64, u64, P)
        self._plan_net = fn("network_memory_plan", C.c_int, P, P)
        if kind == "port":
            self._pool = fn("build_random_pool", C.c_int, u64, u64, f32, f32, u64, C.c_int, P, P)
            self._pool_par = fn("build_random_pool_parallel", C.c_int, u64, u64, f32, f32, u64, C.c_int, P, P)
            self._ff = fn("build_feedforward", C.c_int, P, C.c_size_t, u64, f32, u64, P, P)
            self._layered = fn("build_layered_random", C.c_int, P, C.c_size_t, u64, f32, f32, u64, P, P)
            self._dense_gauss = fn("build_dense_gaussian", C.c_int, P, C.c_size_t, u64, P, P)
            self._run_stream = fn("run_inject_stream", C.c_int, P, P, u64, u64, u64, u64, f32, P, P, P, P)
            self._stream_idx = fn("inject_stream_indices", None, u64, u64, u64, u64, P)
            self._frame = fn("sparse_frame", None, u64, u64, u64, f32, u64, P)
        else:
            self._pool = fn("build_random_pool", C.c_int, P, P, P)
            self._ff = fn("build_feedforward", C.c_int, P, P, P)
            self._copy_voltage = fn("state_copy_voltage", C.c_int, P, P, u64)

    # ---- builders -------------------------------------------------------
    def _wrap(self, st, h) -> Network:
        if st != 0:
            raise RuntimeError(f"build failed: status {st}")
        return Network(self, h.value)

    def random_pool(self, n, fanout, wmin, wmax, seed, allow_self=False, lif=None) -> Network:
        h = P()
        lp = C.byref(lif) if lif is not None else None
        if self.kind == "port":
            st = self._pool(n, fanout, wmin, wmax, seed, int(allow_self), lp, C.byref(h))
        else:
            cfg = RandomPoolConfig(n, fanout, wmin, wmax, seed, int(allow_self))
            st = self._pool(C.byref(cfg), lp, C.byref(h))
        return self._wrap(st, h)

    def random_pool_parallel(self, n, fanout, wmin, wmax, seed, allow_self=False, lif=None) -> Network:
        """random_pool built by all host threads (port only), bit-identical."""
        assert self.kind == "port"
        h = P()
        st = self._pool_par(n, fanout, wmin, wmax, seed, int(allow_self),
                            C.byref(lif) if lif is not None else None, C.byref(h))
        return self._wrap(st, h)

    def feedforward(self, layers, fanout, weight, seed, lif=None) -> Network:
        h = P()
        arr = np.ascontiguousarray(layers, np.uint64)
        lp = C.byref(lif) if lif is not None else None
        if self.kind == "port":
            st = self._ff(_ptr(arr), arr.size, fanout, weight, seed, lp, C.byref(h))
        else:
            cfg = FeedforwardConfig(arr.ctypes.data_as(C.POINTER(u64)), arr.size, fanout, weight, seed)
            st = self._ff(C.byref(cfg), lp, C.byref(h))
        return self._wrap(st, h)

    def custom_csr(self, row_ptr, col_idx, weights, lif=None) -> Network:
        row_ptr = np.ascontiguousarray(row_ptr, np.uint64)
        col_idx = np.ascontiguousarray(col_idx, np.uint64)
        weights = np.ascontiguousarray(weights, np.float32)
        h = P()
        st = self._custom(row_ptr.size - 1, col_idx.size, _ptr(row_ptr), _ptr(col_idx), _ptr(weights),
                          C.byref(lif) if lif is not None else None, C.byref(h))
        return self._wrap(st, h)

    def layered_random(self, layers, fanout, wmin, wmax, seed, lif=None) -> Network:
        assert self.kind == "port"
        arr = np.ascontiguousarray(layers, np.uint64)
        h = P()
        st = self._layered(_ptr(arr), arr.size, fanout, wmin, wmax, seed,
                           C.byref(lif) if lif is not None else None, C.byref(h))
        return self._wrap(st, h)

    def dense_gaussian(self, layers, seed, lif=None) -> Network:
        assert self.kind == "port"
        arr = np.ascontiguousarray(layers, np.uint64)
        h = P()
        st = self._dense_gauss(_ptr(arr), arr.size, seed, C.byref(lif) if lif is not None else None, C.byref(h))
        return self._wrap(st, h)

    # ---- memory plan ----------------------------------------------------
    def plan_counts(self, n, e):
        p = MemoryPlan()
        st = self._plan_counts(n, e, C.byref(p))
        return st, p

    def plan_network(self, net: Network):
        p = MemoryPlan()
        st = self._plan_net(net.handle, C.byref(p))
        return st, p

    # ---- streams (port only) ---------------------------------------------
    def stream_indices(self, seed, step, count, n) -> np.ndarray:
        out = np.zeros(count, np.uint64)
        if self.kind == "port":
            self._stream_idx(seed, step, count, n, _ptr(out))
            return out
        return stream_indices_np(seed, step, count, n)

    def run_inject_stream(self, net: Network, state: State, seed, first_step, steps, count, value,
                          raster=False):
        """Runs `steps` steps of the seeded injection stream. Returns per-step
        spike counts, event counts, spike-vector hashes (and the raster)."""
        sc = np.zeros(steps, np.uint64)
        ev = np.zeros(steps, np.uint64)
        hs = np.zeros(steps, np.uint64)
        rs = np.zeros((steps, net.neuron_count), np.uint8) if raster else None
        if self.kind == "port":
            st = self._run_stream(net.handle, state.handle, seed, first_step, steps, count, value,
                                  _ptr(sc), _ptr(ev), _ptr(hs), _ptr(rs) if raster else None)
            assert st == 0, st
            return sc, ev, hs, rs
        rp = net.row_ptr()
        deg = (rp[1:] - rp[:-1]).astype(np.uint64)
        for t in range(steps):
            idx = stream_indices_np(seed, first_step + t, count, net.neuron_count)
            assert state.inject(idx, np.full(count, value, np.float32)) == 0
            s = state.step()
            sc[t] = int(s.sum())
            ev[t] = int(deg[s.astype(bool)].sum())
            hs[t] = fnv1a(s)
            if raster:
                rs[t] = s
        return sc, ev, hs, rs

    def sparse_frame(self, seed, sample, pixels, zero_prob, n) -> np.ndarray:
        assert self.kind == "port"
        out = np.zeros(n, np.float32)
        self._frame(seed, sample, pixels, zero_prob, n, _ptr(out))
        return out


GAMMA = 0x9E3779B97F4A7C15
M64 = (1 << 64) - 1


def mix64_np(z: np.ndarray) -> np.ndarray:
    z = z.astype(np.uint64)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def stream_indices_np(seed, step, count, n) -> np.ndarray:
    """Same stream as orc_inject_stream_indices, in numpy."""
    with np.errstate(over="ignore"):
        d = np.arange(step * count + 1, step * count + count + 1, dtype=np.uint64)
        z = np.uint64(seed) + d * np.uint64(GAMMA)
        return mix64_np(z) % np.uint64(n)


def fnv1a(b: np.ndarray) -> int:
    h = 0xCBF29CE484222325
    for x in np.asarray(b, np.uint8).tobytes():
        h ^= x
        h = (h * 0x100000001B3) & M64
    return h
