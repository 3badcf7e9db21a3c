"""snn_b200 -- B200 (sm_100a) backend for the Ichigo-Labs/snn LIF simulation step.

The product is the C ABI in include/snn_b200.h, implemented by the in-tree
shared library snn_b200/_lib/libsnn_b200.so (built by ``python -m
snn_b200.build``). This module is a thin ctypes mirror of that interface with
the reference's names and status codes (include/snn/snn.h:17-24, 182-209):

    ctx = CudaContext.create(network, config, options)   # snn_cuda_create / snn_b200_create
    ctx.inject_current(indices, values)                  # snn_cuda_inject_current
    spikes = ctx.step(external=None)                     # snn_cuda_step
    v = ctx.download_voltage()                           # snn_cuda_download_voltage

There is no CPU fallback: importing works anywhere, but every call that needs
the library raises if it is missing, and creating a context without a CUDA
device returns SNN_ERR_CUDA like the reference does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libsnn_b200.so")

u64 = C.c_uint64
f32 = C.c_float
P = C.c_void_p

SNN_OK = 0
SNN_ERR_INVALID_ARGUMENT = -1
SNN_ERR_OUT_OF_MEMORY = -2
SNN_ERR_OVERFLOW = -3
SNN_ERR_CUDA = -4
SNN_ERR_UNSUPPORTED = -5
STATUS_NAMES = {0: "ok", -1: "invalid argument", -2: "out of memory", -3: "integer overflow",
                -4: "cuda error", -5: "unsupported"}

MODE_NONE, MODE_FULL, MODE_STREAMING = 0, 1, 2
NOALLOC_MAX_NEURONS = 1048576  # SNN_B200_NOALLOC_MAX_NEURONS
PROPAGATE_PUSH, PROPAGATE_ORDERED, PROPAGATE_PUSH_ATOMIC, PROPAGATE_PUSH_BINNED = 0, 1, 2, 3
EXCHANGE_NCCL, EXCHANGE_PEER = 0, 1
STREAMING_CHUNKED, STREAMING_SPARSE = 0, 1


class SnnError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        super().__init__(f"{what}: {STATUS_NAMES.get(status, 'unknown status')} ({status})")
        self.status = status


class LifParams(C.Structure):
    """include/snn/snn.h:32-40"""
    _fields_ = [("dt_ms", f32), ("membrane_tau_ms", f32), ("v_rest", f32), ("v_reset", f32),
                ("v_threshold", f32), ("input_scale", f32), ("refractory_steps", C.c_uint32)]

    @classmethod
    def default(cls, **kw) -> "LifParams":
        """The reference defaults (src/snn.c:290-300), overridden by keyword."""
        p = cls(1.0, 20.0, 0.0, 0.0, 1.0, 1.0, 1)
        for k, v in kw.items():
            setattr(p, k, v)
        return p


class CudaConfig(C.Structure):
    """include/snn/snn.h:96-108"""
    _fields_ = [("max_vram_bytes", u64), ("max_stream_synapses", u64), ("max_stream_rows", u64),
                ("prefer_streaming", C.c_int)]


class RandomPoolConfig(C.Structure):
    """include/snn/snn.h:50-57"""
    _fields_ = [("neuron_count", u64), ("fanout_per_neuron", u64), ("weight_min", f32),
                ("weight_max", f32), ("seed", u64), ("allow_self_connections", C.c_int)]


class Options(C.Structure):
    """snn_b200_options_t (include/snn_b200.h)."""
    _fields_ = [("propagation", C.c_int), ("device", C.c_int), ("index_width", C.c_int),
                ("rank", C.c_uint32), ("world_size", C.c_uint32), ("nccl_id", P), ("timing", C.c_int),
                ("exchange", C.c_int), ("streaming", C.c_int), ("batch", C.c_uint32)]


class Stats(C.Structure):
    _fields_ = [("steps", u64), ("spikes", u64), ("events", u64), ("kernel_launches", u64),
                ("step_ms", C.c_double), ("propagate_ms", C.c_double), ("lif_ms", C.c_double),
                ("exchange_ms", C.c_double), ("pull_steps", u64), ("pull_events", u64),
                ("pull_spikes", u64), ("propagate_pull_ms", C.c_double), ("exchange_wait_ms", C.c_double),
                ("exchange_wait_max_ms", C.c_double)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


class Layout(C.Structure):
    _fields_ = [("neuron_count", u64), ("local_begin", u64), ("local_count", u64), ("local_synapses", u64),
                ("index_bits", C.c_uint32), ("propagation", C.c_int), ("device_state_bytes", u64),
                ("device_topology_bytes", u64), ("binned", C.c_uint32), ("binned_passes", C.c_uint32),
                ("ordered_csc", C.c_uint32), ("batch", C.c_uint32), ("topology_rows", u64), ("pull_slots", u64)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


# (name, restype, argtypes) of every exported entry point in include/snn_b200.h.
ENTRY_POINTS = [
    ("snn_cuda_default_config", CudaConfig, []),
    ("snn_cuda_available", C.c_int, []),
    ("snn_cuda_create", C.c_int, [P, P, P]),
    ("snn_cuda_free", None, [P]),
    ("snn_cuda_context_mode", C.c_int, [P]),
    ("snn_cuda_inject_current", C.c_int, [P, P, P, u64]),
    ("snn_cuda_step", C.c_int, [P, P, P]),
    ("snn_cuda_download_voltage", C.c_int, [P, P, u64]),
    ("snn_test_nonnull_cuda_context", P, []),
    ("snn_test_cuda_set_fail_after", None, [C.c_int64]),
    ("snn_test_cuda_disable_failure", None, []),
    ("snn_test_cuda_force_unavailable", None, [C.c_int]),
    ("snn_test_cuda_force_meminfo_fail", None, [C.c_int]),
    ("snn_b200_default_options", Options, []),
    ("snn_b200_create", C.c_int, [P, P, P, P]),
    ("snn_b200_create_random_pool", C.c_int, [P, P, P, P, P]),
    ("snn_b200_create_layered_random", C.c_int, [P, C.c_size_t, u64, f32, f32, u64, P, P, P]),
    ("snn_b200_create_feedforward", C.c_int, [P, C.c_size_t, u64, f32, u64, P, P, P]),
    ("snn_b200_nccl_unique_id", C.c_int, [P]),
    ("snn_b200_ipc_handle", C.c_int, [P, P]),
    ("snn_b200_ipc_connect", C.c_int, [P, P]),
    ("snn_test_b200_peer_loopback", C.c_int, [P, C.c_uint32]),
    ("snn_b200_shard_range", C.c_int, [u64, C.c_uint32, C.c_uint32, P, P]),
    ("snn_b200_last_error", C.c_char_p, []),
    ("snn_b200_step_noalloc", C.c_int, [C.c_int, P, u64, P, f32, P, P, P, P, P, P, P, P, P]),
    ("snn_b200_probe_red_rate", C.c_int, [C.c_int, u64, u64, C.c_uint32, P]),
    ("snn_cuda_create_sharded", C.c_int, [P, P, C.c_int, P, P]),
    ("snn_b200_create_sharded", C.c_int, [P, P, P, C.c_int, P, P]),
    ("snn_b200_reset", C.c_int, [P]),
    ("snn_b200_inject_stream_async", C.c_int, [P, u64, u64, u64, f32]),
    ("snn_b200_run_stream_async", C.c_int, [P, u64, u64, u64, u64, f32]),
    ("snn_b200_step_async", C.c_int, [P]),
    ("snn_b200_set_external", C.c_int, [P, P]),
    ("snn_b200_set_stream_range", C.c_int, [P, u64]),
    ("snn_b200_synchronize", C.c_int, [P]),
    ("snn_b200_get_stats", C.c_int, [P, P]),
    ("snn_b200_reset_stats", C.c_int, [P]),
    ("snn_b200_get_layout", C.c_int, [P, P]),
    ("snn_b200_stream", P, [P]),
    ("snn_b200_download_spikes", C.c_int, [P, P, u64]),
    ("snn_b200_download_current", C.c_int, [P, P, u64]),
    ("snn_b200_download_topology", C.c_int, [P, P, u64, P, P, u64]),
    ("snn_b200_upload_state", C.c_int, [P, P, P, P, u64]),
    ("snn_b200_download_state", C.c_int, [P, P, P, P, u64]),
    ("snn_b200_network_wrap", C.c_int, [u64, u64, P, P, P, P, P]),
    ("snn_b200_network_unwrap", None, [P]),
    ("snn_b200_network_save", C.c_int, [P, C.c_char_p]),
    ("snn_b200_network_map", C.c_int, [C.c_char_p, P]),
]

_LIB = None


def lib() -> C.CDLL:
    """The loaded libsnn_b200.so; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m snn_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, res, args in ENTRY_POINTS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def last_error() -> str:
    """Detail of this thread's most recent CUDA/NCCL failure in the library."""
    return (lib().snn_b200_last_error() or b"").decode(errors="replace")


def _check(st: int, what: str):
    if st != SNN_OK:
        detail = last_error() if st == SNN_ERR_CUDA else ""
        raise SnnError(st, f"{what} [{detail}]" if detail else what)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(P)


def default_config(**kw) -> CudaConfig:
    c = lib().snn_cuda_default_config()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def default_options(**kw) -> Options:
    o = lib().snn_b200_default_options()
    for k, v in kw.items():
        setattr(o, k, v)
    return o


def cuda_available() -> bool:
    return bool(lib().snn_cuda_available())


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """(first neuron, neuron count) owned by `rank` of `world` postsynaptic shards."""
    b, c = u64(), u64()
    _check(lib().snn_b200_shard_range(n, world, rank, C.byref(b), C.byref(c)), "snn_b200_shard_range")
    return int(b.value), int(c.value)


def probe_red_rate(device: int = 0, targets: int = 10_000_000, events: int = 1 << 28, repeats: int = 5) -> float:
    """Reductions per second the device's L2 serves to random float slots
    (snn_b200_probe_red_rate): the ceiling of the atomic push."""
    out = C.c_double()
    _check(lib().snn_b200_probe_red_rate(device, targets, events, repeats, C.byref(out)), "snn_b200_probe_red_rate")
    return out.value


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().snn_b200_nccl_unique_id(buf), "snn_b200_nccl_unique_id")
    return buf.raw


class Network:
    """A network for the backend: either a view over caller CSR arrays
    (snn_b200_network_wrap) or a borrowed handle of a network built by the
    reference's host library."""

    def __init__(self, handle, owner=None, keep=()):
        self.handle = P(handle) if not isinstance(handle, P) else handle
        self._owner = owner
        self._keep = keep

    @classmethod
    def from_csr(cls, row_ptr, col_idx, weights, lif: LifParams | None = None) -> "Network":
        rp = np.ascontiguousarray(row_ptr, np.uint64)
        ci = np.ascontiguousarray(col_idx, np.uint64)
        w = np.ascontiguousarray(weights, np.float32)
        h = P()
        st = lib().snn_b200_network_wrap(rp.size - 1, ci.size, _ptr(rp), _ptr(ci) if ci.size else None,
                                         _ptr(w) if w.size else None, C.byref(lif) if lif else None, C.byref(h))
        _check(st, "snn_b200_network_wrap")
        return cls(h, owner="wrap", keep=(rp, ci, w))

    @classmethod
    def map(cls, path: str) -> "Network":
        """Maps an snn_b200 CSR file read-only (snn_b200_network_map); free() unmaps it."""
        h = P()
        _check(lib().snn_b200_network_map(os.fsencode(path), C.byref(h)), "snn_b200_network_map")
        return cls(h, owner="wrap")

    def free(self):
        if self._owner == "wrap" and self.handle:
            lib().snn_b200_network_unwrap(self.handle)
            self.handle = P(None)

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def save_network(net, path: str) -> None:
    """Writes a network (anything with a .handle: sb.Network or the oracle's) as an snn_b200 CSR file."""
    _check(lib().snn_b200_network_save(net.handle, os.fsencode(path)), "snn_b200_network_save")


class CudaContext:
    """Mirror of snn_cuda_context_t and its entry points."""

    def __init__(self, handle: P, keep=None):
        self.handle = handle
        self._keep = keep
        lay = Layout()
        _check(lib().snn_b200_get_layout(handle, C.byref(lay)), "snn_b200_get_layout")
        self.layout = lay.as_dict()
        self.n = int(lay.neuron_count)
        self.local_begin = int(lay.local_begin)
        self.local_count = int(lay.local_count)

    # ---- creation ------------------------------------------------------
    @classmethod
    def create(cls, network, config: CudaConfig | None = None, options: Options | None = None):
        h = P()
        handle = network.handle if hasattr(network, "handle") else network
        if options is None:
            st = lib().snn_cuda_create(handle, C.byref(config) if config else None, C.byref(h))
        else:
            st = lib().snn_b200_create(handle, C.byref(config) if config else None, C.byref(options), C.byref(h))
        _check(st, "snn_cuda_create")
        return cls(h, keep=network)

    @classmethod
    def create_sharded(cls, network, devices, config: CudaConfig | None = None, options: Options | None = None):
        """One context over several GPUs of this process (snn_cuda_create_sharded)."""
        h = P()
        handle = network.handle if hasattr(network, "handle") else network
        devs = (C.c_int * len(devices))(*devices)
        if options is None:
            st = lib().snn_cuda_create_sharded(handle, C.byref(config) if config else None, len(devices), devs,
                                               C.byref(h))
        else:
            st = lib().snn_b200_create_sharded(handle, C.byref(config) if config else None, C.byref(options),
                                               len(devices), devs, C.byref(h))
        _check(st, "snn_cuda_create_sharded")
        return cls(h, keep=network)

    @classmethod
    def random_pool(cls, n, fanout, wmin, wmax, seed, allow_self=False, lif=None, config=None, options=None):
        cfg = RandomPoolConfig(n, fanout, wmin, wmax, seed, int(allow_self))
        h = P()
        st = lib().snn_b200_create_random_pool(C.byref(cfg), C.byref(lif) if lif else None,
                                               C.byref(config) if config else None,
                                               C.byref(options) if options else None, C.byref(h))
        _check(st, "snn_b200_create_random_pool")
        return cls(h)

    @classmethod
    def layered_random(cls, layers, fanout, wmin, wmax, seed, lif=None, options=None):
        arr = np.ascontiguousarray(layers, np.uint64)
        h = P()
        st = lib().snn_b200_create_layered_random(_ptr(arr), arr.size, fanout, wmin, wmax, seed,
                                                  C.byref(lif) if lif else None,
                                                  C.byref(options) if options else None, C.byref(h))
        _check(st, "snn_b200_create_layered_random")
        return cls(h)

    @classmethod
    def feedforward(cls, layers, fanout, weight, seed, lif=None, options=None):
        """snn_b200_create_feedforward: snn_build_feedforward on the device."""
        arr = np.ascontiguousarray(layers, np.uint64)
        h = P()
        st = lib().snn_b200_create_feedforward(_ptr(arr), arr.size, fanout, weight, seed,
                                               C.byref(lif) if lif else None,
                                               C.byref(options) if options else None, C.byref(h))
        _check(st, "snn_b200_create_feedforward")
        return cls(h)

    # ---- reference entry points ---------------------------------------
    @property
    def mode(self) -> int:
        return lib().snn_cuda_context_mode(self.handle)

    def inject_current(self, indices, values) -> int:
        idx = np.ascontiguousarray(indices, np.uint64)
        val = np.ascontiguousarray(values, np.float32)
        return lib().snn_cuda_inject_current(self.handle, _ptr(idx), _ptr(val), idx.size)

    def step(self, external=None, spikes: bool = True, out: np.ndarray | None = None):
        ext = None if external is None else np.ascontiguousarray(external, np.float32)
        buf = out if out is not None else (np.empty(self.local_count, np.uint8) if spikes else None)
        st = lib().snn_cuda_step(self.handle, _ptr(ext), _ptr(buf))
        _check(st, "snn_cuda_step")
        return buf

    def download_voltage(self) -> np.ndarray:
        out = np.empty(self.local_count, np.float32)
        _check(lib().snn_cuda_download_voltage(self.handle, _ptr(out), out.size), "snn_cuda_download_voltage")
        return out

    # ---- extensions ------------------------------------------------------
    def reset(self):
        _check(lib().snn_b200_reset(self.handle), "snn_b200_reset")

    def inject_stream_async(self, seed, step, count, value):
        _check(lib().snn_b200_inject_stream_async(self.handle, seed, step, count, value), "inject_stream")

    def run_stream_async(self, seed, first_step, steps, count, value):
        _check(lib().snn_b200_run_stream_async(self.handle, seed, first_step, steps, count, value), "run_stream")

    def step_async(self):
        _check(lib().snn_b200_step_async(self.handle), "snn_b200_step_async")

    def set_stream_range(self, n: int):
        """Injection-stream indices in [0, n) (0: all neurons)."""
        _check(lib().snn_b200_set_stream_range(self.handle, n), "snn_b200_set_stream_range")

    def set_external(self, external):
        """Holds an external frame on the device for every later step without its own (None clears)."""
        ext = None if external is None else np.ascontiguousarray(external, np.float32)
        if ext is not None and ext.size < self.local_count:
            raise ValueError("external frame shorter than the local neuron count")
        _check(lib().snn_b200_set_external(self.handle, _ptr(ext)), "snn_b200_set_external")

    def synchronize(self):
        _check(lib().snn_b200_synchronize(self.handle), "snn_b200_synchronize")

    def stats(self) -> dict:
        s = Stats()
        _check(lib().snn_b200_get_stats(self.handle, C.byref(s)), "snn_b200_get_stats")
        return s.as_dict()

    def reset_stats(self):
        _check(lib().snn_b200_reset_stats(self.handle), "snn_b200_reset_stats")

    def stream(self) -> int:
        return int(lib().snn_b200_stream(self.handle) or 0)

    def download_spikes(self) -> np.ndarray:
        out = np.empty(self.local_count, np.uint8)
        _check(lib().snn_b200_download_spikes(self.handle, _ptr(out), out.size), "download_spikes")
        return out

    def download_current(self) -> np.ndarray:
        out = np.empty(self.local_count, np.float32)
        _check(lib().snn_b200_download_current(self.handle, _ptr(out), out.size), "download_current")
        return out

    def upload_state(self, voltage=None, current=None, refractory=None):
        v = None if voltage is None else np.ascontiguousarray(voltage, np.float32)
        c = None if current is None else np.ascontiguousarray(current, np.float32)
        r = None if refractory is None else np.ascontiguousarray(refractory, np.uint32)
        _check(lib().snn_b200_upload_state(self.handle, _ptr(v), _ptr(c), _ptr(r), self.local_count),
               "snn_b200_upload_state")

    def download_state(self):
        v = np.empty(self.local_count, np.float32)
        c = np.empty(self.local_count, np.float32)
        r = np.empty(self.local_count, np.uint32)
        _check(lib().snn_b200_download_state(self.handle, _ptr(v), _ptr(c), _ptr(r), self.local_count),
               "snn_b200_download_state")
        return v, c, r

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(64)
        _check(lib().snn_b200_ipc_handle(self.handle, buf), "snn_b200_ipc_handle")
        return buf.raw

    def ipc_connect(self, handles: list):
        """handles: every rank's ipc_handle() bytes, in rank order."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        _check(lib().snn_b200_ipc_connect(self.handle, blob), "snn_b200_ipc_connect")

    def download_topology(self):
        e = int(self.layout["local_synapses"])
        rp = np.empty(self.n + 1, np.uint64)
        ci = np.empty(max(e, 1), np.uint64)
        w = np.empty(max(e, 1), np.float32)
        _check(lib().snn_b200_download_topology(self.handle, _ptr(rp), rp.size, _ptr(ci), _ptr(w), ci.size),
               "download_topology")
        return rp, ci[:e], w[:e]

    def free(self):
        if self.handle:
            lib().snn_cuda_free(self.handle)
            self.handle = P(None)

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.free()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
