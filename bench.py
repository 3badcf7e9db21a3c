#!/usr/bin/env python
"""Synaptic-event throughput of the snn_b200 simulation step on B200.

Workload ("resident recurrent pool"): 10M LIF neurons,
fixed fanout 1,000 (10B synapses), weights U[-0.2, 0.5] mV, FULL policy;
every step injects 0.5% of the neurons (seeded uniform indices) with 25.0.
The network is generated on the device, bit-identical to the reference's
snn_build_random_pool for the same seed (a host build would need ~120 GB and
minutes). Propagation is the atomic push, with the chunked sliced-ELL pull
taking the steps where more than a quarter of the rows fire (chosen on the
device). At N GPUs the pool is sharded by postsynaptic neuron (strong
scaling: the total network is fixed) and every step's spike bitmap is
exchanged over NVLink by the LIF kernel itself (--exchange peer; --exchange
nccl all-gathers it with NCCL).

    python bench.py [--gpus N --steps K --warmup W]          # snn_b200 arm
    python bench.py --impl reference [--steps K --warmup W]  # reference CPU arm
    torchrun --nproc-per-node N bench.py --gpus N ...        # N > 1

One JSON line is printed by rank 0. value = synaptic events (sum of the
out-degrees of the spiking rows, benchmarks/step_throughput.c:121-126) of all
ranks / device time of exactly K steps (CUDA events on the library's stream,
max over ranks). e2e = the same metric through the reference-facing C ABI
(snn_cuda_inject_current + snn_cuda_step with host index/value buffers and a
host spike download every step).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROPAGATION_LABEL = {"auto": "push (auto)", "atomic": "push (atomic)", "ordered": "ordered (bit-exact, event sort)",
                     "binned": "ordered (bit-exact, bin-fold)"}
L2_NOTE = "inputs larger than L2 (FULL CSR of the shard read sparsely each step; target currents L2-resident by design)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--neurons", type=int, default=10_000_000)
    ap.add_argument("--fanout", type=int, default=1000)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--inject-frac", type=float, default=0.005)
    ap.add_argument("--inject-value", type=float, default=25.0)
    ap.add_argument("--cpu-neurons", type=int, default=1_000_000,
                    help="bounded CPU sample: the same pool scaled to this many neurons")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the ORDERED raster-hash check")
    ap.add_argument("--no-secondary", action="store_true",
                    help="N=1: skip the other workloads (config 0, ORDERED config 2, config 4, STREAMING)")
    ap.add_argument("--parity-neurons", type=int, default=200_000)
    ap.add_argument("--parity-steps", type=int, default=40)
    ap.add_argument("--exchange", choices=["nccl", "peer"], default="peer",
                    help="N>1: spike exchange by ncclAllGather or fused into the LIF kernel over NVLink")
    ap.add_argument("--policy", choices=["full", "streaming"], default="full",
                    help="streaming: STREAMING VRAM policy on a host-resident pool (--stream-neurons), "
                         "measured against the host-link roofline")
    ap.add_argument("--stream-neurons", type=int, default=1_000_000)
    ap.add_argument("--stream-mode", choices=["chunked", "sparse"], default="sparse")
    ap.add_argument("--stream-source", choices=["host", "generated"], default="host",
                    help="host: a numpy-built pool in host memory (1 GPU); generated: each rank's slice of a "
                         "seeded pool generated on its device and moved to host memory (any GPU count)")
    ap.add_argument("--stream-budget-frac", type=float, default=0.25,
                    help="VRAM budget as a fraction of the host CSR bytes (config 3 streams ~15x its budget)")
    ap.add_argument("--workload", choices=["config2", "config1", "config4"], default="config2",
                    help="config1: BASELINE config 1 (784-1000-10 dense, 25 steps per static frame) run as "
                         "--batch samples at once over one shared topology; config4: 8 layers x "
                         "--layer-size, fanout 500 to the next layer, w ~ U[0,1], 5%% of layer 0 injected "
                         "with 30.0 per step")
    ap.add_argument("--layer-size", type=int, default=1_000_000, help="config4: neurons per layer")
    ap.add_argument("--batch", type=int, default=2000, help="config1: samples per batched context")
    ap.add_argument("--propagation", choices=["auto", "binned", "atomic", "ordered"], default="auto",
                    help="auto: the library's push (atomic push, pull on dense steps); atomic: the push alone; "
                         "ordered: bit-exact CSR-order propagation (event sort, pull on dense steps); "
                         "binned: bit-exact bin-fold (no host round trip, pull on dense steps)")
    return ap.parse_args()


# --------------------------------------------------------------- clocks ----
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML during the timed region."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                mask = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def measured_peak_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# DRAM bytes per synaptic event of propagate_push_kernel (32-bit columns):
# dram__bytes_read.sum + dram__bytes_write.sum over the events of one ncu
# capture of the kernel (500k-neuron pool, fanout 1000); scaled by this
# run's events. The pull kernel reads 8 B per slot of its layout.
NCU_DRAM_BYTES_PER_EVENT = 8.68
NCU_PULL_BYTES_PER_SLOT = 8.0


# ------------------------------------------------------------ CPU side ----
def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def pin_cpu_threads():
    """Give the reference's OpenMP step every host core, whatever a launcher
    (torchrun sets OMP_NUM_THREADS=1) left in the environment. Must run before
    the OpenMP runtime is loaded."""
    os.environ["OMP_NUM_THREADS"] = str(host_threads())


def omp_threads() -> int:
    """Threads the loaded OpenMP runtime will use."""
    import ctypes
    try:
        return int(ctypes.CDLL("libgomp.so.1").omp_get_max_threads())
    except OSError:
        return 1


def full_pool_fits(n, fanout) -> bool:
    """Whether the host can hold the full pool (12 B/edge + 8 B/row) with the
    reference's per-thread partial buffers and a margin."""
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        return False
    need = 12 * n * fanout + 8 * (n + 1) + 4 * n * (host_threads() + 8)
    return need < 0.85 * avail


def cpu_sample(args, kind_pref=("ref_omp", "port"), steps=None, warmup=None, seconds=None, neurons=None):
    """Times the reference CPU step (OpenMP build when present) on the pool of
    `neurons` neurons (default --cpu-neurons, a bounded sample of the same
    pool). The network is built by the oracle's multi-threaded builder,
    bit-identical to the reference's snn_build_random_pool, and stepped by
    the reference's own library."""
    import numpy as np

    from oracle.oracle import Oracle, State, baseline_lif, ref_available, stream_indices_np
    kind = next(k for k in kind_pref if k == "port" or ref_available(k))
    orc = Oracle(kind)
    n = neurons or args.cpu_neurons
    net = Oracle("port").random_pool_parallel(n, args.fanout, -0.2, 0.5, args.seed, lif=baseline_lif())
    st = State(net, lib=orc)
    rp = net.row_ptr()
    deg = (rp[1:] - rp[:-1]).astype(np.int64)
    count = max(1, int(round(args.inject_frac * n)))
    val = np.full(count, args.inject_value, np.float32)
    warm = 10 if warmup is None else warmup
    for t in range(warm):
        st.inject(stream_indices_np(args.seed, t, count, n), val)
        st.step()
    events, elapsed, done = 0, 0.0, 0
    idxs = {}
    limit = steps if steps is not None else 10 ** 9
    while done < limit and (seconds is None or elapsed < seconds):
        t = warm + done
        idx = idxs.pop(t, None)
        if idx is None:
            idx = stream_indices_np(args.seed, t, count, n)
        t0 = time.perf_counter()
        st.inject(idx, val)
        s = st.step()
        elapsed += time.perf_counter() - t0
        events += int(deg[s.astype(bool)].sum())
        done += 1
    threads = omp_threads() if kind == "ref_omp" else 1
    scope = "the full pool" if n == args.neurons else f"the same pool scaled to {n} neurons"
    return {"value": events / elapsed if elapsed > 0 else 0.0, "unit": "events/s", "cores": threads,
            "kind": "reference" if kind.startswith("ref") else "port",
            "sample": f"{scope} x fanout {args.fanout}, {done} steps after {warm} warm-up steps, reference "
                      f"src/snn.c snn_step_cpu ({'OpenMP, ' + str(threads) + ' threads' if kind == 'ref_omp' else 'serial'})",
            "steps": done, "seconds": elapsed, "neurons": n}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/liboracle.so not built"}))
        return
    if args.workload != "config2":
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times config 2 only"}))
        return
    pin_cpu_threads()
    warm = max(args.warmup, 0)
    # The full pool when the host can hold it (the reference's own step on
    # the same 10M x 1000 network the GPU arm runs); else the largest
    # bounded sample, and the config says which.
    full = full_pool_fits(args.neurons, args.fanout)
    n = args.neurons if full else args.cpu_neurons
    r = cpu_sample(args, steps=args.steps, warmup=warm, seconds=None, neurons=n)
    if not full:
        args.neurons = n
    cfg = workload_config(args, args.gpus)
    line = {"impl": "reference", "metric": "synaptic_events_per_sec", "value": r["value"], "unit": "events/s",
            "n_gpus": args.gpus, "steps": r["steps"], "warmup": warm,
            "ms_per_step": 1000.0 * r["seconds"] / max(r["steps"], 1), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": r["value"], "unit": "events/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_config(args, world):
    if args.workload == "config4":
        ls = args.layer_size
        return {"workload": "config4_layered", "layers": [ls] * 8, "fanout": 500, "synapses": 7 * ls * 500,
                "weights": "U[0,1] mV", "seed": args.seed,
                "inject": f"5% of layer 0 ({int(round(0.05 * ls))}) x 30 per step",
                "lif": "dt 1 ms, tau 20 ms, rest=reset -65 mV, thr -50 mV, refractory 2", "policy": "FULL",
                "propagation": PROPAGATION_LABEL[args.propagation],
                "parallelism": f"postsynaptic shards x{world}" + (f", {args.exchange} spike exchange" if world > 1 else ""),
                "l2": L2_NOTE}
    return {"workload": "config2_resident_random_pool", "neurons": args.neurons, "fanout": args.fanout,
            "synapses": args.neurons * args.fanout, "weights": "U[-0.2,0.5] mV", "seed": args.seed,
            "inject": f"{args.inject_frac * 100:g}% of neurons x {args.inject_value:g} per step",
            "lif": "dt 1 ms, tau 20 ms, rest=reset -65 mV, thr -50 mV, refractory 2", "policy": "FULL",
            "propagation": PROPAGATION_LABEL[args.propagation], "parallelism": f"postsynaptic shards x{world}" + (f", {args.exchange} spike exchange" if world > 1 else ""), "l2": L2_NOTE}


# ------------------------------------------------------------ GPU side ----
def main():
    args = parse()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.policy == "streaming" and args.stream_source == "generated":
        run_streaming_generated(args)
        return
    if args.policy == "streaming":
        run_streaming(args)
        return
    if args.workload == "config1":
        run_config1(args)
        return
    run_b200(args)


def config1_network(seed):
    """784-1000-10 dense, weights N(0, 1/sqrt(fan_in)) (numpy-seeded synthetic stand-in)."""
    import numpy as np
    layers = [784, 1000, 10]
    rng = np.random.default_rng(seed)
    n = sum(layers)
    rows, cols, ws = [np.zeros(1, np.uint64)], [], []
    off = np.cumsum([0] + layers)
    row_ptr = np.zeros(n + 1, np.uint64)
    for l in range(len(layers) - 1):
        pre, post = layers[l], layers[l + 1]
        w = (rng.standard_normal((pre, post)) / np.sqrt(pre)).astype(np.float32)
        cols.append(np.tile(np.arange(off[l + 1], off[l + 2], dtype=np.uint64), pre))
        ws.append(w.reshape(-1))
        row_ptr[off[l] + 1:off[l + 1] + 1] = np.uint64(post)
    row_ptr = np.cumsum(row_ptr).astype(np.uint64)
    return row_ptr, np.concatenate(cols), np.concatenate(ws), layers


def config1_frames(seed, first, count, n):
    """Static per-sample frames: 784 pixels U[0,1), each zeroed with p = 0.8."""
    import numpy as np
    out = np.zeros((count, n), np.float32)
    for k in range(count):
        rng = np.random.default_rng((seed, first + k))
        px = rng.random(784, dtype=np.float32)
        px[rng.random(784) < 0.8] = 0.0
        out[k, :784] = px
    return out


def run_config1(args):
    """BASELINE config 1 (784-1000-10 dense, 25 steps per static frame, state
    reset between samples) with --batch samples per context sharing one
    topology: per round, one upload of the batch's frames (held on the device),
    a reset, 25 steps. value = events / device time of the timed rounds
    (uploads included); samples/s alongside. ORDERED: bit-exact with the
    reference's serial CPU step sample by sample."""
    import numpy as np
    import torch

    import snn_b200 as sb

    row_ptr, col, w, layers = config1_network(args.seed)
    n, B, T = int(row_ptr.size - 1), args.batch, 25
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 20.0, 2)
    net = sb.Network.from_csr(row_ptr, col, w, lif)
    prop = sb.PROPAGATE_ORDERED if args.propagation == "ordered" else sb.PROPAGATE_PUSH
    ctx = sb.CudaContext.create(net, None, sb.default_options(device=0, timing=1, propagation=prop, batch=B))
    rounds = max(1, args.steps // T)
    warm_rounds = max(1, args.warmup // T)
    frames = [np.ascontiguousarray(config1_frames(args.seed, r * B, B, n).reshape(-1))
              for r in range(warm_rounds + rounds)]
    pinned = [torch.from_numpy(f).pin_memory().numpy() for f in frames]

    def round_(r):
        ctx.set_external(pinned[r])
        ctx.reset()
        for _ in range(T):
            ctx.step_async()

    for r in range(warm_rounds):
        round_(r)
    ctx.synchronize()
    ctx.reset_stats()
    stream = torch.cuda.ExternalStream(ctx.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with ClockSampler(0) as clk:
        ev0.record(stream)
        for r in range(rounds):
            round_(warm_rounds + r)
        ev1.record(stream)
        ctx.synchronize()
    wall = time.perf_counter() - t0
    ms = ev0.elapsed_time(ev1)
    s = ctx.stats()
    samples = rounds * B
    cpu = None
    if not args.no_cpu_baseline:
        try:
            cpu = config1_cpu(row_ptr, col, w, frames[warm_rounds], lif, seconds=min(args.cpu_seconds, 10.0))
        except Exception as exc:  # reported, never required
            cpu = {"value": None, "unavailable": repr(exc)}
    print(json.dumps({
        "metric": "synaptic_events_per_sec", "value": s["events"] / (ms / 1e3), "unit": "events/s", "n_gpus": 1,
        "steps": rounds * T, "warmup": warm_rounds * T, "ms_per_step": ms / (rounds * T), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: numpy-seeded 784-1000-10 gaussian weights and sparse U[0,1) frames",
        "config": {"workload": "config1_batched_samples", "layers": layers, "synapses": int(col.size),
                   "batch": B, "steps_per_sample": T, "propagation": "ordered" if prop == sb.PROPAGATE_ORDERED
                   else "push", "input_scale": 20.0, "l2": "topology (9.5 MB) L2-resident by design"},
        "samples_per_sec": samples / (ms / 1e3), "e2e": {"value": s["events"] / wall, "unit": "events/s",
                                                          "h2d_bytes_per_step": B * n * 4 // T,
                                                          "d2h_bytes_per_step": 0,
                                                          "samples_per_sec": samples / wall},
        "spike_rate": s["spikes"] / (rounds * T * B * n), "events_per_sample": s["events"] / samples,
        "gpu_launches": int(s["kernel_launches"]), "clocks": clk.summary(), "cpu_baseline": cpu,
    }), flush=True)
    ctx.free()


def config1_cpu(row_ptr, col, w, frames, lif, seconds):
    """The reference's serial CPU step (oracle/_ref, else the port) on the same
    network and frames, sample after sample, for a bounded time."""
    import numpy as np

    from oracle.oracle import LifParams, Oracle, State, ref_available
    kind = "ref" if ref_available("ref") else "port"
    orc = Oracle(kind)
    net = orc.custom_csr(row_ptr, col, w, lif=LifParams(lif.dt_ms, lif.membrane_tau_ms, lif.v_rest, lif.v_reset,
                                                        lif.v_threshold, lif.input_scale, lif.refractory_steps))
    n = int(row_ptr.size - 1)
    deg = (row_ptr[1:] - row_ptr[:-1]).astype(np.int64)
    st = State(net)
    events, done, elapsed = 0, 0, 0.0
    frames = frames.reshape(-1, n)
    while elapsed < seconds and done < frames.shape[0]:
        t0 = time.perf_counter()
        st.reset()
        for _ in range(25):
            sp = st.step(frames[done])
            events += int(deg[sp.astype(bool)].sum())
        elapsed += time.perf_counter() - t0
        done += 1
    return {"value": events / elapsed, "unit": "events/s", "cores": 1,
            "kind": "reference" if kind == "ref" else "port",
            "sample": f"{done} samples x 25 steps, serial build", "samples_per_sec": done / elapsed}


def run_streaming(args):
    """STREAMING policy (BASELINE config 3 scaled to host RAM): the CSR lives
    in host memory (page-locked in place by the library) and every step copies
    all of it in bounded chunks, double-buffered so the copy of chunk i+1
    overlaps the propagation of chunk i. Roofline: measured pinned H2D GB/s."""
    import numpy as np
    import torch

    import snn_b200 as sb

    n, f = args.stream_neurons, args.fanout
    e = n * f
    rng = np.random.default_rng(args.seed)
    row_ptr = np.arange(0, e + 1, f, dtype=np.uint64)
    col = rng.integers(0, n, size=e, dtype=np.uint64)
    w = (rng.random(e, dtype=np.float32) * np.float32(0.7) - np.float32(0.2)).astype(np.float32)
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 1.0, 2)
    net = sb.Network.from_csr(row_ptr, col, w, lif)
    csr_bytes = 12 * e + 8 * (n + 1)
    cfg = sb.default_config(prefer_streaming=1, max_vram_bytes=int(args.stream_budget_frac * csr_bytes))
    sparse = args.stream_mode == "sparse"
    ctx = sb.CudaContext.create(net, cfg, sb.default_options(
        device=0, timing=1, streaming=sb.STREAMING_SPARSE if sparse else sb.STREAMING_CHUNKED))
    assert ctx.mode == sb.MODE_STREAMING
    count = max(1, int(round(args.inject_frac * n)))
    # Host-link roofline: pinned host -> device copy of 1 GiB, best of 5.
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    best = 0.0
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        d.copy_(h, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        best = max(best, (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9)
    del h, d
    ctx.run_stream_async(args.seed, 0, args.warmup, count, args.inject_value)
    ctx.synchronize()
    ctx.reset_stats()
    stream = torch.cuda.ExternalStream(ctx.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(0) as clk:
        ev0.record(stream)
        ctx.run_stream_async(args.seed, args.warmup, args.steps, count, args.inject_value)
        ev1.record(stream)
        ctx.synchronize()
    ms = ev0.elapsed_time(ev1)
    s = ctx.stats()
    # Bytes that cross the host link: the whole CSR every step (chunked), or
    # the spiking rows' edges (12 B/event + 16 B/row, sparse).
    streamed = csr_bytes * args.steps if not sparse else 12 * s["events"] + 16 * s["spikes"]
    gbs = streamed / (ms / 1e3) / 1e9
    print(json.dumps({
        "metric": "synaptic_events_per_sec", "value": s["events"] / (ms / 1e3), "unit": "events/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: numpy-seeded uniform pool in host memory",
        "config": {"workload": "config3_streaming_scaled", "neurons": n, "fanout": f, "synapses": e,
                   "host_csr_bytes": csr_bytes, "vram_budget_bytes": int(args.stream_budget_frac * csr_bytes),
                   "policy": f"STREAMING ({args.stream_mode})", "layout": ctx.layout},
        "roofline": {"bound": "host_link", "achieved": gbs, "peak": best, "unit": "GB/s", "frac": gbs / best,
                     "peak_kind": "measured pinned H2D (1 GiB, best of 5)",
                     "algorithmic_bytes_per_step": streamed / args.steps},
        "spike_rate": s["spikes"] / (args.steps * n), "clocks": clk.summary(),
    }), flush=True)
    ctx.free()


def run_streaming_generated(args):
    """STREAMING at N GPUs (config 3's policy at the largest scale the host
    holds): a seeded pool of --stream-neurons x --fanout, sharded by
    postsynaptic neuron; every rank generates its own slice on its device,
    moves it to host memory and streams it every step over its own host link
    (chunked, or sparse reads of the spiking rows), with a VRAM budget of
    --stream-budget-frac of its slice. Reported per GPU against the host-link
    roofline (pinned H2D measured on each rank)."""
    import torch

    import snn_b200 as sb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    n, f = args.stream_neurons, args.fanout
    lo, cnt = sb.shard_range(n, world, rank)
    slice_bytes = 12 * n * f // world + 8 * (n + 1)
    budget = int(args.stream_budget_frac * slice_bytes)
    sparse = args.stream_mode == "sparse"
    opts = sb.default_options(device=local, world_size=world, rank=rank, timing=1,
                              exchange=sb.EXCHANGE_PEER if args.exchange == "peer" else sb.EXCHANGE_NCCL,
                              streaming=sb.STREAMING_SPARSE if sparse else sb.STREAMING_CHUNKED)
    id_buf = None
    if world > 1 and args.exchange == "nccl":
        import ctypes
        obj = [sb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        id_buf = ctypes.create_string_buffer(obj[0], 128)
        opts.nccl_id = ctypes.cast(id_buf, ctypes.c_void_p)
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 1.0, 2)
    t0 = time.time()
    ctx = sb.CudaContext.random_pool(n, f, -0.2, 0.5, args.seed, lif=lif,
                                     config=sb.default_config(prefer_streaming=1, max_vram_bytes=budget),
                                     options=opts)
    gen_s = time.time() - t0
    assert ctx.mode == sb.MODE_STREAMING
    if world > 1 and args.exchange == "peer":
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ipc_handle())
        ctx.ipc_connect(handles)
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    h2d = 0.0
    for _ in range(3):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        d.copy_(h, non_blocking=True)
        a1.record()
        torch.cuda.synchronize()
        h2d = max(h2d, (1 << 30) / (a0.elapsed_time(a1) / 1e3) / 1e9)
    del h, d
    count = max(1, int(round(args.inject_frac * n)))
    ctx.run_stream_async(args.seed, 0, args.warmup, count, args.inject_value)
    ctx.synchronize()
    ctx.reset_stats()
    stream = torch.cuda.ExternalStream(ctx.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        if dist is not None:
            z = torch.zeros(1, device="cuda")
            with torch.cuda.stream(stream):
                dist.all_reduce(z)
        e0.record(stream)
        ctx.run_stream_async(args.seed, args.warmup, args.steps, count, args.inject_value)
        e1.record(stream)
        ctx.synchronize()
        torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1)
    s = ctx.stats()
    lay = ctx.layout
    streamed = (12 * lay["local_synapses"] + 8 * (n + 1)) * args.steps if not sparse else \
        12 * s["events"] + 16 * s["spikes"]
    mine = {"rank": rank, "ms": ms_local, "host_link_gbs": streamed / (ms_local / 1e3) / 1e9, "h2d_peak_gbs": h2d,
            "events": s["events"], "local_synapses": lay["local_synapses"]}
    allr = [mine]
    if dist is not None:
        allr = [None] * world
        dist.all_gather_object(allr, mine)
    ctx.free()
    if rank == 0:
        ms = max(r["ms"] for r in allr)
        events = sum(r["events"] for r in allr)
        fr = [r["host_link_gbs"] / r["h2d_peak_gbs"] for r in allr]
        print(json.dumps({
            "metric": "synaptic_events_per_sec", "value": events / (ms / 1e3), "unit": "events/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded pool generated on each rank's device (bit-identical to snn_build_random_pool)",
            "config": {"workload": "config3_streaming_policy_scaled", "neurons": n, "fanout": f,
                       "synapses": n * f, "host_csr_bytes_total": 12 * n * f + 8 * (n + 1) * world,
                       "vram_budget_bytes_per_gpu": budget, "policy": f"STREAMING ({args.stream_mode})",
                       "parallelism": f"postsynaptic shards x{world}, {args.exchange} spike exchange"},
            "roofline": {"bound": "host_link", "per_gpu_gbs": [r["host_link_gbs"] for r in allr],
                         "per_gpu_peak_gbs": [r["h2d_peak_gbs"] for r in allr], "frac_min": min(fr),
                         "frac_mean": sum(fr) / len(fr), "aggregate_gbs": sum(r["host_link_gbs"] for r in allr)},
            "generate_s": gen_s, "clocks": clk.summary()}), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def run_b200(args):
    import numpy as np
    import torch

    import snn_b200 as sb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    nccl_id = None
    if world > 1 and args.exchange == "nccl":
        obj = [sb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]
    id_buf = None
    prop = {"auto": sb.PROPAGATE_PUSH, "binned": sb.PROPAGATE_PUSH_BINNED, "atomic": sb.PROPAGATE_PUSH_ATOMIC,
            "ordered": sb.PROPAGATE_ORDERED}
    opts = sb.default_options(device=local, world_size=world, rank=rank, timing=1,
                              propagation=prop[args.propagation],
                              exchange=sb.EXCHANGE_PEER if args.exchange == "peer" else sb.EXCHANGE_NCCL)
    if nccl_id is not None:
        import ctypes
        id_buf = ctypes.create_string_buffer(nccl_id, 128)
        opts.nccl_id = ctypes.cast(id_buf, ctypes.c_void_p)
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 1.0, 2)
    t0 = time.time()
    if args.workload == "config4":
        # 8 layers, fanout 500 to the next layer, w ~ U[0, 1]; the seeded
        # injection stream restricted to layer 0 (5% of it, 30.0 each).
        layers = [args.layer_size] * 8
        n, f = sum(layers), 500
        inj_range = args.layer_size
        count = max(1, int(round(0.05 * inj_range)))
        args.inject_value = 30.0
        ctx = sb.CudaContext.layered_random(layers, f, 0.0, 1.0, args.seed, lif=lif, options=opts)
        ctx.set_stream_range(inj_range)
    else:
        n, f = args.neurons, args.fanout
        inj_range = n
        count = max(1, int(round(args.inject_frac * n)))
        ctx = sb.CudaContext.random_pool(n, f, -0.2, 0.5, args.seed, lif=lif, options=opts)
    gen_s = time.time() - t0
    if world > 1 and args.exchange == "peer":
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ipc_handle())
        ctx.ipc_connect(handles)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    # Warm-up (untimed) then exactly K timed steps.
    ctx.run_stream_async(args.seed, 0, args.warmup, count, args.inject_value)
    ctx.synchronize()
    # The state at the start of the timed window, so that the e2e pass below
    # replays the same steps from the same state.
    v0, c0, r0 = ctx.download_state()
    ctx.reset_stats()
    stream = torch.cuda.ExternalStream(ctx.stream())
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rendezvous = torch.zeros(1, dtype=torch.float32, device="cuda") if dist is not None else None
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        if rendezvous is not None:
            # The ranks meet on the device right before the timed window (an
            # all-reduce on the library's stream), so that the host launch
            # skew between processes is not charged to the first exchange.
            with torch.cuda.stream(stream):
                dist.all_reduce(rendezvous)
        ev0.record(stream)
        ctx.run_stream_async(args.seed, args.warmup, args.steps, count, args.inject_value)
        ev1.record(stream)
        ctx.synchronize()
        torch.cuda.synchronize()
    barrier()
    ms_local = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms_local)
    s = ctx.stats()
    events_total = sum_over_ranks(float(s["events"]))
    spikes_total = sum_over_ranks(float(s["spikes"]))
    value = events_total / (ms / 1e3)
    # Roofline of the dominant kernels (propagation) on this rank: the
    # algorithmic bytes are 12 per event (8 B col_idx + 4 B weight, the
    # reference's CSR format) + 16 per spiking row (row_ptr pair). Push steps
    # and pull steps (device-chosen) are reported apart and blended.
    peak, peak_kind = measured_peak_gbs()
    timed = args.steps
    lay = ctx.layout
    # Every rank reads the row_ptr pair of every spiking row (the global list).
    spikes_rows = spikes_total
    prop_bytes = 12.0 * s["events"] + 16.0 * spikes_rows
    kernel_name = "propagate_push_kernel"
    if args.propagation == "ordered":
        kernel_name = "ordered propagation (event sort + in-order fold; pull on dense steps)"
    elif args.propagation == "binned":
        kernel_name = "ordered propagation (bin-fold; pull on dense steps)"
    gated = int(lay.get("ordered_csc", 0)) == 1 and args.propagation == "auto"
    if gated:
        kernel_name = "propagate_push_kernel (sparse steps) + propagate_pull_smem_kernel (dense steps)"
    prop_s = s["propagate_ms"] / 1e3
    achieved = prop_bytes / prop_s / 1e9 if prop_s > 0 else 0.0
    pull_steps = int(s.get("pull_steps", 0))
    pull_ms = s.get("propagate_pull_ms", 0.0)
    push_ms = s["propagate_ms"] - pull_ms
    push_events = s["events"] - s.get("pull_events", 0)
    push_spikes = spikes_rows - s.get("pull_spikes", 0)
    split = {"push_steps": timed - pull_steps, "pull_steps": pull_steps}
    if push_ms > 0:
        b = 12.0 * push_events + 16.0 * push_spikes
        split["push"] = {"achieved": b / (push_ms / 1e3) / 1e9, "frac": b / (push_ms / 1e3) / 1e9 / peak,
                         "ms_per_step": push_ms / max(1, timed - pull_steps),
                         "events_per_s": push_events / (push_ms / 1e3)}
    if pull_ms > 0:
        b = 12.0 * s.get("pull_events", 0) + 16.0 * s.get("pull_spikes", 0)
        slot_bytes = 8.0 * int(lay.get("pull_slots", 0)) * pull_steps
        split["pull"] = {"achieved": b / (pull_ms / 1e3) / 1e9, "frac": b / (pull_ms / 1e3) / 1e9 / peak,
                         "device_bytes_gbs": slot_bytes / (pull_ms / 1e3) / 1e9,
                         "device_frac": slot_bytes / (pull_ms / 1e3) / 1e9 / peak,
                         "ms_per_step": pull_ms / max(1, pull_steps)}
    traffic = None
    if args.propagation not in ("binned", "ordered") and int(lay["index_bits"]) == 32 and timed:
        # DRAM bytes from one ncu capture per kernel: the push kernel moves
        # 8.68 B per event (32-bit columns), the pull kernel 8 B per slot of
        # its layout; scaled by this run's events and pull steps.
        traffic = (NCU_DRAM_BYTES_PER_EVENT * push_events
                   + NCU_PULL_BYTES_PER_SLOT * int(lay.get("pull_slots", 0)) * pull_steps) / timed
    step_bytes = (prop_bytes + 25.0 * ctx.local_count * timed
                  + 12.0 * count * timed)
    launches = int(s["kernel_launches"])
    exchange = None
    if world > 1:
        waits = [max_over_ranks(s.get("exchange_wait_ms", 0.0) / timed),
                 max_over_ranks(s.get("exchange_wait_max_ms", 0.0))]
        exchange = {"kind": args.exchange, "ms_per_step": max_over_ranks(s["exchange_ms"] / timed),
                    "flag_wait_ms_per_step_max_rank": waits[0] if args.exchange == "peer" else None,
                    "longest_flag_wait_ms": waits[1] if args.exchange == "peer" else None,
                    "lif_with_peer_stores_ms_per_step": max_over_ranks(s["lif_ms"] / timed),
                    "propagate_ms_per_step_max_rank": max_over_ranks(s["propagate_ms"] / timed)}

    e2e = None
    if not args.no_e2e:
        # The same K steps as the device window: the state saved at its start
        # is restored, and the seeded stream's indices of those steps are fed
        # from pinned host memory through the reference-facing entry points.
        ctx.upload_state(v0, c0, r0)
        pinned_idx = torch.empty((args.steps, count), dtype=torch.int64).pin_memory()
        from_stream = _stream_indices(args.seed, args.warmup, args.steps, count, inj_range)
        pinned_idx.numpy()[:] = from_stream.view(np.int64)
        pinned_val = torch.full((count,), args.inject_value, dtype=torch.float32).pin_memory()
        spikes_out = torch.empty((ctx.local_count,), dtype=torch.uint8).pin_memory()
        idx_np, val_np, sp_np = pinned_idx.numpy().view(np.uint64), pinned_val.numpy(), spikes_out.numpy()
        ctx.reset_stats()
        barrier()
        t0 = time.perf_counter()
        for k in range(args.steps):
            st = ctx.inject_current(idx_np[k], val_np)
            if st != 0:
                raise sb.SnnError(st, "snn_cuda_inject_current")
            ctx.step(out=sp_np)
        e2e_s = time.perf_counter() - t0
        barrier()
        e2e_s = max_over_ranks(e2e_s)
        s2 = ctx.stats()
        e2e_events = sum_over_ranks(float(s2["events"]))
        e2e = {"value": e2e_events / e2e_s, "unit": "events/s", "h2d_bytes_per_step": count * 12,
               "d2h_bytes_per_step": int(ctx.local_count), "ms_per_step": 1e3 * e2e_s / args.steps,
               "events_per_step": e2e_events / args.steps, "device_events_per_step": events_total / args.steps,
               "window": f"steps {args.warmup}..{args.warmup + args.steps - 1} from the saved state",
               "api": "snn_cuda_inject_current + snn_cuda_step (host buffers, synchronous)"}
    local_count = ctx.local_count
    ctx.free()

    # The atomic push is bound by L2 reduction requests (one per event), not
    # by HBM bytes: measure that ceiling on this device (same target count)
    # and report the push steps against it.
    if "push" in split and args.propagation in ("auto", "atomic"):
        try:
            red = sb.probe_red_rate(local, targets=local_count, events=1 << 28, repeats=5)
            split["push"]["red_ceiling_per_s"] = red
            split["push"]["frac_of_red_ceiling"] = split["push"]["events_per_s"] / red
        except sb.SnnError as exc:  # reported, never required
            split["push"]["red_ceiling_per_s"] = repr(exc)

    parity = None
    if not args.no_parity:
        pid_buf = None
        if world > 1 and args.exchange == "nccl":
            import ctypes
            obj = [sb.nccl_unique_id() if rank == 0 else None]  # a fresh id: one per communicator
            dist.broadcast_object_list(obj, src=0)
            pid_buf = ctypes.create_string_buffer(obj[0], 128)
        parity = raster_check(args, world, rank, local, dist, opts_base=dict(
            device=local, world_size=world, rank=rank,
            exchange=sb.EXCHANGE_PEER if args.exchange == "peer" else sb.EXCHANGE_NCCL), nccl_id_buf=pid_buf)

    secondary = None
    if world == 1 and not args.no_secondary and args.workload == "config2":
        secondary = secondary_workloads(args, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "config4":
        cpu = {"value": None, "unavailable": "no CPU sample for config 4 (the CPU baseline is measured on config 2)"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_sample(args, seconds=args.cpu_seconds)
            cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
        except Exception as exc:  # the baseline is reported, never required
            cpu = {"value": None, "unavailable": repr(exc)}

    if rank == 0:
        line = {
            "metric": "synaptic_events_per_sec", "value": value, "unit": "events/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded random pool generated on device (bit-identical to snn_build_random_pool), "
                    "seeded injection stream",
            "config": workload_config(args, world),
            "index_bits": int(lay["index_bits"]),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": kernel_name,
                         "algorithmic_bytes_per_launch": prop_bytes / timed,
                         "kernel_ms_per_launch": s["propagate_ms"] / timed,
                         "by_step_kind": split},
            "step_roofline": {"achieved": step_bytes / (ms / 1e3) / 1e9 if world == 1 else None,
                              "frac": (step_bytes / (ms / 1e3) / 1e9) / peak if world == 1 else None,
                              "bytes_per_step": step_bytes / timed},
            "spike_rate": spikes_total / (args.steps * n), "events_per_step": events_total / args.steps,
            "kernel_ms": {"lif": s["lif_ms"] / args.steps, "exchange": s["exchange_ms"] / args.steps,
                          "propagate": s["propagate_ms"] / args.steps},
            "pull_steps": pull_steps, "exchange": exchange,
            "gpu_launches": launches, "generate_s": gen_s, "clocks": clk.summary(), "e2e": e2e,
            "cpu_baseline": cpu, "parity": parity, "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def timed_run(ctx, seed, first, steps, count, value, device=0):
    """Device time (CUDA events on the library's stream) of `steps` steps of
    the seeded injection stream through snn_b200_run_stream_async, with the
    SM clocks sampled meanwhile; stats cover exactly those steps."""
    import torch
    ctx.synchronize()
    ctx.reset_stats()
    stream = torch.cuda.ExternalStream(ctx.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with ClockSampler(device) as clk:
        e0.record(stream)
        ctx.run_stream_async(seed, first, steps, count, value)
        e1.record(stream)
        ctx.synchronize()
    return e0.elapsed_time(e1), ctx.stats(), clk.summary()


def secondary_workloads(args, local):
    """The other workloads, measured in the same N=1 run (each bounded to a
    few seconds of device time): config 0 through graph replay, ORDERED
    config 2, config 4, and the STREAMING policy (chunked and sparse) on a
    host-resident pool, each with its own roofline and clock record."""
    import numpy as np
    import torch

    import snn_b200 as sb

    peak, peak_kind = measured_peak_gbs()
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 1.0, 2)
    out = {}

    def roof(bytes_, ms):
        a = bytes_ / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": a, "peak": peak, "unit": "GB/s", "frac": a / peak,
                "peak_kind": peak_kind, "algorithmic_bytes_per_step": bytes_}

    def record(name, fn):
        t0 = time.time()
        try:
            out[name] = fn()
        except Exception as exc:  # a secondary workload never fails the bench
            out[name] = {"unavailable": repr(exc)}
        out[name]["wall_s"] = round(time.time() - t0, 1)

    # Config 0: 100k x fanout 100, w ~ U[0, 0.6], 1% injection of 20.0 per
    # step, 1,000 steps; launch-bound, so timed through the graph-replayed
    # multi-step run (device timing off). PUSH, and the bit-exact bin-fold.
    def config0(prop):
        n, f, steps, count = 100_000, 100, 1000, 1000
        ctx = sb.CudaContext.random_pool(n, f, 0.0, 0.6, 0, lif=lif,
                                         options=sb.default_options(device=local, propagation=prop))
        ctx.run_stream_async(0, 0, 20, count, 20.0)
        ms, s, clk = timed_run(ctx, 0, 20, steps, count, 20.0, local)
        ctx.free()
        b = 12.0 * s["events"] + 16.0 * s["spikes"] + (25.0 * n + 12.0 * count) * steps
        return {"workload": "config0: 100k x 100, 1% x 20.0 per step, graph replay", "value": s["events"] / (ms / 1e3),
                "unit": "events/s", "us_per_step": 1e3 * ms / steps, "steps": steps,
                "gpu_launches": int(s["kernel_launches"]), "spike_rate": s["spikes"] / (steps * n),
                "roofline": roof(b / steps, ms / steps), "clocks": clk}
    record("config0_push_graph", lambda: config0(sb.PROPAGATE_PUSH))
    record("config0_ordered_binfold_graph", lambda: config0(sb.PROPAGATE_PUSH_BINNED))

    # ORDERED (bit-exact) on the headline workload: the same 10M x 1000 pool
    # and window as the main line.
    def config2_ordered():
        n, f = args.neurons, args.fanout
        count = max(1, int(round(args.inject_frac * n)))
        ctx = sb.CudaContext.random_pool(n, f, -0.2, 0.5, args.seed, lif=lif, options=sb.default_options(
            device=local, timing=1, propagation=sb.PROPAGATE_ORDERED))
        ctx.run_stream_async(args.seed, 0, args.warmup, count, args.inject_value)
        ms, s, clk = timed_run(ctx, args.seed, args.warmup, args.steps, count, args.inject_value, local)
        ctx.free()
        b = 12.0 * s["events"] + 16.0 * s["spikes"]
        return {"workload": "config2 ORDERED (event sort + in-order fold; pull on dense steps), same window",
                "value": s["events"] / (ms / 1e3), "unit": "events/s", "ms_per_step": ms / args.steps,
                "steps": args.steps, "pull_steps": int(s["pull_steps"]), "gpu_launches": int(s["kernel_launches"]),
                "roofline": roof(b / args.steps, s["propagate_ms"] / args.steps), "clocks": clk}
    record("config2_ordered", config2_ordered)

    # Config 4: 8 layers x 1M, fanout 500 to the next layer, w ~ U[0, 1], 5%
    # of layer 0 injected with 30.0 per step.
    def config4():
        ls, f = args.layer_size, 500
        layers = [ls] * 8
        count = max(1, int(round(0.05 * ls)))
        ctx = sb.CudaContext.layered_random(layers, f, 0.0, 1.0, args.seed, lif=lif,
                                            options=sb.default_options(device=local, timing=1))
        ctx.set_stream_range(ls)
        ctx.run_stream_async(args.seed, 0, args.warmup, count, 30.0)
        ms, s, clk = timed_run(ctx, args.seed, args.warmup, args.steps, count, 30.0, local)
        ctx.free()
        b = 12.0 * s["events"] + 16.0 * s["spikes"]
        return {"workload": "config4: 8 x 1M layers, fanout 500, 5% of layer 0 x 30.0", "value": s["events"] / (ms / 1e3),
                "unit": "events/s", "ms_per_step": ms / args.steps, "steps": args.steps,
                "spike_rate": s["spikes"] / (args.steps * 8 * ls), "pull_steps": int(s["pull_steps"]),
                "gpu_launches": int(s["kernel_launches"]),
                "roofline": roof(b / args.steps, s["propagate_ms"] / args.steps), "clocks": clk}
    record("config4", config4)

    # STREAMING (config 3's policy, scaled to a host pool of 1M x 1000, 12 GB
    # of CSR in host memory, VRAM budget a quarter of it): chunked streams
    # the whole CSR every step, sparse reads only the spiking rows.
    n, f = args.stream_neurons, args.fanout
    e = n * f
    rng = np.random.default_rng(args.seed)
    row_ptr = np.arange(0, e + 1, f, dtype=np.uint64)
    col = rng.integers(0, n, size=e, dtype=np.uint64)
    w = (rng.random(e, dtype=np.float32) * np.float32(0.7) - np.float32(0.2)).astype(np.float32)
    net = sb.Network.from_csr(row_ptr, col, w, lif)
    csr_bytes = 12 * e + 8 * (n + 1)
    h = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    d = torch.empty(1 << 30, dtype=torch.uint8, device="cuda")
    h2d = 0.0
    for _ in range(5):
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        d.copy_(h, non_blocking=True)
        a1.record()
        torch.cuda.synchronize()
        h2d = max(h2d, (1 << 30) / (a0.elapsed_time(a1) / 1e3) / 1e9)
    del h, d

    def streaming(mode, steps):
        count = max(1, int(round(args.inject_frac * n)))
        cfg = sb.default_config(prefer_streaming=1, max_vram_bytes=int(0.25 * csr_bytes))
        ctx = sb.CudaContext.create(net, cfg, sb.default_options(
            device=local, timing=1, streaming=sb.STREAMING_SPARSE if mode == "sparse" else sb.STREAMING_CHUNKED))
        ctx.run_stream_async(args.seed, 0, 3, count, args.inject_value)
        ms, s, clk = timed_run(ctx, args.seed, 3, steps, count, args.inject_value, local)
        ctx.free()
        streamed = csr_bytes * steps if mode == "chunked" else 12 * s["events"] + 16 * s["spikes"]
        gbs = streamed / (ms / 1e3) / 1e9
        return {"workload": f"STREAMING {mode}: host pool {n} x {f} ({csr_bytes / 1e9:.1f} GB CSR), VRAM budget 25%",
                "value": s["events"] / (ms / 1e3), "unit": "events/s", "ms_per_step": ms / steps, "steps": steps,
                "roofline": {"bound": "host_link", "achieved": gbs, "peak": h2d, "unit": "GB/s", "frac": gbs / h2d,
                             "peak_kind": "measured pinned H2D (1 GiB, best of 5)"},
                "clocks": clk}
    record("streaming_chunked", lambda: streaming("chunked", 4))
    record("streaming_sparse", lambda: streaming("sparse", 20))
    net.free()
    return out


def raster_check(args, world, rank, local, dist, opts_base, nccl_id_buf):
    """Bit-exactness check printed with every bench line: ORDERED propagation
    on a seeded pool of --parity-neurons neurons (fanout and weights as the
    timed workload), sharded over the same ranks, for --parity-steps steps of
    the same injection stream. Rank 0 hashes the whole spike raster (SHA-256
    over the per-step spike vectors); the hash is the same at every GPU count
    and equals the reference's serial CPU step's (computed here when the
    reference library is present)."""
    import hashlib

    import numpy as np
    import torch

    import snn_b200 as sb

    n, steps = args.parity_neurons, args.parity_steps
    count = max(1, int(round(args.inject_frac * n)))
    lif = sb.LifParams(1.0, 20.0, -65.0, -65.0, -50.0, 1.0, 2)
    opts = sb.default_options(propagation=sb.PROPAGATE_ORDERED, **opts_base)
    if nccl_id_buf is not None:
        import ctypes
        opts.nccl_id = ctypes.cast(nccl_id_buf, ctypes.c_void_p)
    ctx = sb.CudaContext.random_pool(n, args.fanout, -0.2, 0.5, args.seed + 1, lif=lif, options=opts)
    if world > 1 and args.exchange == "peer":
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ipc_handle())
        ctx.ipc_connect(handles)
    slot = max(sb.shard_range(n, world, r)[1] for r in range(world))
    sha = hashlib.sha256()
    spikes = 0
    buf = np.zeros(ctx.local_count, np.uint8)
    for t in range(steps):
        idx = _stream_indices(args.seed, t, 1, count, n)[0]
        ctx.inject_current(idx, np.full(count, args.inject_value, np.float32))
        ctx.step(out=buf)
        if world > 1:
            mine = torch.zeros(slot, dtype=torch.uint8, device="cuda")
            mine[:ctx.local_count] = torch.from_numpy(buf).cuda()
            parts = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(parts, mine)
            full = np.concatenate([parts[r].cpu().numpy()[:sb.shard_range(n, world, r)[1]] for r in range(world)])
        else:
            full = buf
        if rank == 0:
            sha.update(full.tobytes())
            spikes += int(full.sum())
    ctx.free()
    if rank != 0:
        return None
    out = {"check": "ORDERED spike raster, SHA-256 over all steps", "neurons": n, "fanout": args.fanout,
           "steps": steps, "seed": args.seed + 1, "raster_sha256": sha.hexdigest(), "spikes": spikes}
    ref = reference_raster_sha(args, n, steps, count)
    if ref is not None:
        out["reference_raster_sha256"] = ref
        out["match"] = ref == out["raster_sha256"]
    return out


def reference_raster_sha(args, n, steps, count):
    """The reference's serial CPU step (oracle/_ref, CSR-order scatter) on the
    same network and inputs: the SHA-256 of its raster, or None when the
    reference library is absent."""
    import hashlib

    import numpy as np

    from oracle.oracle import Oracle, State, baseline_lif, ref_available
    if not ref_available("ref"):
        return None
    net = Oracle("port").random_pool_parallel(n, args.fanout, -0.2, 0.5, args.seed + 1, lif=baseline_lif())
    st = State(net, lib=Oracle("ref"))
    sha = hashlib.sha256()
    val = np.full(count, args.inject_value, np.float32)
    for t in range(steps):
        st.inject(_stream_indices(args.seed, t, 1, count, n)[0], val)
        sha.update(st.step().tobytes())
    return sha.hexdigest()


def _stream_indices(seed, first_step, steps, count, n):
    """Host copy of the seeded injection stream (same formula as
    snn_b200_inject_stream_async) for the host-buffer e2e run."""
    import numpy as np
    g = np.uint64(0x9E3779B97F4A7C15)
    with np.errstate(over="ignore"):
        d = np.arange(first_step * count + 1, (first_step + steps) * count + 1, dtype=np.uint64)
        z = np.uint64(seed) + d * g
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return (z % np.uint64(n)).reshape(steps, count)


if __name__ == "__main__":
    main()
