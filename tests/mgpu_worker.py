"""Worker for the sharded (multi-GPU) parity test, one process per GPU under
torch.distributed.run. Every rank builds the same seeded network with the CPU
oracle, creates a postsynaptic shard of it on its own GPU (NCCL spike
all-gather inside the library), steps it with the seeded injection stream,
and rank 0 compares the concatenated spike slices and voltages with the
oracle's single-process run. Exit code 0 = parity holds.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        --master-port 29511 tests/mgpu_worker.py
"""
import ctypes
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import snn_b200 as sb  # noqa: E402
from oracle.oracle import Oracle, State, baseline_lif, default_lif, stream_indices_np  # noqa: E402
from tests._helpers import lif_to_sb  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    keep = []

    def options(prop, exchange=sb.EXCHANGE_NCCL, streaming=sb.STREAMING_CHUNKED):
        o = sb.default_options(device=local, rank=rank, world_size=world, propagation=prop, exchange=exchange,
                               streaming=streaming)
        if exchange == sb.EXCHANGE_NCCL:
            # A fresh NCCL unique id per context (one communicator each).
            obj = [sb.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            idbuf = ctypes.create_string_buffer(obj[0], 128)
            keep.append(idbuf)
            o.nccl_id = ctypes.cast(idbuf, ctypes.c_void_p)
        return o

    def connect(ctx, exchange):
        # Peer exchange: gather every rank's IPC handle, map the peers.
        if exchange == sb.EXCHANGE_PEER:
            handles = [None] * world
            dist.all_gather_object(handles, ctx.ipc_handle())
            ctx.ipc_connect(handles)

    orc = Oracle("port")
    failures = []
    n, steps, count = 30011, 40, 300
    lif = baseline_lif()
    net = orc.random_pool(n, 120, -0.2, 0.5, 5, lif=lif)
    for prop, exchange in ((sb.PROPAGATE_ORDERED, sb.EXCHANGE_NCCL), (sb.PROPAGATE_PUSH, sb.EXCHANGE_NCCL),
                           (sb.PROPAGATE_ORDERED, sb.EXCHANGE_PEER), (sb.PROPAGATE_PUSH, sb.EXCHANGE_PEER)):
        ctx = sb.CudaContext.create(net, None, options(prop, exchange))
        connect(ctx, exchange)
        lo, cnt = ctx.local_begin, ctx.local_count
        raster = np.zeros((steps, cnt), np.uint8)
        for t in range(steps):
            idx = stream_indices_np(9, t, count, n)
            assert ctx.inject_current(idx, np.full(count, 20.0, np.float32)) == 0
            raster[t] = ctx.step()
        v = ctx.download_voltage()
        stats = ctx.stats()
        parts = [None] * world
        dist.all_gather_object(parts, (lo, raster, v, stats["events"], stats["spikes"]))
        if rank == 0:
            st = State(net)
            sc, ev, hs, ras = orc.run_inject_stream(net, st, 9, 0, steps, count, 20.0, raster=True)
            parts.sort(key=lambda p: p[0])
            g_r = np.concatenate([p[1] for p in parts], axis=1)
            g_v = np.concatenate([p[2] for p in parts])
            exact = prop == sb.PROPAGATE_ORDERED
            if exact:
                if not np.array_equal(g_r, ras):
                    failures.append(f"ordered/{exchange} raster mismatch at step "
                                    f"{np.nonzero((g_r != ras).any(1))[0][:3]}")
                if not np.array_equal(g_v.view(np.uint32), st.voltage().view(np.uint32)):
                    failures.append(f"ordered/{exchange} voltage mismatch")
                if sum(p[3] for p in parts) != int(ev.sum()) or sum(p[4] for p in parts) != int(sc.sum()):
                    failures.append(f"ordered/{exchange} stats mismatch")
            else:
                if not np.array_equal(g_r[0], ras[0]):
                    failures.append(f"push/{exchange} first-step raster mismatch")
        ctx.free()
    # Async multi-step run on the peer exchange equals the NCCL one (ordered: exact).
    finals = []
    for exchange in (sb.EXCHANGE_NCCL, sb.EXCHANGE_PEER):
        ctx = sb.CudaContext.create(net, None, options(sb.PROPAGATE_ORDERED, exchange))
        connect(ctx, exchange)
        ctx.run_stream_async(9, 0, 30, count, 20.0)
        ctx.synchronize()
        finals.append((ctx.download_voltage(), ctx.stats()["spikes"]))
        ctx.free()
    # Device-generated ORDERED shard (CSC built on the device), peer exchange.
    ctx = sb.CudaContext.random_pool(n, 120, -0.2, 0.5, 5, lif=lif_to_sb(lif),
                                     options=options(sb.PROPAGATE_ORDERED, sb.EXCHANGE_PEER))
    connect(ctx, sb.EXCHANGE_PEER)
    ctx.run_stream_async(9, 0, 30, count, 20.0)
    ctx.synchronize()
    finals.append((ctx.download_voltage(), ctx.stats()["spikes"]))
    ctx.free()
    for i, what in ((1, "async peer run differs from NCCL run"), (2, "generated ordered shard differs")):
        if not (np.array_equal(finals[0][0].view(np.uint32), finals[i][0].view(np.uint32)) and
                finals[0][1] == finals[i][1]):
            failures.append(f"rank {rank}: {what}")
    # Device-generated shards tile the host network exactly.
    ctx = sb.CudaContext.random_pool(n, 120, -0.2, 0.5, 5, lif=None, options=options(sb.PROPAGATE_PUSH))
    rp, ci, w = ctx.download_topology()
    parts = [None] * world
    dist.all_gather_object(parts, (ctx.local_begin, ctx.local_count, rp, ci, w))
    if rank == 0:
        hrp, hci, hw = net.row_ptr(), net.col_idx(), net.weights()
        for lo, cnt, rp, ci, w in parts:
            mask = (hci >= lo) & (hci < lo + cnt)
            deg = np.add.reduceat(mask.astype(np.int64), hrp[:-1].astype(np.int64)) if hci.size else None
            exp_rp = np.concatenate([[0], np.cumsum(deg)]).astype(np.uint64)
            if not (np.array_equal(rp, exp_rp) and np.array_equal(ci, hci[mask]) and
                    np.array_equal(w.view(np.uint32), hw[mask].view(np.uint32))):
                failures.append(f"device shard {lo} topology mismatch")
    ctx.free()
    # Dense steps on sharded contexts: the gated pull (PUSH, one dyadic weight so
    # every sum is exact) and the ORDERED pull, over 3-chunk layouts, against
    # the CPU step. Frames alternate between sparse and dense drive.
    os.environ["SNN_B200_PUSH_PULL_MIN_SYNAPSES"] = "0"
    os.environ["SNN_B200_PULL_CHUNK_WORDS"] = "64"
    dlif = default_lif(v_rest=0.0, v_reset=0.0, v_threshold=1.0, input_scale=1.0, refractory_steps=1)
    dn = 6001
    for prop, wlo, whi in ((sb.PROPAGATE_PUSH, 0.0009765625, 0.0009765625), (sb.PROPAGATE_ORDERED, -0.0005, 0.002)):
        dnet = orc.random_pool(dn, 600, wlo, whi, 21, lif=dlif)
        ctx = sb.CudaContext.create(dnet, None, options(prop, sb.EXCHANGE_PEER))
        connect(ctx, sb.EXCHANGE_PEER)
        if ctx.layout["ordered_csc"] != 1:
            failures.append(f"rank {rank}: no pull topology for {prop}")
        lo, cnt = ctx.local_begin, ctx.local_count
        rng = np.random.default_rng(8)
        frames = [(rng.random(dn) < (0.6 if t % 3 == 0 else 0.02)).astype(np.float32) * np.float32(1.5)
                  for t in range(9)]
        raster = np.zeros((9, cnt), np.uint8)
        for t in range(9):
            raster[t] = ctx.step(frames[t][lo:lo + cnt])
        parts = [None] * world
        dist.all_gather_object(parts, (lo, raster, ctx.download_voltage()))
        if rank == 0:
            st = State(dnet)
            ras = np.array([st.step(frames[t]) for t in range(9)])
            parts.sort(key=lambda p: p[0])
            g_r = np.concatenate([p[1] for p in parts], axis=1)
            g_v = np.concatenate([p[2] for p in parts])
            if not (np.array_equal(g_r, ras) and np.array_equal(g_v.view(np.uint32), st.voltage().view(np.uint32))):
                failures.append(f"dense sharded {prop} differs from the CPU step")
            if not (0 < int((ras.sum(axis=1) > dn // 4).sum()) < 9):
                failures.append("dense sharded case lacks a mix of sparse and dense steps")
        ctx.free()
    # Sharded STREAMING: each rank streams only the edges into its neurons
    # (chunked copies, or sparse reads of its mapped slice). One dyadic
    # weight: exact against the CPU step.
    snet = orc.random_pool(20011, 48, 0.046875, 0.046875, 4242, lif=default_lif(refractory_steps=2))
    for smode, exchange in ((sb.STREAMING_CHUNKED, sb.EXCHANGE_PEER), (sb.STREAMING_SPARSE, sb.EXCHANGE_NCCL)):
        cfg = sb.default_config(prefer_streaming=1, max_stream_rows=700)
        ctx = sb.CudaContext.create(snet, cfg, options(sb.PROPAGATE_PUSH, exchange, smode))
        connect(ctx, exchange)
        if ctx.mode != sb.MODE_STREAMING:
            failures.append(f"rank {rank}: sharded context is not STREAMING")
        lo, cnt = ctx.local_begin, ctx.local_count
        rng = np.random.default_rng(11)
        frames = [(rng.random(20011) < 0.08).astype(np.float32) * np.float32(1.5) for _ in range(8)]
        raster = np.zeros((8, cnt), np.uint8)
        for t in range(8):
            raster[t] = ctx.step(frames[t][lo:lo + cnt])
        stats = ctx.stats()
        parts = [None] * world
        dist.all_gather_object(parts, (lo, raster, ctx.download_voltage(), stats["events"], stats["spikes"]))
        if rank == 0:
            st = State(snet)
            ras = np.array([st.step(frames[t]) for t in range(8)])
            parts.sort(key=lambda p: p[0])
            g_r = np.concatenate([p[1] for p in parts], axis=1)
            g_v = np.concatenate([p[2] for p in parts])
            if not (np.array_equal(g_r, ras) and np.array_equal(g_v.view(np.uint32), st.voltage().view(np.uint32))):
                failures.append(f"sharded streaming {smode} differs from the CPU step")
            if sum(p[3] for p in parts) != int(ras.sum()) * 48 or sum(p[4] for p in parts) != int(ras.sum()):
                failures.append(f"sharded streaming {smode} stats differ")
        ctx.free()
    dist.barrier()
    if rank == 0:
        print("FAILURES:" if failures else "MGPU PARITY OK", failures)
    dist.destroy_process_group()
    sys.exit(1 if failures else 0)


if __name__ == "__main__":
    main()
