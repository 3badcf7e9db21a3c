"""World-size-2 gloo test (CPU) of the sharded step's decomposition.

Each rank takes its postsynaptic range from the library's own geometry
(snn_b200_shard_range), keeps the edges that target it in global CSR order,
runs the LIF update on its neurons, all-gathers the packed spike bitmap over
gloo, and folds its targets' inputs in CSR order -- the host-side algorithm
the GPU ranks run with NCCL. Rank 0 checks that the concatenated rasters and
voltages equal the single-process oracle bit for bit, so partition, slicing,
bitmap packing and all-gather layout are validated without a GPU.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import snn_b200 as sb
from oracle.oracle import Oracle, State, baseline_lif, stream_indices_np


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lif(v, cur, ext, refr, p, decay):
    v_int = (np.float32(p.v_rest) + (v - np.float32(p.v_rest)) * np.float32(decay)) + cur + ext
    active = refr == 0
    fired = active & (v_int >= np.float32(p.v_threshold))
    v_new = np.where(active & ~fired, v_int, np.float32(p.v_reset)).astype(np.float32)
    r_new = np.where(fired, p.refractory_steps, refr - (refr != 0)).astype(np.uint32)
    return v_new, r_new, fired


def _worker(rank, world, port, n, steps, count, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    orc = Oracle("port")
    lif = baseline_lif()
    net = orc.random_pool(n, 60, -0.2, 0.5, 3, lif=lif)
    lo, cnt = sb.shard_range(n, world, rank)
    slot_words = -(-(-(-n // world)) // 128) * 4  # ceil(ceil(n/world)/128) * 4 words
    rp, ci, w = net.row_ptr(), net.col_idx(), net.weights()
    rows = np.repeat(np.arange(n, dtype=np.int64), np.diff(rp).astype(np.int64))
    keep = (ci >= lo) & (ci < lo + cnt)
    l_rows, l_tgt, l_w = rows[keep], (ci[keep] - lo).astype(np.int64), w[keep]  # CSR order kept
    v = np.full(cnt, lif.v_rest, np.float32)
    cur = np.zeros(cnt, np.float32)
    refr = np.zeros(cnt, np.uint32)
    rasters = []
    for t in range(steps):
        idx = stream_indices_np(4, t, count, n).astype(np.int64)
        mine = idx[(idx >= lo) & (idx < lo + cnt)] - lo
        np.add.at(cur, mine, np.float32(20.0))  # uniform values: order-free
        v, refr, fired = _lif(v, cur, np.float32(0.0), refr, lif, net.decay)
        rasters.append(fired.astype(np.uint8))
        bits = np.zeros(slot_words * 32, np.uint8)
        bits[:cnt] = fired
        words = torch.from_numpy(np.packbits(bits, bitorder="little").view(np.int32).copy())
        gathered = [torch.zeros_like(words) for _ in range(world)]
        dist.all_gather(gathered, words)
        glob = np.unpackbits(torch.cat(gathered).numpy().view(np.uint8), bitorder="little")[:n].astype(bool)
        nxt = np.zeros(cnt, np.float32)
        act = glob[l_rows]
        np.add.at(nxt, l_tgt[act], l_w[act])  # sequential fold in CSR order
        cur = nxt
    parts = [None] * world
    dist.all_gather_object(parts, (lo, np.array(rasters), v))
    if rank == 0:
        parts.sort(key=lambda p: p[0])
        st = State(net)
        _, _, _, ras = orc.run_inject_stream(net, st, 4, 0, steps, count, 20.0, raster=True)
        g_r = np.concatenate([p[1] for p in parts], axis=1)
        g_v = np.concatenate([p[2] for p in parts])
        out.put((np.array_equal(g_r, ras), np.array_equal(g_v.view(np.uint32), st.voltage().view(np.uint32)),
                 int(ras.sum())))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_sharded_decomposition_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 4099, 25, 60, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    raster_ok, volt_ok, spikes = res
    assert spikes > 100
    assert raster_ok and volt_ok


def test_shard_geometry_tiles_the_network():
    for n in (1, 31, 32, 33, 1000, 10_000_000):
        for world in (1, 2, 3, 4, 8):
            ranges = [sb.shard_range(n, world, r) for r in range(world)]
            pos = 0
            for b, c in ranges:
                assert b == pos or c == 0
                pos = max(pos, b + c)
                assert b % 128 == 0 or c == 0
            assert pos == n
            assert sum(c for _, c in ranges) == n
    with pytest.raises(sb.SnnError):
        sb.shard_range(10, 2, 2)
