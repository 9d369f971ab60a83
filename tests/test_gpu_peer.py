"""GPU tests of the peer-memory exchanges (mgpu_peer_group_*, peer.cu) that the N-GPU decode
step uses in place of collective-library calls: the all-gather of the hidden states and the
all-to-all of the greedy (index, value) pairs."""
import multiprocessing as mp
import os

import numpy as np
import pytest

import mvlm_b200 as mg

pytestmark = pytest.mark.gpu


def test_single_gpu_group_exchanges_and_graph_replay(dev):
    # world = 1: the exchange stores into this GPU's own slot and waits for its own flag; run
    # eagerly and from a captured graph, with the source changing between replays
    K = 2048
    g = mg.PeerGroup(dev, 0, 1, K * 2)
    g.connect_ptrs([g.local_ptr()])
    src = dev.empty(K, mg.BF16)
    slots = g.slots(mg.BF16)
    for it in range(3):
        data = (np.arange(K, dtype=np.uint16) * 7 + it).astype(np.uint16)
        src.write(data)
        g.allgather(src, K * 2).wait()
        assert np.array_equal(slots.read(np.uint16)[:K], data)
    pairs = dev.empty(2, mg.F32)
    gp = mg.PeerGroup(dev, 0, 1, 8)
    gp.connect_ptrs([gp.local_ptr()])
    pslots = gp.slots(mg.F32)
    dev.capture_begin()
    g.allgather(src, K * 2)
    gp.alltoall(pairs, 8)
    graph = dev.capture_end()
    for it in range(4):
        data = (np.arange(K, dtype=np.uint16) * 3 + 11 * it).astype(np.uint16)
        src.write(data)
        pairs.write(np.array([it, 1000 + it], np.int32))
        graph.launch()
        dev.finish()
        assert np.array_equal(slots.read(np.uint16)[:K], data)
        assert np.array_equal(pslots.read(np.int32)[:2], [it, 1000 + it])
    del graph
    g.destroy()
    gp.destroy()


def test_wait_for_a_flag_nothing_sets_times_out(dev):
    # two groups of one device connected to each other, but only rank 0's exchange runs: its
    # stores land in rank 1's slot, and its wait for rank 1's flag (which nothing sets) gives up
    # after the limit with MGPU_ERR_DEVICE_TIMEOUT instead of hanging; the device stays usable
    n = 64
    a = mg.PeerGroup(dev, 0, 2, n)
    b = mg.PeerGroup(dev, 1, 2, n)
    a.connect_ptrs([a.local_ptr(), b.local_ptr()])
    b.connect_ptrs([a.local_ptr(), b.local_ptr()])
    a.set_wait_limit(20_000_000)  # 20 ms
    src = dev.array(np.arange(n // 4, dtype=np.int32), mg.F32)
    a.allgather(src, n)
    with pytest.raises(mg.MgpuError) as e:
        dev.finish()
    assert e.value.code == mg.ERR_DEVICE_TIMEOUT
    assert np.array_equal(b.slots(mg.F32).read(np.int32)[: n // 4], np.arange(n // 4))
    y = dev.empty(4, mg.F32)
    y.write(np.ones(4, np.float32))
    dev.finish()
    assert np.array_equal(y.read(np.float32), np.ones(4, np.float32))
    a.destroy()
    b.destroy()


def _two_gpu_rank(rank, world, port, q):
    try:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        dev = mg.Device(rank)
        K = 2048
        g = mg.PeerGroup(dev, rank, world, K * 2)
        gp = mg.PeerGroup(dev, rank, world, 8)
        for grp in (g, gp):
            handles = [None] * world
            dist.all_gather_object(handles, grp.handle())
            grp.connect(handles)
        src = dev.empty(K, mg.BF16)
        pairs = dev.empty(2 * world, mg.F32)
        slots, pslots = g.slots(mg.BF16), gp.slots(mg.F32)

        def enqueue():
            g.allgather(src, K * 2)
            gp.alltoall(pairs, 8)

        ok = True
        dev.capture_begin()
        enqueue()
        graph = dev.capture_end()
        for it in range(5):
            src.write((np.arange(K) * (rank + 1) + it).astype(np.uint16))
            # pair for sequence s from this rank: (rank * 100 + s, it)
            pairs.write(np.array([[rank * 100 + s, it] for s in range(world)], np.int32).reshape(-1))
            dist.barrier()
            if it < 2:
                enqueue()  # eager
            else:
                graph.launch()
            dev.finish()
            got = slots.read(np.uint16).reshape(world, K)
            for r in range(world):
                ok &= np.array_equal(got[r], (np.arange(K) * (r + 1) + it).astype(np.uint16))
            gotp = pslots.read(np.int32).reshape(world, 2)
            for r in range(world):
                ok &= gotp[r, 0] == r * 100 + rank and gotp[r, 1] == it
            dist.barrier()
        del graph
        g.destroy()
        gp.destroy()
        dist.destroy_process_group()
        q.put((rank, bool(ok), ""))
    except Exception as ex:  # reported to the parent
        q.put((rank, False, repr(ex)))


def test_two_gpu_allgather_and_alltoall():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, 29611 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_two_gpu_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in results), results
