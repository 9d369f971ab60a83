"""Multi-rank host logic of the sharded paths, on CPU with gloo (world size 2 and 3):
column-sharding of a quantised lm_head (each rank takes a contiguous byte range of the packed
GGUF rows), the all-gather of logits, and batch sharding.  The per-rank products come from the
CPU oracle; on the GPU ranks the same ranges feed mgpu_gemv_q (bench.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mvlm_b200.shard import batch_shard, column_shard, gather_columns, shard_sizes, weight_row_bytes_range


def test_partitions_cover_exactly_once():
    for n in (1, 7, 64, 51200, 8192, 51201):
        for world in (1, 2, 3, 4, 8):
            spans = [column_shard(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = shard_sizes(n, world)
            assert max(sizes) - min(sizes) <= 1 and sum(sizes) == n
    assert batch_shard(64, 8, 3) == (24, 32)
    assert weight_row_bytes_range(51200, 1152, 8, 1) == (6400 * 1152, 12800 * 1152)
    with pytest.raises(ValueError):
        column_shard(10, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle as O
        K, N = 256, 101  # N not divisible by the world size
        x = O.normal(K, 11, 1.0)
        W = O.quantize(O.normal(N * K, 12, 0.02), O.Q4_0)
        rb = O.row_bytes(O.Q4_0, K)
        b0, b1 = weight_row_bytes_range(N, rb, world, rank)
        a, b = column_shard(N, world, rank)
        y_local = O.gemm_q(x, W[b0:b1], 1, b - a, K, O.Q4_0)
        full = gather_columns(torch.from_numpy(y_local), N).numpy()
        ref = O.gemm_q(x, W, 1, N, K, O.Q4_0)
        q.put((rank, bool(np.array_equal(full, ref))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_lm_head_column_shard_allgather_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(results.values()), results


def _argmax_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle as O
        from mvlm_b200.shard import combine_argmax_device, distributed_argmax
        N = 101
        ok = True
        for case in range(3):
            logits = O.normal(N, 40 + case, 1.0)
            if case == 1:
                # the same maximum in the last shard and in the first: the smaller index wins
                logits[N - 3] = logits[5] = 9.0
            if case == 2:
                logits[:] = -np.inf  # nothing above -1e30: index 0, as the reference's scan
            a, b = column_shard(N, world, rank)
            i, v = O.argmax_logits(logits[a:b].view(np.uint32), O.F32)
            pair = torch.tensor([i, 0], dtype=torch.int32)
            pair[1] = torch.tensor([v], dtype=torch.float32).view(torch.int32)[0]
            want = O.argmax_logits(logits.view(np.uint32), O.F32)[0]
            got = distributed_argmax(pair, N)
            ok &= got == want
            # the device-side combine the timed decode step uses (no host round trip)
            slots = torch.empty(2 * world, dtype=torch.int32)
            dist.all_gather_into_tensor(slots, pair)
            offsets = torch.tensor([column_shard(N, world, r)[0] for r in range(world)], dtype=torch.int64)
            ok &= int(combine_argmax_device(slots, offsets)) == want
        q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_lm_head_distributed_argmax_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = dict(q.get(timeout=5) for _ in range(world))
    assert all(results.values()), results
