"""World-size-2 gloo tests (CPU) of the multi-GPU bench plumbing: per-rank
shards, max-over-ranks timing and the all-gather verification. The oracle
stands in for the per-rank decode output; a planted error on one rank must be
caught by rank 0's verification and agreed by every rank."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, plant_error, results):
    import sys
    for p in (os.path.join(ROOT, "paged-attention-triton_b200"), ROOT):
        if p not in sys.path:
            sys.path.insert(0, p)
    import bench
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        dev = torch.device("cpu")
        w = bench.build_shard("c5", rank, world, dev, batch=3)
        out, _ = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                         w.block_size, batch_indices=[0, w.batch - 1])
        out = out.to(w.q.dtype)
        if plant_error and rank == 1:
            out[0, 0, 0] += 0.5
        t = bench.max_over_ranks([1.0 + rank, 5.0 - rank], dist, dev)
        ok = bench.gather_and_verify(out, True, "c5", rank, world, dist, dev, batch=3)
        results[rank] = (ok, t, w.num_heads, w.num_kv_heads)
    finally:
        dist.destroy_process_group()


def _run(plant_error):
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, plant_error, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    return dict(results)


def test_two_rank_gather_verify_and_max():
    res = _run(plant_error=False)
    for rank in (0, 1):
        ok, t, hq, hkv = res[rank]
        assert ok
        assert t == [2.0, 5.0]
        assert (hq, hkv) == (32, 4)       # c5 head shard at world 2


def test_two_rank_planted_error_is_caught():
    res = _run(plant_error=True)
    assert res[0][0] is False and res[1][0] is False
