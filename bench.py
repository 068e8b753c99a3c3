"""Decode-step benchmark of the B200 paged-attention operator.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c1|c2|c3|c4|c5]

Workload (default ``c2``): B=32 sequences x 32 query heads = 32 KV heads,
head_dim 128, fp16, 1024 tokens each in 16-token pages shuffled over a pool of
2048 pages, q/K/V i.i.d. N(0,1) -- the high-concurrency steady-state decode
step. One step = one decode call over the whole batch.

Metric: effective KV HBM bandwidth in GB/s (K+V bytes of every cached token
plus q and o bytes, divided by the step's device time) and decode-step us.
L2 (126 MB) is flushed before every timed step by writing a 512 MB buffer;
each step is bracketed by CUDA events on the launching stream.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): weak scaling by
KV head -- rank r holds its own 32-KV-head shard (own seeded pool and block
table) of a 32N-head cache and decodes it independently; no collective touches
the data path. Timing is the max over ranks; after timing, the outputs are
all-gathered over NCCL and rank 0 checks sampled rows of every shard against
the oracle.

``--impl reference`` times the reference algorithm's CPU path (the FP32
gather + softmax attention of the reference's ``tests/correctness.py:17-20``,
restated in ``oracle/``) on the host cores, on a bounded sample of the same
workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "paged-attention-triton_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = ("decode-step µs and effective KV HBM GB/s (% of B200 peak), eager+graph, "
          "1/2/4/8 GPU")
FLUSH_BYTES = 512 * 1024 * 1024
PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "pa_decode_c2_traffic.txt")


# ----------------------------------------------------------------------------- helpers
def _env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _profile_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    if not os.path.exists(PROFILE_TRAFFIC):
        return None
    with open(PROFILE_TRAFFIC) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling (200 ms) during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def __enter__(self):
        cmd = ["nvidia-smi", "-i", str(self.index),
               "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
               "--format=csv,noheader,nounits", "-lms", "200"]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.samples.append([x.strip() for x in line.split(",")])
        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            if self.thread is not None:
                self.thread.join(timeout=2)

    def summary(self):
        rows = [s for s in self.samples if len(s) >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def _stats(ms):
    return {"mean": statistics.fmean(ms), "median": statistics.median(ms), "min": min(ms),
            "max": max(ms)}


# ----------------------------------------------------------------------------- b200 arm
def run_b200(args, rank, world, local_rank):
    import paged_attention as pa
    from paged_attention import workloads
    import oracle

    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)

    # Each rank builds its own shard: c2's shape with a rank-specific seed.
    builder = workloads.CONFIGS[args.config]
    if args.config == "c5":
        w = builder(dev, rank=rank, world=world)
    else:
        w = builder(dev, seed={"c1": 1, "c2": 2, "c3": 3, "c4": 4}[args.config] + 1000 * rank)
    nbytes = w.effective_bytes()
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    ws = pa.DecodeWorkspace(dev)
    stream = torch.cuda.current_stream(dev)

    def op():
        return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                  w.block_size, workspace=ws)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- correctness spot-check before timing (sampled rows vs the oracle)
    out = op()
    torch.cuda.synchronize(dev)
    sample_rows = sorted({0, w.batch // 2, w.batch - 1})
    ro, _ = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                    w.block_size, batch_indices=sample_rows)
    idx = torch.tensor(sample_rows)
    err = (out.float().cpu()[idx] - ro[idx]).abs()
    parity_ok = bool((err <= 2e-3 + 1e-2 * ro[idx].abs()).all())

    # ---- eager, device-timed, L2 flushed before every step
    for _ in range(args.warmup):
        flush.fill_(1)
        op()
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(dev.index) as clocks:
        barrier()
        for k in range(args.steps):
            flush.fill_(1)
            starts[k].record(stream)
            op()
            ends[k].record(stream)
        barrier()
    eager_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    eager = _stats(eager_ms)

    # ---- graph replay (one kernel node), same flush discipline
    runner = pa.PagedAttnGraphRunner(w.batch, w.num_heads, 128, max(w.seq_list()), w.block_size,
                                     w.k_cache.shape[0], device=dev, dtype=w.dtype,
                                     num_kv_heads=w.num_kv_heads,
                                     dynamic_seq_lens=not isinstance(w.seq_len, int),
                                     max_seq_len=w.block_table.shape[1] * w.block_size)
    runner.run(w.q, w.k_cache, w.v_cache, w.block_table, copy_kv=True,
               seq_lens=None if isinstance(w.seq_len, int) else w.seq_len)
    torch.cuda.synchronize(dev)
    graph_ok = torch.equal(runner.static_out, op())
    for _ in range(args.warmup):
        flush.fill_(1)
        runner.replay_only()
    barrier()
    gs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ge = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for k in range(args.steps):
        flush.fill_(1)
        gs[k].record(stream)
        runner.replay_only()
        ge[k].record(stream)
    barrier()
    graph = _stats([s.elapsed_time(e) for s, e in zip(gs, ge)])
    del runner

    # ---- eager with a host sync before each step (reference method: launch
    # overhead included, tests/benchmark_core.py:51-62)
    sync_ms = []
    for k in range(min(args.steps, 50)):
        flush.fill_(1)
        torch.cuda.synchronize(dev)
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        s_ev.record(stream)
        op()
        e_ev.record(stream)
        torch.cuda.synchronize(dev)
        sync_ms.append(s_ev.elapsed_time(e_ev))
    eager_sync = _stats(sync_ms)

    # ---- end to end through the public API with pinned host buffers
    q_host = w.q.cpu().pin_memory()
    bt_host = w.block_table.cpu().pin_memory()
    sl_host = None if isinstance(w.seq_len, int) else w.seq_len.cpu().pin_memory()
    o_host = torch.empty(w.q.shape, dtype=w.q.dtype).pin_memory()
    q_dev = torch.empty_like(w.q)
    bt_dev = torch.empty_like(w.block_table)
    sl_dev = None if sl_host is None else torch.empty_like(w.seq_len)
    h2d = q_host.numel() * q_host.element_size() + bt_host.numel() * 4 + (
        0 if sl_host is None else sl_host.numel() * 4)
    d2h = o_host.numel() * o_host.element_size()

    def e2e_step():
        q_dev.copy_(q_host, non_blocking=True)
        bt_dev.copy_(bt_host, non_blocking=True)
        if sl_dev is not None:
            sl_dev.copy_(sl_host, non_blocking=True)
        o = pa.paged_attention(q_dev, w.k_cache, w.v_cache, bt_dev,
                               w.seq_len if sl_dev is None else sl_dev, w.block_size,
                               workspace=ws)
        o_host.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        flush.fill_(1)
        e2e_step()
    barrier()
    es = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ee = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for k in range(args.steps):
        flush.fill_(1)
        es[k].record(stream)
        e2e_step()
        ee[k].record(stream)
    barrier()
    e2e = _stats([s.elapsed_time(e) for s, e in zip(es, ee)])
    e2e_ok = torch.equal(o_host, out.cpu())

    # ---- max over ranks
    vals = torch.tensor([eager["mean"], graph["mean"], e2e["mean"], eager_sync["median"]],
                        dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    eager_mean, graph_mean, e2e_mean, sync_med = vals.tolist()

    # ---- verification all-gather over NCCL (outside the timed region)
    gathered_ok = True
    if dist is not None:
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        if rank == 0:
            for r in range(world):
                wr = builder(dev, rank=r, world=world) if args.config == "c5" else builder(
                    dev, seed={"c1": 1, "c2": 2, "c3": 3, "c4": 4}[args.config] + 1000 * r)
                rows = [0, wr.batch - 1]
                ro_r, _ = oracle.decode_reference(wr.q, wr.k_cache, wr.v_cache, wr.block_table,
                                                  wr.seq_len, wr.block_size, batch_indices=rows)
                got = gathered[r].float().cpu()[rows]
                gathered_ok &= bool(((got - ro_r[rows]).abs() <=
                                     2e-3 + 1e-2 * ro_r[rows].abs()).all())
                del wr
        flag = torch.tensor([1 if (parity_ok and gathered_ok) else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        parity_ok = bool(flag.item())

    status = ws.read_status()

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return None

    peak, peak_kind = _peaks()
    total_bytes = nbytes * world
    value = total_bytes / (eager_mean * 1e-3) / 1e9
    achieved = nbytes / (eager["mean"] * 1e-3) / 1e9
    traffic = _profile_traffic()
    cpu = cpu_baseline(w, args, sample_seconds=args.cpu_seconds) if world == 1 else None
    res = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(eager_mean, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": str(w.dtype).replace("torch.", "").replace("float16", "f16").replace(
            "bfloat16", "bf16"),
        "data": "synthetic (seeded N(0,1) q/K/V, shuffled page pool)",
        "config": {
            "workload": w.name,
            "batch": w.batch, "num_heads": w.num_heads, "num_kv_heads": w.num_kv_heads,
            "head_dim": 128, "block_size": w.block_size,
            "seq_len": w.seq_len if isinstance(w.seq_len, int) else "per-row",
            "kv_bytes_per_rank": nbytes,
            "l2": "flushed before every step (512 MB write)",
            "schedule": "token-balanced persistent",
            "parallelism": f"kv-head shards x{world}" if world > 1 else "single GPU",
        },
        "us_per_step": {"eager": round(eager_mean * 1e3, 2), "graph": round(graph_mean * 1e3, 2),
                        "eager_host_sync": round(sync_med * 1e3, 2),
                        "eager_median": round(eager["median"] * 1e3, 2),
                        "graph_median": round(graph["median"] * 1e3, 2)},
        "graph_gbs": round(total_bytes / (graph_mean * 1e-3) / 1e9, 1),
        "pct_of_peak": {"eager": round(100 * value / world / peak, 1),
                        "graph": round(100 * total_bytes / world / (graph_mean * 1e-3) / 1e9
                                       / peak, 1),
                        "nominal_8TBs_eager": round(100 * value / world / 8000.0, 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy)"
                     if peak_kind == "measured" else "fallback",
                     "traffic": traffic},
        "e2e": {"value": round(total_bytes / (e2e_mean * 1e-3) / 1e9, 1), "unit": "GB/s",
                "us_per_step": round(e2e_mean * 1e3, 2),
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "note": "KV cache resident in HBM; q, block table (and lengths) in, O out"},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "parity": {"sampled_rows_vs_oracle": parity_ok, "graph_equals_eager": bool(graph_ok),
                   "e2e_equals_device": bool(e2e_ok), "status_word": status},
    }
    print(json.dumps(res), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return res


# ----------------------------------------------------------------------------- CPU arm
def cpu_baseline(w, args, sample_seconds=15.0):
    """The reference algorithm's CPU path on a bounded sample of the workload."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q = w.q.cpu()
    k = w.k_cache.cpu()
    v = w.v_cache.cpu()
    bt = w.block_table.cpu()
    lens = w.seq_list()
    rows_done, bytes_done, t0 = 0, 0, time.perf_counter()
    e = q.element_size()
    while True:
        b = rows_done % w.batch
        oracle.decode_reference(q, k, v, bt, lens, w.block_size, batch_indices=[b])
        bytes_done += (lens[b] * w.num_kv_heads * 128 * e * 2 + w.num_heads * 128 * e * 2)
        rows_done += 1
        if time.perf_counter() - t0 > sample_seconds or rows_done >= 4 * w.batch:
            break
    dt = time.perf_counter() - t0
    return {"value": round(bytes_done / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{rows_done} of {w.batch} rows ({dt:.1f} s), same seeded workload",
            "us_per_row": round(dt / rows_done * 1e6, 1)}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from paged_attention import workloads
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = workloads.CONFIGS[args.config]("cpu")
    q, k, v, bt = w.q, w.k_cache, w.v_cache, w.block_table
    lens = w.seq_list()
    e = q.element_size()
    rows_per_step = max(1, min(w.batch, args.ref_rows))

    def step(i):
        rows = [(i * rows_per_step + j) % w.batch for j in range(rows_per_step)]
        oracle.decode_reference(q, k, v, bt, lens, w.block_size, batch_indices=rows)
        return sum(lens[r] * w.num_kv_heads * 128 * e * 2 + w.num_heads * 128 * e * 2
                   for r in rows)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    nb = 0
    for i in range(args.steps):
        nb += step(i)
    dt = time.perf_counter() - t0
    gbs = nb / dt / 1e9
    sample = (f"{rows_per_step} of {w.batch} rows per step (bounded sample of {w.name}), "
              f"torch CPU FP32, {threads} threads")
    res = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/K/V, shuffled page pool)",
        "config": {"workload": w.name, "batch": w.batch, "num_heads": w.num_heads,
                   "num_kv_heads": w.num_kv_heads, "head_dim": 128, "block_size": w.block_size},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(res), flush=True)
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-rows", type=int, default=2)
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    rank, world, local_rank = _env_rank()
    if world != args.gpus and "RANK" in os.environ:
        print(f"warning: WORLD_SIZE={world} but --gpus {args.gpus}", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
