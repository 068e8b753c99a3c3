"""Decode-step benchmark of the B200 paged-attention operator.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config c1|c2|c3|c4|c5]

Workload (default ``c2``): B=32 sequences x 32 query heads = 32 KV heads,
head_dim 128, fp16, 1024 tokens each in 16-token pages shuffled over a pool of
2048 pages, q/K/V i.i.d. N(0,1) -- the high-concurrency steady-state decode
step. One step = one decode call over the whole batch.

Metric: effective KV HBM bandwidth in GB/s (K+V bytes of every cached token
plus q and o bytes, divided by the step's device time) and decode-step us.
Timing is on the launching stream with CUDA events. When a rank's resident
inputs exceed twice the L2 (126 MB; the default workload holds 537 MB) the K
timed steps run back to back between one event pair (the reference's Layer-3
method, ``tests/benchmark_core.py:133-145``), every step streaming its inputs
from HBM; otherwise L2 is flushed before every timed step by writing a 512 MB
buffer and then reading another 512 MB buffer (so no dirty flush lines are left
in L2) and each step has its own event pair. Per-step, L2-flushed timings are
reported beside the headline either way.

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
L2_BYTES = 126 * 1024 * 1024
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
    """SM clock and throttle-reason sampling during the timed region.

    Polls NVML every 2 ms from a thread (read-only queries); falls back to
    ``nvidia-smi -lms 200`` when NVML is unavailable."""

    # NVML clocks-event reason bits
    _REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
                0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.index = index
        self.samples = []       # (sm_mhz, reason_bits)
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index())
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def poll():
                while not self._stop.is_set():
                    try:
                        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((mhz, bits))
                    except Exception:
                        pass
                    self._stop.wait(0.002)
            self._thread = threading.Thread(target=poll, daemon=True)
            self._thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 1.0:
                time.sleep(0.005)
        except Exception:
            self._thread = None
        return self

    def _physical_index(self):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                return int(vis.split(",")[self.index])
            except (ValueError, IndexError):
                pass
        return self.index

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        rows = list(self.samples)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    "samples": 0}
        reasons = sorted({name for _, bits in rows for bit, name in self._REASONS.items()
                          if bits & bit})
        return {"sm_mhz": statistics.median(m for m, _ in rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(rows), "source": "nvml 2 ms"}


class L2Flush:
    """Evicts L2 (126 MB) before a timed step: writes a 512 MB buffer, then reads
    another 512 MB buffer so the write-back of the flush's own dirty lines
    happens here, outside the timed region, and L2 is left holding only clean,
    unrelated lines. Both run on the timing stream before the start event."""

    def __init__(self, device):
        self.wbuf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.rbuf = torch.ones(FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    def __call__(self):
        self.wbuf.fill_(1)
        # the read half allocates its lines in L2 (a plain reduction), evicting
        # the fill's dirty lines; a streaming (evict-first) read would leave them
        self.rbuf.sum(dtype=torch.int64)


def _stats(ms):
    return {"mean": statistics.fmean(ms), "median": statistics.median(ms), "min": min(ms),
            "max": max(ms)}


# ----------------------------------------------------------------------------- ranks
SEEDS = {"c1": 1, "c2": 2, "c3": 3, "c4": 4, "c5": 5}


def build_shard(config, rank, world, device, batch=None):
    """Rank ``rank``'s shard: c5 splits its 8 KV heads over the ranks (strong
    scaling); the other shapes give every rank a full-size shard with its own
    seed (weak scaling by KV head)."""
    from paged_attention import workloads
    if config == "c5":
        return workloads.c5(device, rank=rank, world=world, batch=batch)
    return workloads.CONFIGS[config](device, seed=SEEDS[config] + 1000 * rank)


def max_over_ranks(values, dist, device):
    """Element-wise max of per-rank timings (all_reduce MAX; identity at N=1)."""
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_and_verify(out, local_ok, config, rank, world, dist, device, batch=None,
                      rows=None):
    """All-gather every rank's output; rank 0 rebuilds each shard's inputs from
    its seed and checks sampled rows against the oracle. Returns the verdict,
    agreed by all ranks (all_reduce MIN)."""
    import oracle
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    ok = bool(local_ok)
    if rank == 0:
        for r in range(world):
            wr = build_shard(config, r, world, device, batch=batch)
            sel = rows if rows is not None else [0, wr.batch - 1]
            ro, _ = oracle.decode_reference(wr.q, wr.k_cache, wr.v_cache, wr.block_table,
                                            wr.seq_len, wr.block_size, batch_indices=sel)
            got = gathered[r].float().cpu()[sel]
            ref = ro[sel]
            ok &= bool(((got - ref).abs() <= 2e-3 + 1e-2 * ref.abs()).all())
            del wr
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


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

    # Each rank builds its own shard (own seed / own KV heads).
    w = build_shard(args.config, rank, world, dev)
    nbytes = w.effective_bytes()
    flusher = L2Flush(dev)
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

    # Inputs larger than twice the L2 stream from HBM in every step: time the
    # steps back to back. Smaller ones get the L2 flushed before every step.
    back_to_back = nbytes > 2 * L2_BYTES

    def timed(fn, flush, steps):
        """Per-step events around every step."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier()
        for k in range(steps):
            if flush:
                flusher()
            starts[k].record(stream)
            fn()
            ends[k].record(stream)
        barrier()
        return _stats([s.elapsed_time(e) for s, e in zip(starts, ends)])

    def timed_back_to_back(fn, steps):
        """One event pair around `steps` consecutive steps (nothing between the
        launches, as in steady-state decoding); mean = elapsed / steps."""
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        barrier()
        s_ev.record(stream)
        for _ in range(steps):
            fn()
        e_ev.record(stream)
        barrier()
        mean = s_ev.elapsed_time(e_ev) / steps
        return {"mean": mean, "median": mean, "min": mean, "max": mean}

    # ---- eager, device-timed (the headline)
    for _ in range(args.warmup):
        if not back_to_back:
            flusher()
        op()
    barrier()
    with ClockSampler(dev.index) as clocks:
        eager = timed_back_to_back(op, args.steps) if back_to_back else timed(op, True, args.steps)
    # the same steps with L2 flushed before each (reported beside the headline)
    eager_flushed = eager if not back_to_back else timed(op, True, args.steps)

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
        flusher()
        runner.replay_only()
    barrier()
    gs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ge = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for k in range(args.steps):
        flusher()
        gs[k].record(stream)
        runner.replay_only()
        ge[k].record(stream)
    barrier()
    graph = _stats([s.elapsed_time(e) for s, e in zip(gs, ge)])
    # reference Layer-3 method (tests/benchmark_core.py:133-145): back-to-back
    # replays averaged, no flush
    reps = 200
    for _ in range(10):
        runner.replay_only()
    b2b_s = torch.cuda.Event(enable_timing=True)
    b2b_e = torch.cuda.Event(enable_timing=True)
    b2b_s.record(stream)
    for _ in range(reps):
        runner.replay_only()
    b2b_e.record(stream)
    torch.cuda.synchronize(dev)
    graph_b2b_ms = b2b_s.elapsed_time(b2b_e) / reps
    del runner

    # ---- eager with a host sync before each step (reference method: launch
    # overhead included, tests/benchmark_core.py:51-62)
    sync_ms = []
    for k in range(min(args.steps, 50)):
        flusher()
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
        if not back_to_back:
            flusher()
        e2e_step()
    barrier()
    e2e_serial = timed_back_to_back(e2e_step, args.steps) if back_to_back else timed(
        e2e_step, True, args.steps)
    e2e_ok = torch.equal(o_host, out.cpu())

    # Serving loop: step k+1's inputs go up on one copy stream and step k-1's
    # output comes down on another while step k's kernel runs (two buffer
    # sets). Every step's copies are inside the timed region. Only for inputs
    # that stream from HBM anyway (no flush to interleave).
    def e2e_pipelined(steps):
        nbuf = 2
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        qb = [torch.empty_like(w.q) for _ in range(nbuf)]
        btb = [torch.empty_like(w.block_table) for _ in range(nbuf)]
        slb = [None if sl_host is None else torch.empty_like(w.seq_len) for _ in range(nbuf)]
        ob = [torch.empty_like(w.q) for _ in range(nbuf)]
        oh = [torch.empty(w.q.shape, dtype=w.q.dtype).pin_memory() for _ in range(nbuf)]
        in_ready = [torch.cuda.Event() for _ in range(nbuf)]
        k_done = [torch.cuda.Event() for _ in range(nbuf)]
        out_done = [torch.cuda.Event() for _ in range(nbuf)]
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        barrier()
        s_ev.record(stream)
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        for k in range(steps):
            i = k % nbuf
            with torch.cuda.stream(s_in):
                if k >= nbuf:
                    s_in.wait_event(k_done[i])          # kernel k-2 is done with buffer i
                qb[i].copy_(q_host, non_blocking=True)
                btb[i].copy_(bt_host, non_blocking=True)
                if slb[i] is not None:
                    slb[i].copy_(sl_host, non_blocking=True)
                in_ready[i].record(s_in)
            stream.wait_event(in_ready[i])
            if k >= nbuf:
                stream.wait_event(out_done[i])          # step k-2's output is on the host
            pa.paged_attention(qb[i], w.k_cache, w.v_cache, btb[i],
                               w.seq_len if slb[i] is None else slb[i], w.block_size,
                               workspace=ws, out=ob[i])
            k_done[i].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(k_done[i])
                oh[i].copy_(ob[i], non_blocking=True)
                out_done[i].record(s_out)
        stream.wait_stream(s_out)
        e_ev.record(stream)
        barrier()
        mean = s_ev.elapsed_time(e_ev) / steps
        ok = all(torch.equal(h, o_host) for h in oh[:min(nbuf, steps)])
        return {"mean": mean, "median": mean, "min": mean, "max": mean}, ok

    if back_to_back:
        e2e_pipelined(args.warmup)
        e2e, pipe_ok = e2e_pipelined(args.steps)
        e2e_ok = e2e_ok and pipe_ok
    else:
        e2e = e2e_serial

    # ---- max over ranks
    eager_mean, graph_mean, e2e_mean, sync_med, graph_b2b, flushed_mean, e2e_serial_mean = (
        max_over_ranks([eager["mean"], graph["mean"], e2e["mean"], eager_sync["median"],
                        graph_b2b_ms, eager_flushed["mean"], e2e_serial["mean"]], dist, dev))

    # ---- verification all-gather over NCCL (outside the timed region)
    if dist is not None:
        parity_ok = gather_and_verify(out, parity_ok, args.config, rank, world, dist, dev)

    status = ws.read_status()

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return None

    peak, peak_kind = _peaks()
    total_bytes = nbytes * world
    value = total_bytes / (eager_mean * 1e-3) / 1e9
    achieved = nbytes / (eager["mean"] * 1e-3) / 1e9
    traffic = _profile_traffic() if args.config == "c2" else None
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
        "scaling": "strong" if args.config == "c5" else "weak",
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
            "l2": (f"inputs {nbytes / 1e6:.0f} MB per rank > 2x L2 (126 MB): the K steps run back "
                   "to back between one event pair, each streaming its inputs from HBM "
                   "(per-step-event timings with L2 flushed under us_per_step)"
                   if back_to_back else
                   "flushed before every step: 512 MB write, then 512 MB read (no dirty lines left)"),
            "schedule": "token-balanced persistent",
            "parallelism": (f"kv-head shards x{world}" if world > 1 else "single GPU"),
        },
        "us_per_step": {"eager": round(eager_mean * 1e3, 2),
                        "eager_l2_flushed": round(flushed_mean * 1e3, 2),
                        "graph_l2_flushed": round(graph_mean * 1e3, 2),
                        "eager_host_sync": round(sync_med * 1e3, 2),
                        "graph_back_to_back": round(graph_b2b * 1e3, 2),
                        "eager_l2_flushed_median": round(eager_flushed["median"] * 1e3, 2),
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
                "us_per_step_copies_serialised": round(e2e_serial_mean * 1e3, 2),
                "note": ("KV cache resident in HBM; q, block table (and lengths) in from pinned "
                         "host memory, O out, every step; "
                         + ("copies double-buffered on two copy streams, overlapping the "
                            "neighbouring steps' kernels" if back_to_back else
                            "copies and kernel serialised on one stream"))},
        "capacity": capacity(w, eager_mean, dev),
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


def capacity(w, step_ms, dev):
    """Layer-2 "paged architecture efficiency" figures (tests/benchmark_core.py:80-107)
    for this workload on this device: KV bytes per request, decode tokens/s per GB
    of KV, and how many such requests fit in 90 % of the device's memory (the
    reference uses a fixed 8 GB budget)."""
    e = w.q.element_size()
    kv = sum(w.seq_list()) * w.num_kv_heads * 128 * e * 2
    per_req = kv / w.batch
    total = torch.cuda.get_device_properties(dev).total_memory
    return {"kv_mb_per_request": round(per_req / 2**20, 2),
            "tokens_per_s_per_gb": round(w.batch / (step_ms * 1e-3) / (kv / 1e9), 1),
            "max_batch_in_90pct_hbm": int(0.9 * total // per_req)}


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
        if time.perf_counter() - t0 > sample_seconds:
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
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=["c1", "c2", "c3", "c4", "c5"], default="c2")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
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
