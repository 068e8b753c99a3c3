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

Beside the headline the JSON line carries:

* ``c5_sharded`` (every N): the 70B-class grouped-query step (B=256, Hq 64 /
  Hkv 8, log-uniform lengths 512-32768, bf16) sharded by KV head -- rank r
  holds KV heads ``[r*8/N, (r+1)*8/N)``, their query heads and its own seeded
  page pool, and decodes them independently (strong scaling: the total work is
  fixed). Per-rank times are the max over ranks; the outputs are all-gathered
  over NCCL after timing and sampled rows of every shard are checked against
  the oracle.
* ``per_config`` (N=1): the three short steps C1 (B1 S128 MHA fp16), C3 (B1
  S4096 page 128 bf16) and C4 (B128 ragged GQA-4 bf16), each L2-flushed per
  step (eager and graph replay), back to back over rotating copies of the
  inputs (distinct seeded workloads whose bytes read per step add up to at
  least twice the L2, so every step reads from HBM without a flush between
  steps), and as back-to-back graph replays of one input (the reference's
  Layer-3 latency method), with fractions of the measured HBM peak.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): the headline is
weak scaling by KV head -- rank r holds its own 32-KV-head shard (own seeded
pool and block table) of a 32N-head cache and decodes it independently; no
collective touches the data path. Timing is the max over ranks; after timing,
the outputs are all-gathered over NCCL and rank 0 checks sampled rows of every
shard against the oracle.

``--impl reference`` times the reference algorithm's CPU path (the FP32
gather + softmax attention of the reference's ``tests/correctness.py:17-20``,
restated in ``oracle/``) on the host cores, on a bounded sample of the same
workload, with the same per-row routine as the b200 arm's ``cpu_baseline``;
under torchrun only rank 0 runs it.
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


def oracle_rows(w, rows):
    """The oracle's O for rows ``rows`` of workload ``w`` (FP32, CPU), computed
    on a compact copy of just those rows' pages: the pages are gathered on
    ``w``'s device, so an 8 GB cache never crosses to the host."""
    import oracle
    lens = w.seq_list()
    outs = []
    for b in rows:
        s_len = lens[b]
        nblk = max(1, (s_len + w.block_size - 1) // w.block_size)
        phys = w.block_table[b, :nblk].long()
        kc = w.k_cache[phys].cpu()
        vc = w.v_cache[phys].cpu()
        bt = torch.arange(nblk, dtype=torch.int32).reshape(1, nblk)
        ro, _ = oracle.decode_reference(w.q[b:b + 1], kc, vc, bt, [s_len], w.block_size)
        outs.append(ro[0])
    return torch.stack(outs)


def rows_match(got_rows, ref_rows):
    """The O tolerance of the parity contract: |got - ref| <= 2e-3 + 1e-2 |ref|."""
    got = got_rows.float().cpu()
    return bool(((got - ref_rows).abs() <= 2e-3 + 1e-2 * ref_rows.abs()).all())


def gather_and_verify(out, local_ok, config, rank, world, dist, device, batch=None,
                      rows=None):
    """All-gather every rank's output; rank 0 rebuilds each shard's inputs from
    its seed and checks sampled rows against the oracle. Returns the verdict,
    agreed by all ranks (all_reduce MIN)."""
    gathered = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(gathered, out)
    ok = bool(local_ok)
    if rank == 0:
        for r in range(world):
            wr = build_shard(config, r, world, device, batch=batch)
            sel = rows if rows is not None else [0, wr.batch - 1]
            ok &= rows_match(gathered[r][sel], oracle_rows(wr, sel))
            del wr
    flag = torch.tensor([1 if ok else 0], device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return bool(flag.item())


def workload_config(w, world, nbytes):
    """The ``config`` object of a JSON line: the same for both arms."""
    back_to_back = nbytes > 2 * L2_BYTES
    return {
        "workload": w.name,
        "batch": w.batch, "num_heads": w.num_heads, "num_kv_heads": w.num_kv_heads,
        "head_dim": w.q.shape[-1], "block_size": w.block_size,
        "seq_len": w.seq_len if isinstance(w.seq_len, int) else "per-row",
        "kv_bytes_per_rank": nbytes,
        "l2": (f"inputs {nbytes / 1e6:.0f} MB per rank > 2x L2 (126 MB): the K steps run back "
               "to back between one event pair, each streaming its inputs from HBM "
               "(per-step-event timings with L2 flushed under us_per_step)"
               if back_to_back else
               "flushed before every step: 512 MB write, then 512 MB read (no dirty lines left)"),
        "schedule": "token-balanced persistent",
        "parallelism": (f"kv-head shards x{world}" if world > 1 else "single GPU"),
    }


# ----------------------------------------------------------------------------- timing
class Timer:
    """CUDA-event timing on one stream, with a barrier (all ranks, then the
    device) on both sides of every timed region."""

    def __init__(self, stream, dev, dist, flusher):
        self.stream, self.dev, self.dist, self.flusher = stream, dev, dist, flusher

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()
        torch.cuda.synchronize(self.dev)

    def per_step(self, fn, steps, flush=True):
        """Per-step events around every step (L2 flushed before each)."""
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        self.barrier()
        for k in range(steps):
            if flush:
                self.flusher()
            starts[k].record(self.stream)
            fn(k)
            ends[k].record(self.stream)
        self.barrier()
        return _stats([a.elapsed_time(b) for a, b in zip(starts, ends)])

    def back_to_back(self, fn, steps):
        """One event pair around `steps` consecutive steps (nothing between the
        launches, as in steady-state decoding); mean = elapsed / steps."""
        s_ev = torch.cuda.Event(enable_timing=True)
        e_ev = torch.cuda.Event(enable_timing=True)
        self.barrier()
        s_ev.record(self.stream)
        for k in range(steps):
            fn(k)
        e_ev.record(self.stream)
        self.barrier()
        mean = s_ev.elapsed_time(e_ev) / steps
        return {"mean": mean, "median": mean, "min": mean, "max": mean}


def capture_graph(w, ws):
    """A CUDA graph of one decode call on ``w``'s tensors (the call's kernel
    node(s)); ``ws`` is sized by an eager call first."""
    import paged_attention as pa

    def call():
        return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                  w.block_size, workspace=ws)
    call()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = call()
    return g, out


# ----------------------------------------------------------------------------- b200 arm
def run_b200(args, rank, world, local_rank):
    import paged_attention as pa

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
    tm = Timer(stream, dev, dist, flusher)
    peak, peak_kind = _peaks()

    def op(_k=0):
        return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                  w.block_size, workspace=ws)

    # ---- correctness spot-check before timing (sampled rows vs the oracle)
    out = op()
    torch.cuda.synchronize(dev)
    sample_rows = sorted({0, w.batch // 2, w.batch - 1})
    parity_ok = rows_match(out[sample_rows], oracle_rows(w, sample_rows))

    # Inputs larger than twice the L2 stream from HBM in every step: time the
    # steps back to back. Smaller ones get the L2 flushed before every step.
    back_to_back = nbytes > 2 * L2_BYTES

    # ---- eager, device-timed (the headline)
    for _ in range(args.warmup):
        if not back_to_back:
            flusher()
        op()
    tm.barrier()
    with ClockSampler(dev.index) as clocks:
        eager = tm.back_to_back(op, args.steps) if back_to_back else tm.per_step(op, args.steps)
    # the same steps with L2 flushed before each (reported beside the headline)
    eager_flushed = eager if not back_to_back else tm.per_step(op, args.steps)

    # ---- graph replay (one kernel node), same flush discipline
    runner = pa.PagedAttnGraphRunner(w.batch, w.num_heads, w.q.shape[-1], max(w.seq_list()),
                                     w.block_size, w.k_cache.shape[0], device=dev, dtype=w.dtype,
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
    graph = tm.per_step(lambda _k: runner.replay_only(), args.steps)
    # reference Layer-3 method (tests/benchmark_core.py:133-145): back-to-back
    # replays averaged, no flush
    for _ in range(10):
        runner.replay_only()
    graph_b2b_ms = tm.back_to_back(lambda _k: runner.replay_only(), 200)["mean"]
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
    e2e, e2e_serial, h2d, d2h, e2e_ok = end_to_end(w, ws, out, tm, args, back_to_back)

    # ---- max over ranks
    eager_mean, graph_mean, e2e_mean, sync_med, graph_b2b, flushed_mean, e2e_serial_mean = (
        max_over_ranks([eager["mean"], graph["mean"], e2e["mean"], eager_sync["median"],
                        graph_b2b_ms, eager_flushed["mean"], e2e_serial["mean"]], dist, dev))

    # ---- verification all-gather over NCCL (outside the timed region)
    if dist is not None:
        parity_ok = gather_and_verify(out, parity_ok, args.config, rank, world, dist, dev)
    status = ws.read_status()
    del w, out

    # ---- the head-sharded C5 step at this N (every rank takes part)
    c5 = c5_sharded(args, rank, world, dist, dev, tm, peak)

    # ---- the short steps, one GPU
    per_cfg = per_config(args, dev, tm, peak) if world == 1 else None

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return None

    total_bytes = nbytes * world
    value = total_bytes / (eager_mean * 1e-3) / 1e9
    achieved = nbytes / (eager["mean"] * 1e-3) / 1e9
    traffic = _profile_traffic() if args.config == "c2" else None
    w0 = build_shard(args.config, 0, world, dev)
    cpu = cpu_baseline(w0, args) if world == 1 else None
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
        "dtype": _dtype_name(w0.dtype),
        "data": "synthetic (seeded N(0,1) q/K/V, shuffled page pool)",
        "config": workload_config(w0, world, nbytes),
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
                     "frac_l2_flushed": round(nbytes / (eager_flushed["mean"] * 1e-3) / 1e9
                                              / peak, 4),
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
        "capacity": capacity(w0, eager_mean, dev),
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "parity": {"sampled_rows_vs_oracle": parity_ok, "graph_equals_eager": bool(graph_ok),
                   "e2e_equals_device": bool(e2e_ok), "status_word": status},
        "c5_sharded": c5,
        "per_config": per_cfg,
    }
    print(json.dumps(res), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return res


def _dtype_name(dt):
    return str(dt).replace("torch.", "").replace("float16", "f16").replace("bfloat16", "bf16")


def end_to_end(w, ws, out, tm, args, back_to_back):
    """The same step through the public API with q, the block table (and the
    lengths) copied in from pinned host memory and O copied out every step."""
    import paged_attention as pa
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
    stream, dev = tm.stream, tm.dev

    def e2e_step(_k=0):
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
            tm.flusher()
        e2e_step()
    tm.barrier()
    e2e_serial = tm.back_to_back(e2e_step, args.steps) if back_to_back else tm.per_step(
        e2e_step, args.steps)
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
        tm.barrier()
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
        tm.barrier()
        mean = s_ev.elapsed_time(e_ev) / steps
        ok = all(torch.equal(h, o_host) for h in oh[:min(nbuf, steps)])
        return {"mean": mean, "median": mean, "min": mean, "max": mean}, ok

    if back_to_back:
        e2e_pipelined(args.warmup)
        e2e, pipe_ok = e2e_pipelined(args.steps)
        e2e_ok = e2e_ok and pipe_ok
    else:
        e2e = e2e_serial
    return e2e, e2e_serial, h2d, d2h, e2e_ok


def c5_sharded(args, rank, world, dist, dev, tm, peak):
    """The head-sharded C5 step at this world size (strong scaling): per-rank
    device times (max over ranks), aggregate bandwidth, and the NCCL gather
    check of every shard against the oracle."""
    import paged_attention as pa
    w = build_shard("c5", rank, world, dev)
    nbytes = w.effective_bytes()
    ws = pa.DecodeWorkspace(dev)

    def op(_k=0):
        return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                  w.block_size, workspace=ws)
    out = op()
    torch.cuda.synchronize(dev)
    rows = [0, w.batch // 2, w.batch - 1]
    local_ok = rows_match(out[rows], oracle_rows(w, rows))
    steps = max(5, min(args.steps, 20))
    for _ in range(args.warmup):
        op()
    eager = tm.back_to_back(op, steps)
    flushed = tm.per_step(op, steps)
    g, g_out = capture_graph(w, ws)
    for _ in range(3):
        g.replay()
    graph_b2b = tm.back_to_back(lambda _k: g.replay(), steps)
    graph_flushed = tm.per_step(lambda _k: g.replay(), steps)
    torch.cuda.synchronize(dev)
    graph_ok = bool(torch.equal(g_out, out))
    del g
    t_eager, t_flushed, t_graph, t_graph_flushed, nb_max = max_over_ranks(
        [eager["mean"], flushed["median"], graph_b2b["mean"], graph_flushed["median"],
         float(nbytes)], dist, dev)
    ok = local_ok and graph_ok
    if dist is not None:
        ok = gather_and_verify(out, ok, "c5", rank, world, dist, dev)
    status = ws.read_status()
    total = nbytes * world
    name = w.name.split("_rank")[0]
    del w, out, g_out
    torch.cuda.empty_cache()
    return {
        "workload": f"{name} (8 KV heads in {world} shard(s))",
        "scaling": "strong", "ranks": world, "kv_heads_per_rank": 8 // world,
        "q_heads_per_rank": 64 // world, "bytes_total": total, "bytes_per_rank": int(nb_max),
        "l2": "inputs per rank > 2x L2: back to back between one event pair; L2-flushed "
              "per-step medians beside",
        "us_per_step": {"eager": round(t_eager * 1e3, 1),
                        "eager_l2_flushed_median": round(t_flushed * 1e3, 1),
                        "graph_back_to_back": round(t_graph * 1e3, 1),
                        "graph_l2_flushed_median": round(t_graph_flushed * 1e3, 1)},
        "gbs_aggregate": round(total / (t_eager * 1e-3) / 1e9, 1),
        "gbs_per_rank": round(nb_max / (t_eager * 1e-3) / 1e9, 1),
        "frac_per_rank": round(nb_max / (t_eager * 1e-3) / 1e9 / peak, 4),
        "frac_per_rank_l2_flushed": round(nb_max / (t_flushed * 1e-3) / 1e9 / peak, 4),
        "verified": bool(ok), "status_word": status, "steps": steps,
    }


PER_CONFIG = ("c1", "c3", "c4")


def per_config(args, dev, tm, peak):
    """C1, C3 and C4 on one GPU: L2-flushed per step (eager, graph), back to
    back over rotating input copies (cold in L2 without a flush), and
    back-to-back graph replays of one input (the reference's Layer-3 method,
    tests/benchmark_core.py:133-145; the latency target of C1)."""
    import paged_attention as pa
    from paged_attention import workloads
    res = {}
    steps = max(args.steps, 50)
    for name in PER_CONFIG:
        base = workloads.CONFIGS[name](dev)
        nbytes = base.effective_bytes()
        copies = max(2, min(128, -(-2 * L2_BYTES // nbytes)))
        ws_list = [base] + [workloads.CONFIGS[name](dev, seed=SEEDS[name] + 100 * i)
                            for i in range(1, copies)]
        spaces = [pa.DecodeWorkspace(dev) for _ in ws_list]

        def op_i(i):
            w = ws_list[i % copies]
            return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                      w.block_size, workspace=spaces[i % copies])
        outs = [op_i(i) for i in range(copies)]
        torch.cuda.synchronize(dev)
        rows = sorted({0, base.batch - 1})
        ok = rows_match(outs[0][rows], oracle_rows(base, rows))
        for _ in range(args.warmup):
            tm.flusher()
            op_i(0)
        flushed = tm.per_step(lambda _k: op_i(0), steps)
        for i in range(copies * 2):
            op_i(i)
        rotating = tm.back_to_back(op_i, steps)
        graphs = [capture_graph(w, sp) for w, sp in zip(ws_list, spaces)]
        for i in range(copies):
            graphs[i][0].replay()
        torch.cuda.synchronize(dev)
        graph_ok = all(torch.equal(g_out, o) for (_, g_out), o in zip(graphs, outs))
        g_flushed = tm.per_step(lambda _k: graphs[0][0].replay(), steps)
        g_rotating = tm.back_to_back(lambda k: graphs[k % copies][0].replay(), steps)
        for _ in range(10):
            graphs[0][0].replay()
        g_warm = tm.back_to_back(lambda _k: graphs[0][0].replay(), 200)
        status = max(sp.read_status() for sp in spaces)
        plan = pa.decode_plan(base.q, base.k_cache, base.v_cache, base.block_table,
                              base.seq_len, base.block_size)

        def entry(ms):
            gbs = nbytes / (ms * 1e-3) / 1e9
            return {"us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4)}
        r = {"workload": base.name, "bytes": nbytes, "dtype": _dtype_name(base.dtype),
             "eager_l2_flushed_median": entry(flushed["median"]),
             "graph_l2_flushed_median": entry(g_flushed["median"]),
             "eager_back_to_back_rotating": entry(rotating["mean"]),
             "graph_back_to_back_rotating": entry(g_rotating["mean"]),
             "graph_back_to_back_same_input": entry(g_warm["mean"]),
             "rotating_copies": copies,
             "kernels_per_call": plan["kernels"],
             "parity": {"sampled_rows_vs_oracle": ok, "graph_equals_eager": bool(graph_ok),
                        "status_word": status}}
        if name == "c1":
            r["target_graph_us"] = 10.0
            r["meets_target"] = bool(g_warm["mean"] * 1e3 <= 10.0)
        res[name] = r
        del graphs, outs, ws_list, spaces, base
        torch.cuda.empty_cache()
    return res


def capacity(w, step_ms, dev):
    """Layer-2 "paged architecture efficiency" figures (tests/benchmark_core.py:80-107)
    for this workload on this device: KV bytes per request, decode tokens/s per GB
    of KV, and how many such requests fit in 90 % of the device's memory (the
    reference uses a fixed 8 GB budget)."""
    e = w.q.element_size()
    kv = sum(w.seq_list()) * w.num_kv_heads * w.q.shape[-1] * e * 2
    per_req = kv / w.batch
    total = torch.cuda.get_device_properties(dev).total_memory
    return {"kv_mb_per_request": round(per_req / 2**20, 2),
            "tokens_per_s_per_gb": round(w.batch / (step_ms * 1e-3) / (kv / 1e9), 1),
            "max_batch_in_90pct_hbm": int(0.9 * total // per_req)}


# ----------------------------------------------------------------------------- CPU arm
class CpuPath:
    """The reference algorithm's CPU path (the oracle's FP32 gather + softmax
    attention, tests/correctness.py:17-20) over one workload held in host
    memory, one row per call on every host thread. Both arms time it with
    this class, so they report the same number for the same workload."""

    WARMUP_ROWS = 4

    def __init__(self, w):
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.q = w.q.cpu()
        self.k = w.k_cache.cpu()
        self.v = w.v_cache.cpu()
        self.bt = w.block_table.cpu()
        self.lens = w.seq_list()
        self.batch, self.block_size = w.batch, w.block_size
        e = self.q.element_size()
        self.row_bytes = [s * w.num_kv_heads * w.q.shape[-1] * e * 2
                          + w.num_heads * w.q.shape[-1] * e * 2 for s in self.lens]
        self.next_row = 0
        for _ in range(self.WARMUP_ROWS):
            self.row()

    def row(self):
        """One row (round robin over the batch); returns its algorithmic bytes."""
        import oracle
        b = self.next_row % self.batch
        self.next_row += 1
        oracle.decode_reference(self.q, self.k, self.v, self.bt, self.lens, self.block_size,
                                batch_indices=[b])
        return self.row_bytes[b]


def cpu_baseline(w, args):
    """The CPU path on a bounded sample (about ``--cpu-seconds`` of work)."""
    cpu = CpuPath(w)
    rows_done, bytes_done, t0 = 0, 0, time.perf_counter()
    while True:
        bytes_done += cpu.row()
        rows_done += 1
        if time.perf_counter() - t0 > args.cpu_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(bytes_done / dt / 1e9, 3), "unit": "GB/s", "cores": cpu.threads,
            "kind": "port",
            "sample": f"{rows_done} rows of {w.batch} round robin ({dt:.1f} s), same seeded "
                      f"workload, torch CPU FP32, {cpu.threads} threads",
            "us_per_row": round(dt / rows_done * 1e6, 1)}


def run_reference(args, rank, world):
    if rank != 0:
        return None
    from paged_attention import workloads
    w = build_shard(args.config, 0, world, "cpu")
    nbytes = w.effective_bytes()
    cpu = CpuPath(w)
    rows_per_step = max(1, args.ref_rows)
    for _ in range(args.warmup):
        for _ in range(rows_per_step):
            cpu.row()
    t0 = time.perf_counter()
    nb = 0
    for _ in range(args.steps):
        for _ in range(rows_per_step):
            nb += cpu.row()
    dt = time.perf_counter() - t0
    gbs = nb / dt / 1e9
    sample = (f"{rows_per_step} rows per step round robin over the {w.batch} rows (bounded "
              f"sample of {w.name}), torch CPU FP32, {cpu.threads} threads")
    res = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if args.config == "c5" else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/K/V, shuffled page pool)",
        "config": workload_config(w, world, nbytes),
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cpu.threads,
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
    ap.add_argument("--ref-rows", type=int, default=8)
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
