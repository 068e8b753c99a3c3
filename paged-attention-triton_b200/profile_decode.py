"""Launch the decode kernel a few times on one benchmark shape, for profilers.

    python profile_decode.py --config c2 [--iters 3] [--num-splits 0] [--flush]
    python profile_decode.py --shape 1,8192,64,8 [--head-dim 128] [--iters 3] [--flush]

Builds the seeded workload, runs one warm-up launch and ``--iters`` timed
launches (L2 flushed before each with ``--flush``) and prints the mean device
time and effective GB/s. Meant to be wrapped by ``ncu`` with ``-k
regex:pa_decode_kernel -s 1 -c <iters>``; small enough for full-metric
captures (c2 holds ~1.1 GB of KV on the device). ``--shape B,S,HQ,HKV`` runs a
same-length bf16 step with block 16 instead of a configuration (when few long
segments cross CTAs the step is two kernels: the decode kernel and the merge
pass, ``merge_segments_kernel``).
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

import paged_attention as pa  # noqa: E402
from paged_attention import workloads  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c2", choices=sorted(workloads.CONFIGS))
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--num-splits", type=int, default=0)
    ap.add_argument("--flush", action="store_true")
    ap.add_argument("--variant", type=int, default=0, help="kernel variant (0 = automatic)")
    ap.add_argument("--batch", type=int, default=0,
                    help="c5 only: the first N of its 256 rows (a smaller shard for profiling)")
    ap.add_argument("--shape", default="", help="B,S,HQ,HKV: a same-length bf16 step, block 16")
    ap.add_argument("--head-dim", type=int, default=128, help="with --shape")
    a = ap.parse_args()
    if a.shape:
        b, s, hq, hkv = (int(x) for x in a.shape.split(","))
        nb = (s + 15) // 16
        w = workloads.build(f"b{b}_s{s}_hq{hq}_hkv{hkv}_d{a.head_dim}_bf16", b, hq, hkv, 16,
                            torch.bfloat16, s, nb, b * nb, 1, "cuda", head_dim=a.head_dim)
    elif a.batch and a.config == "c5":
        w = workloads.c5("cuda", batch=a.batch)
    else:
        w = workloads.CONFIGS[a.config]("cuda")
    ws = pa.DecodeWorkspace("cuda")
    wbuf = torch.empty(512 << 20, dtype=torch.uint8, device="cuda") if a.flush else None
    rbuf = torch.ones(128 << 20, dtype=torch.int32, device="cuda") if a.flush else None

    def flush():
        # evict L2 by writing 512 MB, then read 512 MB so no dirty lines remain
        wbuf.fill_(1)
        rbuf.sum(dtype=torch.int64)

    def op():
        return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                  w.block_size, a.num_splits, workspace=ws,
                                  kernel_variant=a.variant)

    op()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.iters):
        if wbuf is not None:
            flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        op()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    ms = sum(times) / len(times)
    print(f"{w.name} variant {a.variant}: {ms * 1e3:.1f} us/launch, {w.effective_bytes() / ms / 1e6:.1f} GB/s, "
          f"status={ws.read_status()}")


if __name__ == "__main__":
    main()
