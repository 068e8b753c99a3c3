"""HBM peak-bandwidth probe: a CUDA streaming copy (and a streaming read).

Drop-in for ``measure_peak_bw.py`` of bw-won/paged-attention-triton
(reference ``measure_peak_bw.py:24-48``): ``measure_peak_bw(size_mb, repeat)``
copies a ``size_mb`` fp16 buffer ``repeat`` times and returns GB/s counted as
read + write bytes. The Triton copy kernel is replaced by ``pa_stream_copy``
from the C ABI: one 32 KB chunk per 256-thread CTA, eight 16-byte loads in
flight per thread before its stores, the grid covering the buffer once (on
B200 ~6.86 TB/s, above a device-to-device ``copy_`` at ~6.55 TB/s).

B200's L2 is 126 MB, so the buffer should be several times that; the
reference's 256 MB default is kept for call compatibility, the CLI default is
1024 MB.

Usage: python measure_peak_bw.py [--size-mb 1024] [--repeat 200] [--read]
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from paged_attention import _native  # noqa: E402


def _time_ms(fn, repeat: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(repeat):
        fn()
    t1.record()
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / repeat


def measure_peak_bw(size_mb: int = 256, repeat: int = 200, block: int = 1024) -> float:
    """Copy bandwidth in GB/s (read + write bytes), ``measure_peak_bw.py:24-48``.

    ``block`` is accepted for signature compatibility; the CUDA copy kernel
    picks its own launch shape.
    """
    n_bytes = size_mb * 1024 * 1024
    src = torch.empty(n_bytes // 2, dtype=torch.float16, device="cuda")
    dst = torch.empty_like(src)
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream

    def run():
        rc = lib.pa_stream_copy(src.data_ptr(), dst.data_ptr(), n_bytes, stream)
        if rc != _native.PA_OK:
            raise _native.PagedAttentionError("pa_stream_copy", rc)

    ms = _time_ms(run, repeat, warmup=min(50, repeat))
    return 2 * n_bytes / (ms * 1e-3) / 1e9


def measure_read_bw(size_mb: int = 1024, repeat: int = 100) -> float:
    """Read-only streaming bandwidth in GB/s (the decode kernel only reads KV)."""
    n_bytes = size_mb * 1024 * 1024
    src = torch.empty(n_bytes // 2, dtype=torch.float16, device="cuda")
    sink = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream

    def run():
        rc = lib.pa_stream_read(src.data_ptr(), n_bytes, sink.data_ptr(), stream)
        if rc != _native.PA_OK:
            raise _native.PagedAttentionError("pa_stream_read", rc)

    ms = _time_ms(run, repeat, warmup=min(20, repeat))
    return n_bytes / (ms * 1e-3) / 1e9


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description="Measure GPU HBM peak bandwidth")
    parser.add_argument("--size-mb", type=int, default=1024, help="Buffer size in MB (>> L2)")
    parser.add_argument("--repeat", type=int, default=200, help="Timing repetitions")
    parser.add_argument("--read", action="store_true", help="also measure read-only bandwidth")
    args = parser.parse_args()
    bw = measure_peak_bw(args.size_mb, args.repeat)
    print(f"copy: {bw:.1f} GB/s  (buffer {args.size_mb} MB, repeat {args.repeat})")
    if args.read:
        print(f"read: {measure_read_bw(args.size_mb, args.repeat):.1f} GB/s")
