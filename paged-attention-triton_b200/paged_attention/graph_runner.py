"""CUDA Graph static-buffer runner for the decode operator.

Drop-in for ``PagedAttnGraphRunner`` of bw-won/paged-attention-triton
(reference ``paged_attention/graph_runner.py:8-45``): zero-filled static q,
caches and block table (``:13-18``), three warm-up calls on a side stream
(``:20-27``), one captured call (``:29-32``), ``run()`` that copies the inputs
in and replays (``:34-41``) and ``replay_only()`` (``:43-45``).

The captured graph holds ONE kernel node (the reference's holds a fill, the
split and the reduce kernels). Its workspace, arrival counters and status word
belong to the runner and are sized before capture; the counters return to
zero at the end of every replay, so nothing needs re-initialising.

Extensions (keyword-only): ``num_kv_heads`` (GQA caches), ``dynamic_seq_lens``
(a static int32 ``[B]`` length buffer, so one graph serves any lengths up to
``max_seq_len``; the reference bakes its scalar ``seq_len`` into the graph),
``num_splits``, ``scale`` and ``return_lse``.
"""
from __future__ import annotations

from typing import Optional

import torch

from .torch_kernel import DecodeWorkspace, paged_attention


class PagedAttnGraphRunner:
    def __init__(self, B, H, DIM, seq_len, block_size, num_phys_blocks, device="cuda",
                 dtype=torch.float16, *, num_kv_heads: Optional[int] = None,
                 dynamic_seq_lens: bool = False, max_seq_len: Optional[int] = None,
                 num_splits: Optional[int] = None, scale: Optional[float] = None,
                 return_lse: bool = False):
        self.seq_len = seq_len
        self.block_size = block_size
        kv_heads = H if num_kv_heads is None else num_kv_heads
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        cap = max_seq_len if max_seq_len is not None else seq_len
        max_blocks = (cap + block_size - 1) // block_size

        # graph_runner.py:13-18: zero-filled so a replay before run() reads valid blocks.
        self.static_q = torch.zeros(B, H, DIM, device=device, dtype=dtype)
        self.static_k = torch.zeros(num_phys_blocks, block_size, kv_heads, DIM, device=device,
                                    dtype=dtype)
        self.static_v = torch.zeros_like(self.static_k)
        self.static_bt = torch.zeros(B, max_blocks, device=device, dtype=torch.int32)
        self.static_seq_lens = (torch.full((B,), seq_len, device=device, dtype=torch.int32)
                                if dynamic_seq_lens else None)
        self.workspace = DecodeWorkspace(device)
        self._num_splits = num_splits
        self._scale = scale
        self._return_lse = return_lse

        lengths = self.static_seq_lens if dynamic_seq_lens else seq_len

        def call():
            return paged_attention(self.static_q, self.static_k, self.static_v, self.static_bt,
                                   lengths, block_size, num_splits, scale=scale,
                                   return_lse=return_lse, workspace=self.workspace)

        # graph_runner.py:20-27: warm up on a side stream (sizes the workspace).
        warmup_stream = torch.cuda.Stream(device=device)
        warmup_stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(warmup_stream):
            for _ in range(3):
                call()
        torch.cuda.current_stream(device).wait_stream(warmup_stream)
        torch.cuda.synchronize(device)

        # graph_runner.py:29-32
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            res = call()
        if return_lse:
            self.static_out, self.static_lse = res
        else:
            self.static_out, self.static_lse = res, None

    def run(self, q, k_cache, v_cache, block_table, copy_kv=False, seq_lens=None):
        """Copy inputs into the static buffers and replay (``graph_runner.py:34-41``)."""
        self.static_q.copy_(q)
        if block_table.shape == self.static_bt.shape:
            self.static_bt.copy_(block_table)
        else:
            self.static_bt.zero_()
            self.static_bt[:, : block_table.shape[1]].copy_(block_table)
        if seq_lens is not None:
            if self.static_seq_lens is None:
                raise ValueError("seq_lens given but the runner was built without dynamic_seq_lens")
            self.static_seq_lens.copy_(seq_lens)
        if copy_kv:
            self.static_k.copy_(k_cache)
            self.static_v.copy_(v_cache)
        self.graph.replay()
        return self.static_out

    def replay_only(self):
        """Pure graph replay with no host-side copy (``graph_runner.py:43-45``)."""
        self.graph.replay()
