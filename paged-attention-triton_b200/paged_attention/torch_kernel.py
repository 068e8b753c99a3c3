"""PyTorch entry point of the paged-attention decode operator.

Drop-in for ``paged_attention/torch_kernel.py`` of bw-won/paged-attention-triton:
``paged_attention(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size,
num_splits=None)`` (reference ``torch_kernel.py:71-73``) returns ``O`` with the
shape and dtype of ``Q``; ``PagedAttentionV2Function`` keeps the reference's
autograd wrapper whose backward raises (``torch_kernel.py:66-68``).

Underneath is one launch of the sm_100a kernel through the C ABI
(``include/pa_decode.h``), on the current CUDA stream, with no host sync, no
Triton and no CPU fallback.

Superset of the reference API (keyword-only extensions):

* ``seq_len`` may be an ``int`` (reference) or an int32 tensor ``[B]`` of
  per-sequence lengths on the device (ragged batches, graph-replayable).
* ``scale`` (default ``1/sqrt(D)``, the reference's hard-coded value,
  ``split_kv_kernel.py:40``).
* grouped-query attention: ``Hkv = K_Cache.shape[2]`` must divide ``Hq``;
  query head ``h`` reads KV head ``h // (Hq // Hkv)``.
* ``return_lse=True`` also returns the final ``LSE [B, Hq]`` (fp32, natural
  log of the scaled scores; ``-1e30`` for a zero-length row).
* ``return_partials=True`` runs the reference's split schedule and also
  returns ``O_partial [B, Hq, ns, D]`` / ``LSE_partial [B, Hq, ns]`` (fp32;
  empty splits hold LSE ``-1e30``, ``split_kv_kernel.py:7-9,32-33``).
* ``num_splits``: ``None`` or ``0`` selects the token-balanced persistent
  schedule; a positive value selects the reference's split schedule
  (``ns`` equal token ranges per sequence, ``torch_kernel.py:30``).
"""
from __future__ import annotations

import ctypes
import math
import threading
from typing import Dict, Optional, Tuple, Union

import torch

from . import _native
from ._native import DecodeParams, PagedAttentionError
from .split_kv_kernel import LSE_SENTINEL  # noqa: F401  (re-exported constant)

HEAD_DIM = 128

_DTYPES = {torch.float16: _native.PA_F16, torch.bfloat16: _native.PA_BF16}


class DecodeWorkspace:
    """Scratch memory of one stream of decode calls.

    * ``buffer``: partial outputs (size queried from the C ABI per shape),
    * ``counters``: int32 arrival counters, zero-filled once; every launch
      leaves them zero again, so a captured graph can replay without a memset,
    * ``status``: a device word the kernel ORs ``PA_STATUS_*`` bits into.

    Growing reallocates, so a CUDA-graph caller sizes it before capture (the
    graph runner does this in its warm-up).
    """

    def __init__(self, device: Union[torch.device, str, int]):
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.buffer = torch.empty(0, dtype=torch.uint8, device=self.device)
        self.counters = torch.zeros(0, dtype=torch.int32, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

    def ensure(self, nbytes: int, ncounters: int) -> None:
        if nbytes > self.buffer.numel():
            self.buffer = torch.empty(max(nbytes, 2 * self.buffer.numel()), dtype=torch.uint8,
                                      device=self.device)
        if ncounters > self.counters.numel():
            self.counters = torch.zeros(max(ncounters, 2 * self.counters.numel()),
                                        dtype=torch.int32, device=self.device)

    def read_status(self) -> int:
        """Host read of the status word (synchronises the device)."""
        return int(self.status.item())

    def reset(self) -> None:
        """Zero the counters and the status word (after a flagged timeout)."""
        self.counters.zero_()
        self.status.zero_()


_ws_lock = threading.Lock()
_workspaces: Dict[Tuple[int, int], DecodeWorkspace] = {}
_sm_counts: Dict[int, int] = {}


def default_workspace(device: torch.device) -> DecodeWorkspace:
    """The workspace of the current stream on ``device`` (created on first use)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    stream = torch.cuda.current_stream(idx).cuda_stream
    key = (idx, stream)
    ws = _workspaces.get(key)
    if ws is None:
        with _ws_lock:
            ws = _workspaces.get(key)
            if ws is None:
                ws = DecodeWorkspace(torch.device("cuda", idx))
                _workspaces[key] = ws
    return ws


def device_sm_count(device: torch.device) -> int:
    """SM count of ``device`` (the reference reads device 0, ``torch_kernel.py:20``)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = torch.cuda.get_device_properties(idx).multi_processor_count
        _sm_counts[idx] = n
    return n


def num_splits_heuristic(batch: int, heads: int, seq_len: int, block_size: int,
                         sm_count: int) -> int:
    """``torch_kernel.py:19-25``: ``max(1, min(ceil(S/bs), max(1, 4*SM // (B*H))))``."""
    return int(_native.lib().pa_num_splits_heuristic(batch, heads, seq_len, block_size, sm_count))


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _decode(Q: torch.Tensor, K_Cache: torch.Tensor, V_Cache: torch.Tensor,
            Block_Table: torch.Tensor, seq_len: Union[int, torch.Tensor], block_size: int,
            num_splits: Optional[int] = None, scale: Optional[float] = None,
            return_lse: bool = False, return_partials: bool = False,
            workspace: Optional[DecodeWorkspace] = None, out: Optional[torch.Tensor] = None,
            kernel_variant: int = 0):
    _check(Q.is_cuda and K_Cache.is_cuda and V_Cache.is_cuda and Block_Table.is_cuda,
           "paged_attention: Q, K_Cache, V_Cache and Block_Table must be CUDA tensors")
    _check(Q.dim() == 3, "paged_attention: Q must be [B, H, D]")
    _check(K_Cache.dim() == 4 and V_Cache.shape == K_Cache.shape,
           "paged_attention: K_Cache and V_Cache must both be [num_blocks, block_size, Hkv, D]")
    _check(Q.dtype in _DTYPES, f"paged_attention: unsupported dtype {Q.dtype} (fp16 or bf16)")
    _check(K_Cache.dtype == Q.dtype and V_Cache.dtype == Q.dtype,
           "paged_attention: Q, K_Cache and V_Cache must share one dtype")
    _check(Block_Table.dtype == torch.int32 and Block_Table.dim() == 2,
           "paged_attention: Block_Table must be an int32 [B, max_blocks] tensor")
    _check(K_Cache.device == Q.device and V_Cache.device == Q.device
           and Block_Table.device == Q.device, "paged_attention: tensors on different devices")
    batch, heads, dim = Q.shape
    nblocks, bs, kv_heads, kdim = K_Cache.shape
    _check(dim == kdim, "paged_attention: head_dim of Q and the caches differ")
    _check(dim == HEAD_DIM, f"paged_attention: head_dim {dim} is not built (only {HEAD_DIM})")
    _check(int(block_size) == bs, f"paged_attention: block_size {block_size} != cache block {bs}")
    _check(bs % 8 == 0, f"paged_attention: block_size {bs} is not a multiple of 8")
    _check(heads % kv_heads == 0, f"paged_attention: Hq={heads} is not a multiple of Hkv={kv_heads}")
    _check(Block_Table.shape[0] == batch, "paged_attention: Block_Table rows != batch")
    _check(Q.stride(2) == 1 and K_Cache.stride(3) == 1 and V_Cache.stride(3) == 1
           and Block_Table.stride(1) == 1, "paged_attention: last dimensions must be contiguous")
    if Q.stride(1) % 8 or Q.stride(0) % 8 or Q.data_ptr() % 16:
        Q = Q.contiguous()
    max_blocks = Block_Table.shape[1]

    seq_ptr = None
    seq_scalar = 0
    if isinstance(seq_len, torch.Tensor):
        _check(seq_len.numel() == batch, "paged_attention: seq_lens must have B entries")
        if seq_len.device != Q.device or seq_len.dtype != torch.int32 or not seq_len.is_contiguous():
            seq_len = seq_len.to(device=Q.device, dtype=torch.int32).contiguous()
        seq_ptr = seq_len.data_ptr()
    else:
        seq_scalar = int(seq_len)
        _check(0 <= seq_scalar <= max_blocks * bs,
               f"paged_attention: seq_len {seq_scalar} exceeds Block_Table capacity {max_blocks * bs}")

    if scale is None:
        scale = 1.0 / math.sqrt(dim)
    ns = 0 if num_splits is None else int(num_splits)
    _check(ns >= 0, "paged_attention: num_splits must be >= 0")
    if return_partials and ns == 0:
        s_for_heur = seq_scalar if seq_ptr is None else max_blocks * bs
        ns = num_splits_heuristic(batch, heads, s_for_heur, bs, device_sm_count(Q.device))

    if out is None:
        out = torch.empty((batch, heads, dim), dtype=Q.dtype, device=Q.device)
    lse = torch.empty((batch, heads), dtype=torch.float32, device=Q.device) if return_lse else None
    o_part = lse_part = None
    if return_partials:
        o_part = torch.empty((batch, heads, ns, dim), dtype=torch.float32, device=Q.device)
        lse_part = torch.empty((batch, heads, ns), dtype=torch.float32, device=Q.device)

    ws = workspace if workspace is not None else default_workspace(Q.device)
    p = DecodeParams()
    p.q = Q.data_ptr()
    p.q_stride_b, p.q_stride_h = Q.stride(0), Q.stride(1)
    p.k_cache = K_Cache.data_ptr()
    p.k_stride_block, p.k_stride_slot, p.k_stride_head = K_Cache.stride(0), K_Cache.stride(1), K_Cache.stride(2)
    p.v_cache = V_Cache.data_ptr()
    p.v_stride_block, p.v_stride_slot, p.v_stride_head = V_Cache.stride(0), V_Cache.stride(1), V_Cache.stride(2)
    p.block_table = Block_Table.data_ptr()
    p.bt_stride_b = Block_Table.stride(0)
    p.max_blocks = max_blocks
    p.seq_lens = seq_ptr
    p.seq_len = seq_scalar
    p.batch, p.num_heads, p.num_kv_heads = batch, heads, kv_heads
    p.head_dim, p.block_size, p.num_blocks = dim, bs, nblocks
    p.num_splits = ns
    p.scale = float(scale)
    p.dtype = _DTYPES[Q.dtype]
    p.out = out.data_ptr()
    p.out_stride_b, p.out_stride_h = out.stride(0), out.stride(1)
    p.lse = lse.data_ptr() if lse is not None else None
    p.o_partial = o_part.data_ptr() if o_part is not None else None
    p.lse_partial = lse_part.data_ptr() if lse_part is not None else None
    p.kernel_variant = int(kernel_variant)

    lib = _native.lib()
    ws_bytes = ctypes.c_size_t(0)
    n_counters = ctypes.c_size_t(0)
    rc = lib.pa_decode_workspace(ctypes.byref(p), ctypes.byref(ws_bytes), ctypes.byref(n_counters))
    if rc != _native.PA_OK:
        raise PagedAttentionError("pa_decode_workspace", rc)
    ws.ensure(ws_bytes.value, n_counters.value)
    p.workspace = ws.buffer.data_ptr() if ws.buffer.numel() else None
    p.workspace_bytes = ws.buffer.numel()
    p.counters = ws.counters.data_ptr()
    p.counter_count = ws.counters.numel()
    p.status = ws.status.data_ptr()

    stream = torch.cuda.current_stream(Q.device).cuda_stream
    rc = lib.pa_decode(ctypes.byref(p), stream)
    if rc != _native.PA_OK:
        raise PagedAttentionError("pa_decode", rc)

    if not (return_lse or return_partials):
        return out
    res = (out,)
    if return_lse:
        res += (lse,)
    if return_partials:
        res += (o_part, lse_part)
    return res


class PagedAttentionV2Function(torch.autograd.Function):
    """Reference-named autograd wrapper (``torch_kernel.py:13-68``); inference only."""

    @staticmethod
    def forward(ctx, Q, K_Cache, V_Cache, Block_Table, seq_len, block_size,
                num_splits=None, block_n=None):
        # block_n (the reference's Triton tile, torch_kernel.py:27-28) has no
        # meaning for the CUDA kernel, which always streams 32-token tiles.
        return _decode(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits)

    @staticmethod
    def backward(ctx, grad_output):
        raise RuntimeError("PagedAttentionV2 is inference-only.")


def paged_attention(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits=None, *,
                    scale=None, return_lse=False, return_partials=False, workspace=None, out=None,
                    kernel_variant=0):
    """Decode attention of one new token per sequence over a paged KV cache.

    Reference signature: ``paged_attention/torch_kernel.py:71-73``.
    ``kernel_variant`` (0 = automatic) pins one tile/warp/stage variant of the
    CUDA kernel; it exists for tuning and tests.
    """
    if torch.is_grad_enabled() and (Q.requires_grad or K_Cache.requires_grad
                                    or V_Cache.requires_grad):
        if scale is None and not return_lse and not return_partials:
            return PagedAttentionV2Function.apply(Q, K_Cache, V_Cache, Block_Table, seq_len,
                                                  block_size, num_splits)
        raise RuntimeError("PagedAttentionV2 is inference-only.")
    return _decode(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits, scale,
                   return_lse, return_partials, workspace, out, kernel_variant)
