"""PyTorch entry point of the paged-attention decode operator.

Drop-in for ``paged_attention/torch_kernel.py`` of bw-won/paged-attention-triton:
``paged_attention(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size,
num_splits=None)`` (reference ``torch_kernel.py:71-73``) returns ``O`` with the
shape and dtype of ``Q``; ``PagedAttentionV2Function`` keeps the reference's
autograd wrapper whose backward raises (``torch_kernel.py:66-68``).

Underneath is one launch of the sm_100a kernel through the C ABI
(``include/pa_decode.h``), made by a thin C++ extension (``_pa_ext``, built from
``csrc/torch_ext.cpp``) on the current CUDA stream, with no host sync, no
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

HEAD_DIMS = (32, 64, 128, 256)   # head dimensions the kernels are built for

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


def _raw_stream(idx: int) -> int:
    getter = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    return getter(idx) if getter is not None else torch.cuda.current_stream(idx).cuda_stream


def default_workspace(device: torch.device) -> DecodeWorkspace:
    """The workspace of the current stream on ``device`` (created on first use)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    stream = _raw_stream(idx)
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
    # Argument checks, allocation of the outputs and the launch happen in C++
    # (paged_attention/_pa_ext, csrc/torch_ext.cpp) over the C ABI.
    if not (Q.is_cuda and K_Cache.is_cuda and V_Cache.is_cuda and Block_Table.is_cuda):
        raise ValueError("paged_attention: Q, K_Cache, V_Cache and Block_Table must be CUDA tensors")
    ws = workspace if workspace is not None else default_workspace(Q.device)
    if isinstance(seq_len, torch.Tensor):
        seq_t, seq_i = seq_len, 0
    else:
        seq_t, seq_i = None, int(seq_len)
    ns = 0 if num_splits is None else int(num_splits)
    args = (Q, K_Cache, V_Cache, Block_Table, seq_t, seq_i, int(block_size), ns,
            0.0 if scale is None else float(scale), bool(return_lse), bool(return_partials))
    ext = _native.ext()
    status, res, need_bytes, need_counters = ext.decode(
        *args, ws.buffer, ws.counters, ws.status, int(kernel_variant), out)
    if status != 0:
        ws.ensure(need_bytes, need_counters)
        status, res, _, _ = ext.decode(*args, ws.buffer, ws.counters, ws.status,
                                       int(kernel_variant), out)
        if status != 0:
            raise PagedAttentionError("pa_decode", _native.PA_ERR_WORKSPACE)
    return res[0] if len(res) == 1 else tuple(res)


def decode_params(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits=None, *,
                  scale=None, out=None, lse=None, kernel_variant=0) -> DecodeParams:
    """``pa_decode_params`` for these tensors (the C ABI's argument struct), for
    callers that go through ``ctypes`` (``_native.lib()``) instead of the
    extension: device pointers, element strides, shapes and the lengths."""
    p = DecodeParams()
    p.q = Q.data_ptr()
    p.q_stride_b, p.q_stride_h = Q.stride(0), Q.stride(1)
    p.k_cache = K_Cache.data_ptr()
    p.k_stride_block, p.k_stride_slot, p.k_stride_head = K_Cache.stride()[:3]
    p.v_cache = V_Cache.data_ptr()
    p.v_stride_block, p.v_stride_slot, p.v_stride_head = V_Cache.stride()[:3]
    p.block_table = Block_Table.data_ptr()
    p.bt_stride_b = Block_Table.stride(0)
    p.max_blocks = Block_Table.shape[1]
    if isinstance(seq_len, torch.Tensor):
        p.seq_lens, p.seq_len = seq_len.data_ptr(), 0
    else:
        p.seq_lens, p.seq_len = None, int(seq_len)
    p.batch, p.num_heads, p.head_dim = Q.shape
    p.num_kv_heads = K_Cache.shape[2]
    p.block_size, p.num_blocks = int(block_size), K_Cache.shape[0]
    p.num_splits = 0 if num_splits is None else int(num_splits)
    p.scale = (1.0 / math.sqrt(Q.shape[2])) if scale is None else float(scale)
    p.dtype = _DTYPES[Q.dtype]
    if out is not None:
        p.out = out.data_ptr()
        p.out_stride_b, p.out_stride_h = out.stride(0), out.stride(1)
    if lse is not None:
        p.lse = lse.data_ptr()
    p.kernel_variant = int(kernel_variant)
    return p


def decode_plan(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits=None, *,
                kernel_variant=0) -> dict:
    """The schedule one ``paged_attention`` call runs on Q's device
    (``pa_decode_plan``): kernel variant, grid, merge groups, whether the merge
    pass follows the decode kernel, and the workspace it needs."""
    p = decode_params(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size, num_splits,
                      kernel_variant=kernel_variant)
    info = _native.PlanInfo()
    with torch.cuda.device(Q.device):
        rc = _native.lib().pa_decode_plan(ctypes.byref(p), ctypes.byref(info))
    if rc != _native.PA_OK:
        raise PagedAttentionError("pa_decode_plan", rc)
    return {name: getattr(info, name) for name, _ in info._fields_}


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
