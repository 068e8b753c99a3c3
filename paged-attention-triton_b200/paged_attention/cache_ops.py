"""Writing new tokens into the paged KV cache (the step before decode).

The reference fills its caches in test code (``tests/correctness.py:30-36``:
``K_cache[idx] = K_full[0, :, s:e].permute(1, 0, 2)`` per logical block); a
serving loop instead writes each step's new K/V rows into their slots. This
module does that with one CUDA launch (``pa_cache_append`` in the C ABI).

Slots follow vLLM's ``slot_mapping`` convention: token row t goes to
``cache[slot // block_size, slot % block_size]``; a negative slot skips the row.
"""
from __future__ import annotations

import torch

from . import _native


def write_kv_cache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                   v_cache: torch.Tensor, slot_mapping: torch.Tensor,
                   status: torch.Tensor = None) -> None:
    """Copy rows ``key[t], value[t]`` (``[T, Hkv, D]``) into both caches at
    ``slot_mapping[t]`` (int64, device; int32 is widened). In place, async on
    the current stream."""
    if slot_mapping.dtype != torch.int64:
        slot_mapping = slot_mapping.to(torch.int64)
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    _native.ext().cache_append(key, value, k_cache, v_cache, slot_mapping, status)


def slots_for_positions(block_table: torch.Tensor, positions: torch.Tensor,
                        block_size: int) -> torch.Tensor:
    """Slot of token ``positions[b]`` of sequence b through its block table
    (``split_kv_kernel.py:52-58``: block ``pos // bs``, offset ``pos % bs``);
    negative positions give slot -1."""
    pos = positions.to(torch.int64)
    valid = pos >= 0
    safe = torch.where(valid, pos, torch.zeros_like(pos))
    rows = torch.arange(block_table.shape[0], device=block_table.device)
    blocks = block_table[rows, (safe // block_size)].to(torch.int64)
    slots = blocks * block_size + safe % block_size
    return torch.where(valid, slots, torch.full_like(slots, -1))
