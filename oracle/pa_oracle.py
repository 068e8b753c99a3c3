"""FP32 CPU restatement of the reference paged-attention decode algorithm.

TEST INFRASTRUCTURE ONLY: this module is the checker for the CUDA operator and
the timed CPU baseline. The operator itself never imports it.

What it restates (paths are inside the bw-won/paged-attention-triton project):

* ``tests/correctness.py:17-20`` -- ``ref_attention``: scores are
  ``q.float() @ k.float().T * (1/sqrt(D))``, then ``softmax``, then
  ``@ v.float()``. That FP32 gather-then-attend path is the parity oracle.
* ``paged_attention/split_kv_kernel.py:52-66`` -- token ``t`` of sequence
  ``b`` lives at ``cache[block_table[b, t // bs], t % bs, head, :]``.
* ``paged_attention/split_kv_kernel.py:29-33`` and
  ``paged_attention/torch_kernel.py:30`` -- split ``s`` covers tokens
  ``[s*ss, min((s+1)*ss, S))`` with ``ss = ceil(S / num_splits)``; an empty
  split stores nothing, so its LSE keeps the ``-1e30`` fill
  (``torch_kernel.py:34``).
* ``paged_attention/split_kv_kernel.py:79-84`` -- a split stores its
  normalised partial output and ``LSE = m + log(max(l, 1e-20))``.
* ``paged_attention/split_kv_kernel.py:101-122`` -- the reduce skips splits
  with ``lse <= -1e29``, merges the rest by running max, and divides by
  ``max(sum, 1e-20)`` (so a row with no valid split outputs exactly 0).
* ``paged_attention/torch_kernel.py:19-25`` -- the ``num_splits`` heuristic.

Extensions beyond the reference, matching the CUDA operator's superset API:
per-sequence ``seq_lens`` (ragged batches), grouped-query attention with
``kv_head = q_head // (Hq // Hkv)``, an explicit ``scale``, and the final
``LSE = logsumexp(scaled scores)`` per query head (``-1e30`` for an empty row).

Pinned against the reference's own Triton kernels, run on CPU by the Triton
interpreter, through the fixtures in ``tests/golden`` (see
``tests/golden/make_golden.py`` and ``tests/test_oracle.py``).
"""
from __future__ import annotations

import math
from typing import Optional, Sequence, Tuple, Union

import torch

# paged_attention/split_kv_kernel.py:8-9
LSE_SENTINEL = -1e30
LSE_VALID_THRESHOLD = -1e29

SeqLens = Union[int, Sequence[int], torch.Tensor]


def _seq_list(seq_lens: SeqLens, batch: int) -> list:
    if isinstance(seq_lens, int):
        return [int(seq_lens)] * batch
    if isinstance(seq_lens, torch.Tensor):
        return [int(x) for x in seq_lens.detach().cpu().reshape(-1).tolist()]
    return [int(x) for x in seq_lens]


def num_splits_heuristic(batch: int, heads: int, seq_len: int, block_size: int,
                         sm_count: int) -> int:
    """``paged_attention/torch_kernel.py:19-25`` with an explicit SM count."""
    target_programs = sm_count * 4
    return max(1, min((seq_len + block_size - 1) // block_size,
                      max(1, target_programs // (batch * heads))))


def gather_sequence(cache: torch.Tensor, block_table_row: torch.Tensor,
                    seq_len: int, block_size: int) -> torch.Tensor:
    """Token rows ``[S, Hkv, D]`` of one sequence, walked through its block table.

    ``split_kv_kernel.py:52-58``: logical block ``t // bs``, slot ``t % bs``.
    """
    if seq_len == 0:
        return cache.new_zeros((0,) + tuple(cache.shape[2:]))
    nblk = (seq_len + block_size - 1) // block_size
    phys = block_table_row[:nblk].long()
    rows = cache[phys]                      # [nblk, bs, Hkv, D]
    return rows.reshape(nblk * block_size, *cache.shape[2:])[:seq_len]


def _attend(q_b: torch.Tensor, k_rows: torch.Tensor, v_rows: torch.Tensor,
            scale: float, acc_dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """One sequence: q ``[Hq, D]``, K/V rows ``[S, Hkv, D]`` -> O ``[Hq, D]``, LSE ``[Hq]``.

    ``tests/correctness.py:17-20``: FP32 matmul -> softmax -> matmul, with the
    query heads of one KV head grouped (``Hq = Hkv * G``).
    """
    hq, d = q_b.shape
    s_len, hkv, _ = k_rows.shape
    g = hq // hkv
    q = q_b.to(acc_dtype).reshape(hkv, g, d)                 # [Hkv, G, D]
    k = k_rows.to(acc_dtype).permute(1, 2, 0)                # [Hkv, D, S]
    v = v_rows.to(acc_dtype).permute(1, 0, 2)                # [Hkv, S, D]
    s = torch.matmul(q, k) * scale                           # [Hkv, G, S]
    lse = torch.logsumexp(s, dim=-1)                         # [Hkv, G]
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, v)                                   # [Hkv, G, D]
    return o.reshape(hq, d), lse.reshape(hq)


def decode_reference(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     block_table: torch.Tensor, seq_lens: SeqLens, block_size: int,
                     scale: Optional[float] = None,
                     acc_dtype: torch.dtype = torch.float32,
                     batch_indices: Optional[Sequence[int]] = None
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Final output ``O [B, Hq, D]`` and ``LSE [B, Hq]`` in ``acc_dtype`` (CPU).

    ``batch_indices`` restricts the work to some sequences (the other rows stay
    zero / sentinel), so huge batches can be checked on a sample.
    """
    q = q.detach().cpu()
    k_cache = k_cache.detach().cpu()
    v_cache = v_cache.detach().cpu()
    block_table = block_table.detach().cpu()
    b_sz, hq, d = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)           # split_kv_kernel.py:40
    lens = _seq_list(seq_lens, b_sz)
    out = torch.zeros(b_sz, hq, d, dtype=acc_dtype)
    lse = torch.full((b_sz, hq), LSE_SENTINEL, dtype=acc_dtype)
    rows = range(b_sz) if batch_indices is None else batch_indices
    for b in rows:
        s_len = lens[b]
        if s_len == 0:
            continue                          # no valid split -> O = 0 (split_kv_kernel.py:120)
        k_rows = gather_sequence(k_cache, block_table[b], s_len, block_size)
        v_rows = gather_sequence(v_cache, block_table[b], s_len, block_size)
        o_b, l_b = _attend(q[b], k_rows, v_rows, scale, acc_dtype)
        out[b] = o_b
        lse[b] = l_b
    return out, lse


def split_partials(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   block_table: torch.Tensor, seq_lens: SeqLens, block_size: int,
                   num_splits: int, scale: Optional[float] = None,
                   acc_dtype: torch.dtype = torch.float32
                   ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-split ``O_partial [B, Hq, ns, D]`` and ``LSE_partial [B, Hq, ns]``.

    Split ``s`` of sequence ``b`` covers ``[s*ss_b, min((s+1)*ss_b, S_b))`` with
    ``ss_b = ceil(S_b / ns)`` (``torch_kernel.py:30``; per sequence for ragged
    batches). Empty splits keep ``LSE = -1e30`` and a zero partial output.
    """
    q = q.detach().cpu()
    k_cache = k_cache.detach().cpu()
    v_cache = v_cache.detach().cpu()
    block_table = block_table.detach().cpu()
    b_sz, hq, d = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    lens = _seq_list(seq_lens, b_sz)
    o_p = torch.zeros(b_sz, hq, num_splits, d, dtype=acc_dtype)
    lse_p = torch.full((b_sz, hq, num_splits), LSE_SENTINEL, dtype=acc_dtype)
    for b in range(b_sz):
        s_len = lens[b]
        if s_len == 0:
            continue
        ss = (s_len + num_splits - 1) // num_splits
        k_rows = gather_sequence(k_cache, block_table[b], s_len, block_size)
        v_rows = gather_sequence(v_cache, block_table[b], s_len, block_size)
        for s in range(num_splits):
            lo, hi = s * ss, min((s + 1) * ss, s_len)
            if lo >= hi:
                continue                      # split_kv_kernel.py:32-33
            o_s, l_s = _attend(q[b], k_rows[lo:hi], v_rows[lo:hi], scale, acc_dtype)
            o_p[b, :, s] = o_s
            lse_p[b, :, s] = l_s
    return o_p, lse_p


def reduce_partials(o_p: torch.Tensor, lse_p: torch.Tensor
                    ) -> Tuple[torch.Tensor, torch.Tensor]:
    """``split_kv_kernel.py:101-122`` over ``[B, Hq, ns, D]`` partials (FP32).

    Returns ``O [B, Hq, D]`` and the final ``LSE [B, Hq]`` (``g_max + log(g_sum)``,
    or ``-1e30`` when every split of a row is empty).
    """
    o_p = o_p.float()
    lse_p = lse_p.float()
    b_sz, hq, ns, d = o_p.shape
    g_max = torch.full((b_sz, hq), LSE_VALID_THRESHOLD, dtype=torch.float32)
    g_sum = torch.zeros(b_sz, hq, dtype=torch.float32)
    g_acc = torch.zeros(b_sz, hq, d, dtype=torch.float32)
    for s in range(ns):
        lse = lse_p[:, :, s]
        valid = lse > LSE_VALID_THRESHOLD
        new_max = torch.where(valid, torch.maximum(g_max, lse), g_max)
        alpha_old = torch.where(valid, torch.exp(g_max - new_max), torch.ones_like(g_max))
        alpha_new = torch.where(valid, torch.exp(lse - new_max), torch.zeros_like(g_max))
        g_acc = g_acc * alpha_old[..., None] + alpha_new[..., None] * o_p[:, :, s]
        g_sum = g_sum * alpha_old + alpha_new
        g_max = new_max
    out = g_acc / torch.clamp(g_sum, min=1e-20)[..., None]
    lse_final = torch.where(g_sum > 0, g_max + torch.log(torch.clamp(g_sum, min=1e-20)),
                            torch.full_like(g_max, LSE_SENTINEL))
    return out, lse_final


def effective_bytes(seq_lens: SeqLens, batch: int, num_heads: int, num_kv_heads: int,
                    head_dim: int, elem_bytes: int) -> int:
    """Algorithmic bytes of one decode step.

    Generalises ``tests/benchmark_core.py:64-66`` (``kv = B*H*S*D*e*2``,
    ``qo = B*H*D*e*2``) to ragged lengths and GQA: K+V bytes use the KV heads,
    q+o bytes the query heads. Block tables, LSE and partials are excluded.
    """
    lens = _seq_list(seq_lens, batch)
    kv = sum(lens) * num_kv_heads * head_dim * elem_bytes * 2
    qo = batch * num_heads * head_dim * elem_bytes * 2
    return kv + qo
