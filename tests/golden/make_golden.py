"""Generate the golden fixtures in this folder from the reference implementation.

Run from the repository root, in a container that has the reference checked out
(read-only), giving the path of that checkout:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference package ``paged_attention`` and runs its own Triton
kernels on CPU through the Triton interpreter (``TRITON_INTERPRET=1``), with an
explicit ``num_splits`` so the GPU-only SM-count query
(``paged_attention/torch_kernel.py:20``) is never reached. For every case it
stores the seeded inputs and three reference outputs:

* ``o_ref``: ``paged_attention(...)`` (``paged_attention/torch_kernel.py:71-73``),
* ``o_partial`` / ``lse_partial``: the split kernel's per-split outputs, produced
  by launching ``paged_attention_split_kernel`` exactly as
  ``paged_attention/torch_kernel.py:32-51`` does (sentinel-filled LSE buffer,
  grid ``(B*H, ns)``), so empty splits keep ``-1e30``.

fp16/bf16 tensors are stored as their raw 16-bit patterns (``uint16``) next to
a ``dtype`` string. Nothing on a GPU box runs this script; the fixtures travel.
"""
from __future__ import annotations

import os
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))

# name, seed, dtype, B, H, S, block_size, pool blocks, num_splits, table[, head_dim]
CASES = [
    ("mha_f16_b2_s100_bs16_ns3", 1, "float16", 2, 2, 100, 16, 16, 3, "shuffle"),
    ("mha_f16_s9_bs16_ns4_empty_split", 2, "float16", 1, 2, 9, 16, 4, 4, "shuffle"),
    ("mha_bf16_s200_bs32_ns5", 3, "bfloat16", 1, 2, 200, 32, 10, 5, "shuffle"),
    ("mha_f16_s300_bs128_ns2", 4, "float16", 1, 1, 300, 128, 4, 2, "shuffle"),
    ("mha_f16_s1_bs16_ns1", 5, "float16", 2, 2, 1, 16, 4, 1, "shuffle"),
    ("mha_f16_b2_s77_bs8_ns7", 6, "float16", 2, 1, 77, 8, 24, 7, "shuffle"),
    ("mha_bf16_s64_bs16_ns8_scaled_block", 7, "bfloat16", 1, 2, 64, 16, 8, 8, "shuffle"),
    # tests/correctness.py:9-36 style: seed 42, identity block table, heuristic
    # num_splits for a 148-SM part (min(ceil(256/16), 148*4 // (1*4)) = 16).
    ("correctness_f16_b1_h4_s256_bs16_identity", 42, "float16", 1, 4, 256, 16, 16, 16, "identity"),
    # head dimensions other than 128 (the reference kernel takes D as a constexpr)
    ("mha_f16_d64_b2_s100_bs16_ns3", 11, "float16", 2, 2, 100, 16, 16, 3, "shuffle", 64),
    ("mha_bf16_d64_s9_bs8_ns4_empty_split", 12, "bfloat16", 1, 2, 9, 8, 4, 4, "shuffle", 64),
    ("mha_f16_d256_s130_bs16_ns3", 13, "float16", 1, 2, 130, 16, 12, 3, "shuffle", 256),
    ("mha_bf16_d256_b2_s40_bs32_ns2", 14, "bfloat16", 2, 1, 40, 32, 6, 2, "shuffle", 256),
    # pages of 1, 2 and 4 tokens and head_dim 32 (any power of two is a valid
    # tl.arange bound in the reference, split_kv_kernel.py:38,49)
    ("mha_f16_b2_s50_bs4_ns3", 21, "float16", 2, 2, 50, 4, 32, 3, "shuffle"),
    ("mha_bf16_s23_bs2_ns4", 22, "bfloat16", 1, 2, 23, 2, 16, 4, "shuffle"),
    ("mha_f16_s7_bs1_ns2", 23, "float16", 1, 2, 7, 1, 10, 2, "shuffle"),
    ("mha_f16_d32_b2_s70_bs16_ns2", 24, "float16", 2, 2, 70, 16, 12, 2, "shuffle", 32),
    ("mha_bf16_d32_s9_bs4_ns4_empty_split", 25, "bfloat16", 1, 2, 9, 4, 4, 4, "shuffle", 32),
]


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def make_case(ref_pkg, name, seed, dtype_name, b, h, s, bs, pool, ns, table, d=128):
    from paged_attention import paged_attention  # reference package
    from paged_attention.split_kv_kernel import (
        paged_attention_split_kernel, LSE_SENTINEL)

    dtype = getattr(torch, dtype_name)
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, d, generator=g).to(dtype)
    k = torch.randn(pool, bs, h, d, generator=g).to(dtype)
    v = torch.randn(pool, bs, h, d, generator=g).to(dtype)
    nblk = (s + bs - 1) // bs
    if table == "identity":
        bt = torch.arange(b * nblk, dtype=torch.int32).reshape(b, nblk)
    else:
        bt = torch.randperm(pool, generator=g)[: b * nblk].reshape(b, nblk).to(torch.int32)
    if "scaled_block" in name:
        blk = int(bt[0, int(torch.randint(0, nblk, (1,), generator=g))])
        k[blk] = (k[blk].float() * 8).to(dtype)

    o_ref = paged_attention(q, k, v, bt, s, bs, ns)

    split_size = (s + ns - 1) // ns
    # zero-filled so the rows of empty splits (never written) are reproducible
    o_part = torch.zeros(b, h, ns, d, dtype=torch.float16)
    lse_part = torch.empty(b, h, ns, dtype=torch.float32)
    lse_part.fill_(LSE_SENTINEL)
    paged_attention_split_kernel[(b * h, ns)](
        q, k, v, bt, o_part, lse_part,
        q.stride(0), q.stride(1), q.stride(2),
        k.stride(0), k.stride(1), k.stride(2), k.stride(3),
        v.stride(0), v.stride(1), v.stride(2), v.stride(3),
        o_part.stride(0), o_part.stride(1), o_part.stride(2), o_part.stride(3),
        lse_part.stride(0), lse_part.stride(1), lse_part.stride(2),
        h, s, split_size, bt.shape[1], d, bs, bs,
        num_warps=4, num_stages=3,
    )
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(
        path, dtype=np.array(dtype_name), seq_len=np.array(s), block_size=np.array(bs),
        num_splits=np.array(ns), seed=np.array(seed),
        q=_bits(q), k_cache=_bits(k), v_cache=_bits(v), block_table=bt.numpy(),
        o_ref=_bits(o_ref), o_partial=_bits(o_part), lse_partial=lse_part.numpy())
    print(f"wrote {path}")


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    ref = sys.argv[1]
    sys.path.insert(0, ref)
    for case in CASES:
        make_case(ref, *case)


if __name__ == "__main__":
    main()
