"""Seeded synthetic decode workloads (the five benchmark shapes).

Each builder returns a ``Workload`` whose tensors live on ``device``:
q ``[B, Hq, D]``, paged caches ``[num_blocks, block_size, Hkv, D]``, an int32
block table ``[B, max_blocks]`` mapping logical to shuffled physical blocks,
and either a uniform ``seq_len`` (int) or per-row ``seq_lens`` (int32 ``[B]``).
All values are i.i.d. N(0, 1) from ``torch.Generator`` seeds, scale is
``1/sqrt(128)``. There is no public dataset behind these shapes.

* ``c1``: B=1, Hq=Hkv=32, fp16, S=128, block 16, 8 blocks permuted into a
  pool of 64 (the unused 56 hold noise too).
* ``c2``: B=32, Hq=Hkv=32, fp16, S=1024, block 16, pool 2048 = 32 x 64, all
  used, seeded shuffle.
* ``c3``: B=1, Hq=Hkv=32, bf16, S=4096, block 128, 32 blocks from a pool of
  256; the K rows of one random block are scaled by 8.
* ``c4``: B=128, Hq=32 / Hkv=8, bf16, block 16, S ~ U[1, 256], block table
  padded to 16, pool 4096.
* ``c5``: B=256, Hq=64 / Hkv=8, bf16, block 16, S log-uniform in
  [512, 32768], block table padded to 2048; ``shard(rank, world)`` keeps KV heads
  ``[r*8/N, (r+1)*8/N)`` and their query heads, each rank with its own pool.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Union

import torch

HEAD_DIM = 128


@dataclass
class Workload:
    name: str
    q: torch.Tensor
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    block_table: torch.Tensor
    seq_len: Union[int, torch.Tensor]
    block_size: int
    num_kv_heads: int
    seed: int

    @property
    def batch(self) -> int:
        return self.q.shape[0]

    @property
    def num_heads(self) -> int:
        return self.q.shape[1]

    @property
    def dtype(self) -> torch.dtype:
        return self.q.dtype

    def seq_list(self) -> list:
        if isinstance(self.seq_len, int):
            return [self.seq_len] * self.batch
        return [int(x) for x in self.seq_len.cpu().tolist()]

    def effective_bytes(self) -> int:
        """``sum_b S_b * Hkv * D * e * 2 + B * Hq * D * e * 2`` (K+V, then q+o)."""
        e = self.q.element_size()
        d = self.q.shape[-1]
        kv = sum(self.seq_list()) * self.num_kv_heads * d * e * 2
        return kv + self.batch * self.num_heads * d * e * 2

    def flops(self) -> int:
        """``4 * sum_b S_b * Hq * D`` (q.k and p.v multiply-adds)."""
        return 4 * sum(self.seq_list()) * self.num_heads * self.q.shape[-1]


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, g, device, dtype):
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32).to(dtype)


def build(name: str, b: int, hq: int, hkv: int, bs: int, dtype: torch.dtype,
          seq_lens: Union[int, torch.Tensor], max_blocks: int, pool: int, seed: int,
          device="cuda", head_dim: int = HEAD_DIM) -> Workload:
    """Generic builder: shuffled pool, every row's blocks distinct."""
    device = torch.device(device)
    g = _gen(seed, device)
    q = _randn((b, hq, head_dim), g, device, dtype)
    k = _randn((pool, bs, hkv, head_dim), g, device, dtype)
    v = _randn((pool, bs, hkv, head_dim), g, device, dtype)
    need = b * max_blocks
    if need <= pool:
        perm = torch.randperm(pool, generator=g, device=device)[:need]
    else:
        perm = torch.randint(0, pool, (need,), generator=g, device=device)
    bt = perm.reshape(b, max_blocks).to(torch.int32)
    return Workload(name, q, k, v, bt, seq_lens, bs, hkv, seed)


def c1(device="cuda", seed: int = 1) -> Workload:
    return build("c1_b1_h32_s128_bs16_f16", 1, 32, 32, 16, torch.float16, 128, 8, 64, seed, device)


def c2(device="cuda", seed: int = 2) -> Workload:
    return build("c2_b32_h32_s1024_bs16_f16", 32, 32, 32, 16, torch.float16, 1024, 64, 2048, seed,
                 device)


def c3(device="cuda", seed: int = 3) -> Workload:
    w = build("c3_b1_h32_s4096_bs128_bf16", 1, 32, 32, 128, torch.bfloat16, 4096, 32, 256, seed,
              device)
    g = _gen(seed + 1000, torch.device("cpu"))
    blk = int(w.block_table[0, int(torch.randint(0, 32, (1,), generator=g))])
    w.k_cache[blk] = (w.k_cache[blk].float() * 8).to(w.k_cache.dtype)
    return w


def c4(device="cuda", seed: int = 4) -> Workload:
    g = _gen(seed + 1000, torch.device("cpu"))
    lens = torch.randint(1, 257, (128,), generator=g, dtype=torch.int32)
    return build("c4_b128_hq32_hkv8_ragged256_bs16_bf16", 128, 32, 8, 16, torch.bfloat16,
                 lens.to(device), 16, 4096, seed, device)


def c5_lengths(seed: int = 5, batch: int = 256) -> torch.Tensor:
    g = _gen(seed + 1000, torch.device("cpu"))
    u = torch.rand(batch, generator=g, dtype=torch.float64)
    lo, hi = math.log(512), math.log(32768)
    return torch.exp(lo + u * (hi - lo)).round().clamp(512, 32768).to(torch.int32)


def c5(device="cuda", seed: int = 5, rank: int = 0, world: int = 1,
       batch: Optional[int] = None) -> Workload:
    """Head-sharded C5: rank ``rank`` of ``world`` holds 8/world KV heads and
    64/world query heads; each rank's pool is its own seeded shuffle holding
    exactly the blocks its rows use."""
    b = 256 if batch is None else batch
    assert 8 % world == 0, "world size must divide the 8 KV heads"
    lens = c5_lengths(seed, 256)[:b]
    nblk = ((lens + 15) // 16).tolist()
    pool = int(sum(nblk))
    hkv, hq = 8 // world, 64 // world
    device = torch.device(device)
    g = _gen(seed * 100 + rank, device)
    q = _randn((b, hq, HEAD_DIM), g, device, torch.bfloat16)
    k = _randn((pool, 16, hkv, HEAD_DIM), g, device, torch.bfloat16)
    v = _randn((pool, 16, hkv, HEAD_DIM), g, device, torch.bfloat16)
    perm = torch.randperm(pool, generator=g, device=device).to(torch.int32)
    bt = torch.zeros(b, 2048, dtype=torch.int32, device=device)
    off = 0
    for i, n in enumerate(nblk):
        bt[i, :n] = perm[off:off + n]
        off += n
    return Workload(f"c5_b{b}_hq{hq}_hkv{hkv}_loguniform_bs16_bf16_rank{rank}of{world}", q, k, v,
                    bt, lens.to(device), 16, hkv, seed)


CONFIGS = {"c1": c1, "c2": c2, "c3": c3, "c4": c4, "c5": c5}
