"""GPU tests of the head-sharded C5 shards that the multi-GPU benchmark runs.

`bench.py --gpus N` gives rank r the KV heads [r*8/N, (r+1)*8/N) of C5 (B 256,
64 query heads over 8 KV heads, log-uniform lengths 512-32768, page 16, bf16)
with their query heads and its own page pool. Here each shard of N = 2, 4 and
8 (first and last rank) runs on one GPU, one after the other, and sampled rows
(the shortest, the longest and a few fixed ones) are checked against the
oracle; the whole shard is checked against the split schedule.
"""
import pytest
import torch

from helpers import assert_lse_close, assert_o_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pa():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    import paged_attention
    return paged_attention


@pytest.fixture(scope="module")
def oracle():
    import oracle as o
    return o


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 0), (4, 3), (8, 0), (8, 7)])
def test_c5_shard(pa, oracle, world, rank):
    from paged_attention import workloads
    w = workloads.c5("cuda", rank=rank, world=world)
    assert w.num_kv_heads == 8 // world and w.num_heads == 64 // world
    lens = w.seq_list()
    rows = sorted({0, 100, 255, min(range(len(lens)), key=lambda i: lens[i]),
                   max(range(len(lens)), key=lambda i: lens[i])})
    ws = pa.DecodeWorkspace("cuda")
    o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                w.block_size, return_lse=True, workspace=ws)
    o_split = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                 w.block_size, 8)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    assert torch.isfinite(o.float()).all()
    assert_o_close(o_split, o.float(), f"{w.name} split vs balanced schedule")
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                     w.block_size, batch_indices=rows)
    idx = torch.tensor(rows)
    assert_o_close(o.cpu()[idx], ro[idx], f"{w.name} O")
    assert_lse_close(lse.cpu()[idx], rl[idx], f"{w.name} LSE")
    del w, o, o_split
    torch.cuda.empty_cache()
