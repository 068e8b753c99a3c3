"""CPU tests of the Python host API: argument checking fails loudly, and the
reference-named exports exist. Nothing here launches a kernel."""
import pytest
import torch

import paged_attention as pa
from paged_attention import split_kv_kernel, workloads


def test_reference_exports():
    assert callable(pa.paged_attention)
    assert pa.PagedAttnGraphRunner.__name__ == "PagedAttnGraphRunner"
    assert set(pa.__all__) == {"paged_attention", "PagedAttnGraphRunner"}
    assert split_kv_kernel.LSE_SENTINEL == -1e30
    assert split_kv_kernel.LSE_VALID_THRESHOLD == -1e29


def test_cpu_tensors_rejected_no_fallback():
    q = torch.randn(1, 2, 128, dtype=torch.float16)
    k = torch.randn(2, 16, 2, 128, dtype=torch.float16)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA tensors"):
        pa.paged_attention(q, k, k, bt, 16, 16)


def test_heuristic_binding():
    assert pa.num_splits_heuristic(1, 32, 128, 16, 148) == 8
    assert pa.num_splits_heuristic(1, 32, 4096, 128, 148) == 18


def test_workload_cpu_shapes():
    w = workloads.c1("cpu")
    assert w.q.shape == (1, 32, 128) and w.k_cache.shape == (64, 16, 32, 128)
    assert w.block_table.shape == (1, 8) and len(set(w.block_table[0].tolist())) == 8
    assert w.effective_bytes() == 2_113_536
    w4 = workloads.c4("cpu")
    lens = w4.seq_list()
    assert min(lens) >= 1 and max(lens) <= 256 and w4.num_kv_heads == 8
    lens5 = workloads.c5_lengths()
    assert lens5.min() >= 512 and lens5.max() <= 32768


def test_c5_shards_partition_heads():
    full = workloads.c5("cpu", batch=4)
    parts = [workloads.c5("cpu", rank=r, world=4, batch=4) for r in range(4)]
    assert sum(p.num_heads for p in parts) == full.num_heads
    assert sum(p.num_kv_heads for p in parts) == full.num_kv_heads
    assert all(p.seq_list() == full.seq_list() for p in parts)
