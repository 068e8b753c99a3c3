"""GPU tests of the cluster schedule.

Same-length rows whose segments (one row, one KV head, up to 8 of its query
heads) are longer than a CTA's share of the step run as thread-block clusters:
one cluster of 2-8 CTAs per segment, each CTA one contiguous part of it, the
CTAs' pieces merged by the cluster's rank 0 from distributed shared memory.
When the device cannot hold every cluster at once the call falls back to the
plain schedule. Every case is checked against the oracle, twice on one
workspace, and against the reference's split schedule.
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


# (batch, seq_len, query heads, KV heads, page size, dtype, head_dim)
CASES = [
    (1, 4096, 32, 32, 128, torch.bfloat16, 128),   # 32 segments: clusters of 4
    (2, 2048, 32, 32, 16, torch.float16, 128),     # 64 segments: clusters of 2
    (1, 1000, 20, 20, 16, torch.bfloat16, 128),    # 20 segments: clusters of 7, ragged last tile
    (1, 4096, 64, 64, 128, torch.bfloat16, 64),    # head_dim 64
    (1, 4096, 16, 16, 128, torch.bfloat16, 256),   # head_dim 256: clusters of 8, or the fallback
    (1, 8192, 128, 16, 16, torch.bfloat16, 128),   # query-head groups of 8
    (1, 3000, 96, 6, 32, torch.float16, 128),      # groups of 16: two chunks of 8 per KV head
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_cluster_schedule_matches_oracle(pa, oracle, case):
    from paged_attention import workloads
    b, s, hq, hkv, bs, dtype, d = CASES[case]
    nb = (s + bs - 1) // bs
    w = workloads.build(f"cluster{case}", b, hq, hkv, bs, dtype, s, nb, b * nb + 5,
                        seed=100 + case, device="cuda", head_dim=d)
    plan = pa.decode_plan(w.q, w.k_cache, w.v_cache, w.block_table, s, bs, None)
    if case in (0, 1, 2, 3):
        # these fit on a 148-SM part (fewer SMs: no clusters, or smaller ones)
        assert plan["cluster_size"] >= 2 or torch.cuda.get_device_properties(0).multi_processor_count < 148, plan
    if plan["cluster_size"]:
        assert plan["kernels"] == 1 and plan["merge_pass"] == 0, plan
    ws = pa.DecodeWorkspace("cuda")
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, s, bs)
    outs = []
    for call in range(2):
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, s, bs,
                                    return_lse=True, workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
        assert_o_close(o, ro, f"O call {call}")
        assert_lse_close(lse, rl, f"LSE call {call}")
        outs.append(o.clone())
    assert torch.equal(outs[0], outs[1]), "two calls on one workspace differ"
    o_split = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, s, bs, 5)
    torch.cuda.synchronize()
    assert_o_close(o_split, ro, "O split schedule")


def test_cluster_schedule_in_graph(pa, oracle):
    """A captured graph replays the cluster launch (its cluster shape is part
    of the kernel node)."""
    from paged_attention import workloads
    b, s, hq, hkv, bs = 1, 4096, 32, 32, 128
    w = workloads.build("cluster_graph", b, hq, hkv, bs, torch.bfloat16, s, s // bs, s // bs,
                        seed=7, device="cuda")
    ws = pa.DecodeWorkspace("cuda")
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, s, bs, workspace=ws)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            og = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, s, bs,
                                    workspace=ws)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(og, o)
    ro, _ = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, s, bs)
    assert_o_close(og, ro, "O graph")
