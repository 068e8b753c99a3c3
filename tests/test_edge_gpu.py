"""GPU edge shapes: wide query-head groups, one very long sequence (a segment
spread over many CTAs: the general cross-CTA merge), more ragged rows than the
per-CTA prefix sum holds (the plan falls back to the split schedule), large
pages, and caches with padded strides. Every case against the oracle.
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


def _run_and_check(pa, oracle, q, k, v, bt, lens, bs, rows=None, num_splits=None):
    ws = pa.DecodeWorkspace(q.device)
    o, lse = pa.paged_attention(q, k, v, bt, lens, bs, num_splits, return_lse=True, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(q, k, v, bt, lens, bs, batch_indices=rows)
    if rows is not None:
        idx = torch.tensor(rows)
        o, lse, ro, rl = o.cpu()[idx], lse.cpu()[idx], ro[idx], rl[idx]
    assert_o_close(o, ro, "O")
    assert_lse_close(lse, rl, "LSE")


@pytest.mark.parametrize("hq,hkv", [(64, 1), (32, 1), (24, 2)])
def test_wide_query_groups(pa, oracle, hq, hkv):
    """G = 64, 32, 12: several chunks of 8 query heads per KV head."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(hq)
    lens = torch.randint(0, 700, (9,), generator=g, dtype=torch.int32)
    w = workloads.build("wide_g", 9, hq, hkv, 16, torch.bfloat16, lens.cuda(), 44, 9 * 44,
                        seed=hq, device="cuda")
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), 16)
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, 650, 16)
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, 650, 16, num_splits=4)


@pytest.mark.parametrize("hq,hkv,dtype", [(8, 8, torch.float16), (32, 4, torch.bfloat16)])
def test_one_long_sequence(pa, oracle, hq, hkv, dtype):
    """B = 1, S = 131072: each KV head's segment spans many CTAs, so its pieces
    merge through the general (more than 8 rows) cross-CTA path."""
    from paged_attention import workloads
    s, bs = 131072, 16
    w = workloads.build("long_seq", 1, hq, hkv, bs, dtype, s, s // bs, s // bs, seed=hq,
                        device="cuda")
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, s, bs)
    lens = torch.tensor([s - 77], dtype=torch.int32, device="cuda")
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, lens, bs)


def test_more_ragged_rows_than_prefix_sum(pa, oracle):
    """1500 rows with per-row lengths (over the 1024-row prefix sum): the plan
    runs the split schedule with the reference heuristic; sampled rows."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(3)
    b = 1500
    lens = torch.randint(0, 96, (b,), generator=g, dtype=torch.int32)
    w = workloads.build("many_rows", b, 8, 2, 16, torch.float16, lens.cuda(), 6, b * 6,
                        seed=3, device="cuda")
    rows = [0, 1, 511, 1023, 1024, 1499]
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), 16,
                   rows=rows)


@pytest.mark.parametrize("bs", [256, 512])
@pytest.mark.parametrize("group", [1, 8])
def test_large_pages(pa, oracle, bs, group):
    from paged_attention import workloads
    g = torch.Generator().manual_seed(bs + group)
    lens = torch.randint(1, 3 * bs, (5,), generator=g, dtype=torch.int32)
    w = workloads.build("large_pages", 5, 2 * group, 2, bs, torch.bfloat16, lens.cuda(), 3, 20,
                        seed=bs, device="cuda")
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), bs)
    _run_and_check(pa, oracle, w.q, w.k_cache, w.v_cache, w.block_table, 2 * bs + 5, bs,
                   num_splits=3)


@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_padded_cache_strides(pa, oracle, head_dim):
    """K/V views with padded head and slot strides (head dimension contiguous)."""
    g = torch.Generator(device="cuda").manual_seed(head_dim)
    nb, bs, hkv, hq, b, s = 32, 16, 2, 8, 3, 150
    pad_d, pad_h = head_dim + 32, hkv + 1
    kbuf = torch.randn(nb, bs, pad_h, pad_d, generator=g, device="cuda").to(torch.bfloat16)
    vbuf = torch.randn(nb, bs, pad_h, pad_d, generator=g, device="cuda").to(torch.bfloat16)
    k = kbuf[:, :, :hkv, :head_dim]
    v = vbuf[:, :, :hkv, :head_dim]
    assert k.stride(3) == 1 and not k.is_contiguous()
    q = torch.randn(b, hq, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    bt = torch.randperm(nb, generator=g, device="cuda")[: b * 10].reshape(b, 10).int()
    _run_and_check(pa, oracle, q, k, v, bt, s, bs)
    _run_and_check(pa, oracle, q, k, v, bt, s, bs, num_splits=2)


@pytest.mark.parametrize("head_dim,hq,hkv,b,s,per_row", [
    (128, 64, 8, 1, 8192, False), (128, 64, 8, 1, 8192, True), (128, 32, 4, 1, 32768, False),
    (128, 32, 8, 4, 2048, True), (128, 24, 2, 2, 9000, False), (128, 8, 8, 1, 131072, False),
    (64, 64, 8, 1, 16384, False), (64, 16, 2, 3, 5000, True), (256, 16, 2, 1, 12000, False),
    (256, 16, 16, 1, 16384, True), (128, 32, 8, 4, 2048, "zero_ends"),
    (128, 64, 8, 3, 6000, "zero_ends")])
def test_few_long_segments_merge_pass(pa, oracle, head_dim, hq, hkv, b, s, per_row):
    """Few segments, each spread over many CTAs: the pieces merge in the
    separate merge kernel that follows the decode kernel (one CTA per crossing
    segment, its warps over the columns and pieces), for query-head groups of
    2-8 columns and partial column chunks (G = 12), single columns spanning
    more than 8 groups, same-length and per-row lengths (with zero-length
    first and last rows, which own no tile and that pass skips), D = 64, 128,
    256. The plan query confirms that every case takes the merge pass."""
    from paged_attention import workloads
    bs = 16
    nblk = (s + bs - 1) // bs
    w = workloads.build("merge_pass", b, hq, hkv, bs, torch.bfloat16, s, nblk, b * nblk,
                        seed=hq + s, device="cuda", head_dim=head_dim)
    if per_row:
        lens = torch.tensor([s - 7 * i for i in range(b)], dtype=torch.int32, device="cuda")
        if per_row == "zero_ends":
            lens[0] = 0
            lens[-1] = 0
    else:
        lens = s
    plan = pa.decode_plan(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs)
    assert plan["merge_pass"] == 1 and plan["kernels"] == 2, plan
    ws = pa.DecodeWorkspace("cuda")
    for rep in range(2):   # the second call reuses the workspace as left by the first
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs,
                                    return_lse=True, workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs)
    assert_o_close(o, ro, "O")
    assert_lse_close(lse, rl, "LSE")
    # the split schedule on the same inputs (no merge pass) agrees too
    o2 = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs, 7)
    torch.cuda.synchronize()
    assert_o_close(o2, ro, "O split")


@pytest.mark.parametrize("head_dim,hq,hkv,variant", [(128, 32, 8, 3), (64, 64, 8, 8),
                                                    (256, 16, 2, 9)])
def test_long_segments_merge_rows_in_workspace(pa, oracle, head_dim, hq, hkv, variant):
    """Variants whose warps' merge rows do not fit in shared memory beside the
    stages, with segments far longer than 8 tiles: the CTA-level merge goes
    through the workspace (same-length and per-row lengths, both checked)."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(head_dim + variant)
    b, s, bs = 3, 20000, 16
    lens = torch.randint(s // 2, s, (b,), generator=g, dtype=torch.int32)
    nblk = (s + bs - 1) // bs
    w = workloads.build("long_ws", b, hq, hkv, bs, torch.bfloat16, lens.cuda(), nblk, b * nblk,
                        seed=variant, device="cuda", head_dim=head_dim)
    for lengths in (lens.cuda(), s - 3):
        ws = pa.DecodeWorkspace("cuda")
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lengths, bs,
                                    return_lse=True, workspace=ws, kernel_variant=variant)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
        ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lengths, bs)
        assert_o_close(o, ro, "O")
        assert_lse_close(lse, rl, "LSE")


@pytest.mark.parametrize("hq,hkv,b,smax,variant", [
    (32, 8, 128, 256, 0), (32, 8, 128, 256, 5), (32, 8, 300, 100, 5), (16, 16, 200, 300, 0),
    (16, 16, 64, 2000, 0), (64, 8, 96, 200, 0)])
def test_ragged_short_segments_group_boundaries(pa, oracle, hq, hkv, b, smax, variant):
    """Ragged batches of short rows (zero-length rows included): with
    whole-CTA merge groups the group boundaries move to segment boundaries, so
    every segment merges inside one CTA; with longer rows they stay put and the
    cross-CTA merge runs. Every row against the oracle."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(b + smax)
    lens = torch.randint(0, smax + 1, (b,), generator=g, dtype=torch.int32)
    lens[0] = 0
    lens[b // 2] = smax
    lens[-1] = 0
    nblk = (smax + 15) // 16
    w = workloads.build("ragged_short", b, hq, hkv, 16, torch.bfloat16, lens.cuda(), nblk,
                        b * nblk, seed=b, device="cuda")
    ws = pa.DecodeWorkspace("cuda")
    for _ in range(2):
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), 16,
                                    return_lse=True, workspace=ws, kernel_variant=variant)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lens, 16)
    assert_o_close(o, ro, "O")
    assert_lse_close(lse, rl, "LSE")
