"""GPU parity for head dimensions 64 and 256 (the reference kernel takes the
head dimension as a compile-time constant, ``split_kv_kernel.py:12-30``; its
golden fixtures for both are in ``tests/golden``): both schedules against the
oracle over block sizes, query-head groups, ragged and zero lengths; the
single-token KAT; explicit variants; same-length batches large enough for
segment-aligned groups; graph replay.
"""
import pytest
import torch

from helpers import assert_lse_close, assert_o_close

pytestmark = pytest.mark.gpu

SENTINEL = torch.tensor(-1e30, dtype=torch.float32)


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


def _check(pa, oracle, w, num_splits=None, **kw):
    ws = pa.DecodeWorkspace(w.q.device)
    o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                w.block_size, num_splits, return_lse=True, workspace=ws, **kw)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                     w.block_size)
    assert_o_close(o, ro, f"{w.name} ns={num_splits} O")
    assert_lse_close(lse, rl, f"{w.name} ns={num_splits} LSE")
    return o


@pytest.mark.parametrize("head_dim", [64, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bs", [8, 16, 32, 128])
@pytest.mark.parametrize("group", [1, 2, 3, 4, 8])
def test_sweep_head_dim(pa, oracle, head_dim, dtype, bs, group):
    from paged_attention import workloads
    hkv, b = 2, 5
    g = torch.Generator().manual_seed(head_dim + bs * 100 + group)
    lens = torch.randint(0, 300, (b,), generator=g, dtype=torch.int32)
    lens[0] = 1
    lens[1] = 0
    max_blocks = (300 + bs - 1) // bs
    w = workloads.build(f"d{head_dim}_bs{bs}_g{group}", b, hkv * group, hkv, bs, dtype,
                        lens.cuda(), max_blocks, b * max_blocks + 3, seed=bs + group,
                        device="cuda", head_dim=head_dim)
    _check(pa, oracle, w)
    _check(pa, oracle, w, num_splits=3)
    # same-length rows (the uniform-length schedule)
    w.seq_len = 250
    _check(pa, oracle, w)


@pytest.mark.parametrize("head_dim", [64, 256])
def test_kat_single_token_bit_exact_head_dim(pa, head_dim):
    """S=1: O equals the V row bit-exactly (block-table, head and dim indexing)."""
    from paged_attention import workloads
    for hq, hkv in [(16, 16), (16, 4), (32, 4)]:
        w = workloads.build("kat_s1", 4, hq, hkv, 16, torch.bfloat16, 1, 4, 64, seed=21,
                            device="cuda", head_dim=head_dim)
        for ns in (None, 1, 3):
            o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 1, 16, ns)
            torch.cuda.synchronize()
            phys = w.block_table[:, 0].long()
            kvh = torch.arange(hq, device="cuda") // (hq // hkv)
            expect = w.v_cache[phys][:, 0][:, kvh]
            assert torch.equal(o, expect), f"D={head_dim} hq={hq} hkv={hkv} ns={ns}"


@pytest.mark.parametrize("head_dim", [64, 256])
def test_zero_length_and_empty_split_head_dim(pa, head_dim):
    from paged_attention import workloads
    lens = torch.tensor([0, 9, 0, 33], dtype=torch.int32, device="cuda")
    w = workloads.build("kat_s0", 4, 8, 2, 16, torch.float16, lens, 4, 32, seed=22,
                        device="cuda", head_dim=head_dim)
    for ns in (None, 4):
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens, 16, ns,
                                    return_lse=True)
        torch.cuda.synchronize()
        for b in (0, 2):
            assert torch.equal(o[b], torch.zeros_like(o[b]))
            assert torch.equal(lse[b].cpu(), SENTINEL.expand(8))
    # S=9, ns=4 (split size 3): the fourth split of row 1 is empty
    _, _, lse_p = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 9, 16, 4,
                                     return_partials=True)
    torch.cuda.synchronize()
    assert torch.equal(lse_p[1, :, 3].cpu(), SENTINEL.expand(8))


@pytest.mark.parametrize("variant", [3, 5, 8])
@pytest.mark.parametrize("group", [1, 4, 8])
def test_head_dim_64_variants(pa, oracle, variant, group):
    from paged_attention import workloads
    g = torch.Generator().manual_seed(variant * 10 + group)
    lens = torch.randint(0, 400, (6,), generator=g, dtype=torch.int32)
    w = workloads.build("d64_variant", 6, 2 * group, 2, 16, torch.bfloat16, lens.cuda(), 25, 150,
                        seed=variant, device="cuda", head_dim=64)
    _check(pa, oracle, w, kernel_variant=variant)
    _check(pa, oracle, w, num_splits=5, kernel_variant=variant)


@pytest.mark.parametrize("variant", [6, 7, 9])
@pytest.mark.parametrize("group", [1, 4, 8])
def test_head_dim_256_variants(pa, oracle, variant, group):
    from paged_attention import workloads
    g = torch.Generator().manual_seed(variant * 10 + group)
    lens = torch.randint(0, 400, (6,), generator=g, dtype=torch.int32)
    w = workloads.build("d256_variant", 6, 2 * group, 2, 16, torch.float16, lens.cuda(), 25, 150,
                        seed=variant, device="cuda", head_dim=256)
    _check(pa, oracle, w, kernel_variant=variant)
    _check(pa, oracle, w, num_splits=5, kernel_variant=variant)


def test_unbuilt_variant_rejected(pa):
    from paged_attention import workloads
    w = workloads.build("d256", 2, 4, 4, 16, torch.float16, 40, 4, 8, seed=1, device="cuda",
                        head_dim=256)
    with pytest.raises(Exception):
        pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 40, 16, kernel_variant=3)


@pytest.mark.parametrize("head_dim,hq,hkv", [(64, 16, 16), (64, 32, 4), (256, 8, 8), (256, 16, 2)])
def test_segment_aligned_groups_head_dim(pa, oracle, head_dim, hq, hkv):
    """Same-length batch with at least one segment per CTA: groups aligned to
    whole segments (no cross-CTA merges)."""
    from paged_attention import workloads
    b = 592 // hkv          # 592 = 4 x 148 segments: whole segments per CTA
    w = workloads.build("aligned", b, hq, hkv, 16, torch.bfloat16, 192, 12, b * 12,
                        seed=head_dim + hq, device="cuda", head_dim=head_dim)
    rows = [0, b // 2, b - 1]
    ws = pa.DecodeWorkspace("cuda")
    o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 192, 16,
                                return_lse=True, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, 192, 16,
                                     batch_indices=rows)
    idx = torch.tensor(rows)
    assert_o_close(o.cpu()[idx], ro[idx], "aligned O")
    assert_lse_close(lse.cpu()[idx], rl[idx], "aligned LSE")


@pytest.mark.parametrize("head_dim", [64, 256])
def test_graph_runner_head_dim(pa, oracle, head_dim):
    B, H, S, bs, nblk = 3, 4, 200, 16, 40
    g = torch.Generator(device="cuda").manual_seed(head_dim)
    runner = pa.PagedAttnGraphRunner(B, H, head_dim, S, bs, nblk, device="cuda",
                                     dtype=torch.float16)
    q = torch.randn(B, H, head_dim, generator=g, device="cuda").half()
    k = torch.randn(nblk, bs, H, head_dim, generator=g, device="cuda").half()
    v = torch.randn(nblk, bs, H, head_dim, generator=g, device="cuda").half()
    bt = torch.randperm(nblk, generator=g, device="cuda")[: B * 13].reshape(B, 13).int()
    out = runner.run(q, k, v, bt, copy_kv=True).clone()
    runner.replay_only()
    torch.cuda.synchronize()
    ro, _ = oracle.decode_reference(q, k, v, bt, S, bs)
    assert_o_close(out, ro, "graph O")
    assert torch.equal(runner.static_out, out)
