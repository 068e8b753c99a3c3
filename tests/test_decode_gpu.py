"""GPU parity tests: the sm_100a operator against the CPU oracle and the golden
fixtures made from the reference's own kernels.

Every call goes through ``paged_attention`` -> the C ABI (``pa_decode``).
"""
import math

import pytest
import torch

from helpers import (assert_lse_close, assert_o_close, golden_paths, load_golden)

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


def _status_ok(ws):
    return ws is None or ws.read_status() == 0


# --------------------------------------------------------------------------- golden
@pytest.mark.parametrize("path", golden_paths(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_split_schedule(pa, path):
    """Reference split schedule (same num_splits as the fixture): O, partial LSE,
    partial O and the -1e30 sentinel against the reference Triton kernels."""
    g = load_golden(path, "cuda")
    ws = pa.DecodeWorkspace("cuda")
    o, lse, o_p, lse_p = pa.paged_attention(
        g["q"], g["k_cache"], g["v_cache"], g["block_table"], g["seq_len"], g["block_size"],
        g["num_splits"], return_lse=True, return_partials=True, workspace=ws)
    torch.cuda.synchronize()
    assert _status_ok(ws)
    assert o.dtype == g["q"].dtype and o.shape == g["q"].shape
    assert_o_close(o, g["o_ref"], "O vs reference")
    ref_lse = g["lse_partial"].cpu()
    valid = ref_lse > -1e29
    got_lse = lse_p.cpu()
    # sentinel bit-exact where the reference split was empty
    assert torch.equal(got_lse[~valid], ref_lse[~valid])
    assert (got_lse[valid] > -1e29).all()
    assert_lse_close(got_lse[valid], ref_lse[valid], "partial LSE")
    assert_o_close(o_p.cpu()[valid], g["o_partial"].cpu()[valid], "partial O")


@pytest.mark.parametrize("path", golden_paths(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_balanced_schedule(pa, oracle, path):
    g = load_golden(path, "cuda")
    o, lse = pa.paged_attention(g["q"], g["k_cache"], g["v_cache"], g["block_table"],
                                g["seq_len"], g["block_size"], return_lse=True)
    torch.cuda.synchronize()
    assert_o_close(o, g["o_ref"], "O vs reference")
    ro, rl = oracle.decode_reference(g["q"], g["k_cache"], g["v_cache"], g["block_table"],
                                     g["seq_len"], g["block_size"])
    assert_o_close(o, ro, "O vs oracle")
    assert_lse_close(lse, rl, "LSE vs oracle")


# --------------------------------------------------------------------------- configs
def _check_workload(pa, oracle, w, num_splits=None, batch_indices=None):
    ws = pa.DecodeWorkspace(w.q.device)
    o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                w.block_size, num_splits, return_lse=True, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                     w.block_size, batch_indices=batch_indices)
    if batch_indices is not None:
        idx = torch.tensor(batch_indices)
        o, lse, ro, rl = o.cpu()[idx], lse.cpu()[idx], ro[idx], rl[idx]
    assert_o_close(o, ro, f"{w.name} O")
    assert_lse_close(lse, rl, f"{w.name} LSE")
    return o, lse


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c4"])
def test_config_balanced(pa, oracle, cfg):
    from paged_attention import workloads
    w = workloads.CONFIGS[cfg]("cuda")
    _check_workload(pa, oracle, w)


@pytest.mark.parametrize("cfg", ["c1", "c2", "c3", "c4"])
def test_config_reference_split_heuristic(pa, oracle, cfg):
    """num_splits from the reference heuristic with this device's SM count."""
    from paged_attention import workloads
    w = workloads.CONFIGS[cfg]("cuda")
    s = max(w.seq_list())
    ns = pa.num_splits_heuristic(w.batch, w.num_heads, s, w.block_size,
                                 pa.device_sm_count(w.q.device))
    _check_workload(pa, oracle, w, num_splits=ns)


@pytest.mark.parametrize("ns", [4, 16])
def test_c4_forced_splits_sentinel(pa, oracle, ns):
    """Ragged GQA with forced splits: short rows have empty splits (-1e30)."""
    from paged_attention import workloads
    w = workloads.c4("cuda")
    o, lse, o_p, lse_p = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                            w.block_size, ns, return_lse=True,
                                            return_partials=True)
    torch.cuda.synchronize()
    ref_op, ref_lp = oracle.split_partials(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                           w.block_size, ns)
    ref_valid = ref_lp > -1e29
    got = lse_p.cpu()
    assert (~ref_valid).any(), "workload must contain empty splits"
    assert torch.equal(got[~ref_valid], torch.full_like(got[~ref_valid], -1e30))
    assert_lse_close(got[ref_valid], ref_lp[ref_valid], "partial LSE")
    assert_o_close(o_p.cpu()[ref_valid], ref_op[ref_valid], "partial O")
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                     w.block_size)
    assert_o_close(o, ro, "O")
    assert_lse_close(lse, rl, "LSE")


def test_c5_full_size_sampled(pa, oracle):
    """Full C5 (N=1 shard) on the GPU; the oracle checks a sample of rows, the
    rest is checked for finiteness and against the split schedule."""
    from paged_attention import workloads
    w = workloads.c5("cuda")
    rows = [0, 1, 77, 128, 200, 255]
    lens = w.seq_list()
    rows += [int(min(range(len(lens)), key=lambda i: lens[i])),
             int(max(range(len(lens)), key=lambda i: lens[i]))]
    o, lse = _check_workload(pa, oracle, w, batch_indices=rows)
    o_all, lse_all = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                        w.block_size, return_lse=True)
    o_split = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                 w.block_size, 8)
    torch.cuda.synchronize()
    assert torch.isfinite(o_all.float()).all()
    assert_o_close(o_split, o_all.float(), "split vs balanced schedule")


# --------------------------------------------------------------------------- sweeps
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bs", [8, 16, 24, 32, 64, 128, 256])
@pytest.mark.parametrize("group", [1, 2, 3, 4, 8, 16])
def test_sweep_block_size_group(pa, oracle, dtype, bs, group):
    from paged_attention import workloads
    hkv = 2
    b = 5
    g = torch.Generator().manual_seed(bs * 100 + group)
    lens = torch.randint(0, 300, (b,), generator=g, dtype=torch.int32)
    lens[0] = 1
    lens[1] = 0 if group != 3 else 2
    max_blocks = (300 + bs - 1) // bs
    w = workloads.build(f"sweep_bs{bs}_g{group}", b, hkv * group, hkv, bs, dtype, lens.cuda(),
                        max_blocks, b * max_blocks + 3, seed=bs + group, device="cuda")
    _check_workload(pa, oracle, w)
    _check_workload(pa, oracle, w, num_splits=3)


@pytest.mark.parametrize("group,bs,dtype", [(1, 16, torch.float16), (4, 16, torch.bfloat16),
                                            (8, 32, torch.bfloat16), (2, 128, torch.float16)])
def test_ragged_mixed_long_and_short_rows(pa, oracle, group, bs, dtype):
    """Per-row lengths mixing rows that span several CTAs (cross-CTA merges)
    with short rows (CTA boundaries moved to segment edges), every row checked."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(group * 1000 + bs)
    b, hkv = 48, 2
    lens = torch.randint(1, 120, (b,), generator=g, dtype=torch.int32)
    long_rows = torch.randperm(b, generator=g)[:6]
    lens[long_rows] = torch.randint(3000, 6000, (6,), generator=g, dtype=torch.int32)
    lens[5] = 0
    max_blocks = (6000 + bs - 1) // bs
    w = workloads.build("ragged_mixed", b, hkv * group, hkv, bs, dtype, lens.cuda(), max_blocks,
                        int(((lens + bs - 1) // bs).sum()) + 8, seed=group + bs, device="cuda")
    _check_workload(pa, oracle, w)


@pytest.mark.parametrize("variant", [1, 2, 3, 4, 5, 10])
@pytest.mark.parametrize("group,bs,dtype", [(1, 16, torch.float16), (4, 24, torch.bfloat16),
                                            (8, 128, torch.bfloat16), (3, 8, torch.float16)])
def test_kernel_variants(pa, oracle, variant, group, bs, dtype):
    """Every tile/warp/stage variant, both schedules, against the oracle."""
    from paged_attention import workloads
    g = torch.Generator().manual_seed(variant * 10 + group)
    b, hkv = 7, 2
    lens = torch.randint(0, 400, (b,), generator=g, dtype=torch.int32)
    lens[2] = 0
    max_blocks = (400 + bs - 1) // bs
    w = workloads.build("variant", b, hkv * group, hkv, bs, dtype, lens.cuda(), max_blocks,
                        b * max_blocks, seed=variant, device="cuda")
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs)
    for ns in (None, 5):
        ws = pa.DecodeWorkspace("cuda")
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len, bs, ns,
                                    return_lse=True, workspace=ws, kernel_variant=variant)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
        assert_o_close(o, ro, f"variant {variant} ns={ns}")
        assert_lse_close(lse, rl, f"variant {variant} ns={ns} LSE")
    # uniform-length path of the balanced schedule
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 300, bs,
                           kernel_variant=variant)
    ro2, _ = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, 300, bs)
    assert_o_close(o, ro2, f"variant {variant} uniform")


# --------------------------------------------------------------------------- KATs
def test_kat_single_token_bit_exact(pa):
    """S=1: the softmax weight is exactly 1, so O equals the V row bit-exactly
    (pins block-table and head indexing)."""
    from paged_attention import workloads
    for hq, hkv in [(32, 32), (32, 8), (64, 8)]:
        w = workloads.build("kat_s1", 4, hq, hkv, 16, torch.bfloat16, 1, 4, 64, seed=11,
                            device="cuda")
        for ns in (None, 1, 3):
            o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 1, 16, ns)
            torch.cuda.synchronize()
            phys = w.block_table[:, 0].long()
            kvh = torch.arange(hq, device="cuda") // (hq // hkv)
            expect = w.v_cache[phys][:, 0][:, kvh]          # [B, Hq, D]
            assert torch.equal(o, expect), f"hq={hq} hkv={hkv} ns={ns}"


def test_kat_zero_length_rows(pa):
    """S=0 rows: O exactly 0 and final LSE exactly -1e30 (split_kv_kernel.py:120)."""
    from paged_attention import workloads
    lens = torch.tensor([0, 37, 0, 5], dtype=torch.int32, device="cuda")
    w = workloads.build("kat_s0", 4, 8, 2, 16, torch.float16, lens, 4, 32, seed=12, device="cuda")
    for ns in (None, 2):
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens, 16, ns,
                                    return_lse=True)
        torch.cuda.synchronize()
        for b in (0, 2):
            assert torch.equal(o[b], torch.zeros_like(o[b]))
            assert torch.equal(lse[b].cpu(), SENTINEL.expand(8))
        assert (o[1].float().abs().sum() > 0)
    # uniform zero length
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 0, 16)
    torch.cuda.synchronize()
    assert torch.equal(o, torch.zeros_like(o))


def test_kat_zero_query_is_mean_of_values(pa, oracle):
    """q = 0: all scores equal, so O is the mean of the row's V vectors."""
    from paged_attention import workloads
    w = workloads.build("kat_q0", 2, 4, 4, 16, torch.float16, 100, 7, 16, seed=13, device="cuda")
    w.q.zero_()
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 100, 16)
    torch.cuda.synchronize()
    for b in range(2):
        rows = oracle.gather_sequence(w.v_cache.cpu(), w.block_table[b].cpu(), 100, 16)
        assert_o_close(o[b], rows.float().mean(0), "mean of V")


def test_kat_empty_split_sentinel_exact(pa):
    """S=9, ns=4 (split size 3): split 3 is empty and keeps LSE == float32(-1e30)."""
    from paged_attention import workloads
    w = workloads.build("kat_empty", 1, 2, 2, 16, torch.float16, 9, 1, 4, seed=14, device="cuda")
    _, _, lse_p = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 9, 16, 4,
                                     return_partials=True)
    torch.cuda.synchronize()
    assert torch.equal(lse_p[0, :, 3].cpu(), SENTINEL.expand(2))
    assert (lse_p[0, :, :3] > -1e29).all()


# --------------------------------------------------------------------------- API
def test_determinism_and_workspace_reuse(pa):
    from paged_attention import workloads
    w = workloads.c4("cuda")
    outs = [pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len, 16)
            for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_strided_query(pa, oracle):
    from paged_attention import workloads
    w = workloads.build("strided", 3, 8, 8, 16, torch.float16, 70, 5, 20, seed=15, device="cuda")
    big = torch.randn(3, 8, 2 * 128, device="cuda", dtype=torch.float16)
    q = big[:, :, 64:192].contiguous()
    qs = big[:, :, :128]          # stride(1) = 256, last dim contiguous
    qs.copy_(q)
    o = pa.paged_attention(qs, w.k_cache, w.v_cache, w.block_table, 70, 16)
    ro, _ = oracle.decode_reference(qs, w.k_cache, w.v_cache, w.block_table, 70, 16)
    assert_o_close(o, ro, "strided q")


def test_bad_block_index_flagged_not_faulting(pa):
    """A block-table entry outside the pool is skipped and flagged in the status
    word (no device trap, no out-of-bounds read)."""
    from paged_attention import workloads
    w = workloads.build("badblk", 2, 4, 4, 16, torch.float16, 40, 3, 8, seed=16, device="cuda")
    w.block_table[1, 1] = 1_000_000
    ws = pa.DecodeWorkspace("cuda")
    pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 40, 16, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() & 1
    ws.reset()
    w.block_table[1, 1] = 0
    pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 40, 16, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0


def test_seq_len_over_capacity_flagged(pa):
    from paged_attention import workloads
    lens = torch.tensor([10, 500], dtype=torch.int32, device="cuda")
    w = workloads.build("overcap", 2, 4, 4, 16, torch.float16, lens, 2, 8, seed=17, device="cuda")
    ws = pa.DecodeWorkspace("cuda")
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens, 16, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() & 2
    assert torch.isfinite(o.float()).all()


def test_backward_raises(pa):
    from paged_attention import workloads
    w = workloads.build("bwd", 1, 2, 2, 16, torch.float16, 16, 1, 2, seed=18, device="cuda")
    q = w.q.clone().requires_grad_(True)
    o = pa.paged_attention(q, w.k_cache, w.v_cache, w.block_table, 16, 16)
    with pytest.raises(RuntimeError, match="inference-only"):
        o.float().sum().backward()


# --------------------------------------------------------------------------- graphs
def test_graph_runner_matches_eager(pa, oracle):
    """Reference tests/correctness.py:44-48 flow: build, run(copy_kv=True), compare."""
    torch.manual_seed(42)
    B, H, D, S, bs, NB = 1, 8, 128, 4096, 16, 4096
    runner = pa.PagedAttnGraphRunner(B, H, D, S, bs, NB)
    q = torch.randn(B, H, D, device="cuda", dtype=torch.float16)
    k = torch.randn(NB, bs, H, D, device="cuda", dtype=torch.float16)
    v = torch.randn(NB, bs, H, D, device="cuda", dtype=torch.float16)
    bt = torch.randperm(NB, device="cuda")[: S // bs].reshape(1, -1).to(torch.int32)
    out = runner.run(q, k, v, bt, copy_kv=True)
    eager = pa.paged_attention(q, k, v, bt, S, bs)
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    ro, _ = oracle.decode_reference(q, k, v, bt, S, bs)
    assert_o_close(out, ro, "graph")
    # replay again with new q: counters must have reset
    q2 = torch.randn_like(q)
    out2 = runner.run(q2, k, v, bt).clone()
    torch.cuda.synchronize()
    ro2, _ = oracle.decode_reference(q2, k, v, bt, S, bs)
    assert_o_close(out2, ro2, "graph replay 2")


def test_graph_runner_dynamic_lengths_gqa(pa, oracle):
    B, Hq, Hkv, D, bs, NB, cap = 6, 16, 4, 128, 16, 256, 512
    runner = pa.PagedAttnGraphRunner(B, Hq, D, 100, bs, NB, dtype=torch.bfloat16,
                                     num_kv_heads=Hkv, dynamic_seq_lens=True, max_seq_len=cap,
                                     return_lse=True)
    k = torch.randn(NB, bs, Hkv, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn_like(k)
    bt = torch.randperm(NB, device="cuda")[: B * (cap // bs)].reshape(B, -1).to(torch.int32)
    runner.static_k.copy_(k)
    runner.static_v.copy_(v)
    for it in range(3):
        lens = torch.randint(0, cap + 1, (B,), dtype=torch.int32)
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        out = runner.run(q, k, v, bt, seq_lens=lens.cuda()).clone()
        lse = runner.static_lse.clone()
        torch.cuda.synchronize()
        ro, rl = oracle.decode_reference(q, k, v, bt, lens, bs)
        assert_o_close(out, ro, f"graph dyn it{it}")
        assert_lse_close(lse, rl, f"graph dyn lse it{it}")
    assert runner.workspace.read_status() == 0


def test_peak_bw_probe_copies_exactly_and_at_least_at_memcpy_speed(pa):
    """The probe's copy is exact (odd sizes included) and, on 1 GiB buffers,
    no slower than 0.97x a device-to-device copy_ timed the same way -- it is
    the roofline denominator, so reading low would flatter every fraction."""
    import measure_peak_bw
    from paged_attention import _native
    lib = _native.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for nbytes in (16, 4096 + 48, (32 << 10) * 3 + 16, 64 << 20):
        src = torch.randint(-2 ** 31, 2 ** 31 - 1, (nbytes // 4,), dtype=torch.int32,
                            device="cuda")
        dst = torch.zeros_like(src)
        assert lib.pa_stream_copy(src.data_ptr(), dst.data_ptr(), nbytes, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(src, dst), nbytes
    size_mb = 1024
    ours = measure_peak_bw.measure_peak_bw(size_mb, 20)
    a = torch.empty(size_mb << 19, dtype=torch.float16, device="cuda")
    b = torch.empty_like(a)
    ms = measure_peak_bw._time_ms(lambda: b.copy_(a), 20, warmup=5)
    theirs = 2 * a.numel() * 2 / (ms * 1e-3) / 1e9
    assert ours >= 0.97 * theirs, (ours, theirs)
