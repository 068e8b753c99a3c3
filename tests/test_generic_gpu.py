"""GPU tests of the CUDA-core path for the shapes the tile kernels do not take:
head_dim 32, and pages whose size is not a multiple of 8 tokens (1, 2, 4, and
any other positive size). The reference accepts any power of two for both
(split_kv_kernel.py:38,49); its fixtures for pages of 1, 2 and 4 tokens and
head_dim 32 are checked by the golden tests of test_decode_gpu.py. Here:
grouped query heads, ragged and zero lengths, the split schedule's partials
and the single-token known answer, against the oracle."""
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


@pytest.mark.parametrize("bs,d,hq,hkv,dtype", [
    (1, 128, 8, 8, torch.float16), (2, 64, 8, 2, torch.bfloat16), (4, 128, 16, 4, torch.bfloat16),
    (12, 128, 8, 1, torch.float16), (16, 32, 32, 8, torch.bfloat16), (4, 32, 4, 4, torch.float16),
    (64, 32, 16, 2, torch.float16), (3, 256, 4, 2, torch.bfloat16)])
def test_generic_path_against_oracle(pa, bs, d, hq, hkv, dtype):
    import oracle
    from paged_attention import workloads
    g = torch.Generator().manual_seed(bs * 1000 + d + hq)
    b = 7
    smax = 150
    lens = torch.randint(0, smax + 1, (b,), generator=g, dtype=torch.int32)
    lens[0] = 0
    lens[3] = smax
    nblk = (smax + bs - 1) // bs
    w = workloads.build("generic", b, hq, hkv, bs, dtype, lens.cuda(), nblk, b * nblk,
                        seed=bs + d, device="cuda", head_dim=d)
    plan = pa.decode_plan(w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), bs)
    assert plan["generic_path"] == 1 and plan["kernels"] == 2, plan
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lens, bs)
    ws = pa.DecodeWorkspace("cuda")
    for ns in (None, 3):
        o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, lens.cuda(), bs,
                                    ns, return_lse=True, workspace=ws)
        torch.cuda.synchronize()
        assert ws.read_status() == 0
        assert_o_close(o, ro, f"O ns={ns}")
        assert_lse_close(lse, rl, f"LSE ns={ns}")
    # uniform length and the split schedule's partials (sentinel rows bit-exact)
    s = 41
    o, lse, op, lp = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, s, bs, 5,
                                        return_lse=True, return_partials=True, workspace=ws)
    torch.cuda.synchronize()
    rop, rlp = oracle.split_partials(w.q, w.k_cache, w.v_cache, w.block_table, s, bs, 5)
    assert_o_close(op, rop, "partials")
    sentinel = rlp == -1e30
    assert torch.equal(lp.cpu()[sentinel], rlp[sentinel].float())
    assert_lse_close(lp.cpu()[~sentinel], rlp[~sentinel], "partial LSE")
    ro2, rl2 = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, s, bs)
    assert_o_close(o, ro2, "O uniform")


@pytest.mark.parametrize("bs,d", [(1, 32), (4, 128), (6, 64)])
def test_generic_path_single_token_is_the_value_row(pa, bs, d):
    """S = 1: the softmax weight is exactly 1, so O equals V[bt[b, 0], 0, kv head]
    bit for bit (block-table and head indexing)."""
    from paged_attention import workloads
    w = workloads.build("generic_s1", 3, 8, 2, bs, torch.bfloat16, 1, 2, 12, seed=d,
                        device="cuda", head_dim=d)
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 1, bs)
    torch.cuda.synchronize()
    for b in range(3):
        for h in range(8):
            assert torch.equal(o[b, h], w.v_cache[int(w.block_table[b, 0]), 0, h // 4])
