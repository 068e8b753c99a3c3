"""GPU tests of the KV-cache append (``write_kv_cache`` -> ``pa_cache_append``)."""
import pytest
import torch

from helpers import assert_lse_close, assert_o_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bs,hkv,d", [(16, 8, 128), (24, 2, 128), (128, 4, 128), (16, 4, 64)])
def test_append_matches_indexing(dtype, bs, hkv, d):
    import paged_attention as pa
    g = torch.Generator(device="cuda").manual_seed(bs + hkv)
    nb, t = 40, 57
    kc = torch.randn(nb, bs, hkv, d, device="cuda", generator=g).to(dtype)
    vc = torch.randn_like(kc)
    key = torch.randn(t, hkv, d, device="cuda", generator=g).to(dtype)
    val = torch.randn_like(key)
    slots = torch.randperm(nb * bs, device="cuda", generator=g)[:t].to(torch.int64)
    slots[::7] = -1                                  # padding rows are skipped
    ek, ev = kc.clone(), vc.clone()
    keep = slots >= 0
    ek.view(-1, hkv, d)[slots[keep]] = key[keep]
    ev.view(-1, hkv, d)[slots[keep]] = val[keep]
    pa.write_kv_cache(key, val, kc, vc, slots)
    torch.cuda.synchronize()
    assert torch.equal(kc, ek) and torch.equal(vc, ev)


def test_append_strided_qkv_and_int32_slots():
    import paged_attention as pa
    hkv, d, bs, nb, t = 4, 128, 16, 16, 9
    qkv = torch.randn(t, 3, hkv, d, device="cuda", dtype=torch.bfloat16)
    kc = torch.zeros(nb, bs, hkv, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.arange(3, 3 + t, device="cuda", dtype=torch.int32) * 5
    pa.write_kv_cache(qkv[:, 1], qkv[:, 2], kc, vc, slots)
    torch.cuda.synchronize()
    assert torch.equal(kc.view(-1, hkv, d)[slots.long()], qkv[:, 1])
    assert torch.equal(vc.view(-1, hkv, d)[slots.long()], qkv[:, 2])


def test_append_out_of_pool_slot_flagged():
    import paged_attention as pa
    kc = torch.zeros(4, 16, 2, 128, device="cuda", dtype=torch.float16)
    vc = torch.zeros_like(kc)
    key = torch.ones(2, 2, 128, device="cuda", dtype=torch.float16)
    slots = torch.tensor([3, 4 * 16 + 5], device="cuda", dtype=torch.int64)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    pa.write_kv_cache(key, key, kc, vc, slots, status)
    torch.cuda.synchronize()
    assert status.item() & 1
    assert kc.abs().sum().item() == 2 * 128  # only the in-pool row was written


def test_append_then_decode_matches_oracle():
    """A decode step after appending each row's newest token through its block table."""
    import oracle
    import paged_attention as pa
    from paged_attention import workloads
    lens = torch.tensor([1, 17, 64, 200, 33], dtype=torch.int32)
    w = workloads.build("append", 5, 16, 4, 16, torch.bfloat16, lens.cuda(), 13, 80, seed=21,
                        device="cuda")
    new_k = torch.randn(5, 4, 128, device="cuda", dtype=torch.bfloat16)
    new_v = torch.randn_like(new_k)
    pos = (lens - 1).cuda()                                  # overwrite each row's last token
    slots = pa.slots_for_positions(w.block_table, pos, 16)
    pa.write_kv_cache(new_k, new_v, w.k_cache, w.v_cache, slots)
    o, lse = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len, 16,
                                return_lse=True)
    torch.cuda.synchronize()
    for b in range(5):
        s = int(lens[b])
        rows_k = oracle.gather_sequence(w.k_cache.cpu(), w.block_table[b].cpu(), s, 16)
        assert torch.equal(rows_k[s - 1], new_k[b].cpu())
    ro, rl = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, lens, 16)
    assert_o_close(o, ro, "decode after append")
    assert_lse_close(lse, rl, "decode after append LSE")
