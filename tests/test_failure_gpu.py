"""Device-side failure handling, exercised without faulting the GPU.

The decode kernel's only device-side failure path is a copy barrier whose
phase never completes: its bounded wait gives up (after 2 s in the decode
kernel), ORs PA_STATUS_TIMEOUT into the status word, waits (bounded) for the
copies still in flight on the other ring stages and returns, so that the
context stays usable. ``pa_selftest_wait_timeout`` runs those same device
functions on a barrier that nothing completes (one arrival of the two it
expects), with a 1 ms limit. The test checks the status word, that the copy in
flight on the other stage landed before the warp returned, and that a normal
decode call on the same stream afterwards is correct and clean."""
import ctypes

import pytest
import torch

from helpers import assert_o_close

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_flags_and_returns():
    import paged_attention as pa
    from paged_attention import _native, workloads
    import oracle
    lib = _native.lib()
    src = torch.arange(64, dtype=torch.int32, device="cuda") * 7 + 3
    dst = torch.zeros(64, dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    for limit_ns in (10 ** 6, 10 ** 5):
        status.zero_()
        dst.zero_()
        rc = lib.pa_selftest_wait_timeout(src.data_ptr(), dst.data_ptr(), limit_ns,
                                          status.data_ptr(), stream.cuda_stream)
        assert rc == _native.PA_OK
        torch.cuda.synchronize()
        assert int(status.item()) == _native.PA_STATUS_TIMEOUT
        assert torch.equal(dst, src)       # the other stage's copy landed before the return
    # the context is still usable: a decode step on the same stream is correct and clean
    w = workloads.build("after_timeout", 3, 8, 2, 16, torch.bfloat16, 300, 19, 57, seed=9,
                        device="cuda")
    ws = pa.DecodeWorkspace("cuda")
    o = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, 300, 16, workspace=ws)
    torch.cuda.synchronize()
    assert ws.read_status() == 0
    ro, _ = oracle.decode_reference(w.q, w.k_cache, w.v_cache, w.block_table, 300, 16)
    assert_o_close(o, ro, "decode after the timeout self-test")
