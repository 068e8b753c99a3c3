"""Same-GPU comparison with library paged-attention decode kernels.

    python compare_libs.py [--configs c1,c2,c3,c4,c5] [--iters 50]
    python compare_libs.py --head-dims 64,256 [--iters 50]
    python compare_libs.py --long [--iters 50]
    python compare_libs.py --small-batch [--iters 50]
    python compare_libs.py --reference [PATH] [--configs c1,c2,c3] [--iters 50]

``--head-dims`` runs C2-sized MHA steps (B=32, S=1024, block 16, fp16, 537 MB
of K/V) at other head dimensions instead of the five configurations (query
heads chosen so the bytes match: 64 heads at D=64, 16 at D=256). ``--long``
runs long-context shapes: one 131072-token sequence (MHA 8 heads fp16, and
Hq 32 / Hkv 8 bf16), 8 sequences of 32768 tokens and 64 ragged sequences of
1K-8K tokens (Hq 32 / Hkv 8 bf16), block 16. ``--small-batch`` runs
grouped-query shapes with few sequences (1-64 rows of 512-32768 tokens,
Hq 32 or 64 over Hkv 4 or 8, bf16, block 16), where few long segments spread
over many CTAs and the cross-CTA merge is the step's tail.

For each benchmark shape it times this operator, vLLM's
``paged_attention_v1`` / ``paged_attention_v2`` (the kernels the reference's
Layer-4 benchmark calls, ``tests/benchmark_vllm.py:9-89``) and FlashInfer's
``BatchDecodeWithPagedKVCacheWrapper``, all on the same inputs, and checks that
their outputs agree with this operator's within the parity tolerance. The
reference passes v2's arguments as ``(out, tmp_out, exp_sums, max_logits, ...)``
(``tests/benchmark_vllm.py:58``); vLLM's signature is
``(out, exp_sum, max_logits, tmp_out, ...)``, which is what is used here.

vLLM stores K as ``[blocks, Hkv, D/x, block, x]`` and V as ``[blocks, Hkv, D,
block]``; the caches are re-laid out once, outside the timed region. FlashInfer
reads the ``[blocks, block, Hkv, D]`` (NHD) layout this operator uses.
Timing: L2 flushed before every call (512 MB write, then 512 MB read), CUDA
events around the call only, median of ``--iters`` calls.

``--reference [PATH]`` times the reference's own Triton operator instead: the
unmodified ``paged_attention`` package of bw-won/paged-attention-triton,
imported from ``PATH`` (default ``baseline/_ref`` at the repository root, where
it is pip-installed) under another module name, on the shapes it supports
(C1-C3: one KV head per query head, one length for every row). Its stock call
``paged_attention(Q, K_Cache, V_Cache, Block_Table, seq_len, block_size)``
(``paged_attention/torch_kernel.py:71-73``; the ``num_splits`` heuristic of
``torch_kernel.py:19-25`` on this GPU) and its ``PagedAttnGraphRunner``
(``paged_attention/graph_runner.py:8-45``) are timed beside this operator's
eager call and graph runner: L2 flushed per call (eager and graph replay), and
back-to-back graph replays with nothing between them (the reference's Layer-3
method, ``tests/benchmark_core.py:133-145``). The reference's outputs (eager and
graph) are checked against this operator's within the parity tolerance.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

import paged_attention as pa  # noqa: E402
from paged_attention import workloads  # noqa: E402


class _Flush:
    def __init__(self):
        self.w = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
        self.r = torch.ones(128 << 20, dtype=torch.int32, device="cuda")

    def __call__(self):
        self.w.fill_(1)
        self.r.sum(dtype=torch.int64)


def _time(fn, flush, iters):
    fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) * 1e3)
    times.sort()
    return times[len(times) // 2]


def _close(a, b):
    a = a.float()
    b = b.float()
    return bool(((a - b).abs() <= 2e-3 + 1e-2 * b.abs()).all())


def _vllm_runners(w, lens, max_s, scale):
    try:
        from vllm import _custom_ops as ops
    except Exception as e:  # vLLM missing or not built for this GPU
        return {}, f"vllm unavailable: {type(e).__name__}"
    q, k, v = w.q, w.k_cache, w.v_cache
    nb, bs, hkv, d = k.shape
    x = 16 // k.element_size()
    kv = k.view(nb, bs, hkv, d // x, x).permute(0, 2, 3, 1, 4).contiguous()
    vv = v.permute(0, 2, 3, 1).contiguous()
    out = torch.empty_like(q)
    one = torch.tensor(1.0, dtype=torch.float32, device="cuda")
    runners = {}

    def v1():
        ops.paged_attention_v1(out, q, kv, vv, hkv, scale, w.block_table, lens, bs, max_s, None,
                               "auto", one, one)
        return out

    if max_s <= 8192:
        runners["vllm_v1"] = v1
    parts = (max_s + 511) // 512
    exp_sum = torch.empty(q.shape[0], q.shape[1], parts, dtype=torch.float32, device="cuda")
    max_logits = torch.empty_like(exp_sum)
    tmp = torch.empty(q.shape[0], q.shape[1], parts, d, dtype=q.dtype, device="cuda")

    def v2():
        ops.paged_attention_v2(out, exp_sum, max_logits, tmp, q, kv, vv, hkv, scale,
                               w.block_table, lens, bs, max_s, None, "auto", one, one)
        return out

    runners["vllm_v2"] = v2
    return runners, None


def _flashinfer_runner(w, lens_list, scale):
    try:
        import flashinfer
    except Exception as e:
        return None, f"flashinfer unavailable: {type(e).__name__}"
    q, k, v = w.q, w.k_cache, w.v_cache
    bs = w.block_size
    npages = [(s + bs - 1) // bs for s in lens_list]
    indptr = [0]
    for n in npages:
        indptr.append(indptr[-1] + n)
    bt = w.block_table.cpu()
    indices = torch.cat([bt[i, :n] for i, n in enumerate(npages)]).to(torch.int32)
    last = torch.tensor([s - (n - 1) * bs if n else 0 for s, n in zip(lens_list, npages)],
                        dtype=torch.int32)
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD",
                                                            use_tensor_cores=w.num_heads != w.num_kv_heads)
    wrapper.plan(torch.tensor(indptr, dtype=torch.int32, device="cuda"), indices.cuda(),
                 last.cuda(), w.num_heads, w.num_kv_heads, q.shape[-1], bs, q_data_type=q.dtype,
                 kv_data_type=k.dtype, sm_scale=scale)

    def run():
        return wrapper.run(q, (k, v))
    return run, None


REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _import_reference(path):
    """The reference package ``paged_attention`` found under ``path``, imported
    as ``reference_paged_attention`` (this package owns the name
    ``paged_attention``)."""
    import importlib.util
    init = os.path.join(path, "paged_attention", "__init__.py")
    if not os.path.exists(init):
        return None, f"reference package not found under {path}"
    spec = importlib.util.spec_from_file_location(
        "reference_paged_attention", init,
        submodule_search_locations=[os.path.dirname(init)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["reference_paged_attention"] = mod
    try:
        spec.loader.exec_module(mod)
    except Exception as e:  # noqa: BLE001 -- e.g. Triton missing
        return None, f"reference import failed: {type(e).__name__}: {str(e)[:160]}"
    return mod, None


def _time_back_to_back(fn, reps=200):
    """Mean of ``reps`` calls between one event pair, nothing between them."""
    for _ in range(10):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / reps


def run_reference(a, flush):
    """This operator against the reference's Triton operator, same inputs; the
    reference's outputs are checked against this operator's (whose parity with
    the oracle the GPU tests establish)."""
    ref, err = _import_reference(a.reference)
    if err:
        print(json.dumps({"reference": "unavailable", "why": err}), flush=True)
        return
    for name in a.configs.split(","):
        w = workloads.CONFIGS[name]("cuda")
        if w.num_heads != w.num_kv_heads or not isinstance(w.seq_len, int):
            print(json.dumps({"config": w.name, "reference": "shape not supported by the "
                              "reference (grouped KV heads or per-row lengths)"}), flush=True)
            continue
        nb = w.k_cache.shape[0]
        res = {"config": w.name, "bytes": w.effective_bytes()}

        # this operator
        ws = pa.DecodeWorkspace("cuda")

        def mine():
            return pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                      w.block_size, workspace=ws)
        mine_out = mine().clone()
        res["this_eager_us"] = _time(mine, flush, a.iters)
        runner = pa.PagedAttnGraphRunner(w.batch, w.num_heads, w.q.shape[-1], w.seq_len,
                                         w.block_size, nb, device="cuda", dtype=w.dtype)
        runner.run(w.q, w.k_cache, w.v_cache, w.block_table, copy_kv=True)
        res["this_graph_us"] = _time(runner.replay_only, flush, a.iters)
        res["this_graph_back_to_back_us"] = _time_back_to_back(runner.replay_only)
        del runner

        # the reference, stock call and stock graph runner
        def theirs():
            return ref.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                       w.block_size)
        try:
            res["reference_matches"] = _close(theirs(), mine_out)
            res["reference_eager_us"] = _time(theirs, flush, a.iters)
            rr = ref.PagedAttnGraphRunner(w.batch, w.num_heads, w.q.shape[-1], w.seq_len,
                                          w.block_size, nb, device="cuda", dtype=w.dtype)
            o = rr.run(w.q, w.k_cache, w.v_cache, w.block_table, copy_kv=True)
            torch.cuda.synchronize()
            res["reference_graph_matches"] = _close(o, mine_out)
            res["reference_graph_us"] = _time(rr.replay_only, flush, a.iters)
            res["reference_graph_back_to_back_us"] = _time_back_to_back(rr.replay_only)
            del rr
        except Exception as e:  # noqa: BLE001
            res["reference"] = f"failed: {type(e).__name__}: {str(e)[:160]}"
        for key in list(res):
            if key.endswith("_us"):
                res[key.replace("_us", "_gbs")] = round(res["bytes"] / res[key] / 1e3, 1)
                res[key] = round(res[key], 2)
        print(json.dumps(res), flush=True)
        del w


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--configs", default="c1,c2,c3,c4,c5")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--head-dims", default="", help="e.g. 64,256: C2-sized MHA at these D")
    ap.add_argument("--long", action="store_true", help="long-context shapes")
    ap.add_argument("--small-batch", action="store_true", help="few-sequence GQA shapes")
    ap.add_argument("--reference", nargs="?", const=os.path.join(REPO, "baseline", "_ref"),
                    default=None, help="time the reference's Triton operator (package path)")
    a = ap.parse_args()
    flush = _Flush()
    if a.reference is not None:
        if a.configs == "c1,c2,c3,c4,c5":
            a.configs = "c1,c2,c3"
        run_reference(a, flush)
        return
    if a.long:
        g = torch.Generator().manual_seed(7)
        ragged = torch.randint(1024, 8193, (64,), generator=g, dtype=torch.int32)
        bf16, f16 = torch.bfloat16, torch.float16
        builders = [
            ("b1_s131072_h8_mha_f16", lambda: workloads.build(
                "b1_s131072_h8_mha_f16", 1, 8, 8, 16, f16, 131072, 8192, 8192, 1, "cuda")),
            ("b1_s131072_hq32_hkv8_bf16", lambda: workloads.build(
                "b1_s131072_hq32_hkv8_bf16", 1, 32, 8, 16, bf16, 131072, 8192, 8192, 2, "cuda")),
            ("b8_s32768_hq32_hkv8_bf16", lambda: workloads.build(
                "b8_s32768_hq32_hkv8_bf16", 8, 32, 8, 16, bf16, 32768, 2048, 16384, 3, "cuda")),
            ("b64_ragged1k-8k_hq32_hkv8_bf16", lambda: workloads.build(
                "b64_ragged1k-8k_hq32_hkv8_bf16", 64, 32, 8, 16, bf16, ragged.cuda(), 512,
                64 * 512, 4, "cuda")),
        ]
    elif a.small_batch:
        shapes = [(1, 1024, 32, 8), (1, 4096, 32, 8), (4, 2048, 32, 8), (16, 1024, 32, 8),
                  (64, 512, 32, 8), (1, 8192, 64, 8), (8, 4096, 64, 8), (1, 32768, 32, 4)]
        builders = [(f"b{b}_s{s}_hq{hq}_hkv{hkv}_bf16", (lambda b=b, s=s, hq=hq, hkv=hkv:
                     workloads.build(f"b{b}_s{s}_hq{hq}_hkv{hkv}_bf16", b, hq, hkv, 16,
                                     torch.bfloat16, s, (s + 15) // 16, b * ((s + 15) // 16),
                                     1, "cuda")))
                    for b, s, hq, hkv in shapes]
    elif a.head_dims:
        heads = {64: 64, 128: 32, 256: 16}
        builders = [(f"c2size_d{d}", (lambda d=d: workloads.build(
            f"c2size_mha_d{d}_h{heads[d]}_s1024_bs16_f16", 32, heads[d], heads[d], 16,
            torch.float16, 1024, 64, 2048, 2, "cuda", head_dim=d)))
            for d in (int(x) for x in a.head_dims.split(","))]
    else:
        builders = [(name, (lambda name=name: workloads.CONFIGS[name]("cuda")))
                    for name in a.configs.split(",")]
    for name, make in builders:
        w = make()
        lens_list = w.seq_list()
        lens = torch.tensor(lens_list, dtype=torch.int32, device="cuda")
        max_s = max(lens_list)
        scale = 1.0 / math.sqrt(w.q.shape[-1])
        ws = pa.DecodeWorkspace("cuda")
        mine_out = pa.paged_attention(w.q, w.k_cache, w.v_cache, w.block_table, w.seq_len,
                                      w.block_size, workspace=ws)
        res = {"config": w.name, "bytes": w.effective_bytes()}
        res["this_us"] = _time(lambda: pa.paged_attention(w.q, w.k_cache, w.v_cache,
                                                          w.block_table, w.seq_len, w.block_size,
                                                          workspace=ws), flush, a.iters)
        runners, err = _vllm_runners(w, lens, max_s, scale)
        if err:
            res["vllm"] = err
        for key, fn in runners.items():
            try:
                o = fn().clone()
                res[key + "_us"] = _time(fn, flush, a.iters)
                res[key + "_matches"] = _close(o, mine_out)
            except Exception as e:  # noqa: BLE001
                res[key] = f"failed: {type(e).__name__}: {str(e)[:120]}"
        try:
            fi, err = _flashinfer_runner(w, lens_list, scale)
            if err:
                res["flashinfer"] = err
            else:
                o = fi().clone()
                res["flashinfer_us"] = _time(fi, flush, a.iters)
                res["flashinfer_matches"] = _close(o, mine_out)
        except Exception as e:  # noqa: BLE001
            res["flashinfer"] = f"failed: {type(e).__name__}: {str(e)[:120]}"
        for key in list(res):
            if key.endswith("_us"):
                res[key.replace("_us", "_gbs")] = round(res["bytes"] / res[key] / 1e3, 1)
                res[key] = round(res[key], 1)
        print(json.dumps(res), flush=True)
        del w


if __name__ == "__main__":
    main()
