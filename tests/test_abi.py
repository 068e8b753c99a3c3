"""CPU tests of the C-ABI boundary: the library loads without a GPU, exports
every function the header declares, and the ctypes struct matches the C layout."""
import ctypes
import os
import re
import shutil
import subprocess

import pytest

import oracle
from paged_attention import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pa_decode.h")


def _declared_functions():
    text = open(HEADER).read()
    return re.findall(r"PA_API\s+[\w\s\*]+?\b(pa_\w+)\s*\(", text)


def test_header_declares_expected_entry_points():
    names = set(_declared_functions())
    assert {"pa_decode", "pa_decode_workspace", "pa_num_splits_heuristic", "pa_stream_copy",
            "pa_stream_read", "pa_device_sm_count", "pa_status_string",
            "pa_abi_version", "pa_cache_append", "pa_decode_plan",
            "pa_selftest_wait_timeout", "pa_decode_noalloc"} <= names


def test_ctypes_binding_covers_every_declared_function():
    assert set(_declared_functions()) == set(_native._SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in _declared_functions():
        assert hasattr(lib, name), f"{name} not exported by {_native.library_path()}"
    assert lib.pa_abi_version() == 1


def test_library_has_no_cudart_runtime_dependency():
    ldd = shutil.which("ldd")
    if not ldd:
        pytest.skip("ldd not available")
    out = subprocess.run([ldd, _native.library_path()], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


@pytest.mark.parametrize("cname,pyname", [("pa_decode_params", "DecodeParams"),
                                          ("pa_append_params", "AppendParams"),
                                          ("pa_decode_plan_info", "PlanInfo")])
def test_struct_layout_matches_header(tmp_path, cname, pyname):
    gcc = shutil.which("gcc")
    if not gcc:
        pytest.skip("gcc not available")
    cls = getattr(_native, pyname)
    fields = [f[0] for f in cls._fields_]
    src = ['#include <stdio.h>', '#include <stddef.h>', '#include "pa_decode.h"',
           'int main(void) {', f'printf("size %zu\\n", sizeof({cname}));']
    for f in fields:
        src.append(f'printf("{f} %zu\\n", offsetof({cname}, {f}));')
    src += ["return 0;", "}"]
    c = tmp_path / "probe.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "probe"
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run([gcc, "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, str(c), "-o",
                    str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    got = dict(line.split() for line in out.strip().splitlines())
    assert int(got["size"]) == ctypes.sizeof(cls)
    for f in fields:
        assert int(got[f]) == getattr(cls, f).offset, f


@pytest.mark.parametrize("b,h,s,bs,sm", [(1, 32, 128, 16, 148), (32, 32, 1024, 16, 148),
                                         (1, 32, 4096, 128, 148), (128, 32, 256, 16, 148),
                                         (1, 8, 4096, 16, 20), (3, 5, 7, 8, 1), (1, 1, 0, 16, 148)])
def test_heuristic_matches_reference_formula(b, h, s, bs, sm):
    assert _native.lib().pa_num_splits_heuristic(b, h, s, bs, sm) == \
        oracle.num_splits_heuristic(b, h, s, bs, sm)


def _params(**kw):
    p = _native.DecodeParams()
    p.batch, p.num_heads, p.num_kv_heads, p.head_dim = 2, 8, 2, 128
    p.block_size, p.num_blocks, p.max_blocks, p.seq_len = 16, 8, 4, 50
    p.scale, p.dtype = 0.088, _native.PA_F16
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize("kw,code", [
    ({"num_heads": 6, "num_kv_heads": 4}, _native.PA_ERR_ARG),     # Hq % Hkv != 0
    ({"dtype": 7}, _native.PA_ERR_ARG),
    ({"seq_len": 65}, _native.PA_ERR_ARG),                          # > max_blocks * bs
    ({"num_splits": -1}, _native.PA_ERR_ARG),
    ({"head_dim": 96}, _native.PA_ERR_UNSUPPORTED),
    ({"head_dim": 16}, _native.PA_ERR_UNSUPPORTED),
    ({"head_dim": 32, "kernel_variant": 3}, _native.PA_ERR_UNSUPPORTED),    # CUDA-core path only
    ({"head_dim": 256, "kernel_variant": 3}, _native.PA_ERR_UNSUPPORTED),   # not built for 256
    ({"head_dim": 64, "kernel_variant": 1}, _native.PA_ERR_UNSUPPORTED),    # not built for 64
    ({"head_dim": 128, "kernel_variant": 6}, _native.PA_ERR_UNSUPPORTED),   # not built for 128
    ({"kernel_variant": 11}, _native.PA_ERR_ARG),                           # no such variant
    ({"kernel_variant": 8}, _native.PA_ERR_UNSUPPORTED),                    # head_dim 64 only
    ({"block_size": 12, "seq_len": 40, "kernel_variant": 5}, _native.PA_ERR_UNSUPPORTED),
    ({"block_size": 1 << 21, "max_blocks": 1, "seq_len": 40}, _native.PA_ERR_UNSUPPORTED),
])
def test_host_validation_without_gpu(kw, code):
    lib = _native.lib()
    p = _params(**kw)
    a, b = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.pa_decode_workspace(ctypes.byref(p), ctypes.byref(a), ctypes.byref(b)) == code
    assert lib.pa_decode(ctypes.byref(p), None) == code


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_workspace_scales_with_head_dim(head_dim):
    """Split-schedule partials are [B, Hq, ns, D] floats plus one LSE each."""
    lib = _native.lib()
    p = _params(head_dim=head_dim, num_splits=3)
    a, b = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.pa_decode_workspace(ctypes.byref(p), ctypes.byref(a), ctypes.byref(b)) == 0
    assert a.value == 2 * 8 * 3 * (head_dim + 1) * 4
    assert b.value == 2 * 2          # one counter per (row, KV head)


def test_null_params_rejected():
    lib = _native.lib()
    assert lib.pa_decode(None, None) == _native.PA_ERR_ARG
    assert lib.pa_stream_copy(None, None, 16, None) == _native.PA_ERR_ARG


def test_status_strings():
    assert _native.status_string(0) == "ok"
    assert "unsupported" in _native.status_string(2)


@pytest.mark.parametrize("limit_ns", [0, 999, 100000001, 2 ** 63])
def test_wait_timeout_selftest_rejects_limits_out_of_range(limit_ns):
    """Validated on the host before any CUDA call (so this runs without a GPU)."""
    lib = _native.lib()
    buf = ctypes.create_string_buffer(512)
    addr = (ctypes.addressof(buf) + 15) & ~15
    assert lib.pa_selftest_wait_timeout(addr, addr + 256, limit_ns, addr, None) == _native.PA_ERR_ARG


def test_wait_timeout_selftest_rejects_null_and_misaligned_pointers():
    lib = _native.lib()
    buf = ctypes.create_string_buffer(512)
    addr = (ctypes.addressof(buf) + 15) & ~15
    assert lib.pa_selftest_wait_timeout(None, addr, 10 ** 6, addr, None) == _native.PA_ERR_ARG
    assert lib.pa_selftest_wait_timeout(addr, None, 10 ** 6, addr, None) == _native.PA_ERR_ARG
    assert lib.pa_selftest_wait_timeout(addr, addr, 10 ** 6, None, None) == _native.PA_ERR_ARG
    assert lib.pa_selftest_wait_timeout(addr + 4, addr, 10 ** 6, addr, None) == _native.PA_ERR_ARG
