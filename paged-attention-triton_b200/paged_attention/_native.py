"""ctypes binding of the C ABI in ``include/pa_decode.h`` (``libpa_decode.so``).

The shared library sits next to this file (built by ``build.py``). Loading
fails loudly when it is missing: there is no CPU or Triton fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_LIB_NAME = "libpa_decode.so"
_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), _LIB_NAME)

PA_OK = 0
PA_ERR_ARG = 1
PA_ERR_UNSUPPORTED = 2
PA_ERR_LAUNCH = 3
PA_ERR_WORKSPACE = 4

PA_F16 = 0
PA_BF16 = 1

PA_STATUS_BAD_BLOCK = 1
PA_STATUS_BAD_SEQLEN = 2
PA_STATUS_TIMEOUT = 4

# size of the scratch array pa_decode_noalloc uses (PA_NOALLOC_SCRATCH_BYTES)
PA_NOALLOC_SCRATCH_BYTES = 16 << 20


class DecodeParams(ctypes.Structure):
    """Mirror of ``pa_decode_params`` (field order and types must match)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_b", ctypes.c_int64),
        ("q_stride_h", ctypes.c_int64),
        ("k_cache", ctypes.c_void_p),
        ("k_stride_block", ctypes.c_int64),
        ("k_stride_slot", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_cache", ctypes.c_void_p),
        ("v_stride_block", ctypes.c_int64),
        ("v_stride_slot", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("block_table", ctypes.c_void_p),
        ("bt_stride_b", ctypes.c_int64),
        ("max_blocks", ctypes.c_int32),
        ("seq_lens", ctypes.c_void_p),
        ("seq_len", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("dtype", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("out_stride_b", ctypes.c_int64),
        ("out_stride_h", ctypes.c_int64),
        ("lse", ctypes.c_void_p),
        ("o_partial", ctypes.c_void_p),
        ("lse_partial", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("counters", ctypes.c_void_p),
        ("counter_count", ctypes.c_size_t),
        ("status", ctypes.c_void_p),
        ("kernel_variant", ctypes.c_int32),
    ]


class AppendParams(ctypes.Structure):
    """Mirror of ``pa_append_params``."""

    _fields_ = [
        ("key", ctypes.c_void_p),
        ("key_stride_t", ctypes.c_int64),
        ("key_stride_h", ctypes.c_int64),
        ("value", ctypes.c_void_p),
        ("value_stride_t", ctypes.c_int64),
        ("value_stride_h", ctypes.c_int64),
        ("k_cache", ctypes.c_void_p),
        ("k_stride_block", ctypes.c_int64),
        ("k_stride_slot", ctypes.c_int64),
        ("k_stride_head", ctypes.c_int64),
        ("v_cache", ctypes.c_void_p),
        ("v_stride_block", ctypes.c_int64),
        ("v_stride_slot", ctypes.c_int64),
        ("v_stride_head", ctypes.c_int64),
        ("slot_mapping", ctypes.c_void_p),
        ("num_tokens", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


class PlanInfo(ctypes.Structure):
    """Mirror of ``pa_decode_plan_info``."""

    _fields_ = [
        ("kernel_variant", ctypes.c_int32),
        ("tile_tokens", ctypes.c_int32),
        ("warps", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("group_warps", ctypes.c_int32),
        ("merge_rows_global", ctypes.c_int32),
        ("merge_pass", ctypes.c_int32),
        ("kernels", ctypes.c_int32),
        ("smem_bytes", ctypes.c_int32),
        ("generic_path", ctypes.c_int32),
        ("workspace_bytes", ctypes.c_size_t),
        ("counter_count", ctypes.c_size_t),
        ("cluster_size", ctypes.c_int32),
    ]


# name -> (restype, argtypes); every function declared in include/pa_decode.h.
_SIGNATURES = {
    "pa_decode_workspace": (ctypes.c_int, [ctypes.POINTER(DecodeParams),
                                           ctypes.POINTER(ctypes.c_size_t),
                                           ctypes.POINTER(ctypes.c_size_t)]),
    "pa_decode_plan": (ctypes.c_int, [ctypes.POINTER(DecodeParams), ctypes.POINTER(PlanInfo)]),
    "pa_decode": (ctypes.c_int, [ctypes.POINTER(DecodeParams), ctypes.c_void_p]),
    "pa_decode_noalloc": (ctypes.c_int, [ctypes.POINTER(DecodeParams), ctypes.c_void_p]),
    "pa_cache_append": (ctypes.c_int, [ctypes.POINTER(AppendParams), ctypes.c_void_p]),
    "pa_num_splits_heuristic": (ctypes.c_int32, [ctypes.c_int32] * 5),
    "pa_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_uint64, ctypes.c_void_p,
                                                ctypes.c_void_p]),
    "pa_stream_copy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                      ctypes.c_void_p]),
    "pa_stream_read": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                      ctypes.c_void_p]),
    "pa_device_sm_count": (ctypes.c_int32, []),
    "pa_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "pa_abi_version": (ctypes.c_int32, []),
}

_lock = threading.Lock()
_lib = None


class NativeLibraryMissing(RuntimeError):
    pass


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                raise NativeLibraryMissing(
                    f"{_LIB_PATH} is missing: build it with "
                    "`python paged-attention-triton_b200/build.py` (there is no fallback)")
            handle = ctypes.CDLL(_LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


_ext = None


def ext():
    """The PyTorch extension module ``_pa_ext`` (next to this file; no fallback)."""
    global _ext
    if _ext is None:
        lib()   # the extension links libpa_decode.so; report it first if missing
        try:
            from . import _pa_ext as mod
        except ImportError as e:
            raise NativeLibraryMissing(
                f"paged_attention/_pa_ext is missing or broken ({e}): build it with "
                "`python paged-attention-triton_b200/build.py` (there is no fallback)") from e
        _ext = mod
    return _ext


def status_string(code: int) -> str:
    return lib().pa_status_string(code).decode()


class PagedAttentionError(RuntimeError):
    def __init__(self, where: str, code: int):
        super().__init__(f"{where} failed: {status_string(code)} (code {code})")
        self.code = code
