"""B200 (sm_100a) paged-attention decode operator.

Drop-in for the ``paged_attention`` package of bw-won/paged-attention-triton
(reference ``paged_attention/__init__.py:1-4``): the same two exports, backed by
hand-written CUDA through the C ABI in ``include/pa_decode.h``.
"""
from .torch_kernel import (  # noqa: F401
    paged_attention,
    PagedAttentionV2Function,
    DecodeWorkspace,
    num_splits_heuristic,
    device_sm_count,
    decode_params,
    decode_plan,
)
from .graph_runner import PagedAttnGraphRunner  # noqa: F401
from .cache_ops import write_kv_cache, slots_for_positions  # noqa: F401
from .split_kv_kernel import LSE_SENTINEL, LSE_VALID_THRESHOLD  # noqa: F401

__all__ = ["paged_attention", "PagedAttnGraphRunner"]
