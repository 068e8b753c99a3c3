"""CPU oracle for the paged-attention decode op.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only to check or time the CUDA path. The shipped operator
(``paged_attention``) never imports it and has no CPU fallback.
"""
from .pa_oracle import (  # noqa: F401
    LSE_SENTINEL,
    LSE_VALID_THRESHOLD,
    decode_reference,
    split_partials,
    reduce_partials,
    num_splits_heuristic,
    gather_sequence,
    effective_bytes,
)
