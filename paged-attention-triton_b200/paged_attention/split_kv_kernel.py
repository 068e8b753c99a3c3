"""Constants of the split / reduce stages.

The reference module of this name (``paged_attention/split_kv_kernel.py`` of
bw-won/paged-attention-triton) holds the two Triton kernels and the LSE
sentinel constants. Here both stages are one sm_100a CUDA kernel
(``csrc/pa_decode.cu``, launched through ``pa_decode`` in
``include/pa_decode.h``); this module keeps the constants under their
reference names so code that imports them keeps working.
"""

# split_kv_kernel.py:8-9 -- an empty split's partial LSE reads as -1e30; the
# reduce treats any LSE <= -1e29 as "no tokens in this split".
LSE_SENTINEL = -1e30
LSE_VALID_THRESHOLD = -1e29

# Tokens per pipeline stage of the CUDA kernel (the reference's BLOCK_N was the
# page size; the CUDA kernel decouples its tile from the page size).
TILE_TOKENS = 32
