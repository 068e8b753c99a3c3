/*
 * pa_decode.h -- C ABI of the B200 (sm_100a) paged-attention decode operator.
 *
 * Plain pointers and sizes only; no PyTorch types. Every pointer argument that
 * names tensor data is a CUDA device pointer on the current device; every call
 * is asynchronous on `stream` and never synchronises the host.
 *
 * Reference interfaces replaced (paths inside bw-won/paged-attention-triton):
 *   pa_decode                 <- paged_attention(Q, K_Cache, V_Cache, Block_Table,
 *                                seq_len, block_size, num_splits)
 *                                (paged_attention/torch_kernel.py:71-73), i.e.
 *                                PagedAttentionV2Function.forward
 *                                (paged_attention/torch_kernel.py:14-64): the
 *                                split kernel (paged_attention/split_kv_kernel.py:12-84)
 *                                and the LSE reduce kernel (split_kv_kernel.py:87-122).
 *   pa_decode_workspace       <- the partial-buffer allocation of
 *                                paged_attention/torch_kernel.py:32-35.
 *   pa_num_splits_heuristic   <- paged_attention/torch_kernel.py:19-25.
 *   pa_stream_copy            <- _copy_kernel / measure_peak_bw
 *                                (measure_peak_bw.py:15-48).
 */
#ifndef PA_DECODE_H_
#define PA_DECODE_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PA_ABI_VERSION 1

#if defined(__GNUC__)
#define PA_API __attribute__((visibility("default")))
#else
#define PA_API
#endif

/* Return codes. The reference raises Python/Triton errors or reads out of
 * bounds silently; this ABI validates on the host and never traps on device. */
typedef enum pa_status {
  PA_OK = 0,
  PA_ERR_ARG = 1,          /* null pointer, inconsistent shape, bad stride/alignment */
  PA_ERR_UNSUPPORTED = 2,  /* legal but not built: head_dim not 32/64/128/256, an explicit
                              kernel_variant the shape has no kernel for */
  PA_ERR_LAUNCH = 3,       /* CUDA runtime/driver error while launching */
  PA_ERR_WORKSPACE = 4     /* workspace or counter buffer smaller than queried */
} pa_status_t;

typedef enum pa_dtype { PA_F16 = 0, PA_BF16 = 1 } pa_dtype_t;

/* Bits of the optional device status word (OR-ed by the kernel). */
#define PA_STATUS_BAD_BLOCK 1u    /* a block-table entry outside [0, num_blocks) */
#define PA_STATUS_BAD_SEQLEN 2u   /* seq_lens[b] < 0 or > max_blocks * block_size (clamped) */
#define PA_STATUS_TIMEOUT 4u      /* a bounded wait on a copy barrier gave up (2 s) */

/* One decode step: O[b, h] = softmax(q[b, h] . K_b^T * scale) V_b, where token t
 * of sequence b lives at cache[block_table[b, t / block_size], t % block_size,
 * h / (num_heads / num_kv_heads), :].
 * All strides are in elements; the last (head_dim) dimension is contiguous. */
typedef struct pa_decode_params {
  /* query [batch, num_heads, head_dim] */
  const void* q;
  int64_t q_stride_b, q_stride_h;
  /* paged caches [num_blocks, block_size, num_kv_heads, head_dim] */
  const void* k_cache;
  int64_t k_stride_block, k_stride_slot, k_stride_head;
  const void* v_cache;
  int64_t v_stride_block, v_stride_slot, v_stride_head;
  /* block table [batch, max_blocks] int32 */
  const int32_t* block_table;
  int64_t bt_stride_b;
  int32_t max_blocks;
  /* lengths: seq_lens[batch] (device, int32) or, when NULL, seq_len for every row */
  const int32_t* seq_lens;
  int32_t seq_len;
  int32_t batch, num_heads, num_kv_heads, head_dim, block_size, num_blocks;
  /* 0: token-balanced persistent schedule (default).
   * >0: the reference's split schedule: split s of row b covers tokens
   *     [s*ceil(S_b/ns), min((s+1)*ceil(S_b/ns), S_b)); empty splits store LSE -1e30. */
  int32_t num_splits;
  float scale;                 /* softmax scale; the reference uses 1/sqrt(head_dim) */
  int32_t dtype;               /* pa_dtype_t of q, caches and out */
  /* output [batch, num_heads, head_dim] in dtype */
  void* out;
  int64_t out_stride_b, out_stride_h;
  float* lse;                  /* optional [batch, num_heads]: natural-log LSE, -1e30 if S_b == 0 */
  /* optional split-schedule partials (num_splits > 0): [batch, num_heads, ns, head_dim]
   * and [batch, num_heads, ns] fp32, contiguous. NULL: taken from the workspace. */
  float* o_partial;
  float* lse_partial;
  /* scratch: query sizes with pa_decode_workspace */
  void* workspace;
  size_t workspace_bytes;
  int32_t* counters;           /* zero-filled once by the caller; the kernel leaves it zeroed */
  size_t counter_count;
  uint32_t* status;            /* optional device word, PA_STATUS_* bits OR-ed in */
  /* 0: automatic. 1..10: a fixed kernel variant (tile tokens x warps x ring
   * depth), for tuning; see the variant table in csrc/pa_decode.cu (1-5 and
   * 10 for head_dim 128; 3, 5 and 8 for 64; 6, 7 and 9 for 256; others, and
   * any variant for head_dim 32 or pages not a multiple of 8 tokens, return
   * PA_ERR_UNSUPPORTED). */
  int32_t kernel_variant;
} pa_decode_params;

/* Bytes of workspace and number of int32 arrival counters pa_decode needs for
 * these parameters (pointers are not read). */
PA_API pa_status_t pa_decode_workspace(const pa_decode_params* p, size_t* workspace_bytes,
                                size_t* counter_count);

/* The schedule pa_decode would run for these parameters (pointers are not
 * read). Replaces nothing in the reference, whose schedule is fixed by the
 * num_splits heuristic (paged_attention/torch_kernel.py:19-25) and its two
 * launch grids (torch_kernel.py:37-62); it lets a caller or a test see which
 * kernels one call launches. */
typedef struct pa_decode_plan_info {
  int32_t kernel_variant;     /* 1..10: tile tokens x warps per CTA x ring depth */
  int32_t tile_tokens, warps, stages;
  int32_t grid;               /* CTAs of the decode kernel */
  int32_t num_splits;         /* 0: token-balanced persistent schedule; >0: split schedule */
  int32_t group_warps;        /* balanced: warps per merge group (1, or every warp of a CTA) */
  int32_t merge_rows_global;  /* balanced: the warps' merge rows live in the workspace */
  int32_t merge_pass;         /* 1: merge_segments_kernel follows the decode kernel */
  int32_t kernels;            /* launches of one call: 0 (batch 0), 1 or 2 */
  int32_t smem_bytes;         /* dynamic shared memory per CTA */
  int32_t generic_path;       /* 1: head_dim 32 or pages not a multiple of 8 tokens: the
                                 CUDA-core split + reduce kernels (kernel_variant 0) */
  size_t workspace_bytes, counter_count;   /* as pa_decode_workspace reports */
  int32_t cluster_size;       /* CTAs per thread-block cluster (0: no clusters). The device
                                 may not fit the clusters at once, in which case pa_decode
                                 falls back to the plain schedule. */
} pa_decode_plan_info;

PA_API pa_status_t pa_decode_plan(const pa_decode_params* p, pa_decode_plan_info* info);

/* Launch one decode step on `stream`: the decode kernel, followed (in the same
 * stream, as a programmatic dependent launch) by merge_segments_kernel when the
 * plan has a merge pass. If the call returns PA_ERR_LAUNCH after the first
 * kernel was queued, `out` and `lse` are undefined for that step. */
PA_API pa_status_t pa_decode(const pa_decode_params* p, cudaStream_t stream);

/* New tokens' K/V rows into the paged caches (the step before decode in a
 * serving loop; the reference fills its caches in test code,
 * tests/correctness.py:30-36). Row t of key/value ([num_tokens, num_kv_heads,
 * head_dim], element strides, head_dim contiguous) goes to
 * cache[slot / block_size, slot % block_size, :, :] with slot = slot_mapping[t];
 * a negative slot skips the row (padding). A slot beyond the pool skips the row
 * and ORs PA_STATUS_BAD_BLOCK into *status (when given). */
typedef struct pa_append_params {
  const void* key;
  int64_t key_stride_t, key_stride_h;
  const void* value;
  int64_t value_stride_t, value_stride_h;
  void* k_cache;
  int64_t k_stride_block, k_stride_slot, k_stride_head;
  void* v_cache;
  int64_t v_stride_block, v_stride_slot, v_stride_head;
  const int64_t* slot_mapping;   /* [num_tokens], device */
  int32_t num_tokens, num_kv_heads, head_dim, block_size, num_blocks;
  int32_t dtype;                 /* pa_dtype_t (element size 2) */
  uint32_t* status;              /* optional device word */
} pa_append_params;

PA_API pa_status_t pa_cache_append(const pa_append_params* p, cudaStream_t stream);

/* Allocation-free variant of pa_decode. It has no counterpart in the reference.
 *
 * pa_decode needs scratch memory (partial outputs of split segments and the
 * arrival counters) that the caller allocates. Some callers cannot allocate
 * device memory: a plugin or operator host that hands a kernel only its
 * input and output buffers, a runtime whose device memory is carved up once at
 * start-up with no allocator reachable afterwards, or a C caller without
 * access to a device allocator. pa_decode_noalloc takes the same parameters,
 * ignores `workspace`, `workspace_bytes`, `counters` and `counter_count`, and
 * uses a fixed scratch array that the library itself holds in device memory:
 *
 *  - The array is PA_NOALLOC_SCRATCH_BYTES (16 MiB) and every GPU that loads
 *    the library keeps it until the process exits. A call whose scratch
 *    (partials + counters, as pa_decode_workspace reports) does not fit is
 *    rejected with PA_ERR_WORKSPACE, before anything is launched.
 *    Rejections for bad arguments, strides or alignment (PA_ERR_ARG) and for
 *    size happen before anything is queued on `stream`.
 *  - The first call on each device looks up the array's device address once
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before any stream capture.
 *  - Every call on a device shares the one array, and the array keeps the
 *    last call's contents. Each call clears the counter part (an async memset
 *    on `stream`) before its kernel. Calls whose executions overlap on the GPU
 *    (different streams without ordering between them) race on the array and
 *    give wrong results; order them on one stream.
 *  - It calls no cudaMalloc, cudaFree or other allocating routine. */
#define PA_NOALLOC_SCRATCH_BYTES (16u << 20)
PA_API pa_status_t pa_decode_noalloc(const pa_decode_params* p, cudaStream_t stream);

/* max(1, min(ceil(S / block_size), max(1, 4 * sm_count / (batch * heads)))). */
PA_API int32_t pa_num_splits_heuristic(int32_t batch, int32_t heads, int32_t seq_len,
                                int32_t block_size, int32_t sm_count);

/* Self-test of the decode kernel's bounded barrier wait, its only device-side
 * failure handling (the reference has none). One warp waits on a barrier that
 * nothing completes: after `limit_ns` (1 us .. 100 ms, else PA_ERR_ARG) the
 * wait gives up, ORs PA_STATUS_TIMEOUT into *status and, as the decode kernel
 * does, waits (bounded) for its other copy in flight -- 256 bytes from `src`,
 * which it writes to `dst` (16-byte aligned) -- and returns. The context stays
 * usable. */
PA_API pa_status_t pa_selftest_wait_timeout(const void* src, void* dst, uint64_t limit_ns,
                                            uint32_t* status, cudaStream_t stream);

/* Streaming copy of `bytes` (multiple of 16, 16-byte aligned pointers): the
 * HBM peak-bandwidth probe. */
PA_API pa_status_t pa_stream_copy(const void* src, void* dst, size_t bytes, cudaStream_t stream);

/* Streaming read of `bytes` (multiple of 16, 16-byte aligned) folded into
 * `sink[0]` (one uint32 on the device): the read-only bandwidth probe. */
PA_API pa_status_t pa_stream_read(const void* src, size_t bytes, uint32_t* sink, cudaStream_t stream);

/* Number of streaming multiprocessors of the current device (cached). */
PA_API int32_t pa_device_sm_count(void);

PA_API const char* pa_status_string(pa_status_t s);
PA_API int32_t pa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PA_DECODE_H_ */
