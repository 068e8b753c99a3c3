// torch_ext.cpp -- thin PyTorch extension over the C ABI (include/pa_decode.h).
//
// One Python call = argument checks, output allocation from the caching
// allocator, a workspace-size query and one pa_decode launch on the current
// CUDA stream, all in C++ (the equivalent Python/ctypes path costs ~15 us per
// call). The launcher itself lives in libpa_decode.so; this module only maps
// at::Tensor arguments onto pa_decode_params.
//
// Reference interface: paged_attention(Q, K_Cache, V_Cache, Block_Table,
// seq_len, block_size, num_splits) (paged_attention/torch_kernel.py:71-73).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <tuple>
#include <vector>

#include "pa_decode.h"

namespace {

void check(bool cond, const char* msg) { TORCH_CHECK_VALUE(cond, "paged_attention: ", msg); }

int dtype_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kHalf) return PA_F16;
  if (t.scalar_type() == at::kBFloat16) return PA_BF16;
  TORCH_CHECK_VALUE(false, "paged_attention: unsupported dtype ", t.scalar_type(),
                    " (fp16 or bf16)");
  return -1;
}

// Returns (status, tensors): status 0 and [out[, lse][, o_partial, lse_partial]]
// on success; when the workspace is too small nothing is launched and the
// result is (-1, []) with the needed sizes in the last two fields.
std::tuple<int64_t, std::vector<at::Tensor>, int64_t, int64_t> decode(
    const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& bt,
    const c10::optional<at::Tensor>& seq_lens, int64_t seq_len, int64_t block_size,
    int64_t num_splits, double scale, bool return_lse, bool return_partials,
    const at::Tensor& ws_buffer, const at::Tensor& ws_counters, const at::Tensor& ws_status,
    int64_t kernel_variant, const c10::optional<at::Tensor>& out_opt) {
  check(q.is_cuda() && k.is_cuda() && v.is_cuda() && bt.is_cuda(),
        "Q, K_Cache, V_Cache and Block_Table must be CUDA tensors");
  check(q.dim() == 3, "Q must be [B, H, D]");
  check(k.dim() == 4 && v.sizes() == k.sizes(),
        "K_Cache and V_Cache must both be [num_blocks, block_size, Hkv, D]");
  const int dt = dtype_code(q);
  check(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
        "Q, K_Cache and V_Cache must share one dtype");
  check(bt.scalar_type() == at::kInt && bt.dim() == 2,
        "Block_Table must be an int32 [B, max_blocks] tensor");
  const auto dev = q.device();
  check(k.device() == dev && v.device() == dev && bt.device() == dev,
        "tensors on different devices");
  const int64_t batch = q.size(0), heads = q.size(1), dim = q.size(2);
  const int64_t nblocks = k.size(0), bs = k.size(1), kv_heads = k.size(2);
  check(k.size(3) == dim, "head_dim of Q and the caches differ");
  check(dim == 32 || dim == 64 || dim == 128 || dim == 256,
        "head_dim must be 32, 64, 128 or 256");
  check(block_size == bs, "block_size differs from the cache's block dimension");
  check(bs >= 1, "block_size must be positive");
  check(heads % kv_heads == 0, "Hq must be a multiple of Hkv");
  check(bt.size(0) == batch, "Block_Table rows != batch");
  check(q.stride(2) == 1 && k.stride(3) == 1 && v.stride(3) == 1 && bt.stride(1) == 1,
        "last dimensions must be contiguous");
  at::Tensor Q = q;
  if (q.stride(0) % 8 || q.stride(1) % 8 || reinterpret_cast<uintptr_t>(q.data_ptr()) % 16)
    Q = q.contiguous();
  const int64_t max_blocks = bt.size(1);

  c10::cuda::CUDAGuard guard(dev);
  at::Tensor lens;
  if (seq_lens.has_value()) {
    lens = *seq_lens;
    check(lens.numel() == batch, "seq_lens must have B entries");
    if (lens.device() != dev || lens.scalar_type() != at::kInt || !lens.is_contiguous())
      lens = lens.to(dev, at::kInt).contiguous();
  } else {
    check(seq_len >= 0 && seq_len <= max_blocks * bs, "seq_len exceeds the Block_Table capacity");
  }
  check(num_splits >= 0, "num_splits must be >= 0");
  int64_t ns = num_splits;
  if (return_partials && ns == 0) {
    const int64_t s = seq_lens.has_value() ? max_blocks * bs : seq_len;
    ns = pa_num_splits_heuristic(static_cast<int32_t>(batch), static_cast<int32_t>(heads),
                                 static_cast<int32_t>(s), static_cast<int32_t>(bs),
                                 pa_device_sm_count());
  }

  const auto opts = Q.options();
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({batch, heads, dim}, opts);
  check(out.sizes() == Q.sizes() && out.scalar_type() == Q.scalar_type() && out.stride(2) == 1,
        "out must match Q's shape and dtype");
  const auto f32 = opts.dtype(at::kFloat);
  at::Tensor lse, o_part, lse_part;
  if (return_lse) lse = at::empty({batch, heads}, f32);
  if (return_partials) {
    o_part = at::empty({batch, heads, ns, dim}, f32);
    lse_part = at::empty({batch, heads, ns}, f32);
  }

  pa_decode_params p{};
  p.q = Q.data_ptr();
  p.q_stride_b = Q.stride(0);
  p.q_stride_h = Q.stride(1);
  p.k_cache = k.data_ptr();
  p.k_stride_block = k.stride(0);
  p.k_stride_slot = k.stride(1);
  p.k_stride_head = k.stride(2);
  p.v_cache = v.data_ptr();
  p.v_stride_block = v.stride(0);
  p.v_stride_slot = v.stride(1);
  p.v_stride_head = v.stride(2);
  p.block_table = bt.data_ptr<int32_t>();
  p.bt_stride_b = bt.stride(0);
  p.max_blocks = static_cast<int32_t>(max_blocks);
  p.seq_lens = seq_lens.has_value() ? lens.data_ptr<int32_t>() : nullptr;
  p.seq_len = seq_lens.has_value() ? 0 : static_cast<int32_t>(seq_len);
  p.batch = static_cast<int32_t>(batch);
  p.num_heads = static_cast<int32_t>(heads);
  p.num_kv_heads = static_cast<int32_t>(kv_heads);
  p.head_dim = static_cast<int32_t>(dim);
  p.block_size = static_cast<int32_t>(bs);
  p.num_blocks = static_cast<int32_t>(nblocks);
  p.num_splits = static_cast<int32_t>(ns);
  p.scale = static_cast<float>(scale > 0 ? scale : 1.0 / std::sqrt(static_cast<double>(dim)));
  p.dtype = dt;
  p.out = out.data_ptr();
  p.out_stride_b = out.stride(0);
  p.out_stride_h = out.stride(1);
  p.lse = return_lse ? lse.data_ptr<float>() : nullptr;
  p.o_partial = return_partials ? o_part.data_ptr<float>() : nullptr;
  p.lse_partial = return_partials ? lse_part.data_ptr<float>() : nullptr;
  p.kernel_variant = static_cast<int32_t>(kernel_variant);

  size_t ws_bytes = 0, n_counters = 0;
  pa_status_t rc = pa_decode_workspace(&p, &ws_bytes, &n_counters);
  TORCH_CHECK(rc == PA_OK, "pa_decode_workspace failed: ", pa_status_string(rc));
  if (ws_bytes > static_cast<size_t>(ws_buffer.numel()) ||
      n_counters > static_cast<size_t>(ws_counters.numel())) {
    return {-1, {}, static_cast<int64_t>(ws_bytes), static_cast<int64_t>(n_counters)};
  }
  p.workspace = ws_buffer.numel() ? ws_buffer.data_ptr() : nullptr;
  p.workspace_bytes = static_cast<size_t>(ws_buffer.numel());
  p.counters = ws_counters.data_ptr<int32_t>();
  p.counter_count = static_cast<size_t>(ws_counters.numel());
  p.status = reinterpret_cast<uint32_t*>(ws_status.data_ptr<int32_t>());

  rc = pa_decode(&p, c10::cuda::getCurrentCUDAStream(dev.index()).stream());
  TORCH_CHECK(rc == PA_OK, "pa_decode failed: ", pa_status_string(rc));

  std::vector<at::Tensor> res{out};
  if (return_lse) res.push_back(lse);
  if (return_partials) {
    res.push_back(o_part);
    res.push_back(lse_part);
  }
  return {0, std::move(res), 0, 0};
}

// Writes key/value rows [T, Hkv, D] into the paged caches at slot_mapping[t]
// (negative: skipped) through pa_cache_append.
void cache_append(const at::Tensor& key, const at::Tensor& value, const at::Tensor& k_cache,
                  const at::Tensor& v_cache, const at::Tensor& slot_mapping,
                  const c10::optional<at::Tensor>& status) {
  check(key.is_cuda() && value.is_cuda() && k_cache.is_cuda() && v_cache.is_cuda() &&
            slot_mapping.is_cuda(),
        "cache_append: all tensors must be CUDA tensors");
  check(key.dim() == 3 && value.sizes() == key.sizes(), "key and value must be [T, Hkv, D]");
  check(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes(),
        "caches must be [num_blocks, block_size, Hkv, D]");
  check(key.size(1) == k_cache.size(2) && key.size(2) == k_cache.size(3),
        "key rows and cache rows differ in Hkv or D");
  const int dt = dtype_code(key);
  check(value.scalar_type() == key.scalar_type() && k_cache.scalar_type() == key.scalar_type() &&
            v_cache.scalar_type() == key.scalar_type(),
        "key, value and caches must share one dtype");
  check(slot_mapping.scalar_type() == at::kLong && slot_mapping.dim() == 1 &&
            slot_mapping.size(0) == key.size(0) && slot_mapping.is_contiguous(),
        "slot_mapping must be a contiguous int64 [T] tensor");
  check(key.stride(2) == 1 && value.stride(2) == 1 && k_cache.stride(3) == 1 &&
            v_cache.stride(3) == 1,
        "head_dim must be contiguous");
  c10::cuda::CUDAGuard guard(key.device());
  pa_append_params a{};
  a.key = key.data_ptr();
  a.key_stride_t = key.stride(0);
  a.key_stride_h = key.stride(1);
  a.value = value.data_ptr();
  a.value_stride_t = value.stride(0);
  a.value_stride_h = value.stride(1);
  a.k_cache = k_cache.data_ptr();
  a.k_stride_block = k_cache.stride(0);
  a.k_stride_slot = k_cache.stride(1);
  a.k_stride_head = k_cache.stride(2);
  a.v_cache = v_cache.data_ptr();
  a.v_stride_block = v_cache.stride(0);
  a.v_stride_slot = v_cache.stride(1);
  a.v_stride_head = v_cache.stride(2);
  a.slot_mapping = slot_mapping.data_ptr<int64_t>();
  a.num_tokens = static_cast<int32_t>(key.size(0));
  a.num_kv_heads = static_cast<int32_t>(key.size(1));
  a.head_dim = static_cast<int32_t>(key.size(2));
  a.block_size = static_cast<int32_t>(k_cache.size(1));
  a.num_blocks = static_cast<int32_t>(k_cache.size(0));
  a.dtype = dt;
  a.status = status.has_value() ? reinterpret_cast<uint32_t*>(status->data_ptr<int32_t>())
                                : nullptr;
  const pa_status_t rc =
      pa_cache_append(&a, c10::cuda::getCurrentCUDAStream(key.device().index()).stream());
  TORCH_CHECK(rc == PA_OK, "pa_cache_append failed: ", pa_status_string(rc));
}

}  // namespace

PYBIND11_MODULE(_pa_ext, m) {
  m.def("cache_append", &cache_append, "write K/V rows into the paged caches by slot");
  m.doc() = "PyTorch binding of the sm_100a paged-attention decode C ABI";
  m.def("decode", &decode, "one paged-attention decode step (see torch_kernel.py)");
}
