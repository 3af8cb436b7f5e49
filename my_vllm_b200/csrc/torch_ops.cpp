// torch_ops.cpp — the B200 kernels as PyTorch operators (torch.ops.b200.*).
//
// A thin C++ layer over the C ABI of include/b200_paged_attn.h, registered
// with TORCH_LIBRARY the way the reference engine exposes its own CUDA op
// (csrc/silu_and_mul.cpp:24-29, built by setup.py:7-14 with
// torch.utils.cpp_extension). Every op works in place on caller tensors, on
// the current CUDA stream, and returns nothing; the Meta implementations do
// nothing (no shape changes, no outputs), so the ops trace under FakeTensor /
// torch.compile. Argument checks raise through TORCH_CHECK (RuntimeError in
// Python); an ABI error carries b200_last_error().
//
//   kv_append      <- store_kvcache (nanovllm/layers/attention.py:34-41)
//   paged_decode   <- BatchDecodeWithPagedKVCacheWrapper.run (attention_backend.py:995-997)
//   paged_prefill  <- BatchPrefillWithPagedKVCacheWrapper.run (attention_backend.py:992-994)
#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <optional>

#include "../../include/b200_paged_attn.h"

namespace {

int32_t activation_dtype(at::ScalarType t) {
  if (t == at::kBFloat16) return B200_DTYPE_BFLOAT16;
  if (t == at::kHalf) return B200_DTYPE_FLOAT16;
  TORCH_CHECK(false, "b200: q, key and value must be float16 or bfloat16, got ", t);
  return -1;
}

void check_abi(int rc, const char* what) {
  TORCH_CHECK(rc == B200_OK, "b200: ", what, " failed: ", b200_last_error());
}

void* current_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void require_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "b200: ", name,
              " must be a CUDA tensor (the B200 path has no CPU fallback)");
}

const float* scale_ptr(const std::optional<at::Tensor>& s, const char* name) {
  if (!s.has_value()) return nullptr;
  TORCH_CHECK(s->is_cuda() && s->scalar_type() == at::kFloat && s->numel() == 1, "b200: ",
              name, " must be a 1-element float32 CUDA tensor");
  return s->data_ptr<float>();
}

int32_t* status_ptr(const std::optional<at::Tensor>& s) {
  if (!s.has_value()) return nullptr;
  TORCH_CHECK(s->is_cuda() && s->scalar_type() == at::kInt && s->numel() >= 1,
              "b200: status must be an int32 CUDA tensor");
  return s->data_ptr<int32_t>();
}

void require_int32_vector(const at::Tensor& t, const char* name) {
  require_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == at::kInt, "b200: ", name, " must be int32");
  TORCH_CHECK(t.dim() == 1 && (t.numel() <= 1 || t.stride(0) == 1), "b200: ", name,
              " must be a contiguous 1-D tensor");
}

void require_block_tables(const at::Tensor& t) {
  require_cuda(t, "block_tables");
  TORCH_CHECK(t.scalar_type() == at::kInt, "b200: block_tables must be int32");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "b200: block_tables rows must be contiguous");
}

// The NHD cache pair [num_blocks, block_size, num_kv_heads, head_dim].
b200_paged_cache cache_desc(const at::Tensor& k, const at::Tensor& v, at::ScalarType q_dtype,
                            const std::optional<at::Tensor>& k_scale,
                            const std::optional<at::Tensor>& v_scale) {
  require_cuda(k, "k_cache");
  require_cuda(v, "v_cache");
  TORCH_CHECK(k.dim() == 4 && k.sizes() == v.sizes(),
              "b200: key and value caches must have shape "
              "[pages, block_size, num_kv_heads, head_dim]");
  TORCH_CHECK(k.strides() == v.strides(), "b200: key and value caches must have identical strides");
  TORCH_CHECK(k.scalar_type() == v.scalar_type(), "b200: key and value caches must share one dtype");
  TORCH_CHECK(k.stride(3) == 1, "b200: cache head_dim must be contiguous");
  const bool fp8 = k.scalar_type() == at::kFloat8_e4m3fn;
  b200_paged_cache c{};
  c.k_cache = k.data_ptr();
  c.v_cache = v.data_ptr();
  c.num_blocks = k.size(0);
  c.block_size = static_cast<int32_t>(k.size(1));
  c.num_kv_heads = static_cast<int32_t>(k.size(2));
  c.head_dim = static_cast<int32_t>(k.size(3));
  c.dtype = activation_dtype(q_dtype);
  c.block_stride = k.stride(0);
  c.slot_stride = k.stride(1);
  c.head_stride = k.stride(2);
  c.kv_fp8 = fp8 ? 1 : 0;
  if (fp8) {
    c.k_scale = scale_ptr(k_scale, "k_scale");
    c.v_scale = scale_ptr(v_scale, "v_scale");
  } else {
    TORCH_CHECK(k.scalar_type() == q_dtype,
                "b200: query, output and 16-bit caches must share one dtype");
    TORCH_CHECK(!k_scale.has_value() && !v_scale.has_value(),
                "b200: k_scale / v_scale apply to FP8 caches only");
  }
  return c;
}

// ---------------------------------------------------------------- kv_append --
void kv_append(const at::Tensor& key, const at::Tensor& value, at::Tensor& k_cache,
               at::Tensor& v_cache, const at::Tensor& slot_mapping,
               const std::optional<at::Tensor>& k_scale,
               const std::optional<at::Tensor>& v_scale,
               const std::optional<at::Tensor>& status) {
  for (auto [t, name] : {std::pair<const at::Tensor&, const char*>{key, "key"},
                         {value, "value"}, {k_cache, "k_cache"}, {v_cache, "v_cache"},
                         {slot_mapping, "slot_mapping"}})
    require_cuda(t, name);
  TORCH_CHECK(key.dim() == 3 && value.sizes() == key.sizes(),
              "b200: key and value must be [tokens, num_kv_heads, head_dim] of one shape");
  const int64_t n = key.size(0), head_dim = key.size(2), row = key.size(1) * head_dim;
  // the reference launcher's assertions (attention.py:37-40)
  TORCH_CHECK(key.stride(-1) == 1 && value.stride(-1) == 1,
              "b200: key/value must be contiguous in head_dim");
  TORCH_CHECK(key.stride(1) == head_dim && value.stride(1) == head_dim,
              "b200: key/value heads must be packed (stride(1) == head_dim)");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.sizes() == v_cache.sizes() &&
                  k_cache.strides() == v_cache.strides(),
              "b200: key and value caches must have the same [num_blocks, block_size, "
              "num_kv_heads, head_dim] shape and strides");
  TORCH_CHECK(k_cache.stride(1) == row && v_cache.stride(1) == row,
              "b200: cache slots must be packed (stride(1) == num_kv_heads*head_dim)");
  TORCH_CHECK(k_cache.stride(0) == k_cache.size(1) * row,
              "b200: cache blocks must be contiguous");
  TORCH_CHECK(slot_mapping.numel() == n, "b200: slot_mapping must contain one slot per token");
  TORCH_CHECK(slot_mapping.dim() == 1 && (n <= 1 || slot_mapping.stride(0) == 1),
              "b200: slot_mapping must be a contiguous 1-D tensor");
  if (n == 0) return;
  const int64_t num_slots = k_cache.size(0) * k_cache.size(1);
  if (k_cache.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(v_cache.scalar_type() == at::kFloat8_e4m3fn, "b200: both caches must be FP8");
    TORCH_CHECK(slot_mapping.scalar_type() == at::kInt, "b200: FP8 appends take int32 slots");
    check_abi(b200_store_kvcache_fp8(
                  key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
                  activation_dtype(key.scalar_type()), k_cache.data_ptr(), v_cache.data_ptr(),
                  row, slot_mapping.data_ptr<int32_t>(), n, row, scale_ptr(k_scale, "k_scale"),
                  scale_ptr(v_scale, "v_scale"), num_slots, status_ptr(status),
                  current_stream(key)),
              "b200_store_kvcache_fp8");
    return;
  }
  TORCH_CHECK(key.scalar_type() == k_cache.scalar_type() &&
                  value.scalar_type() == v_cache.scalar_type() &&
                  key.scalar_type() == value.scalar_type(),
              "b200: key, value and caches must share one dtype");
  TORCH_CHECK(!k_scale.has_value() && !v_scale.has_value(),
              "b200: k_scale / v_scale apply to FP8 caches only");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kInt || slot_mapping.scalar_type() == at::kLong,
              "b200: slot_mapping must be int32 or int64");
  check_abi(b200_store_kvcache(key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
                               k_cache.data_ptr(), v_cache.data_ptr(), row,
                               slot_mapping.data_ptr(),
                               slot_mapping.scalar_type() == at::kLong ? 1 : 0, n, row,
                               static_cast<int32_t>(key.element_size()), num_slots,
                               status_ptr(status), current_stream(key)),
            "b200_store_kvcache");
}

// ------------------------------------------------------------- paged_decode --
void paged_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                  const at::Tensor& block_tables, const at::Tensor& seq_lens, at::Tensor& out,
                  int64_t num_parts, int64_t part_tokens, double softmax_scale,
                  const std::optional<at::Tensor>& workspace,
                  const std::optional<at::Tensor>& k_scale,
                  const std::optional<at::Tensor>& v_scale,
                  const std::optional<at::Tensor>& status) {
  require_cuda(q, "q");
  require_cuda(out, "out");
  TORCH_CHECK(q.dim() == 3 && out.sizes() == q.sizes() && q.stride(2) == 1 && out.stride(2) == 1,
              "b200: q and out must be [tokens, num_q_heads, head_dim], head_dim contiguous");
  TORCH_CHECK(out.scalar_type() == q.scalar_type(), "b200: out must have the query dtype");
  require_block_tables(block_tables);
  require_int32_vector(seq_lens, "seq_lens");
  const int64_t b = q.size(0);
  TORCH_CHECK(block_tables.size(0) >= b && seq_lens.numel() >= b,
              "b200: block_tables / seq_lens must have one row per sequence");
  const b200_paged_cache cache = cache_desc(k_cache, v_cache, q.scalar_type(), k_scale, v_scale);
  void* ws = nullptr;
  int64_t ws_bytes = 0;
  if (workspace.has_value()) {
    require_cuda(*workspace, "workspace");
    ws = workspace->data_ptr();
    ws_bytes = workspace->numel() * workspace->element_size();
  }
  b200_decode_plan plan{static_cast<int32_t>(num_parts), static_cast<int32_t>(part_tokens), 0};
  check_abi(b200_paged_decode(q.data_ptr(), q.stride(0), q.stride(1), &cache,
                              block_tables.data_ptr<int32_t>(), block_tables.stride(0),
                              seq_lens.data_ptr<int32_t>(), static_cast<int32_t>(b),
                              static_cast<int32_t>(q.size(1)), out.data_ptr(), out.stride(0),
                              out.stride(1), static_cast<float>(softmax_scale), &plan, ws,
                              ws_bytes, status_ptr(status), current_stream(q)),
            "b200_paged_decode");
}

// ------------------------------------------------------------ paged_prefill --
void paged_prefill(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                   const at::Tensor& block_tables, const at::Tensor& seq_lens,
                   const at::Tensor& query_start_loc, at::Tensor& out, int64_t max_q_len,
                   double softmax_scale, int64_t num_seqs,
                   const std::optional<at::Tensor>& k_scale,
                   const std::optional<at::Tensor>& v_scale,
                   const std::optional<at::Tensor>& status,
                   const std::optional<at::Tensor>& workspace) {
  require_cuda(q, "q");
  require_cuda(out, "out");
  TORCH_CHECK(q.dim() == 3 && out.sizes() == q.sizes() && q.stride(2) == 1 && out.stride(2) == 1,
              "b200: q and out must be [tokens, num_q_heads, head_dim], head_dim contiguous");
  TORCH_CHECK(out.scalar_type() == q.scalar_type(), "b200: out must have the query dtype");
  require_block_tables(block_tables);
  require_int32_vector(seq_lens, "seq_lens");
  require_int32_vector(query_start_loc, "query_start_loc");
  TORCH_CHECK(num_seqs >= 0 && query_start_loc.numel() >= num_seqs + 1 &&
                  block_tables.size(0) >= num_seqs && seq_lens.numel() >= num_seqs,
              "b200: query_start_loc / block_tables / seq_lens too short for num_seqs");
  const b200_paged_cache cache = cache_desc(k_cache, v_cache, q.scalar_type(), k_scale, v_scale);
  void* ws = nullptr;
  int64_t ws_bytes = 0;
  if (workspace.has_value()) {
    require_cuda(*workspace, "workspace");
    ws = workspace->data_ptr();
    ws_bytes = workspace->numel() * workspace->element_size();
  }
  check_abi(b200_paged_prefill(q.data_ptr(), q.stride(0), q.stride(1), &cache,
                               block_tables.data_ptr<int32_t>(), block_tables.stride(0),
                               seq_lens.data_ptr<int32_t>(), query_start_loc.data_ptr<int32_t>(),
                               static_cast<int32_t>(num_seqs), static_cast<int32_t>(q.size(0)),
                               static_cast<int32_t>(max_q_len),
                               static_cast<int32_t>(q.size(1)), out.data_ptr(), out.stride(0),
                               out.stride(1), static_cast<float>(softmax_scale), ws, ws_bytes,
                               status_ptr(status), current_stream(q)),
            "b200_paged_prefill");
}

// ------------------------------------------------ Meta (FakeTensor) kernels --
void kv_append_meta(const at::Tensor&, const at::Tensor&, at::Tensor&, at::Tensor&,
                    const at::Tensor&, const std::optional<at::Tensor>&,
                    const std::optional<at::Tensor>&, const std::optional<at::Tensor>&) {}

void paged_decode_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                       const at::Tensor&, const at::Tensor&, at::Tensor&, int64_t, int64_t,
                       double, const std::optional<at::Tensor>&,
                       const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                       const std::optional<at::Tensor>&) {}

void paged_prefill_meta(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        const at::Tensor&, const at::Tensor&, const at::Tensor&, at::Tensor&,
                        int64_t, double, int64_t, const std::optional<at::Tensor>&,
                        const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                        const std::optional<at::Tensor>&) {}

}  // namespace

TORCH_LIBRARY(b200, m) {
  m.def(
      "kv_append(Tensor key, Tensor value, Tensor(a!) k_cache, Tensor(b!) v_cache, "
      "Tensor slot_mapping, Tensor? k_scale=None, Tensor? v_scale=None, "
      "Tensor(c!)? status=None) -> ()");
  m.def(
      "paged_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, Tensor(a!) out, int num_parts, int part_tokens, float softmax_scale, "
      "Tensor(b!)? workspace=None, Tensor? k_scale=None, Tensor? v_scale=None, "
      "Tensor(c!)? status=None) -> ()");
  m.def(
      "paged_prefill(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, "
      "Tensor seq_lens, Tensor query_start_loc, Tensor(a!) out, int max_q_len, "
      "float softmax_scale, int num_seqs, Tensor? k_scale=None, Tensor? v_scale=None, "
      "Tensor(b!)? status=None, Tensor(c!)? workspace=None) -> ()");
}

TORCH_LIBRARY_IMPL(b200, CUDA, m) {
  m.impl("kv_append", &kv_append);
  m.impl("paged_decode", &paged_decode);
  m.impl("paged_prefill", &paged_prefill);
}

TORCH_LIBRARY_IMPL(b200, Meta, m) {
  m.impl("kv_append", &kv_append_meta);
  m.impl("paged_decode", &paged_decode_meta);
  m.impl("paged_prefill", &paged_prefill_meta);
}
