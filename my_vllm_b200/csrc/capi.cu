// capi.cu — the extern "C" boundary of the paged-attention path.
//
// Validates arguments (the checks the reference does in Python before its
// kernels run: attention.py:37-40 for the append,
// attention_backend.py:1522-1553 for attention inputs), builds and caches
// the TMA tensor maps of the paged caches, plans the decode split and
// launches the kernels on the caller's stream.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/b200_paged_attn.h"
#include "paged_decode.cuh"
#include "paged_prefill.cuh"
#include "rope_append.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    else
      cudaGetLastError();
  });
  return fn;
}

struct MapKey {
  uint64_t ptr;
  int64_t dims[4];
  int64_t strides[3];
  int32_t dtype;
  bool operator==(const MapKey& o) const {
    return std::memcmp(this, &o, sizeof(MapKey)) == 0;
  }
};

struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash>& map_cache() {
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> m;
  return m;
}

int cache_elem_bytes(const b200_paged_cache& c) { return c.kv_fp8 ? 1 : 2; }

// Tensor map over one paged cache tensor viewed as (head_dim, kv_head, slot,
// block), 128-byte swizzle; box = 64 elements (16-bit) or 128 elements
// (FP8) x 1 head x 16 slots x 1 block, i.e. 128-byte rows either way.
int cache_tensor_map(const void* base, const b200_paged_cache& c, CUtensorMap* out) {
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.ptr = reinterpret_cast<uint64_t>(base);
  key.dims[0] = c.head_dim;
  key.dims[1] = c.num_kv_heads;
  key.dims[2] = c.block_size;
  key.dims[3] = c.num_blocks;
  key.strides[0] = c.head_stride;
  key.strides[1] = c.slot_stride;
  key.strides[2] = c.block_stride;
  key.dtype = c.kv_fp8 ? B200_DTYPE_FP8_E4M3 : c.dtype;
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    auto it = map_cache().find(key);
    if (it != map_cache().end()) {
      *out = it->second;
      return B200_OK;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr)
    return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[4] = {(cuuint64_t)c.head_dim, (cuuint64_t)c.num_kv_heads,
                              (cuuint64_t)c.block_size, (cuuint64_t)c.num_blocks};
  const cuuint64_t eb = (cuuint64_t)cache_elem_bytes(c);
  const cuuint64_t strides[3] = {(cuuint64_t)c.head_stride * eb, (cuuint64_t)c.slot_stride * eb,
                                 (cuuint64_t)c.block_stride * eb};
  const cuuint32_t box[4] = {(cuuint32_t)(128 / eb), 1, (cuuint32_t)b200::kTileTokens, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType type = c.kv_fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : c.dtype == B200_DTYPE_BFLOAT16
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap m;
  CUresult r = fn(&m, type, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " +
                                   std::to_string(static_cast<int>(r)));
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    if (map_cache().size() > 4096) map_cache().clear();
    map_cache().emplace(key, m);
  }
  *out = m;
  return B200_OK;
}

// Tensor map over q or out (16-bit) viewed as (head_dim, q head, token), 128-byte
// swizzle; box = 64 elements x group heads x 128 / group tokens, i.e. one
// d-half of a prefill Q tile's 128 (token, head) rows in row order.
int q_tensor_map(const void* q, int dtype, int num_q_heads, int num_tokens,
                 int64_t q_head_stride, int64_t q_token_stride, int group, CUtensorMap* out) {
  MapKey key;
  std::memset(&key, 0, sizeof(key));
  key.ptr = reinterpret_cast<uint64_t>(q);
  key.dims[0] = b200::kHeadDim;
  key.dims[1] = num_q_heads;
  key.dims[2] = num_tokens;
  key.dims[3] = group;
  key.strides[0] = q_head_stride;
  key.strides[1] = q_token_stride;
  key.dtype = 1000 + dtype;  // never equal to a cache map's key
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    auto it = map_cache().find(key);
    if (it != map_cache().end()) {
      *out = it->second;
      return B200_OK;
    }
  }
  auto fn = encode_fn();
  if (fn == nullptr)
    return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t dims[3] = {(cuuint64_t)b200::kHeadDim, (cuuint64_t)num_q_heads,
                              (cuuint64_t)num_tokens};
  const cuuint64_t strides[2] = {(cuuint64_t)q_head_stride * 2, (cuuint64_t)q_token_stride * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)group, (cuuint32_t)(128 / group)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType type = dtype == B200_DTYPE_BFLOAT16
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap m;
  CUresult r = fn(&m, type, 3, const_cast<void*>(q), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled (q) failed with CUresult " +
                                   std::to_string(static_cast<int>(r)));
  {
    std::lock_guard<std::mutex> lock(g_map_mu);
    if (map_cache().size() > 4096) map_cache().clear();
    map_cache().emplace(key, m);
  }
  *out = m;
  return B200_OK;
}

int validate_cache(const b200_paged_cache* c) {
  if (c == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "cache descriptor is NULL");
  if (c->k_cache == nullptr || c->v_cache == nullptr)
    return fail(B200_ERR_INVALID_ARGUMENT, "key and value caches must both be present");
  if (c->dtype != B200_DTYPE_BFLOAT16 && c->dtype != B200_DTYPE_FLOAT16)
    return fail(B200_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  if (c->kv_fp8 != 0 && c->kv_fp8 != 1)
    return fail(B200_ERR_INVALID_ARGUMENT, "kv_fp8 must be 0 or 1");
  if (!c->kv_fp8 && (c->k_scale != nullptr || c->v_scale != nullptr))
    return fail(B200_ERR_INVALID_ARGUMENT, "k_scale / v_scale apply to FP8 caches only");
  if (c->head_dim != b200::kHeadDim)
    return fail(B200_ERR_UNSUPPORTED, "head_dim must be 128");
  if (c->block_size <= 0 || c->block_size % b200::kTileTokens != 0)
    return fail(B200_ERR_UNSUPPORTED, "block_size must be a positive multiple of 16");
  if (c->num_kv_heads <= 0 || c->num_blocks <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "num_kv_heads and num_blocks must be positive");
  if (c->num_blocks > (int64_t(1) << 31) - 1)
    return fail(B200_ERR_UNSUPPORTED, "num_blocks must fit in int32");
  if (((reinterpret_cast<uintptr_t>(c->k_cache) | reinterpret_cast<uintptr_t>(c->v_cache)) &
       15) != 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "cache base pointers must be 16-byte aligned");
  const int64_t per16 = 16 / cache_elem_bytes(*c);  // elements per 16 bytes
  if (c->head_stride % per16 || c->slot_stride % per16 || c->block_stride % per16 ||
      c->head_stride <= 0 || c->slot_stride <= 0 || c->block_stride <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "cache strides must be positive multiples of 16 bytes");
  return B200_OK;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return 148;
  }
  return n;
}

int64_t decode_workspace_bytes(int64_t num_seqs, int64_t num_q_heads, int64_t num_parts) {
  if (num_parts <= 1) return 0;
  const int64_t slots = num_seqs * num_q_heads * num_parts;
  const int64_t o_bytes = (slots * b200::kHeadDim * 4 + 255) / 256 * 256;
  return o_bytes + (slots * 4 + 255) / 256 * 256;
}

}  // namespace

namespace b200 {
void set_last_error(const std::string& message) { g_last_error = message; }
}  // namespace b200

extern "C" {

int b200_abi_version(void) { return 300; }

const char* b200_last_error(void) { return g_last_error.c_str(); }

int b200_store_kvcache(const void* key, int64_t key_row_stride, const void* value,
                       int64_t value_row_stride, void* k_cache, void* v_cache,
                       int64_t cache_slot_stride, const void* slot_mapping,
                       int32_t slot_is_int64, int64_t num_tokens, int64_t row_elems,
                       int32_t elem_bytes, int64_t num_slots, int32_t* status,
                       void* stream) {
  g_last_error.clear();
  if (num_tokens < 0 || row_elems <= 0 || num_slots < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "negative size");
  if (elem_bytes != 2 && elem_bytes != 4)
    return fail(B200_ERR_UNSUPPORTED, "element size must be 2 or 4 bytes");
  if (num_tokens == 0) return B200_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (key_row_stride < row_elems || value_row_stride < row_elems ||
      cache_slot_stride < row_elems)
    return fail(B200_ERR_INVALID_ARGUMENT, "row strides must cover row_elems");
  cudaError_t e = b200::launch_kv_append(
      key, key_row_stride, value, value_row_stride, k_cache, v_cache, cache_slot_stride,
      slot_mapping, slot_is_int64 != 0, num_tokens, row_elems, elem_bytes, num_slots, status,
      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv append launch");
  return B200_OK;
}

}  // extern "C"

namespace {
// Shared by b200_qk_norm_rope_append and its FP8-cache variant (fp8: caches
// hold one byte per element; cache_slot_stride counts bytes then).
int rope_append_impl(const void* q, int64_t q_token_stride, int64_t q_head_stride,
                             const void* k, int64_t k_token_stride, const void* v,
                             int64_t v_token_stride, void* q_out, int64_t q_out_token_stride,
                             int64_t q_out_head_stride, const void* q_weight,
                             const void* k_weight, float eps, const int64_t* positions,
                             const float* cos_sin_cache, int64_t max_position, void* k_cache,
                             void* v_cache, int64_t cache_slot_stride,
                             const int32_t* slot_mapping, int64_t num_tokens,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             int32_t dtype, int64_t num_slots, bool fp8, const float* k_scale,
                             const float* v_scale, int32_t* status, void* stream) {
  g_last_error.clear();
  if (head_dim != b200::kRopeHeadDim) return fail(B200_ERR_UNSUPPORTED, "head_dim must be 128");
  if (dtype != B200_DTYPE_BFLOAT16 && dtype != B200_DTYPE_FLOAT16)
    return fail(B200_ERR_UNSUPPORTED, "dtype must be float16 or bfloat16");
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_position <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  if (num_tokens == 0) return B200_OK;
  if (!q || !k || !v || !q_out || !q_weight || !k_weight || !positions || !cos_sin_cache ||
      !k_cache || !v_cache || !slot_mapping)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(q_out) |
        reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
        reinterpret_cast<uintptr_t>(q_weight) | reinterpret_cast<uintptr_t>(k_weight) |
        reinterpret_cast<uintptr_t>(cos_sin_cache)) & 15) ||
      (q_token_stride | q_head_stride | k_token_stride | v_token_stride | q_out_token_stride |
       q_out_head_stride | cache_slot_stride) & 7)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "tensors must be 16-byte aligned with strides that are multiples of 8 "
                "elements (rows move as 16-byte vectors)");
  if (cache_slot_stride < (int64_t)num_kv_heads * head_dim)
    return fail(B200_ERR_INVALID_ARGUMENT, "cache slot stride must cover all KV heads");
  b200::RopeAppendParams p;
  p.q = q;
  p.q_token_stride = q_token_stride;
  p.q_head_stride = q_head_stride;
  p.k = k;
  p.k_token_stride = k_token_stride;
  p.v = v;
  p.v_token_stride = v_token_stride;
  p.q_out = q_out;
  p.q_out_token_stride = q_out_token_stride;
  p.q_out_head_stride = q_out_head_stride;
  p.q_weight = q_weight;
  p.k_weight = k_weight;
  p.eps = eps;
  p.positions = positions;
  p.cos_sin_cache = cos_sin_cache;
  p.max_position = max_position;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.cache_slot_stride = cache_slot_stride;
  p.slot_mapping = slot_mapping;
  p.num_tokens = num_tokens;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.num_slots = num_slots;
  p.k_scale = k_scale;
  p.v_scale = v_scale;
  p.status = status;
  cudaError_t e =
      b200::launch_qk_norm_rope_append(p, dtype, fp8, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "q/k norm + rope + append launch");
  return B200_OK;
}

}  // namespace

extern "C" {

int b200_qk_norm_rope_append(const void* q, int64_t q_token_stride, int64_t q_head_stride,
                             const void* k, int64_t k_token_stride, const void* v,
                             int64_t v_token_stride, void* q_out, int64_t q_out_token_stride,
                             int64_t q_out_head_stride, const void* q_weight,
                             const void* k_weight, float eps, const int64_t* positions,
                             const float* cos_sin_cache, int64_t max_position, void* k_cache,
                             void* v_cache, int64_t cache_slot_stride,
                             const int32_t* slot_mapping, int64_t num_tokens,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             int32_t dtype, int64_t num_slots, int32_t* status, void* stream) {
  return rope_append_impl(q, q_token_stride, q_head_stride, k, k_token_stride, v, v_token_stride,
                          q_out, q_out_token_stride, q_out_head_stride, q_weight, k_weight, eps,
                          positions, cos_sin_cache, max_position, k_cache, v_cache,
                          cache_slot_stride, slot_mapping, num_tokens, num_q_heads,
                          num_kv_heads, head_dim, dtype, num_slots, false, nullptr, nullptr,
                          status, stream);
}

int b200_qk_norm_rope_append_fp8(
    const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
    int64_t k_token_stride, const void* v, int64_t v_token_stride, void* q_out,
    int64_t q_out_token_stride, int64_t q_out_head_stride, const void* q_weight,
    const void* k_weight, float eps, const int64_t* positions, const float* cos_sin_cache,
    int64_t max_position, void* k_cache, void* v_cache, int64_t cache_slot_stride,
    const int32_t* slot_mapping, int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype, const float* k_scale, const float* v_scale,
    int64_t num_slots, int32_t* status, void* stream) {
  return rope_append_impl(q, q_token_stride, q_head_stride, k, k_token_stride, v, v_token_stride,
                          q_out, q_out_token_stride, q_out_head_stride, q_weight, k_weight, eps,
                          positions, cos_sin_cache, max_position, k_cache, v_cache,
                          cache_slot_stride, slot_mapping, num_tokens, num_q_heads,
                          num_kv_heads, head_dim, dtype, num_slots, true, k_scale, v_scale,
                          status, stream);
}

int b200_build_slot_mapping(const int32_t* block_tables, int64_t block_table_stride,
                            int32_t max_blocks, int64_t num_blocks, const int32_t* seq_lens,
                            const int32_t* query_start_loc, int32_t num_seqs,
                            int32_t num_tokens, int32_t block_size, int32_t* slot_mapping,
                            int32_t* status, void* stream) {
  g_last_error.clear();
  if (num_seqs < 0 || num_tokens < 0 || block_size <= 0 || max_blocks < 0 || num_blocks < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "sizes must be non-negative, block_size positive");
  if (num_tokens == 0) return B200_OK;
  if (num_seqs == 0) return fail(B200_ERR_INVALID_ARGUMENT, "tokens without sequences");
  if (!block_tables || !seq_lens || !query_start_loc || !slot_mapping)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (max_blocks > block_table_stride)
    return fail(B200_ERR_INVALID_ARGUMENT, "max_blocks exceeds the block-table row stride");
  cudaError_t e = b200::launch_build_slot_mapping(
      block_tables, block_table_stride, max_blocks, num_blocks, seq_lens, query_start_loc,
      num_seqs, num_tokens, block_size, slot_mapping, status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "slot mapping launch");
  return B200_OK;
}

int b200_build_block_tables(const int32_t* block_ids, const int32_t* offsets,
                            int32_t num_seqs, int32_t max_blocks, int32_t* block_tables,
                            int64_t block_table_stride, int32_t* status, void* stream) {
  g_last_error.clear();
  if (num_seqs < 0 || max_blocks < 0 || block_table_stride < max_blocks)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "sizes must be non-negative and the row stride at least max_blocks");
  if (num_seqs == 0 || max_blocks == 0) return B200_OK;
  if (!block_ids || !offsets || !block_tables)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  cudaError_t e = b200::launch_build_block_tables(block_ids, offsets, num_seqs, max_blocks,
                                                  block_tables, block_table_stride, status,
                                                  static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "block table launch");
  return B200_OK;
}

int b200_store_kvcache_fp8(const void* key, int64_t key_row_stride, const void* value,
                           int64_t value_row_stride, int32_t src_dtype, void* k_cache,
                           void* v_cache, int64_t cache_slot_stride, const int32_t* slot_mapping,
                           int64_t num_tokens, int64_t row_elems, const float* k_scale,
                           const float* v_scale, int64_t num_slots, int32_t* status,
                           void* stream) {
  g_last_error.clear();
  if (src_dtype != B200_DTYPE_BFLOAT16 && src_dtype != B200_DTYPE_FLOAT16)
    return fail(B200_ERR_UNSUPPORTED, "source rows must be float16 or bfloat16");
  if (num_tokens < 0 || row_elems <= 0 || num_slots < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "sizes must be non-negative");
  if (row_elems % 16)
    return fail(B200_ERR_INVALID_ARGUMENT, "row_elems must be a multiple of 16");
  if (num_tokens == 0) return B200_OK;
  if (!key || !value || !k_cache || !v_cache || !slot_mapping)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (((reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
        reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) ||
      (key_row_stride | value_row_stride) % 8 || cache_slot_stride % 16)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "rows and caches must be 16-byte aligned (row strides multiples of 8 "
                "elements, cache slot stride a multiple of 16 bytes)");
  if (cache_slot_stride < row_elems)
    return fail(B200_ERR_INVALID_ARGUMENT, "cache slot stride must cover a row");
  cudaError_t e = b200::launch_kv_append_fp8(key, key_row_stride, value, value_row_stride,
                                             src_dtype, k_cache, v_cache, cache_slot_stride,
                                             slot_mapping, num_tokens, row_elems, k_scale,
                                             v_scale, num_slots, status,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fp8 KV append launch");
  return B200_OK;
}

int b200_paged_decode_plan(int32_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                           int32_t head_dim, int32_t block_size, int32_t max_kv_len,
                           int64_t total_kv_tokens, int32_t force_num_parts,
                           int32_t kv_fp8, b200_decode_plan* plan) {
  g_last_error.clear();
  if (plan == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (num_seqs <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || max_kv_len <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "sizes must be positive");
  if (head_dim != b200::kHeadDim) return fail(B200_ERR_UNSUPPORTED, "head_dim must be 128");
  if (block_size <= 0 || block_size % b200::kTileTokens)
    return fail(B200_ERR_UNSUPPORTED, "block_size must be a positive multiple of 16");
  if (num_q_heads % num_kv_heads)
    return fail(B200_ERR_INVALID_ARGUMENT, "num_q_heads must be divisible by num_kv_heads");
  const int64_t tiles = (max_kv_len + b200::kTileTokens - 1) / b200::kTileTokens;
  const int64_t max_part_tiles = b200::kMaxPartTokens / b200::kTileTokens;
  const int64_t min_parts = (tiles + max_part_tiles - 1) / max_part_tiles;
  int64_t parts;
  if (force_num_parts > 0) {
    parts = force_num_parts;
    if (parts < min_parts)
      return fail(B200_ERR_INVALID_ARGUMENT,
                  "forced split leaves partitions longer than 8192 tokens");
    if (parts > tiles) parts = tiles;
  } else {
    // The kernel is HBM-bound: it needs bytes in flight, not full waves of
    // CTAs, and every extra partition costs a pipeline ramp plus partial
    // outputs. So split only (a) to give every SM at least one CTA (two for
    // FP8 caches, whose kernel holds 4 CTAs per SM: one KV head of 256
    // sequences measured 0.056 ms split in two against 0.068 ms whole), and
    // (b) for ragged batches, so no CTA holds more than 1/12 of the average
    // per-SM work (the longest sequences would otherwise finish last on a few
    // SMs; 1/12 measured best on a 124-sequence batch of U[128, 8192]).
    const int64_t units = (int64_t)num_seqs * num_kv_heads;
    const int64_t sms = sm_count();
    const int64_t cover = kv_fp8 ? 2 * sms : sms;
    parts = min_parts;
    if (units * parts < cover) parts = (cover + units - 1) / units;
    const int64_t max_tokens = (int64_t)num_seqs * max_kv_len;
    const int64_t total = (total_kv_tokens > 0 && total_kv_tokens < max_tokens)
                              ? total_kv_tokens : max_tokens;
    if (total < max_tokens) {
      const int64_t total_tiles = (total + b200::kTileTokens - 1) / b200::kTileTokens;
      const double per_sm = double(total_tiles) * num_kv_heads / double(sms);
      int64_t balance = (int64_t)(12.0 * double(tiles) / per_sm + 0.999999);
      const int64_t cap = tiles / 4 > 1 ? tiles / 4 : 1;  // >= 4 tiles per partition
      if (balance > cap) balance = cap;
      if (balance > parts) parts = balance;
    }
  }
  const int64_t part_tiles = (tiles + parts - 1) / parts;
  parts = (tiles + part_tiles - 1) / part_tiles;
  plan->num_parts = static_cast<int32_t>(parts);
  plan->part_tokens = static_cast<int32_t>(part_tiles * b200::kTileTokens);
  plan->workspace_bytes = decode_workspace_bytes(num_seqs, num_q_heads, parts);
  return B200_OK;
}

int b200_paged_decode(const void* q, int64_t q_seq_stride, int64_t q_head_stride,
                      const b200_paged_cache* cache, const int32_t* block_tables,
                      int64_t block_table_stride, const int32_t* seq_lens, int32_t num_seqs,
                      int32_t num_q_heads, void* out, int64_t out_seq_stride,
                      int64_t out_head_stride, float softmax_scale,
                      const b200_decode_plan* plan, void* workspace, int64_t workspace_bytes,
                      int32_t* status, void* stream) {
  g_last_error.clear();
  int rc = validate_cache(cache);
  if (rc != B200_OK) return rc;
  if (plan == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "plan is NULL");
  if (num_seqs < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_seqs must be >= 0");
  if (num_seqs == 0) return B200_OK;
  if (!q || !out || !block_tables || !seq_lens)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (num_q_heads <= 0 || num_q_heads % cache->num_kv_heads)
    return fail(B200_ERR_INVALID_ARGUMENT, "num_q_heads must be divisible by num_kv_heads");
  const int group = num_q_heads / cache->num_kv_heads;
  if (group > 16) return fail(B200_ERR_UNSUPPORTED, "at most 16 q heads per KV head");
  if (plan->num_parts < 1 || plan->part_tokens <= 0 ||
      plan->part_tokens % b200::kTileTokens || plan->part_tokens > b200::kMaxPartTokens)
    return fail(B200_ERR_INVALID_ARGUMENT, "malformed decode plan");
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 3) ||
      (q_seq_stride | q_head_stride | out_seq_stride | out_head_stride) & 1)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "q/out must be 4-byte aligned with even strides");
  const int64_t need = decode_workspace_bytes(num_seqs, num_q_heads, plan->num_parts);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(B200_ERR_INVALID_ARGUMENT,
                "decode workspace too small: need " + std::to_string(need) + " bytes");
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(B200_ERR_INVALID_ARGUMENT, "decode workspace must be 256-byte aligned");
  CUtensorMap mk, mv;
  if ((rc = cache_tensor_map(cache->k_cache, *cache, &mk)) != B200_OK) return rc;
  if ((rc = cache_tensor_map(cache->v_cache, *cache, &mv)) != B200_OK) return rc;

  b200::DecodeParams p;
  p.q = q;
  p.q_seq_stride = q_seq_stride;
  p.q_head_stride = q_head_stride;
  p.block_tables = block_tables;
  p.block_table_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.out = out;
  p.out_seq_stride = out_seq_stride;
  p.out_head_stride = out_head_stride;
  const int64_t slots = (int64_t)num_seqs * num_q_heads * plan->num_parts;
  p.part_o = need > 0 ? static_cast<float*>(workspace) : nullptr;
  p.part_lse = need > 0 ? reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                                   (slots * b200::kHeadDim * 4 + 255) / 256 * 256)
                        : nullptr;
  p.num_parts = plan->num_parts;
  p.part_tokens = plan->part_tokens;
  p.block_size = cache->block_size;
  p.group = group;
  p.num_q_heads = num_q_heads;
  p.num_blocks = cache->num_blocks;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.k_scale = cache->k_scale;
  p.v_scale = cache->v_scale;
  p.status = status;
  cudaError_t e =
      b200::launch_paged_decode(mk, mv, p, cache->dtype, cache->kv_fp8 != 0,
                                cache->num_kv_heads, num_seqs, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged decode launch");
  return B200_OK;
}

int64_t b200_paged_prefill_workspace_bytes(void) { return b200::prefill_workspace_bytes(); }

int b200_paged_prefill(const void* q, int64_t q_token_stride, int64_t q_head_stride,
                       const b200_paged_cache* cache, const int32_t* block_tables,
                       int64_t block_table_stride, const int32_t* seq_lens,
                       const int32_t* query_start_loc, int32_t num_seqs, int32_t num_q_tokens,
                       int32_t max_q_len, int32_t num_q_heads, void* out,
                       int64_t out_token_stride, int64_t out_head_stride, float softmax_scale,
                       void* workspace, int64_t workspace_bytes, int32_t* status,
                       void* stream) {
  g_last_error.clear();
  int rc = validate_cache(cache);
  if (rc != B200_OK) return rc;
  if (num_seqs < 0 || num_q_tokens < 0 || max_q_len < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "sizes must be >= 0");
  if (num_seqs == 0 || num_q_tokens == 0) return B200_OK;
  if (!q || !out || !block_tables || !seq_lens || !query_start_loc)
    return fail(B200_ERR_INVALID_ARGUMENT, "NULL tensor pointer");
  if (num_q_heads <= 0 || num_q_heads % cache->num_kv_heads)
    return fail(B200_ERR_INVALID_ARGUMENT, "num_q_heads must be divisible by num_kv_heads");
  const int group = num_q_heads / cache->num_kv_heads;
  if (max_q_len <= 0) return fail(B200_ERR_INVALID_ARGUMENT, "max_q_len must be positive");
  if (group > 128) return fail(B200_ERR_UNSUPPORTED, "at most 128 q heads per KV head");
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15) ||
      (q_token_stride | q_head_stride | out_token_stride | out_head_stride) & 7)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "q/out must be 16-byte aligned with strides that are multiples of 8");
  if (workspace != nullptr) {
    if (workspace_bytes < b200::prefill_workspace_bytes())
      return fail(B200_ERR_INVALID_ARGUMENT,
                  "prefill workspace smaller than b200_paged_prefill_workspace_bytes()");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
      return fail(B200_ERR_INVALID_ARGUMENT, "prefill workspace must be 256-byte aligned");
  }
  CUtensorMap mk, mv;
  if ((rc = cache_tensor_map(cache->k_cache, *cache, &mk)) != B200_OK) return rc;
  if ((rc = cache_tensor_map(cache->v_cache, *cache, &mv)) != B200_OK) return rc;
  b200::PrefillParams p{};
  p.q = q;
  p.q_token_stride = q_token_stride;
  p.q_head_stride = q_head_stride;
  p.block_tables = block_tables;
  p.block_table_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.query_start_loc = query_start_loc;
  p.out = out;
  p.out_token_stride = out_token_stride;
  p.out_head_stride = out_head_stride;
  p.out_v8 = (reinterpret_cast<uintptr_t>(out) % 32 == 0 &&
              ((out_token_stride | out_head_stride) & 15) == 0) ? 1 : 0;
  p.block_size = cache->block_size;
  p.group = group;
  p.num_q_heads = num_q_heads;
  p.num_blocks = cache->num_blocks;
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.k_scale = cache->k_scale;
  p.v_scale = cache->v_scale;
  p.status = status;
  // split-KV of long units needs the workspace (tickets, then part records)
  p.split_records = nullptr;
  p.split_tickets = nullptr;
  p.split_cap = 0;
  p.num_sms = 0;
  if (workspace != nullptr) {
    p.split_tickets = static_cast<int*>(workspace);
    p.split_records = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                               b200::prefill_split_ticket_bytes());
    p.split_cap = b200::kPrefillSplitCap;
  }
  // Q by TMA when a tile's rows are one box of the q tensor: a GQA group that
  // divides 128 (FP8 caches convert the landed Q to fp16 in shared memory).
  CUtensorMap mq;
  std::memset(&mq, 0, sizeof(mq));
  p.q_tma = 128 % group == 0 ? 1 : 0;
  if (p.q_tma && q_tensor_map(q, cache->dtype, num_q_heads, num_q_tokens, q_head_stride,
                              q_token_stride, group, &mq) != B200_OK) {
    p.q_tma = 0;  // strides the driver does not accept: the softmax warps stage Q
    g_last_error.clear();
  }
  // Whole output tiles leave by TMA stores under the same condition.
  CUtensorMap mo;
  std::memset(&mo, 0, sizeof(mo));
  p.o_tma = 128 % group == 0 ? 1 : 0;
  if (p.o_tma && q_tensor_map(out, cache->dtype, num_q_heads, num_q_tokens, out_head_stride,
                              out_token_stride, group, &mo) != B200_OK) {
    p.o_tma = 0;  // per-thread stores
    g_last_error.clear();
  }
  cudaError_t e = b200::launch_paged_prefill_tc(mk, mv, mq, mo, p, cache->dtype,
                                                cache->kv_fp8 != 0,
                                                cache->num_kv_heads, num_seqs, max_q_len,
                                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "paged prefill launch");
  return B200_OK;
}

}  // extern "C"
