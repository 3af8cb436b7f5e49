// kv_append.cu — KV-cache append: scatter new K/V rows into paged cache slots.
//
// Semantics follow nanovllm/layers/attention.py:11-41 (Triton
// store_kvcache_kernel + launcher) and attention.py:69-85 (forward_native):
// token i with slot s != -1 copies its K row to k_cache[s] and its V row to
// v_cache[s]; slots of -1 (CUDA-graph padding) are skipped.
//
// Design: the work is pure HBM traffic (read one row, write one row), so the
// kernel maps one 16-byte vector per thread, with consecutive threads on
// consecutive vectors of the same row for coalesced 16-byte loads/stores.
// A block covers whole rows of both K and V; the vector width falls back to
// 8/4/2 bytes only when a pointer or stride is not 16-byte aligned.
#include <cuda_runtime.h>

#include "common.cuh"

namespace b200 {

template <int kVec>
struct VecType;
template <>
struct VecType<16> {
  using type = uint4;
};
template <>
struct VecType<8> {
  using type = uint2;
};
template <>
struct VecType<4> {
  using type = uint32_t;
};
template <>
struct VecType<2> {
  using type = uint16_t;
};

template <int kVec, typename SlotT>
__global__ void __launch_bounds__(256)
    kv_append_kernel(const char* __restrict__ key, int64_t key_row_bytes_stride,
                     const char* __restrict__ value,
                     int64_t value_row_bytes_stride, char* __restrict__ k_cache,
                     char* __restrict__ v_cache, int64_t cache_slot_bytes_stride,
                     const SlotT* __restrict__ slot_mapping, int64_t num_tokens,
                     int64_t vecs_per_row, int64_t num_slots,
                     int32_t* status) {
  using V = typename VecType<kVec>::type;
  // the decode that follows may start its prologue now; it waits for this
  // grid to complete before it reads the cache
  pdl_launch_dependents();
  // Work item = (token, tensor in {K, V}, vector within row).
  const int64_t per_token = 2 * vecs_per_row;
  const int64_t total = num_tokens * per_token;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t token = idx / per_token;
    const int64_t rem = idx - token * per_token;
    const int is_v = rem >= vecs_per_row;
    const int64_t vec = rem - (is_v ? vecs_per_row : 0);
    const int64_t slot = static_cast<int64_t>(slot_mapping[token]);
    if (slot == -1) continue;
    if (slot < 0 || slot >= num_slots) {
      if (vec == 0 && !is_v) report_status(status, B200_STATUS_SLOT_OUT_OF_RANGE);
      continue;
    }
    const char* src = (is_v ? value : key) +
                      token * (is_v ? value_row_bytes_stride : key_row_bytes_stride) +
                      vec * kVec;
    char* dst = (is_v ? v_cache : k_cache) + slot * cache_slot_bytes_stride + vec * kVec;
    *reinterpret_cast<V*>(dst) = __ldg(reinterpret_cast<const V*>(src));
  }
}

template <int kVec>
static cudaError_t launch_vec(const void* key, int64_t key_stride_b,
                              const void* value, int64_t value_stride_b,
                              void* k_cache, void* v_cache, int64_t slot_stride_b,
                              const void* slots, bool slot64, int64_t num_tokens,
                              int64_t row_bytes, int64_t num_slots,
                              int32_t* status, cudaStream_t stream) {
  const int64_t vecs = row_bytes / kVec;
  const int64_t total = num_tokens * 2 * vecs;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  // Enough blocks to cover every SM several times over; the grid-stride loop
  // handles the rest.
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  if (slot64) {
    kv_append_kernel<kVec, int64_t><<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const char*>(key), key_stride_b,
        static_cast<const char*>(value), value_stride_b,
        static_cast<char*>(k_cache), static_cast<char*>(v_cache), slot_stride_b,
        static_cast<const int64_t*>(slots), num_tokens, vecs, num_slots, status);
  } else {
    kv_append_kernel<kVec, int32_t><<<(unsigned)blocks, threads, 0, stream>>>(
        static_cast<const char*>(key), key_stride_b,
        static_cast<const char*>(value), value_stride_b,
        static_cast<char*>(k_cache), static_cast<char*>(v_cache), slot_stride_b,
        static_cast<const int32_t*>(slots), num_tokens, vecs, num_slots, status);
  }
  return cudaGetLastError();
}

// Picks the widest vector every pointer, stride and the row length allow.
cudaError_t launch_kv_append(const void* key, int64_t key_row_stride,
                             const void* value, int64_t value_row_stride,
                             void* k_cache, void* v_cache,
                             int64_t cache_slot_stride, const void* slot_mapping,
                             bool slot64, int64_t num_tokens, int64_t row_elems,
                             int32_t elem_bytes, int64_t num_slots,
                             int32_t* status, cudaStream_t stream) {
  const int64_t row_bytes = row_elems * elem_bytes;
  const int64_t ks = key_row_stride * elem_bytes;
  const int64_t vs = value_row_stride * elem_bytes;
  const int64_t cs = cache_slot_stride * elem_bytes;
  uint64_t align_bits = reinterpret_cast<uintptr_t>(key) |
                        reinterpret_cast<uintptr_t>(value) |
                        reinterpret_cast<uintptr_t>(k_cache) |
                        reinterpret_cast<uintptr_t>(v_cache) |
                        static_cast<uint64_t>(ks) | static_cast<uint64_t>(vs) |
                        static_cast<uint64_t>(cs) | static_cast<uint64_t>(row_bytes);
  if ((align_bits & 15) == 0)
    return launch_vec<16>(key, ks, value, vs, k_cache, v_cache, cs, slot_mapping,
                          slot64, num_tokens, row_bytes, num_slots, status, stream);
  if ((align_bits & 7) == 0)
    return launch_vec<8>(key, ks, value, vs, k_cache, v_cache, cs, slot_mapping,
                         slot64, num_tokens, row_bytes, num_slots, status, stream);
  if ((align_bits & 3) == 0)
    return launch_vec<4>(key, ks, value, vs, k_cache, v_cache, cs, slot_mapping,
                         slot64, num_tokens, row_bytes, num_slots, status, stream);
  return launch_vec<2>(key, ks, value, vs, k_cache, v_cache, cs, slot_mapping,
                       slot64, num_tokens, row_bytes, num_slots, status, stream);
}

// Append into an FP8 E4M3 cache: each thread quantises 16 consecutive
// elements of one K or V row (two 16-byte loads, one 16-byte store):
// stored = e4m3(x * inv), inv = 1 / scale rounded once to fp32 (one multiply
// per element instead of a division), round to nearest even with
// saturation to +-448 (cvt.rn.satfinite; NaN stays NaN).
template <typename T>
__device__ __forceinline__ float2 widen2(uint32_t w);
template <>
__device__ __forceinline__ float2 widen2<__nv_bfloat16>(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 widen2<__half>(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// two floats -> two E4M3 bytes (lo in the low byte)
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T>
__global__ void __launch_bounds__(256)
    kv_append_fp8_kernel(const T* __restrict__ key, int64_t key_row_stride,
                         const T* __restrict__ value, int64_t value_row_stride,
                         uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache,
                         int64_t cache_slot_stride, const int32_t* __restrict__ slot_mapping,
                         int64_t num_tokens, int64_t vecs_per_row, const float* k_scale,
                         const float* v_scale, int64_t num_slots, int32_t* status) {
  pdl_launch_dependents();
  // reciprocals of the dequantisation scales, correctly rounded to fp32
  const float ks = __frcp_rn(k_scale != nullptr ? __ldg(k_scale) : 1.f);
  const float vs = __frcp_rn(v_scale != nullptr ? __ldg(v_scale) : 1.f);
  const int64_t per_token = 2 * vecs_per_row;
  const int64_t total = num_tokens * per_token;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t token = idx / per_token;
    const int64_t rem = idx - token * per_token;
    const int is_v = rem >= vecs_per_row;
    const int64_t vec = rem - (is_v ? vecs_per_row : 0);
    const int64_t slot = slot_mapping[token];
    if (slot == -1) continue;
    if (slot < 0 || slot >= num_slots) {
      if (vec == 0 && !is_v) report_status(status, B200_STATUS_SLOT_OUT_OF_RANGE);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(
        (is_v ? value + token * value_row_stride : key + token * key_row_stride) + vec * 16);
    const uint4 a = __ldg(src), b = __ldg(src + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const float sc = is_v ? vs : ks;
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x0 = widen2<T>(w[2 * i]);
      const float2 x1 = widen2<T>(w[2 * i + 1]);
      const uint32_t lo = e4m3x2(__fmul_rn(x0.x, sc), __fmul_rn(x0.y, sc));
      const uint32_t hi = e4m3x2(__fmul_rn(x1.x, sc), __fmul_rn(x1.y, sc));
      out[i] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>((is_v ? v_cache : k_cache) + slot * cache_slot_stride + vec * 16) =
        make_uint4(out[0], out[1], out[2], out[3]);
  }
}

cudaError_t launch_kv_append_fp8(const void* key, int64_t key_row_stride, const void* value,
                                 int64_t value_row_stride, int src_dtype, void* k_cache,
                                 void* v_cache, int64_t cache_slot_stride,
                                 const int32_t* slot_mapping, int64_t num_tokens,
                                 int64_t row_elems, const float* k_scale, const float* v_scale,
                                 int64_t num_slots, int32_t* status, cudaStream_t stream) {
  const int64_t vecs = row_elems / 16;
  const int64_t total = num_tokens * 2 * vecs;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  if (src_dtype == B200_DTYPE_BFLOAT16)
    kv_append_fp8_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(key), key_row_stride,
        static_cast<const __nv_bfloat16*>(value), value_row_stride,
        static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache), cache_slot_stride,
        slot_mapping, num_tokens, vecs, k_scale, v_scale, num_slots, status);
  else
    kv_append_fp8_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(
        static_cast<const __half*>(key), key_row_stride, static_cast<const __half*>(value),
        value_row_stride, static_cast<uint8_t*>(k_cache), static_cast<uint8_t*>(v_cache),
        cache_slot_stride, slot_mapping, num_tokens, vecs, k_scale, v_scale, num_slots, status);
  return cudaGetLastError();
}

// Slot of every new token, from the batch metadata (see b200_build_slot_mapping).
// A position past the table row (pos / block_size >= max_blocks) or a page
// id outside the pool gives slot -1 and sets B200_STATUS_SLOT_OUT_OF_RANGE.
__global__ void __launch_bounds__(256)
    build_slot_mapping_kernel(const int32_t* __restrict__ block_tables, int64_t bt_stride,
                              int max_blocks, int64_t num_blocks,
                              const int32_t* __restrict__ seq_lens,
                              const int32_t* __restrict__ query_start_loc, int num_seqs,
                              int num_tokens, int block_size, int32_t* __restrict__ slots,
                              int32_t* status) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= num_tokens) return;
  // sequence s with query_start_loc[s] <= t < query_start_loc[s + 1]
  int lo = 0, hi = num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(query_start_loc + mid) <= t) lo = mid;
    else hi = mid - 1;
  }
  const int s = lo;
  const int q0 = __ldg(query_start_loc + s);
  const int q_len = __ldg(query_start_loc + s + 1) - q0;
  const int pos = __ldg(seq_lens + s) - q_len + (t - q0);
  int32_t slot = -1;
  if (pos >= 0) {
    const int col = pos / block_size;
    if (col >= max_blocks) {
      report_status(status, B200_STATUS_SLOT_OUT_OF_RANGE);
    } else {
      const int32_t page = __ldg(block_tables + (int64_t)s * bt_stride + col);
      if (page >= (int64_t)num_blocks) report_status(status, B200_STATUS_SLOT_OUT_OF_RANGE);
      else if (page >= 0) slot = page * block_size + pos % block_size;
    }
  }
  slots[t] = slot;
}

cudaError_t launch_build_slot_mapping(const int32_t* block_tables, int64_t bt_stride,
                                      int max_blocks, int64_t num_blocks,
                                      const int32_t* seq_lens, const int32_t* query_start_loc,
                                      int num_seqs, int num_tokens, int block_size,
                                      int32_t* slots, int32_t* status, cudaStream_t stream) {
  const int threads = 256;
  const int blocks = (num_tokens + threads - 1) / threads;
  build_slot_mapping_kernel<<<blocks, threads, 0, stream>>>(
      block_tables, bt_stride, max_blocks, num_blocks, seq_lens, query_start_loc, num_seqs,
      num_tokens, block_size, slots, status);
  return cudaGetLastError();
}

// Padded block tables from the packed per-sequence block lists (see
// b200_build_block_tables). One warp per row, lanes on consecutive columns:
// every store is a coalesced 128-byte line, entries past the row's count are
// -1. A row whose list is longer than the table is cut at max_blocks and
// reported (B200_STATUS_PAGE_OUT_OF_RANGE).
__global__ void __launch_bounds__(256)
    build_block_tables_kernel(const int32_t* __restrict__ block_ids,
                              const int32_t* __restrict__ offsets, int num_seqs,
                              int max_blocks, int32_t* __restrict__ tables, int64_t stride,
                              int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_seqs; row += warps) {
    const int begin = __ldg(offsets + row);
    const int count = __ldg(offsets + row + 1) - begin;
    if (count > max_blocks && lane == 0) report_status(status, B200_STATUS_PAGE_OUT_OF_RANGE);
    int32_t* dst = tables + (int64_t)row * stride;
    for (int col = lane; col < max_blocks; col += 32)
      dst[col] = col < count ? __ldg(block_ids + begin + col) : -1;
  }
}

cudaError_t launch_build_block_tables(const int32_t* block_ids, const int32_t* offsets,
                                      int num_seqs, int max_blocks, int32_t* tables,
                                      int64_t stride, int32_t* status, cudaStream_t stream) {
  const int threads = 256;
  const int rows_per_block = threads / 32;
  int blocks = (num_seqs + rows_per_block - 1) / rows_per_block;
  if (blocks > 148 * 8) blocks = 148 * 8;
  build_block_tables_kernel<<<blocks, threads, 0, stream>>>(block_ids, offsets, num_seqs,
                                                            max_blocks, tables, stride, status);
  return cudaGetLastError();
}

}  // namespace b200
