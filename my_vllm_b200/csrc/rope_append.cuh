// rope_append.cuh — parameters of the fused q/k RMSNorm + rotary + append kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

constexpr int kRopeHeadDim = 128;

struct RopeAppendParams {
  const void* q;  // [T, Hq, 128], strides (q_token_stride, q_head_stride, 1)
  int64_t q_token_stride;
  int64_t q_head_stride;
  const void* k;  // [T, Hkv, 128], heads packed, token stride k_token_stride
  int64_t k_token_stride;
  const void* v;  // [T, Hkv, 128], heads packed
  int64_t v_token_stride;
  void* q_out;    // [T, Hq, 128]
  int64_t q_out_token_stride;
  int64_t q_out_head_stride;
  const void* q_weight;  // [128], 16-bit
  const void* k_weight;  // [128], 16-bit
  float eps;
  const int64_t* positions;     // [T]
  const float* cos_sin_cache;   // [max_position, 128]: cos | sin
  int64_t max_position;
  void* k_cache;
  void* v_cache;
  int64_t cache_slot_stride;    // cache elements between consecutive slots (Hkv * 128)
  const int32_t* slot_mapping;  // [T], -1 = no cache write
  int64_t num_tokens;
  int num_q_heads;
  int num_kv_heads;
  int64_t num_slots;
  const float* k_scale;  // FP8 caches: quantisation scales (nullptr = 1)
  const float* v_scale;
  int32_t* status;
};

cudaError_t launch_qk_norm_rope_append(const RopeAppendParams& p, int dtype, bool fp8_cache,
                                       cudaStream_t stream);

}  // namespace b200
