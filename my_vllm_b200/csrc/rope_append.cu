// rope_append.cu — fused q/k RMSNorm + rotary embedding + KV append.
//
// The step before attention in the engine (nanovllm/models/qwen3.py:96-100)
// runs q_norm, k_norm (layers/layernorm.py:30-41), the neox-style rotary
// embedding (layers/rotary_embedding.py:7-15, 40-51) and then the KV append
// (layers/attention.py:34-41) as separate kernels, each reading and writing
// q/k through HBM. Here one warp owns one (token, head) row of 128 elements:
//   q rows: normalise, scale by q_weight, rotate -> q_out
//   k rows: normalise, scale by k_weight, rotate -> k_cache[slot]
//   v rows: copied to v_cache[slot]
// so the rotated k never exists outside the cache. Rounding follows the
// reference's eager math: the normalised row is rounded to the 16-bit type,
// multiplied by the 16-bit weight and rounded again, then rotated in fp32 from
// those values (no fused multiply-adds, IEEE square root and division) and
// rounded once more.
#include <cuda_runtime.h>

#include "common.cuh"
#include "rope_append.cuh"

namespace b200 {

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f<__half>(__half x) {
  return __half2float(x);
}

template <typename T>
__device__ __forceinline__ float round_t(float x) {
  return to_f<T>(Elem<T>::from_float(x));
}

template <typename T>
__global__ void __launch_bounds__(256)
    qk_norm_rope_append_kernel(const RopeAppendParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t rows_per_token = p.num_q_heads + 2 * p.num_kv_heads;
  const int64_t total = p.num_tokens * rows_per_token;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < total;
       r += warps) {
    const int64_t t = r / rows_per_token;
    const int j = static_cast<int>(r - t * rows_per_token);
    const int32_t slot = p.slot_mapping[t];
    if (j >= p.num_q_heads + p.num_kv_heads) {
      // v row: plain copy into the cache slot (16 lanes x 16 bytes)
      if (slot < 0) continue;
      if (slot >= p.num_slots) {
        if (lane == 0) report_status(p.status, B200_STATUS_SLOT_OUT_OF_RANGE);
        continue;
      }
      const int h = j - p.num_q_heads - p.num_kv_heads;
      const T* src = reinterpret_cast<const T*>(p.v) + t * p.v_token_stride + h * kRopeHeadDim;
      T* dst = reinterpret_cast<T*>(p.v_cache) + (int64_t)slot * p.cache_slot_stride +
               h * kRopeHeadDim;
      if (lane < 16)
        reinterpret_cast<uint4*>(dst)[lane] = __ldg(reinterpret_cast<const uint4*>(src) + lane);
      continue;
    }
    const bool is_q = j < p.num_q_heads;
    const int h = is_q ? j : j - p.num_q_heads;
    if (!is_q && slot < 0) continue;
    if (!is_q && slot >= p.num_slots) {
      if (lane == 0) report_status(p.status, B200_STATUS_SLOT_OUT_OF_RANGE);
      continue;
    }
    const T* src = is_q ? reinterpret_cast<const T*>(p.q) + t * p.q_token_stride +
                              h * p.q_head_stride
                        : reinterpret_cast<const T*>(p.k) + t * p.k_token_stride +
                              h * kRopeHeadDim;
    // lane owns rotary pairs i = 2*lane, 2*lane + 1: x1 = row[i], x2 = row[64 + i]
    const int i0 = 2 * lane;
    const uint32_t w1 = __ldg(reinterpret_cast<const uint32_t*>(src + i0));
    const uint32_t w2 = __ldg(reinterpret_cast<const uint32_t*>(src + 64 + i0));
    const T* e1 = reinterpret_cast<const T*>(&w1);
    const T* e2 = reinterpret_cast<const T*>(&w2);
    float x[4] = {to_f<T>(e1[0]), to_f<T>(e1[1]), to_f<T>(e2[0]), to_f<T>(e2[1])};
    float ss = __fmul_rn(x[0], x[0]);
    ss = __fadd_rn(ss, __fmul_rn(x[1], x[1]));
    ss = __fadd_rn(ss, __fmul_rn(x[2], x[2]));
    ss = __fadd_rn(ss, __fmul_rn(x[3], x[3]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
    const float var = __fdiv_rn(ss, static_cast<float>(kRopeHeadDim));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
    const T* wt = reinterpret_cast<const T*>(is_q ? p.q_weight : p.k_weight);
    const int dims[4] = {i0, i0 + 1, 64 + i0, 64 + i0 + 1};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float normed = round_t<T>(__fmul_rn(x[e], inv));
      x[e] = round_t<T>(__fmul_rn(normed, to_f<T>(wt[dims[e]])));
    }
    const int64_t pos = p.positions[t];
    if (pos < 0 || pos >= p.max_position) {  // no rotation row for it: skip, report
      if (lane == 0) report_status(p.status, B200_STATUS_POSITION_OUT_OF_RANGE);
      continue;
    }
    const float* cs = p.cos_sin_cache + pos * kRopeHeadDim;
    float y[4];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float c = cs[i0 + e];
      const float s = cs[64 + i0 + e];
      y[e] = __fsub_rn(__fmul_rn(x[e], c), __fmul_rn(x[2 + e], s));      // x1 cos - x2 sin
      y[2 + e] = __fadd_rn(__fmul_rn(x[2 + e], c), __fmul_rn(x[e], s));  // x2 cos + x1 sin
    }
    T* dst = is_q ? reinterpret_cast<T*>(p.q_out) + t * p.q_out_token_stride +
                        h * p.q_out_head_stride
                  : reinterpret_cast<T*>(p.k_cache) + (int64_t)slot * p.cache_slot_stride +
                        h * kRopeHeadDim;
    *reinterpret_cast<uint32_t*>(dst + i0) = Elem<T>::pack(y[0], y[1]);
    *reinterpret_cast<uint32_t*>(dst + 64 + i0) = Elem<T>::pack(y[2], y[3]);
  }
}

cudaError_t launch_qk_norm_rope_append(const RopeAppendParams& p, int dtype,
                                       cudaStream_t stream) {
  const int64_t rows = p.num_tokens * (p.num_q_heads + 2 * p.num_kv_heads);
  int64_t blocks = (rows + 7) / 8;  // 8 warps per block, one row per warp
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  if (dtype == B200_DTYPE_BFLOAT16)
    qk_norm_rope_append_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(p);
  else
    qk_norm_rope_append_kernel<__half><<<(unsigned)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace b200
