// rope_append.cu — fused q/k RMSNorm + rotary embedding + KV append.
//
// The step before attention in the engine (nanovllm/models/qwen3.py:96-100)
// runs q_norm, k_norm (layers/layernorm.py:30-41), the neox-style rotary
// embedding (layers/rotary_embedding.py:7-15, 40-51) and then the KV append
// (layers/attention.py:34-41) as separate kernels, each reading and writing
// q/k through HBM. Here one pass over the token's rows does all of it:
//   q rows: normalise, scale by q_weight, rotate -> q_out
//   k rows: normalise, scale by k_weight, rotate -> k_cache[slot]
//   v rows: copied to v_cache[slot]
// so the rotated k never exists outside the cache. With an FP8 E4M3 pool the
// k and v rows are quantised on the way in, exactly as the FP8 append would
// quantise the 16-bit rows (k after its rounding to the 16-bit type). Rounding follows the
// reference's eager math: the normalised row is rounded to the 16-bit type,
// multiplied by the 16-bit weight and rounded again, then rotated in fp32 from
// those values (no fused multiply-adds, IEEE square root and division) and
// rounded once more.
#include <cuda_runtime.h>

#include <type_traits>

#include "common.cuh"
#include "rope_append.cuh"

namespace b200 {

// f32x2 helpers (f2, f2_split, f2_mul, f2_add, f2_sub, f2_fma) are in common.cuh

template <typename T>
struct Pair;
template <>
struct Pair<__nv_bfloat16> {
  __device__ __forceinline__ static uint64_t widen(uint32_t w) {  // exact
    return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  __device__ __forceinline__ static uint32_t narrow(uint64_t x) {  // round to nearest even
    float lo, hi;
    f2_split(x, lo, hi);
    return Elem<__nv_bfloat16>::pack(lo, hi);
  }
  // 16-bit x 16-bit product rounded once to 16 bits (exact in fp32 first)
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};
template <>
struct Pair<__half> {
  __device__ __forceinline__ static uint64_t widen(uint32_t w) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return f2(f.x, f.y);
  }
  __device__ __forceinline__ static uint32_t narrow(uint64_t x) {
    float lo, hi;
    f2_split(x, lo, hi);
    return Elem<__half>::pack(lo, hi);
  }
  __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Work layout: one warp per token; its 32 lanes form 4 groups of 8, each
// group one (token, head) row per pass: lane l of a group owns elements
// [8l, 8l + 8) (x1) and [64 + 8l, 64 + 8l + 8) (x2) of the 128-element row,
// i.e. 8 complete rotary pairs, moved as two 16-byte vectors. The token's
// cos/sin values stay in registers across its Hq + 2 Hkv rows, the two norm
// weights in shared memory; the mean of squares is reduced over the group's
// 8 lanes. Each group loads kRowsInFlight rows before computing any, so
// every warp keeps 2 KiB of loads in flight; three 8-warp blocks per SM (24
// warps, register-limited) keep more in flight per SM than two blocks with
// batches of four rows.
constexpr int kRowsInFlight = 2;  // rows each lane group loads before computing
constexpr int kRopeCtasPerSm = 3;

// FP8 E4M3 cache rows: 8 values of T (4 words) -> 8 bytes, each
// e4m3(x * inv) with inv = 1 / scale rounded once to fp32, round to nearest even and
// saturation to +-448 (the semantics of b200_store_kvcache_fp8).
template <typename T>
__device__ __forceinline__ uint2 quantize8(const uint32_t (&w)[4], float inv) {
  uint32_t out[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t bytes = 0;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      float lo, hi;
      f2_split(Pair<T>::widen(w[2 * h + i]), lo, hi);
      uint16_t r;
      asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;"
          : "=h"(r)
          : "f"(__fmul_rn(hi, inv)), "f"(__fmul_rn(lo, inv)));
      bytes |= static_cast<uint32_t>(r) << (16 * i);
    }
    out[h] = bytes;
  }
  return make_uint2(out[0], out[1]);
}

template <typename T, bool kFp8>
__global__ void __launch_bounds__(256, kRopeCtasPerSm)
    qk_norm_rope_append_kernel(const RopeAppendParams p) {
  using P = Pair<T>;
  // cache element type: T, or one byte (E4M3) per element
  using C = typename std::conditional<kFp8, uint8_t, T>::type;
  // FP8: reciprocals of the dequantisation scales, correctly rounded to fp32
  const float k_inv = __frcp_rn(kFp8 && p.k_scale != nullptr ? __ldg(p.k_scale) : 1.f);
  const float v_inv = __frcp_rn(kFp8 && p.v_scale != nullptr ? __ldg(p.v_scale) : 1.f);
  __shared__ uint4 weights[2][16];  // q_weight, k_weight
  if (threadIdx.x < 32)
    weights[threadIdx.x >> 4][threadIdx.x & 15] = __ldg(
        reinterpret_cast<const uint4*>(threadIdx.x < 16 ? p.q_weight : p.k_weight) +
        (threadIdx.x & 15));
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int grp = lane >> 3;
  const int l = lane & 7;
  const uint32_t gmask = 0xffu << (grp * 8);
  const int hq = p.num_q_heads;
  const int hqk = p.num_q_heads + p.num_kv_heads;
  const int rows = hqk + p.num_kv_heads;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);

  for (int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
       t < p.num_tokens; t += warps) {
    const int32_t slot = __ldg(p.slot_mapping + t);
    const int64_t pos = __ldg(p.positions + t);
    const bool slot_ok = slot >= 0 && slot < p.num_slots;
    const bool pos_ok = pos >= 0 && pos < p.max_position;
    if (lane == 0) {
      if (slot >= p.num_slots || slot < -1) report_status(p.status, B200_STATUS_SLOT_OUT_OF_RANGE);
      if (!pos_ok) report_status(p.status, B200_STATUS_POSITION_OUT_OF_RANGE);
    }
    uint64_t cs[4], sn[4];  // cos / sin of this lane's 8 pairs, as f32x2
    if (pos_ok) {
      const float4* row = reinterpret_cast<const float4*>(p.cos_sin_cache + pos * kRopeHeadDim);
      const float4 c0 = __ldg(row + 2 * l), c1 = __ldg(row + 2 * l + 1);
      const float4 s0 = __ldg(row + 16 + 2 * l), s1 = __ldg(row + 16 + 2 * l + 1);
      cs[0] = f2(c0.x, c0.y); cs[1] = f2(c0.z, c0.w); cs[2] = f2(c1.x, c1.y); cs[3] = f2(c1.z, c1.w);
      sn[0] = f2(s0.x, s0.y); sn[1] = f2(s0.z, s0.w); sn[2] = f2(s1.x, s1.y); sn[3] = f2(s1.z, s1.w);
    }
    // Source row j of this token, or nullptr when nothing is written for it:
    // k and v rows need a valid slot, q and k rows a valid position.
    auto src_of = [&](int j) -> const uint4* {
      if (j >= rows) return nullptr;
      if (j < hq)
        return pos_ok ? reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                                        t * p.q_token_stride + j * p.q_head_stride)
                      : nullptr;
      if (!slot_ok) return nullptr;
      if (j < hqk)
        return pos_ok ? reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.k) +
                                                        t * p.k_token_stride +
                                                        (j - hq) * kRopeHeadDim)
                      : nullptr;
      return reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.v) +
                                            t * p.v_token_stride + (j - hqk) * kRopeHeadDim);
    };
    for (int j0 = grp; j0 < rows; j0 += 4 * kRowsInFlight) {
      const uint4* src[kRowsInFlight];
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) src[u] = src_of(j0 + 4 * u);
      uint4 a[kRowsInFlight], b[kRowsInFlight];
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u)
        if (src[u]) {
          a[u] = __ldg(src[u] + l);
          b[u] = __ldg(src[u] + 8 + l);
        }
#pragma unroll
      for (int u = 0; u < kRowsInFlight; ++u) {
        if (!src[u]) continue;
        const int j = j0 + 4 * u;
        if (j >= hqk) {  // v row: copied (or quantised) into the cache slot
          C* dst = reinterpret_cast<C*>(p.v_cache) + (int64_t)slot * p.cache_slot_stride +
                   (j - hqk) * kRopeHeadDim;
          if constexpr (kFp8) {
            const uint32_t wa[4] = {a[u].x, a[u].y, a[u].z, a[u].w};
            const uint32_t wb[4] = {b[u].x, b[u].y, b[u].z, b[u].w};
            reinterpret_cast<uint2*>(dst)[l] = quantize8<T>(wa, v_inv);
            reinterpret_cast<uint2*>(dst)[8 + l] = quantize8<T>(wb, v_inv);
          } else {
            reinterpret_cast<uint4*>(dst)[l] = a[u];
            reinterpret_cast<uint4*>(dst)[8 + l] = b[u];
          }
          continue;
        }
        const bool is_q = j < hq;
        uint64_t x1[4], x2[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x1[i] = P::widen(word(a[u], i));
          x2[i] = P::widen(word(b[u], i));
        }
        // mean of squares over the 128 elements (the group's 8 lanes)
        uint64_t acc = f2_mul(x1[0], x1[0]);
#pragma unroll
        for (int i = 1; i < 4; ++i) acc = f2_fma(x1[i], x1[i], acc);
#pragma unroll
        for (int i = 0; i < 4; ++i) acc = f2_fma(x2[i], x2[i], acc);
        float ss_lo, ss_hi;
        f2_split(acc, ss_lo, ss_hi);
        float ss = ss_lo + ss_hi;
        ss += __shfl_xor_sync(gmask, ss, 1);
        ss += __shfl_xor_sync(gmask, ss, 2);
        ss += __shfl_xor_sync(gmask, ss, 4);
        const float var = ss * (1.0f / kRopeHeadDim);  // exact: power of two
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.eps)));
        const uint64_t inv2 = f2(inv, inv);
        const uint4 w1 = weights[is_q ? 0 : 1][l];
        const uint4 w2 = weights[is_q ? 0 : 1][8 + l];
        uint32_t y1w[4], y2w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          // normalise, round to T, scale by the T weight (one rounding), widen
          const uint64_t n1 = P::widen(P::mul(P::narrow(f2_mul(x1[i], inv2)), word(w1, i)));
          const uint64_t n2 = P::widen(P::mul(P::narrow(f2_mul(x2[i], inv2)), word(w2, i)));
          // y1 = x1 cos - x2 sin, y2 = x2 cos + x1 sin (fp32, each op rounded)
          y1w[i] = P::narrow(f2_sub(f2_mul(n1, cs[i]), f2_mul(n2, sn[i])));
          y2w[i] = P::narrow(f2_add(f2_mul(n2, cs[i]), f2_mul(n1, sn[i])));
        }
        if (kFp8 && !is_q) {  // rotated k, rounded to T, then quantised like the append
          uint2* dst = reinterpret_cast<uint2*>(reinterpret_cast<C*>(p.k_cache) +
                                                (int64_t)slot * p.cache_slot_stride +
                                                (j - hq) * kRopeHeadDim);
          dst[l] = quantize8<T>(y1w, k_inv);
          dst[8 + l] = quantize8<T>(y2w, k_inv);
          continue;
        }
        uint4* dst = reinterpret_cast<uint4*>(
            is_q ? reinterpret_cast<T*>(p.q_out) + t * p.q_out_token_stride +
                       j * p.q_out_head_stride
                 : reinterpret_cast<T*>(p.k_cache) + (int64_t)slot * p.cache_slot_stride +
                       (j - hq) * kRopeHeadDim);
        dst[l] = make_uint4(y1w[0], y1w[1], y1w[2], y1w[3]);
        dst[8 + l] = make_uint4(y2w[0], y2w[1], y2w[2], y2w[3]);
      }
    }
  }
}

cudaError_t launch_qk_norm_rope_append(const RopeAppendParams& p, int dtype, bool fp8_cache,
                                       cudaStream_t stream) {
  // 8 warps per block, one token per warp; at most the 3 blocks per SM that
  // fit at once, the grid-stride loop covers the rest
  int64_t blocks = (p.num_tokens + 7) / 8;
  if (blocks > 148 * kRopeCtasPerSm) blocks = 148 * kRopeCtasPerSm;
  if (blocks < 1) blocks = 1;
  if (dtype == B200_DTYPE_BFLOAT16) {
    if (fp8_cache)
      qk_norm_rope_append_kernel<__nv_bfloat16, true><<<(unsigned)blocks, 256, 0, stream>>>(p);
    else
      qk_norm_rope_append_kernel<__nv_bfloat16, false><<<(unsigned)blocks, 256, 0, stream>>>(p);
  } else {
    if (fp8_cache)
      qk_norm_rope_append_kernel<__half, true><<<(unsigned)blocks, 256, 0, stream>>>(p);
    else
      qk_norm_rope_append_kernel<__half, false><<<(unsigned)blocks, 256, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace b200
