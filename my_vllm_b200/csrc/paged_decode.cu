// paged_decode.cu — paged GQA decode attention (flash-decoding) for sm_100a.
//
// Semantics: for sequence b and query head h (KV head h / group),
//   out[b, h] = softmax(q[b, h] . K[0:len]^T * scale) . V[0:len]
// with K/V gathered from the NHD paged cache through block_tables[b]
// (nanovllm/layers/attention_backend.py:995-997 runs FlashInfer's decode
// wrapper for this; the fp32 oracle is tests/test_attention_backend.py:660-699).
//
// Design (HBM-bound: ~4 FLOP per byte of KV):
//   * One CTA per (sequence, KV head, KV partition). The group of q heads
//     that share the KV head are the rows of a 16-row MMA tile, so each K/V
//     byte is read from HBM exactly once per step.
//   * 4 warps per CTA, each an independent flash-decoding worker over an
//     interleaved subset of the partition's 16-token tiles. Lane 0 of each
//     warp streams its tiles into a 3-stage ring of shared-memory buffers
//     with 4 TMA box loads per tile (K/V x two 64-element halves of
//     head_dim, 128-byte swizzle), completing on one mbarrier per stage.
//   * QK^T and PV run on mma.sync m16n8k16 with fp32 accumulation; K comes
//     through ldmatrix, V through ldmatrix.trans; P stays in registers
//     (accumulator layout of QK^T == A-operand layout of PV).
//   * Online softmax in the exp2 domain with quad-lane shuffles; warps are
//     merged through shared memory at the end. With more than one
//     partition the CTA writes an fp32 partial output plus log2-sum-exp and
//     decode_reduce_kernel merges partitions.
//   * Every mbarrier wait is bounded (kWaitTimeoutNs); a timeout sets
//     B200_STATUS_WAIT_TIMEOUT, drains the warp's outstanding TMA loads with
//     bounded waits, and finishes without hanging the GPU.
#include <cuda_runtime.h>
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "paged_decode.cuh"

namespace b200 {

__device__ __forceinline__ uint32_t ld_u32(const void* p) {
  return __ldg(reinterpret_cast<const uint32_t*>(p));
}

// Zeroes the 16-bit halves of a packed pair whose token index (tok for the
// low half, tok + 1 for the high half) is >= valid.
__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int tok, int valid) {
  const uint32_t lo = tok < valid ? 0x0000ffffu : 0u;
  const uint32_t hi = tok + 1 < valid ? 0xffff0000u : 0u;
  return v & (lo | hi);
}

__device__ __forceinline__ uint32_t to_f16_pair(uint32_t w, __half) { return w; }
__device__ __forceinline__ uint32_t to_f16_pair(uint32_t w, __nv_bfloat16) {
  const float lo = __uint_as_float(w << 16), hi = __uint_as_float(w & 0xffff0000u);
  return Elem<__half>::pack(lo, hi);
}

template <bool kFp8, typename T>
__device__ __forceinline__ uint32_t to_f16_or_same(uint32_t w, T tag) {
  if constexpr (kFp8) return to_f16_pair(w, tag);
  else return w;
}

// kFp8 = false: K/V tiles in T, QK^T and PV on T MMAs.
// kFp8 = true: K/V stored as FP8 E4M3; each 16-token tile is one 2 KiB TMA
// box per tensor. E4M3 values convert exactly to fp16, so the MMAs run in
// fp16: q is converted once (exact for |q| in [2^-14, 65504]), P is packed
// as fp16, and the dequantisation scales fold into the softmax scale (K)
// and the final normalisation (V). Fragment layouts for FP8:
//   K: ldmatrix (no transpose) over 16-byte rows gives lane (g, q) the 4
//      bytes d = 16c + 4q .. 4q+3 of token g; they serve as the B fragment's
//      k indices {2q, 2q+1} and {8+2q, 9+2q}, so the q fragment is loaded
//      with the same permutation of d within each 16-element chunk c.
//   V: ldmatrix.trans at 16-bit granularity gives lane (g, q) the byte pairs
//      (d = 16c + 2g, 16c + 2g + 1) of tokens 2q and 2q+1; one byte permute
//      regroups them by d, giving B fragments for column d = 16c + 2g (even
//      MMA) and 16c + 2g + 1 (odd MMA). The accumulator of chunk c's even
//      and odd MMAs together holds d = 16c + 4q .. 16c + 4q + 3.
template <typename T, bool kHiRows, bool kFp8>
__global__ void __launch_bounds__(kDecodeWarps * 32, kFp8 ? 3 : 2)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v,
                        const DecodeParams p) {
  using M = typename std::conditional<kFp8, __half, T>::type;  // MMA operand type
  constexpr int kStages = kFp8 ? kFp8Stages : kDecodeStages;
  constexpr int kStageBytes = kFp8 ? kFp8StageBytes : kDecodeStageBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      smem + (kFp8 ? kFp8StageArenaBytes : kDecodeStageArenaBytes));
  int32_t* bt_s = reinterpret_cast<int32_t*>(bars + kDecodeWarps * kStages);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.z;
  const int kvh = blockIdx.y;
  const int part = blockIdx.x;

  const int seq_len = p.seq_lens[b];
  const int tok_begin = part * p.part_tokens;
  if (tok_begin >= seq_len) {
    // Only reachable for partition 0 with seq_len <= 0 (invalid metadata):
    // write zeros so the output is defined. Later partitions of shorter
    // sequences are ignored by the reduce.
    if (part == 0 && p.num_parts == 1) {
      T* ob = reinterpret_cast<T*>(p.out) + (int64_t)b * p.out_seq_stride +
              (int64_t)(kvh * p.group) * p.out_head_stride;
      for (int i = threadIdx.x; i < p.group * kHeadDim; i += blockDim.x)
        ob[(i >> 7) * p.out_head_stride + (i & 127)] = Elem<T>::from_float(0.f);
    }
    return;
  }
  if (part == p.num_parts - 1 && seq_len > tok_begin + p.part_tokens &&
      threadIdx.x == 0)
    report_status(p.status, B200_STATUS_PLAN_EXCEEDED);
  const int tok_end = min(seq_len, tok_begin + p.part_tokens);
  const int ntiles = (tok_end - tok_begin + kTileTokens - 1) / kTileTokens;
  const int page_begin = tok_begin / p.block_size;
  const int npages = (tok_end - 1) / p.block_size - page_begin + 1;

  // Block-table slice of this partition -> shared memory (coalesced), so the
  // TMA-issuing lane never waits on a global load.
  const int32_t* bt_row =
      p.block_tables + (int64_t)b * p.block_table_stride + page_begin;
  for (int i = threadIdx.x; i < npages; i += blockDim.x) bt_s[i] = bt_row[i];
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    for (int i = 0; i < kDecodeWarps * kStages; ++i)
      mbar_init(smem_u32(&bars[i]), 1);
    mbar_init_fence();
  }
  __syncthreads();

  // ---- Q fragments (A operand, rows = q heads of this KV head's group) ----
  const int gr = lane >> 2;  // row within the MMA tile
  const int tq = lane & 3;   // column pair index
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_seq_stride +
                (int64_t)(kvh * p.group) * p.q_head_stride;
  uint32_t qa[8][4];
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    // 16-bit caches: k pairs (2q, 2q+1) and (8+2q, 9+2q) of chunk kk are
    // d = 16kk + 2q (+1) and 16kk + 8 + 2q (+1). FP8: d = 16kk + 4q .. 4q+3.
    const int d0 = kFp8 ? kk * 16 + tq * 4 : kk * 16 + tq * 2;
    const int d1 = kFp8 ? d0 + 2 : d0 + 8;
    const bool lo_ok = gr < p.group;
    qa[kk][0] = lo_ok ? to_f16_or_same<kFp8>(ld_u32(qb + gr * p.q_head_stride + d0), T()) : 0u;
    qa[kk][2] = lo_ok ? to_f16_or_same<kFp8>(ld_u32(qb + gr * p.q_head_stride + d1), T()) : 0u;
    if (kHiRows) {
      const bool hi_ok = gr + 8 < p.group;
      qa[kk][1] =
          hi_ok ? to_f16_or_same<kFp8>(ld_u32(qb + (gr + 8) * p.q_head_stride + d0), T()) : 0u;
      qa[kk][3] =
          hi_ok ? to_f16_or_same<kFp8>(ld_u32(qb + (gr + 8) * p.q_head_stride + d1), T()) : 0u;
    } else {
      qa[kk][1] = 0u;
      qa[kk][3] = 0u;
    }
  }
  float scale_log2 = p.scale_log2;
  float out_scale = 1.f;
  if (kFp8) {
    if (p.k_scale != nullptr) scale_log2 *= __ldg(p.k_scale);
    if (p.v_scale != nullptr) out_scale = __ldg(p.v_scale);
  }

  // ---- per-warp TMA ring ----
  const int my_tiles =
      ntiles > warp ? (ntiles - warp + kDecodeWarps - 1) / kDecodeWarps : 0;
  uint8_t* ring = smem + warp * kStages * kStageBytes;
  const uint32_t ring_u32 = smem_u32(ring);
  const uint32_t bar0 = smem_u32(&bars[warp * kStages]);

  auto issue = [&](int j) {
    const int stage = j % kStages;
    const int t = warp + j * kDecodeWarps;
    const int tok = tok_begin + t * kTileTokens;
    const int page = bt_s[tok / p.block_size - page_begin];
    const int row = tok % p.block_size;
    if (page < 0 || page >= p.num_blocks)
      report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
    // Out-of-range coordinates are zero-filled by TMA, never dereferenced.
    const uint32_t dst = ring_u32 + stage * kStageBytes;
    const uint32_t bar = bar0 + stage * 8;
    mbar_arrive_expect_tx(bar, kStageBytes);
    if constexpr (kFp8) {
      tma_load_4d(dst, &tmap_k, bar, 0, kvh, row, page);
      tma_load_4d(dst + kFp8TileBytes, &tmap_v, bar, 0, kvh, row, page);
    } else {
      tma_load_4d(dst, &tmap_k, bar, 0, kvh, row, page);
      tma_load_4d(dst + kHalfTileBytes, &tmap_k, bar, 64, kvh, row, page);
      tma_load_4d(dst + 2 * kHalfTileBytes, &tmap_v, bar, 0, kvh, row, page);
      tma_load_4d(dst + 3 * kHalfTileBytes, &tmap_v, bar, 64, kvh, row, page);
    }
  };

  const int prologue = my_tiles < kStages ? my_tiles : kStages;
  if (lane == 0)
    for (int j = 0; j < prologue; ++j) issue(j);
  int issued = prologue;

  const float kNegInf = -INFINITY;
  float m_lo = kNegInf, m_hi = kNegInf, l_lo = 0.f, l_hi = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  int consumed = 0;
  bool ok = true;
  for (int j = 0; j < my_tiles; ++j) {
    const int stage = j % kStages;
    const uint32_t parity = (j / kStages) & 1;
    const bool got = mbar_wait(bar0 + stage * 8, parity);
    if (!__all_sync(0xffffffffu, got)) {
      ok = false;
      break;
    }
    consumed = j + 1;
    const uint32_t kb = ring_u32 + stage * kStageBytes;
    const uint32_t vb = kb + (kFp8 ? kFp8TileBytes : 2 * kHalfTileBytes);
    const int t = warp + j * kDecodeWarps;
    const int valid = min(kTileTokens, tok_end - (tok_begin + t * kTileTokens));

    // ---- S = Q K^T (16 rows x 16 tokens) ----
    float s0[4] = {0.f, 0.f, 0.f, 0.f};
    float s1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int r = (lane & 7) + ((lane >> 4) << 3);
      const int csel = (lane >> 3) & 1;
      if constexpr (kFp8) {
        // matrices: (tokens 0-7 | 8-15) x (chunk cc | cc+1) of 16 d each
#pragma unroll
        for (int cc = 0; cc < 8; cc += 2) {
          uint32_t r0, r1, r2, r3, b0, b1;
          ldmatrix_x4(kb + swz128(r, cc + csel), r0, r1, r2, r3);
          e4m3x4_to_f16(r0, b0, b1);
          Elem<M>::mma(s0, qa[cc], b0, b1);
          e4m3x4_to_f16(r1, b0, b1);
          Elem<M>::mma(s0, qa[cc + 1], b0, b1);
          e4m3x4_to_f16(r2, b0, b1);
          Elem<M>::mma(s1, qa[cc], b0, b1);
          e4m3x4_to_f16(r3, b0, b1);
          Elem<M>::mma(s1, qa[cc + 1], b0, b1);
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t addr = kb + (kk >> 2) * kHalfTileBytes +
                                swz128(r, ((kk & 3) << 1) + csel);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(addr, b0, b1, b2, b3);
          Elem<M>::mma(s0, qa[kk], b0, b1);
          Elem<M>::mma(s1, qa[kk], b2, b3);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s0[i] *= scale_log2;
      s1[i] *= scale_log2;
    }
    if (valid < kTileTokens) {
      const int c0 = tq * 2;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (c0 + (i & 1) >= valid) s0[i] = kNegInf;
        if (8 + c0 + (i & 1) >= valid) s1[i] = kNegInf;
      }
    }

    // ---- online softmax (rows gr and gr + 8) ----
    uint32_t pa[4];
    {
      float mx = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_lo, mx);
      const float base = m_new == kNegInf ? 0.f : m_new;
      const float alpha = fast_exp2(m_lo - base);
      const float p0 = fast_exp2(s0[0] - base), p1 = fast_exp2(s0[1] - base);
      const float p2 = fast_exp2(s1[0] - base), p3 = fast_exp2(s1[1] - base);
      l_lo = l_lo * alpha + (p0 + p1) + (p2 + p3);
      // alpha is exactly 1 unless the running max moved: skip the 32
      // multiplies on the (usual) tiles where no row's max moved
      if (__any_sync(0xffffffffu, m_new != m_lo)) {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][0] *= alpha;
          o[n][1] *= alpha;
        }
      }
      m_lo = m_new;
      pa[0] = Elem<M>::pack(p0, p1);
      pa[2] = Elem<M>::pack(p2, p3);
    }
    if (kHiRows) {
      float mx = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_hi, mx);
      const float base = m_new == kNegInf ? 0.f : m_new;
      const float alpha = fast_exp2(m_hi - base);
      const float p0 = fast_exp2(s0[2] - base), p1 = fast_exp2(s0[3] - base);
      const float p2 = fast_exp2(s1[2] - base), p3 = fast_exp2(s1[3] - base);
      l_hi = l_hi * alpha + (p0 + p1) + (p2 + p3);
      if (__any_sync(0xffffffffu, m_new != m_hi)) {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          o[n][2] *= alpha;
          o[n][3] *= alpha;
        }
      }
      m_hi = m_new;
      pa[1] = Elem<M>::pack(p0, p1);
      pa[3] = Elem<M>::pack(p2, p3);
    } else {
      pa[1] = 0u;
      pa[3] = 0u;
    }

    // ---- O += P V (16 rows x 128 dims) ----
    if constexpr (kFp8) {
      const int r = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int csel = lane >> 4;
#pragma unroll
      for (int cc = 0; cc < 8; cc += 2) {
        // v0 / v1: tokens 0-7 / 8-15 of chunk cc; v2 / v3: the same of cc+1
        uint32_t v[4];
        ldmatrix_x4_trans(vb + swz128(r, cc + csel), v[0], v[1], v[2], v[3]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t e0, o0, e1, o1;  // even / odd d column, tokens 2q.. / 8+2q..
          e4m3x4_to_f16(__byte_perm(v[2 * h], 0, 0x3120), e0, o0);
          e4m3x4_to_f16(__byte_perm(v[2 * h + 1], 0, 0x3120), e1, o1);
          if (valid < kTileTokens) {
            // never-written slots past the sequence end may hold NaN bytes
            e0 = mask_pair(e0, tq * 2, valid);
            o0 = mask_pair(o0, tq * 2, valid);
            e1 = mask_pair(e1, 8 + tq * 2, valid);
            o1 = mask_pair(o1, 8 + tq * 2, valid);
          }
          Elem<M>::mma(o[2 * (cc + h)], pa, e0, e1);
          Elem<M>::mma(o[2 * (cc + h) + 1], pa, o0, o1);
        }
      }
    } else {
      const int r = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int csel = lane >> 4;
#pragma unroll
      for (int dn = 0; dn < 8; ++dn) {
        const int c = dn * 2 + csel;
        const uint32_t addr = vb + (c >> 3) * kHalfTileBytes + swz128(r, c & 7);
        uint32_t v0, v1, v2, v3;
        ldmatrix_x4_trans(addr, v0, v1, v2, v3);
        if (valid < kTileTokens) {
          // Rows past the sequence end may hold never-written cache memory
          // (possibly NaN bit patterns) and P = 0 does not cancel NaN, so
          // clear those V elements in registers: v0/v2 hold tokens 2tq and
          // 2tq+1 (low/high half), v1/v3 tokens 8+2tq and 9+2tq.
          v0 = mask_pair(v0, tq * 2, valid);
          v2 = mask_pair(v2, tq * 2, valid);
          v1 = mask_pair(v1, 8 + tq * 2, valid);
          v3 = mask_pair(v3, 8 + tq * 2, valid);
        }
        Elem<M>::mma(o[2 * dn], pa, v0, v1);
        Elem<M>::mma(o[2 * dn + 1], pa, v2, v3);
      }
    }

    // ---- refill this stage with the warp's tile j + kStages ----
    fence_proxy_async_smem();
    __syncwarp();
    if (issued < my_tiles) {
      if (lane == 0) issue(issued);
      ++issued;
    }
  }

  if (!ok) {
    // A wait ran out: report, then drain this warp's loads still in flight
    // (each wait bounded again) so no TMA writes into smem after exit.
    if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
    for (int j = consumed; j < issued; ++j)
      mbar_wait(bar0 + (j % kStages) * 8, (j / kStages) & 1);
  }

  // ---- merge the warps' partial softmax states ----
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  __syncthreads();  // every warp is done with the stage buffers

  float* ml = reinterpret_cast<float*>(smem);                   // [W][2][16]
  float* mo = reinterpret_cast<float*>(smem) + kDecodeWarps * 32;  // [W][16][kMergeStride]
  if (tq == 0) {
    if (gr < p.group) {
      ml[warp * 32 + gr] = m_lo;
      ml[warp * 32 + 16 + gr] = l_lo;
    }
    if (kHiRows && gr + 8 < p.group) {
      ml[warp * 32 + gr + 8] = m_hi;
      ml[warp * 32 + 16 + gr + 8] = l_hi;
    }
  }
  if constexpr (kFp8) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = c * 16 + tq * 4;
      if (gr < p.group)
        *reinterpret_cast<float4*>(&mo[(warp * 16 + gr) * kMergeStride + d]) =
            make_float4(o[2 * c][0], o[2 * c + 1][0], o[2 * c][1], o[2 * c + 1][1]);
      if (kHiRows && gr + 8 < p.group)
        *reinterpret_cast<float4*>(&mo[(warp * 16 + gr + 8) * kMergeStride + d]) =
            make_float4(o[2 * c][2], o[2 * c + 1][2], o[2 * c][3], o[2 * c + 1][3]);
    }
  } else {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int d = n * 8 + tq * 2;
      if (gr < p.group)
        *reinterpret_cast<float2*>(&mo[(warp * 16 + gr) * kMergeStride + d]) =
            make_float2(o[n][0], o[n][1]);
      if (kHiRows && gr + 8 < p.group)
        *reinterpret_cast<float2*>(&mo[(warp * 16 + gr + 8) * kMergeStride + d]) =
            make_float2(o[n][2], o[n][3]);
    }
  }
  __syncthreads();

  for (int idx = threadIdx.x; idx < p.group * kHeadDim; idx += blockDim.x) {
    const int row = idx >> 7;
    const int d = idx & 127;
    float m = kNegInf;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) m = fmaxf(m, ml[w * 32 + row]);
    float acc = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) {
      const float mw = ml[w * 32 + row];
      if (mw == kNegInf) continue;
      const float sc = fast_exp2(mw - m);
      acc += mo[(w * 16 + row) * kMergeStride + d] * sc;
      l += ml[w * 32 + 16 + row] * sc;
    }
    const float val = l > 0.f ? acc / l * out_scale : 0.f;
    const int head = kvh * p.group + row;
    if (p.num_parts == 1) {
      T* ob = reinterpret_cast<T*>(p.out) + (int64_t)b * p.out_seq_stride +
              (int64_t)head * p.out_head_stride;
      ob[d] = Elem<T>::from_float(val);
    } else {
      const int64_t slot = ((int64_t)b * p.num_q_heads + head) * p.num_parts + part;
      p.part_o[slot * kHeadDim + d] = val;
      if (d == 0) p.part_lse[slot] = l > 0.f ? m + log2f(l) : kNegInf;
    }
  }
}

// Merges the KV partitions of one (sequence, q head) per CTA, one thread
// per head_dim element.
template <typename T>
__global__ void __launch_bounds__(kHeadDim)
    decode_reduce_kernel(const DecodeParams p) {
  const int b = blockIdx.y;
  const int head = blockIdx.x;
  const int d = threadIdx.x;
  const int seq_len = p.seq_lens[b];
  int nvalid = seq_len > 0 ? (seq_len + p.part_tokens - 1) / p.part_tokens : 0;
  if (nvalid > p.num_parts) nvalid = p.num_parts;
  const int64_t base = ((int64_t)b * p.num_q_heads + head) * p.num_parts;
  float m = -INFINITY;
  for (int i = 0; i < nvalid; ++i) m = fmaxf(m, p.part_lse[base + i]);
  float acc = 0.f, l = 0.f;
  for (int i = 0; i < nvalid; ++i) {
    const float lse = p.part_lse[base + i];
    if (lse == -INFINITY) continue;
    const float w = fast_exp2(lse - m);
    acc += w * p.part_o[(base + i) * kHeadDim + d];
    l += w;
  }
  T* ob = reinterpret_cast<T*>(p.out) + (int64_t)b * p.out_seq_stride +
          (int64_t)head * p.out_head_stride;
  ob[d] = Elem<T>::from_float(l > 0.f ? acc / l : 0.f);
}

template <typename T, bool kHiRows, bool kFp8>
static cudaError_t launch_typed(const CUtensorMap& mk, const CUtensorMap& mv,
                                const DecodeParams& p, int num_kv_heads,
                                int num_seqs, cudaStream_t stream) {
  auto kernel = paged_decode_kernel<T, kHiRows, kFp8>;
  constexpr int kSmem = decode_smem_bytes(kFp8);
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kSmem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.num_parts, num_kv_heads, num_seqs);
  kernel<<<grid, kDecodeWarps * 32, kSmem, stream>>>(mk, mv, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.num_parts > 1) {
    decode_reduce_kernel<T><<<dim3(p.num_q_heads, num_seqs), kHeadDim, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

template <bool kFp8>
static cudaError_t launch_kv(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeParams& p,
                             int dtype, int num_kv_heads, int num_seqs, cudaStream_t stream) {
  const bool hi = p.group > 8;
  if (dtype == B200_DTYPE_BFLOAT16)
    return hi ? launch_typed<__nv_bfloat16, true, kFp8>(mk, mv, p, num_kv_heads, num_seqs, stream)
              : launch_typed<__nv_bfloat16, false, kFp8>(mk, mv, p, num_kv_heads, num_seqs,
                                                         stream);
  return hi ? launch_typed<__half, true, kFp8>(mk, mv, p, num_kv_heads, num_seqs, stream)
            : launch_typed<__half, false, kFp8>(mk, mv, p, num_kv_heads, num_seqs, stream);
}

cudaError_t launch_paged_decode(const CUtensorMap& mk, const CUtensorMap& mv,
                                const DecodeParams& p, int dtype, bool kv_fp8,
                                int num_kv_heads, int num_seqs, cudaStream_t stream) {
  return kv_fp8 ? launch_kv<true>(mk, mv, p, dtype, num_kv_heads, num_seqs, stream)
                : launch_kv<false>(mk, mv, p, dtype, num_kv_heads, num_seqs, stream);
}

}  // namespace b200
