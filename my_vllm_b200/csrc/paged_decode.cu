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
//     that share the KV head are the columns (N = 8 per MMA) of every MMA,
//     so each K/V byte is read from HBM exactly once per step.
//   * 4 warps per CTA, each an independent flash-decoding worker over an
//     interleaved subset of the partition's 16-token tiles. Lane 0 of each
//     warp streams its tiles into a 3-stage ring of shared-memory buffers
//     with 4 TMA box loads per tile (K/V x two 64-element halves of
//     head_dim, 128-byte swizzle), completing on one mbarrier per stage.
//   * The KV tile is the A operand (M = 16 tokens or 16 d rows): S^T = K Q^T
//     with K through ldmatrix and Q^T (N = 8 heads) in registers, then
//     O^T += V^T P^T with V through ldmatrix.trans. P^T comes out of the QK
//     accumulator as (token, head) and two movmatrix.trans per tile turn it
//     into the B operand. A GQA group of 4 fills half of each MMA's N.
//   * Online softmax in the exp2 domain per head column: the tile maximum is
//     an in-thread max over 2 tokens plus 3 shuffles over the 8 lanes holding
//     the other tokens; warps are merged through shared memory at the end. With more than one
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

// Transpose of an 8x8 16-bit matrix held one packed pair per lane in the MMA
// accumulator layout (lane (g, q): row g, columns 2q, 2q+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
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
//      bytes d = 16c + 4q .. 4q+3 of token g; they serve as the A fragment's
//      k indices {2q, 2q+1} and {8+2q, 9+2q}, so the Q^T fragment is loaded
//      with the same permutation of d within each 16-element chunk c.
//   V: ldmatrix.trans at 16-bit granularity gives lane (g, q) the byte pairs
//      (d = 16c + 2g, 16c + 2g + 1) of tokens 2q and 2q+1; one byte permute
//      regroups them by d, giving A fragments whose row g is d = 16c + 2g
//      (even m-tile) or 16c + 2g + 1 (odd m-tile); rows g + 8 come from
//      chunk c + 1. The merge writes each accumulator to its d.
// kWideGroup: more than 8 q heads per KV head, two 8-head n-tiles per MMA step.
template <typename T, bool kWideGroup, bool kFp8>
__global__ void __launch_bounds__(kDecodeWarps * 32, kFp8 ? (kWideGroup ? 3 : 4) : 2)
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

  // ---- Q^T fragments (B operand: k = head_dim, n = 8 q heads of the group) ----
  constexpr int NT = kWideGroup ? 2 : 1;  // 8-head n-tiles
  const int gr = lane >> 2;  // fragment row (token or d) / column (head) index
  const int tq = lane & 3;   // column-pair index
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_seq_stride +
                (int64_t)(kvh * p.group) * p.q_head_stride;
  uint32_t qf[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int h = nt * 8 + gr;
    const bool ok_h = h < p.group;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // 16-bit caches: k pairs (2q, 2q+1) and (8+2q, 9+2q) of chunk kk are
      // d = 16kk + 2q (+1) and 16kk + 8 + 2q (+1). FP8: d = 16kk + 4q .. 4q+3.
      const int d0 = kFp8 ? kk * 16 + tq * 4 : kk * 16 + tq * 2;
      const int d1 = kFp8 ? d0 + 2 : d0 + 8;
      qf[nt][kk][0] = ok_h ? to_f16_or_same<kFp8>(ld_u32(qb + h * p.q_head_stride + d0), T()) : 0u;
      qf[nt][kk][1] = ok_h ? to_f16_or_same<kFp8>(ld_u32(qb + h * p.q_head_stride + d1), T()) : 0u;
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

  // Everything above reads only metadata and q. The cache may still be
  // receiving this step's rows from the append kernel launched just before
  // (this kernel is launched as its programmatic dependent): wait for it.
  pdl_wait();
  const int prologue = my_tiles < kStages ? my_tiles : kStages;
  if (lane == 0)
    for (int j = 0; j < prologue; ++j) issue(j);
  int issued = prologue;

  const float kNegInf = -INFINITY;
  // softmax state per head column of this thread: heads nt*8 + 2q + c
  float m_run[NT][2], l_run[NT][2];
  // O^T accumulators: per n-tile, 8 m-tiles of 16 d rows x 8 heads
  float o[NT][8][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m_run[nt][0] = m_run[nt][1] = kNegInf;
    l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
  }

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

    // ---- S^T = K Q^T (16 tokens x 8 heads per n-tile); A = K from the tile ----
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    {
      // matrices of one x4 load: (tokens 0-7 | 8-15) x (k columns 0-7 | 8-15)
      const int r = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int csel = lane >> 4;
      if constexpr (kFp8) {
        // one 16-byte row chunk holds 16 d of one token: chunks cc and cc+1
#pragma unroll
        for (int cc = 0; cc < 8; cc += 2) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(kb + swz128(r, cc + csel), r0, r1, r2, r3);
          uint32_t a[4];
          e4m3x4_to_f16(r0, a[0], a[2]);  // tokens g: d 16cc + 4q .. 4q+3
          e4m3x4_to_f16(r1, a[1], a[3]);  // tokens g + 8
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Elem<M>::mma(sc[nt], a, qf[nt][cc][0], qf[nt][cc][1]);
          e4m3x4_to_f16(r2, a[0], a[2]);
          e4m3x4_to_f16(r3, a[1], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            Elem<M>::mma(sc[nt], a, qf[nt][cc + 1][0], qf[nt][cc + 1][1]);
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t addr = kb + (kk >> 2) * kHalfTileBytes +
                                swz128(r, ((kk & 3) << 1) + csel);
          uint32_t a[4];
          ldmatrix_x4(addr, a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Elem<M>::mma(sc[nt], a, qf[nt][kk][0], qf[nt][kk][1]);
        }
      }
    }

    // ---- online softmax per head column (max over the 16 tokens of the tile) ----
    uint32_t pb[NT][2];  // P^T as the B operand of PV (after the transpose)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) sc[nt][i] *= scale_log2;
      if (valid < kTileTokens) {
        if (gr >= valid) sc[nt][0] = sc[nt][1] = kNegInf;
        if (gr + 8 >= valid) sc[nt][2] = sc[nt][3] = kNegInf;
      }
      float pr[2][2];  // [token g | g+8][head column c]
      bool moved = false;
      float alpha[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float mx = fmaxf(sc[nt][c], sc[nt][2 + c]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[nt][c], mx);
        const float base = m_new == kNegInf ? 0.f : m_new;
        alpha[c] = fast_exp2(m_run[nt][c] - base);
        pr[0][c] = fast_exp2(sc[nt][c] - base);
        pr[1][c] = fast_exp2(sc[nt][2 + c] - base);
        l_run[nt][c] = l_run[nt][c] * alpha[c] + (pr[0][c] + pr[1][c]);
        moved |= m_new != m_run[nt][c];
        m_run[nt][c] = m_new;
      }
      // alpha is exactly 1 unless a running max moved: skip the multiplies
      // on the (usual) tiles where none did
      if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          o[nt][mt][0] *= alpha[0];
          o[nt][mt][1] *= alpha[1];
          o[nt][mt][2] *= alpha[0];
          o[nt][mt][3] *= alpha[1];
        }
      }
      // P^T rows (tokens) x columns (heads) in accumulator layout -> transpose
      // to the B layout (k = tokens 2q, 2q+1 | 8+2q, 9+2q; n = head g)
      pb[nt][0] = movmatrix_trans(Elem<M>::pack(pr[0][0], pr[0][1]));
      pb[nt][1] = movmatrix_trans(Elem<M>::pack(pr[1][0], pr[1][1]));
    }

    // ---- O^T += V^T P^T (16 d rows x 8 heads per m-tile); A = V^T ----
    {
      // matrices of one x4.trans load: (tokens 0-7 | 8-15) x (two 8-column
      // chunks); lane (g, q) receives tokens 2q, 2q+1 of column g
      const int r = (lane & 7) + ((lane >> 4) << 3);
      const int csel = (lane >> 3) & 1;
      if constexpr (kFp8) {
#pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          // chunks 2pp, 2pp+1 (d 32pp .. 32pp + 31): even / odd d m-tiles
          uint32_t v[4];
          ldmatrix_x4_trans(vb + swz128(r, 2 * pp + csel), v[0], v[1], v[2], v[3]);
          uint32_t ae[4], ao[4];
          e4m3x4_to_f16(__byte_perm(v[0], 0, 0x3120), ae[0], ao[0]);  // d 32pp + 2g, tok 2q..
          e4m3x4_to_f16(__byte_perm(v[1], 0, 0x3120), ae[1], ao[1]);  // d 32pp + 16 + 2g
          e4m3x4_to_f16(__byte_perm(v[2], 0, 0x3120), ae[2], ao[2]);  // tokens 8 + 2q..
          e4m3x4_to_f16(__byte_perm(v[3], 0, 0x3120), ae[3], ao[3]);
          if (valid < kTileTokens) {  // never-written slots may hold NaN bytes
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int tok = (i >> 1) * 8 + tq * 2;
              ae[i] = mask_pair(ae[i], tok, valid);
              ao[i] = mask_pair(ao[i], tok, valid);
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Elem<M>::mma(o[nt][2 * pp], ae, pb[nt][0], pb[nt][1]);
            Elem<M>::mma(o[nt][2 * pp + 1], ao, pb[nt][0], pb[nt][1]);
          }
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int c = mt * 2 + csel;  // 8-element column chunk (d 8c .. 8c + 7)
          const uint32_t addr = vb + (c >> 3) * kHalfTileBytes + swz128(r, c & 7);
          uint32_t a[4];
          ldmatrix_x4_trans(addr, a[0], a[1], a[2], a[3]);
          if (valid < kTileTokens) {
            // Rows past the sequence end may hold never-written cache memory
            // (possibly NaN bit patterns) and P = 0 does not cancel NaN, so
            // clear those V elements in registers.
            a[0] = mask_pair(a[0], tq * 2, valid);
            a[1] = mask_pair(a[1], tq * 2, valid);
            a[2] = mask_pair(a[2], 8 + tq * 2, valid);
            a[3] = mask_pair(a[3], 8 + tq * 2, valid);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Elem<M>::mma(o[nt][mt], a, pb[nt][0], pb[nt][1]);
        }
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
  // each lane summed only its two tokens per tile: add over the 8 lanes g
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      l_run[nt][c] += __shfl_xor_sync(0xffffffffu, l_run[nt][c], 4);
      l_run[nt][c] += __shfl_xor_sync(0xffffffffu, l_run[nt][c], 8);
      l_run[nt][c] += __shfl_xor_sync(0xffffffffu, l_run[nt][c], 16);
    }
  __syncthreads();  // every warp is done with the stage buffers

  float* ml = reinterpret_cast<float*>(smem);                   // [W][2][16]
  float* mo = reinterpret_cast<float*>(smem) + kDecodeWarps * 32;  // [W][16][kMergeStride]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int head = nt * 8 + tq * 2 + c;
      if (head < p.group) {
        if (gr == 0) {
          ml[warp * 32 + head] = m_run[nt][c];
          ml[warp * 32 + 16 + head] = l_run[nt][c];
        }
        float* row = &mo[(warp * 16 + head) * kMergeStride];
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          // bf16: m-tile mt holds d = 16 mt + g (+8); FP8: m-tile 2pp + e
          // holds d = 32 pp + 2g + e (+16)
          const int d_lo = kFp8 ? 32 * (mt >> 1) + 2 * gr + (mt & 1) : 16 * mt + gr;
          const int d_hi = kFp8 ? d_lo + 16 : d_lo + 8;
          row[d_lo] = o[nt][mt][c];
          row[d_hi] = o[nt][mt][2 + c];
        }
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

template <typename T, bool kWideGroup, bool kFp8>
static cudaError_t launch_typed(const CUtensorMap& mk, const CUtensorMap& mv,
                                const DecodeParams& p, int num_kv_heads,
                                int num_seqs, cudaStream_t stream) {
  auto kernel = paged_decode_kernel<T, kWideGroup, kFp8>;
  constexpr int kSmem = decode_smem_bytes(kFp8);
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kSmem);
  if (e != cudaSuccess) return e;
  // Launched as a programmatic dependent of the previous kernel on the
  // stream (the KV append of the same step): the CTAs' prologue overlaps the
  // append, and pdl_wait() holds the cache reads until it has completed.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.num_parts, num_kv_heads, num_seqs);
  cfg.blockDim = dim3(kDecodeWarps * 32);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, mk, mv, p);
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
