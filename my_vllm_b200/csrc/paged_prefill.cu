// paged_prefill.cu — paged prefill / chunked-prefill attention for sm_100a.
//
// Semantics (tests/test_attention_backend.py:660-699, the fp32 reference the
// reference's FlashInfer prefill route is checked against): sequence s has
// q_len = query_start_loc[s+1] - query_start_loc[s] new query tokens and
// seq_len = seq_lens[s] KV tokens in the paged cache (prefix-cache hits plus
// the new chunk, already appended). Query token i sits at KV position
// seq_len - q_len + i and attends to positions <= that one.
//
// Design:
//   * One CTA per (sequence, KV head, block of 128 packed rows), a row being
//     a (query token, q head of the GQA group) pair: the group's heads share
//     every K/V tile, so K/V cross HBM/L2 once per group rather than once per
//     q head. Heavier row blocks (more visible keys) launch first.
//   * Warp 8 is the producer: it reads the block table and streams 64-token
//     K/V tiles (4 x 16-token sub-tiles, 128-byte swizzled TMA boxes) into a
//     4-stage ring (full / empty mbarriers). Warps 0-7 each own 16 rows.
//   * QK^T and PV on mma.sync m16n8k16 with fp32 accumulation, online softmax
//     in the exp2 domain; the causal mask is applied only on tiles that cross
//     the diagonal. V elements past the sequence end are zeroed in registers.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "paged_decode.cuh"
#include "paged_prefill.cuh"

namespace b200 {

constexpr int kPfConsumerWarps = 8;
constexpr int kPfThreads = (kPfConsumerWarps + 1) * 32;
constexpr int kPfRows = kPfConsumerWarps * 16;  // packed rows per CTA
constexpr int kPfTileTokens = 64;               // KV tokens per stage
constexpr int kPfSubTiles = kPfTileTokens / kTileTokens;
constexpr int kPfSubBytes = 4 * kHalfTileBytes;  // K lo/hi + V lo/hi of 16 tokens
constexpr int kPfStageBytes = kPfSubTiles * kPfSubBytes;  // 32 KiB
constexpr int kPfStages = 4;
constexpr int kPfSmemBytes = 1024 + kPfStages * kPfStageBytes + 2 * kPfStages * 8;

int prefill_rows_per_cta() { return kPfRows; }

__device__ __forceinline__ uint32_t pf_ld_u32(const void* p) {
  return __ldg(reinterpret_cast<const uint32_t*>(p));
}

__device__ __forceinline__ uint32_t pf_mask_pair(uint32_t v, int tok, int valid) {
  const uint32_t lo = tok < valid ? 0x0000ffffu : 0u;
  const uint32_t hi = tok + 1 < valid ? 0xffff0000u : 0u;
  return v & (lo | hi);
}

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_v,
                         const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfStages * kPfStageBytes);
  uint64_t* empty = full + kPfStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.z;
  const int kvh = blockIdx.y;
  const int rb = gridDim.x - 1 - blockIdx.x;  // heavier blocks first

  const int q_start = p.query_start_loc[s];
  const int q_len = p.query_start_loc[s + 1] - q_start;
  const int seq_len = p.seq_lens[s];
  const int total_rows = q_len * p.group;
  const int row0 = rb * kPfRows;
  if (row0 >= total_rows || seq_len <= 0) return;
  const int ctx = seq_len - q_len;  // KV position of query token 0
  const int last_row = min(row0 + kPfRows, total_rows) - 1;
  const int kv_limit = min(seq_len, max(0, ctx + last_row / p.group + 1));
  const int n_tiles = (kv_limit + kPfTileTokens - 1) / kPfTileTokens;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kPfConsumerWarps);
    }
    mbar_init_fence();
  }
  __syncthreads();

  const uint32_t ring = smem_u32(smem);

  if (warp == kPfConsumerWarps) {
    // ------------------------------------------------------------ producer --
    const int32_t* bt_row = p.block_tables + (int64_t)s * p.block_table_stride;
    int issued = 0;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int stage = i % kPfStages;
      if (i >= kPfStages) {
        const bool got = mbar_wait(smem_u32(&empty[stage]), ((i / kPfStages) - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
      }
      const uint32_t bar = smem_u32(&full[stage]);
      if (lane == 0) mbar_arrive_expect_tx(bar, kPfStageBytes);
      __syncwarp();
      if (lane < kPfSubTiles) {
        const int tok = i * kPfTileTokens + lane * kTileTokens;
        // Sub-tiles past the last page read block 0's coordinates clamped to
        // a valid page: their tokens are >= seq_len and are masked anyway.
        const int max_page_idx = (seq_len - 1) / p.block_size;
        int pidx = tok / p.block_size;
        if (pidx > max_page_idx) pidx = max_page_idx;
        const int page = bt_row[pidx];
        const int row = tok % p.block_size;
        if (page < 0 || page >= p.num_blocks)
          report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
        const uint32_t dst = ring + stage * kPfStageBytes + lane * kPfSubBytes;
        tma_load_4d(dst, &tmap_k, bar, 0, kvh, row, page);
        tma_load_4d(dst + kHalfTileBytes, &tmap_k, bar, 64, kvh, row, page);
        tma_load_4d(dst + 2 * kHalfTileBytes, &tmap_v, bar, 0, kvh, row, page);
        tma_load_4d(dst + 3 * kHalfTileBytes, &tmap_v, bar, 64, kvh, row, page);
      }
      issued = i + 1;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      // Drain the loads this warp issued before leaving (bounded waits).
      for (int i = (issued > kPfStages ? issued - kPfStages : 0); i < issued; ++i)
        mbar_wait(smem_u32(&full[i % kPfStages]), (i / kPfStages) & 1);
    }
    return;
  }

  // -------------------------------------------------------------- consumers --
  const int gr = lane >> 2;
  const int tq = lane & 3;
  const int r_lo = row0 + warp * 16 + gr;
  const int r_hi = r_lo + 8;
  const bool v_lo = r_lo < total_rows;
  const bool v_hi = r_hi < total_rows;
  const int tok_lo = v_lo ? r_lo / p.group : 0;
  const int tok_hi = v_hi ? r_hi / p.group : 0;
  const int head_lo = kvh * p.group + (v_lo ? r_lo % p.group : 0);
  const int head_hi = kvh * p.group + (v_hi ? r_hi % p.group : 0);
  const int qpos_lo = v_lo ? ctx + tok_lo : -1;
  const int qpos_hi = v_hi ? ctx + tok_hi : -1;

  // Rows owned by this warp: visible-key range and first masked position.
  const int warp_first = row0 + warp * 16;
  const int warp_last = min(warp_first + 15, total_rows - 1);
  const int warp_min_qpos = warp_first < total_rows ? ctx + warp_first / p.group : -1;
  const int warp_max_qpos = warp_first < total_rows ? ctx + warp_last / p.group : -1;

  uint32_t qa[8][4];
  {
    const T* ql = reinterpret_cast<const T*>(p.q) +
                  (int64_t)(q_start + tok_lo) * p.q_token_stride +
                  (int64_t)head_lo * p.q_head_stride;
    const T* qh = reinterpret_cast<const T*>(p.q) +
                  (int64_t)(q_start + tok_hi) * p.q_token_stride +
                  (int64_t)head_hi * p.q_head_stride;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + tq * 2;
      qa[kk][0] = v_lo ? pf_ld_u32(ql + d0) : 0u;
      qa[kk][2] = v_lo ? pf_ld_u32(ql + d0 + 8) : 0u;
      qa[kk][1] = v_hi ? pf_ld_u32(qh + d0) : 0u;
      qa[kk][3] = v_hi ? pf_ld_u32(qh + d0 + 8) : 0u;
    }
  }

  const float kNegInf = -INFINITY;
  float m_lo = kNegInf, m_hi = kNegInf, l_lo = 0.f, l_hi = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  bool ok = true;
  for (int i = 0; i < n_tiles; ++i) {
    const int stage = i % kPfStages;
    const bool got = mbar_wait(smem_u32(&full[stage]), (i / kPfStages) & 1);
    if (!__all_sync(0xffffffffu, got)) {
      ok = false;
      break;
    }
    const int tile_start = i * kPfTileTokens;
    if (tile_start <= warp_max_qpos) {
      const uint32_t base = ring + stage * kPfStageBytes;
      float sc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
      {
        const int r = (lane & 7) + ((lane >> 4) << 3);
        const int csel = (lane >> 3) & 1;
#pragma unroll
        for (int sub = 0; sub < kPfSubTiles; ++sub) {
          const uint32_t kb = base + sub * kPfSubBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(kb + (kk >> 2) * kHalfTileBytes + swz128(r, ((kk & 3) << 1) + csel),
                        b0, b1, b2, b3);
            Elem<T>::mma(sc[2 * sub], qa[kk], b0, b1);
            Elem<T>::mma(sc[2 * sub + 1], qa[kk], b2, b3);
          }
        }
      }
      const bool need_mask = tile_start + kPfTileTokens > warp_min_qpos + 1;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = sc[n][e] * p.scale_log2;
          if (need_mask) {
            const int kpos = tile_start + n * 8 + tq * 2 + (e & 1);
            const int qpos = (e < 2) ? qpos_lo : qpos_hi;
            if (kpos > qpos) v = kNegInf;
          }
          sc[n][e] = v;
        }
      }
      // Online softmax, rows lo (elements 0,1) and hi (elements 2,3).
      float mx_lo = kNegInf, mx_hi = kNegInf;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        mx_lo = fmaxf(mx_lo, fmaxf(sc[n][0], sc[n][1]));
        mx_hi = fmaxf(mx_hi, fmaxf(sc[n][2], sc[n][3]));
      }
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
      const float mn_lo = fmaxf(m_lo, mx_lo);
      const float mn_hi = fmaxf(m_hi, mx_hi);
      const float b_lo = mn_lo == kNegInf ? 0.f : mn_lo;
      const float b_hi = mn_hi == kNegInf ? 0.f : mn_hi;
      const float a_lo = fast_exp2(m_lo - b_lo);
      const float a_hi = fast_exp2(m_hi - b_hi);
      m_lo = mn_lo;
      m_hi = mn_hi;
      float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        sc[n][0] = fast_exp2(sc[n][0] - b_lo);
        sc[n][1] = fast_exp2(sc[n][1] - b_lo);
        sc[n][2] = fast_exp2(sc[n][2] - b_hi);
        sc[n][3] = fast_exp2(sc[n][3] - b_hi);
        sum_lo += sc[n][0] + sc[n][1];
        sum_hi += sc[n][2] + sc[n][3];
      }
      l_lo = l_lo * a_lo + sum_lo;
      l_hi = l_hi * a_hi + sum_hi;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        o[n][0] *= a_lo;
        o[n][1] *= a_lo;
        o[n][2] *= a_hi;
        o[n][3] *= a_hi;
      }
      // O += P V over the 4 sub-tiles.
      const int r = (lane & 7) + (((lane >> 3) & 1) << 3);
      const int csel = lane >> 4;
#pragma unroll
      for (int sub = 0; sub < kPfSubTiles; ++sub) {
        uint32_t pa[4];
        pa[0] = Elem<T>::pack(sc[2 * sub][0], sc[2 * sub][1]);
        pa[1] = Elem<T>::pack(sc[2 * sub][2], sc[2 * sub][3]);
        pa[2] = Elem<T>::pack(sc[2 * sub + 1][0], sc[2 * sub + 1][1]);
        pa[3] = Elem<T>::pack(sc[2 * sub + 1][2], sc[2 * sub + 1][3]);
        const uint32_t vb = base + sub * kPfSubBytes + 2 * kHalfTileBytes;
        const int valid = seq_len - (tile_start + sub * kTileTokens);
#pragma unroll
        for (int dn = 0; dn < 8; ++dn) {
          const int c = dn * 2 + csel;
          uint32_t v0, v1, v2, v3;
          ldmatrix_x4_trans(vb + (c >> 3) * kHalfTileBytes + swz128(r, c & 7), v0, v1, v2,
                            v3);
          if (valid < kTileTokens) {
            v0 = pf_mask_pair(v0, tq * 2, valid);
            v2 = pf_mask_pair(v2, tq * 2, valid);
            v1 = pf_mask_pair(v1, 8 + tq * 2, valid);
            v3 = pf_mask_pair(v3, 8 + tq * 2, valid);
          }
          Elem<T>::mma(o[2 * dn], pa, v0, v1);
          Elem<T>::mma(o[2 * dn + 1], pa, v2, v3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&empty[stage]));
  }
  if (!ok && lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);

  // ---- epilogue: normalise and store the valid rows ----
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
  const float inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  T* out_lo = reinterpret_cast<T*>(p.out) + (int64_t)(q_start + tok_lo) * p.out_token_stride +
              (int64_t)head_lo * p.out_head_stride;
  T* out_hi = reinterpret_cast<T*>(p.out) + (int64_t)(q_start + tok_hi) * p.out_token_stride +
              (int64_t)head_hi * p.out_head_stride;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = n * 8 + tq * 2;
    if (v_lo)
      *reinterpret_cast<uint32_t*>(out_lo + d) = Elem<T>::pack(o[n][0] * inv_lo, o[n][1] * inv_lo);
    if (v_hi)
      *reinterpret_cast<uint32_t*>(out_hi + d) = Elem<T>::pack(o[n][2] * inv_hi, o[n][3] * inv_hi);
  }
}

template <typename T>
static cudaError_t launch_typed(const CUtensorMap& mk, const CUtensorMap& mv,
                                const PrefillParams& p, int num_kv_heads, int num_seqs,
                                int max_q_len, cudaStream_t stream) {
  auto kernel = paged_prefill_kernel<T>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kPfSmemBytes);
  if (e != cudaSuccess) return e;
  const int64_t rows = (int64_t)max_q_len * p.group;
  const int blocks = (int)((rows + kPfRows - 1) / kPfRows);
  if (blocks <= 0) return cudaSuccess;
  dim3 grid(blocks, num_kv_heads, num_seqs);
  kernel<<<grid, kPfThreads, kPfSmemBytes, stream>>>(mk, mv, p);
  return cudaGetLastError();
}

cudaError_t launch_paged_prefill(const CUtensorMap& mk, const CUtensorMap& mv,
                                 const PrefillParams& p, int dtype, int num_kv_heads,
                                 int num_seqs, int max_q_len, cudaStream_t stream) {
  if (dtype == B200_DTYPE_BFLOAT16)
    return launch_typed<__nv_bfloat16>(mk, mv, p, num_kv_heads, num_seqs, max_q_len, stream);
  return launch_typed<__half>(mk, mv, p, num_kv_heads, num_seqs, max_q_len, stream);
}

}  // namespace b200
