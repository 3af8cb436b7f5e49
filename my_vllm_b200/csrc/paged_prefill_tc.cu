// paged_prefill_tc.cu — paged prefill / chunked-prefill attention on the
// 5th-generation tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Semantics (tests/test_attention_backend.py:660-699): sequence s has
// q_len = query_start_loc[s+1] - query_start_loc[s] new query tokens and
// seq_len = seq_lens[s] KV tokens in the paged cache (prefix-cache hits plus
// the new chunk, already appended). Query token i sits at KV position
// seq_len - q_len + i and attends to positions <= that one.
//
// Design (one CTA per (sequence, KV head, block of 128 packed rows)):
//   * A row is a (query token, q head of the GQA group) pair; 128 rows form
//     the M = 128 side of every UMMA, so the group's heads share each K/V
//     tile that crosses HBM/L2.
//   * warps 0-3 (128 threads): softmax and epilogue, thread t owns row t =
//     TMEM lane t, so row max / row sum need no shuffles. They stage Q into
//     shared memory (K-major, 128-byte swizzle) at the start.
//   * warp 4: TMA producer, 128-token K/V tiles of the paged cache (8 x
//     16-token sub-tiles, one lane each) into a 2-stage ring.
//   * warp 5: TMEM allocation (256 columns: S | O) and the single thread that
//     issues tcgen05.mma: S = Q K^T (A, B K-major) into TMEM, then
//     O += P V with P (bf16, written by the softmax warps into shared memory,
//     K-major) and V read N-major straight from the TMA tile.
//   * Online softmax in the exp2 domain with a lazy rescale: the running
//     maximum only moves when a tile's maximum exceeds it by more than 2^8,
//     so O (in TMEM) is rarely rescaled; O / l is independent of that choice.
//   * The bottom-right causal mask and the sequence end are applied in
//     registers; V rows past the sequence end are zeroed in shared memory
//     before the last PV MMA (never-written cache slots may hold NaN).
//   * Every mbarrier wait is bounded; on a timeout the CTA reports
//     B200_STATUS_WAIT_TIMEOUT, drains its TMA loads and MMAs with bounded
//     waits, frees its tensor memory and exits.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "paged_decode.cuh"
#include "paged_prefill.cuh"
#include "tcgen05.cuh"

namespace b200 {

constexpr int kTcRows = 128;   // UMMA M
constexpr int kTcKv = 128;     // KV tokens per tile (N of QK^T, K of PV)
constexpr int kTcThreads = 192;
constexpr int kTcHalf = kTcRows * 128;           // [128 rows x 64 elements] = 16 KiB
constexpr int kTcQ = 0;
constexpr int kTcStage0 = 2 * kTcHalf;           // 32 KiB after Q
constexpr int kTcStageBytes = 4 * kTcHalf;       // K lo/hi + V lo/hi = 64 KiB
constexpr int kTcP = kTcStage0 + 2 * kTcStageBytes;
constexpr int kTcBars = kTcP + 2 * kTcHalf;
constexpr int kTcSmemBytes = 1024 + kTcBars + 128;
constexpr uint32_t kTcTmemCols = 256;            // S: [0, 128), O: [128, 256)
constexpr float kRescaleThreshold = 8.0f;        // log2 units

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 r;
  r.x = Elem<__nv_bfloat16>::pack(v[0], v[1]);
  r.y = Elem<__nv_bfloat16>::pack(v[2], v[3]);
  r.z = Elem<__nv_bfloat16>::pack(v[4], v[5]);
  r.w = Elem<__nv_bfloat16>::pack(v[6], v[7]);
  return r;
}

template <typename T>
__device__ __forceinline__ uint4 pack8_t(const float* v) {
  uint4 r;
  r.x = Elem<T>::pack(v[0], v[1]);
  r.y = Elem<T>::pack(v[2], v[3]);
  r.z = Elem<T>::pack(v[4], v[5]);
  r.w = Elem<T>::pack(v[6], v[7]);
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_v,
                            const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcBars);
  // barrier slots
  uint64_t* kv_full = bars + 0;    // [2] TMA -> MMA
  uint64_t* kv_empty = bars + 2;   // [2] MMA (commit) -> TMA
  uint64_t* s_full = bars + 4;     // MMA (commit) -> softmax
  uint64_t* p_ready = bars + 5;    // softmax (128 arrivals) -> MMA
  uint64_t* o_done = bars + 6;     // MMA (commit) -> softmax
  uint64_t* mma_drain = bars + 7;  // MMA (commit) -> MMA, before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int s = blockIdx.z;
  const int kvh = blockIdx.y;
  const int rb = gridDim.x - 1 - blockIdx.x;  // heavier row blocks first

  const int q_start = p.query_start_loc[s];
  const int q_len = p.query_start_loc[s + 1] - q_start;
  const int seq_len = p.seq_lens[s];
  const int group = p.group;
  const int tpc = kTcRows / group;  // query tokens per CTA
  const int tok_begin = rb * tpc;
  if (tok_begin >= q_len || seq_len <= 0) return;  // CTA-uniform, before any sync
  const int ctx = seq_len - q_len;
  const int tok_last = min(q_len, tok_begin + tpc) - 1;
  const int kv_limit = min(seq_len, max(1, ctx + tok_last + 1));
  const int n_tiles = (kv_limit + kTcKv - 1) / kTcKv;

  const uint32_t sbase = smem_u32(smem);
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&kv_full[0]), 1);
    mbar_init(smem_u32(&kv_full[1]), 1);
    mbar_init(smem_u32(&kv_empty[0]), 1);
    mbar_init(smem_u32(&kv_empty[1]), 1);
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(p_ready), 128);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(mma_drain), 1);
    mbar_init_fence();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }

  // ---- softmax warps: this thread's row and its Q into shared memory ----
  const int t = threadIdx.x;
  int row_token = -1, row_head = 0, qpos = -1;
  if (warp < 4) {
    const int tl = t / group;
    if (tl < tpc && tok_begin + tl < q_len) {
      row_token = tok_begin + tl;
      row_head = kvh * group + (t - tl * group);
      qpos = ctx + row_token;
    }
    const uint4* src = reinterpret_cast<const uint4*>(
        reinterpret_cast<const T*>(p.q) + (int64_t)(q_start + max(row_token, 0)) * p.q_token_stride +
        (int64_t)row_head * p.q_head_stride);
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint4 v = row_token >= 0 ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(smem + kTcQ + (c >> 3) * kTcHalf + swz128(t, c & 7)) = v;
    }
    fence_proxy_async_smem();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tS = tmem_base;
  const uint32_t tO = tmem_base + 128;
  bool ok = true;

  if (warp == 4) {
    // ------------------------------------------------------------ producer --
    const int32_t* bt_row = p.block_tables + (int64_t)s * p.block_table_stride;
    const int max_page_idx = (seq_len - 1) / p.block_size;
    int issued = 0;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (j >= 2) {
        const bool got = mbar_wait(smem_u32(&kv_empty[st]), ((j >> 1) - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
      }
      const uint32_t bar = smem_u32(&kv_full[st]);
      if (lane == 0) mbar_arrive_expect_tx(bar, kTcStageBytes);
      __syncwarp();
      if (lane < kTcKv / kTileTokens) {
        const int tok = j * kTcKv + lane * kTileTokens;
        int pidx = tok / p.block_size;
        int row = tok % p.block_size;
        if (pidx > max_page_idx) {  // past the sequence end: any valid page, masked later
          pidx = max_page_idx;
          row = 0;
        }
        const int page = bt_row[pidx];
        if (page < 0 || page >= p.num_blocks)
          report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
        const uint32_t dst = sbase + kTcStage0 + st * kTcStageBytes + lane * kHalfTileBytes;
        tma_load_4d(dst, &tmap_k, bar, 0, kvh, row, page);
        tma_load_4d(dst + kTcHalf, &tmap_k, bar, 64, kvh, row, page);
        tma_load_4d(dst + 2 * kTcHalf, &tmap_v, bar, 0, kvh, row, page);
        tma_load_4d(dst + 3 * kTcHalf, &tmap_v, bar, 64, kvh, row, page);
      }
      issued = j + 1;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      for (int j = max(0, issued - 2); j < issued; ++j)
        mbar_wait(smem_u32(&kv_full[j & 1]), (j >> 1) & 1);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr bool kBf16 = Elem<T>::kDtype == B200_DTYPE_BFLOAT16;
      const uint32_t idesc_s = f16_instr_desc(kTcRows, kTcKv, kBf16, false);
      const uint32_t idesc_pv = f16_instr_desc(kTcRows, kHeadDim, kBf16, true);
      auto kmajor = [&](uint32_t addr, int k) {  // K-major, 16-element k-step k
        return smem_desc(addr + (k >> 2) * kTcHalf + (k & 3) * 32, 16, 1024);
      };
      auto issue_pv = [&](int j) {
        const uint32_t vbase = sbase + kTcStage0 + (j & 1) * kTcStageBytes + 2 * kTcHalf;
#pragma unroll
        for (int k = 0; k < kTcKv / 16; ++k)
          umma_f16(tO, kmajor(sbase + kTcP, k),
                   smem_desc(vbase + k * 16 * 128, kTcHalf, 1024), idesc_pv,
                   (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(smem_u32(o_done));
        umma_commit(smem_u32(&kv_empty[j & 1]));
      };
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(smem_u32(&kv_full[st]), (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        if (j > 0) {
          if (!mbar_wait(smem_u32(p_ready), (j - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          issue_pv(j - 1);
        }
        const uint32_t kbase = sbase + kTcStage0 + st * kTcStageBytes;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k)
          umma_f16(tS, kmajor(sbase + kTcQ, k), kmajor(kbase, k), idesc_s, k > 0 ? 1u : 0u);
        umma_commit(smem_u32(s_full));
      }
      if (ok) {
        if (mbar_wait(smem_u32(p_ready), (n_tiles - 1) & 1)) {
          tc_fence_after_sync();
          issue_pv(n_tiles - 1);
        } else {
          ok = false;
        }
      }
      if (!ok) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(smem_u32(mma_drain));
      mbar_wait(smem_u32(mma_drain), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- softmax warps --
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float kNegInf = -INFINITY;
    float m_used = kNegInf, l = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      const bool got = mbar_wait(smem_u32(s_full), j & 1);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld32(tS + lane_off + c * 32, *reinterpret_cast<float(*)[32]>(&sv[c * 32]));
      const int kbase = j * kTcKv;
      const bool need_mask = kbase + kTcKv - 1 > qpos || kbase + kTcKv > seq_len;
      float m_tile = kNegInf;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        float v = sv[i] * p.scale_log2;
        if (need_mask && (kbase + i > qpos || kbase + i >= seq_len)) v = kNegInf;
        sv[i] = v;
        m_tile = fmaxf(m_tile, v);
      }
      float alpha = 1.f;
      bool rescale = false;
      if (m_tile > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - m_tile);
        m_used = m_tile;
        rescale = true;
      }
      const float base = m_used == kNegInf ? 0.f : m_used;
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        const float pv = fast_exp2(sv[i] - base);
        sv[i] = pv;
        sum += pv;
      }
      l = l * alpha + sum;

      if (j > 0) {
        // PV of the previous tile must be done: it reads the P buffer and
        // writes O.
        const bool done = mbar_wait(smem_u32(o_done), (j - 1) & 1);
        if (!__all_sync(0xffffffffu, done)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float ov[32];
            tmem_ld32(tO + lane_off + c * 32, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) ov[i] *= alpha;
            tmem_st32(tO + lane_off + c * 32, ov);
          }
          tmem_wait_st();
        }
      }
      if (kbase + kTcKv > seq_len) {
        // Last tile: V rows past the sequence end may hold never-written
        // cache slots (possibly NaN) and P = 0 does not cancel NaN.
        const bool landed = mbar_wait(smem_u32(&kv_full[j & 1]), (j >> 1) & 1);
        if (!__all_sync(0xffffffffu, landed)) {
          ok = false;
          break;
        }
        if (kbase + t >= seq_len) {
          uint8_t* vrow = smem + kTcStage0 + (j & 1) * kTcStageBytes + 2 * kTcHalf + t * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + kTcHalf + c * 16) = make_uint4(0, 0, 0, 0);
          }
        }
      }
      // P (16-bit) into shared memory, K-major, 128-byte swizzle
#pragma unroll
      for (int c = 0; c < 16; ++c)
        *reinterpret_cast<uint4*>(smem + kTcP + (c >> 3) * kTcHalf + swz128(t, c & 7)) =
            pack8_t<T>(&sv[c * 8]);
      fence_proxy_async_smem();
      tc_fence_before_sync();
      mbar_arrive(smem_u32(p_ready));
    }
    if (ok) {
      const bool done = mbar_wait(smem_u32(o_done), (n_tiles - 1) & 1);
      if (!__all_sync(0xffffffffu, done)) ok = false;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
    } else {
      tc_fence_after_sync();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.out) + (int64_t)(q_start + max(row_token, 0)) * p.out_token_stride +
                (int64_t)row_head * p.out_head_stride;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tO + lane_off + c * 32, ov);
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= inv_l;
        if (row_token >= 0) {
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            *reinterpret_cast<uint4*>(orow + c * 32 + q8 * 8) = pack8_t<T>(&ov[q8 * 8]);
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

template <typename T>
static cudaError_t launch_tc_typed(const CUtensorMap& mk, const CUtensorMap& mv,
                                   const PrefillParams& p, int num_kv_heads, int num_seqs,
                                   int max_q_len, cudaStream_t stream) {
  auto kernel = paged_prefill_tc_kernel<T>;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kTcSmemBytes);
  if (e != cudaSuccess) return e;
  const int tpc = kTcRows / p.group;
  const int blocks = (max_q_len + tpc - 1) / tpc;
  if (blocks <= 0) return cudaSuccess;
  dim3 grid(blocks, num_kv_heads, num_seqs);
  kernel<<<grid, kTcThreads, kTcSmemBytes, stream>>>(mk, mv, p);
  return cudaGetLastError();
}

cudaError_t launch_paged_prefill_tc(const CUtensorMap& mk, const CUtensorMap& mv,
                                    const PrefillParams& p, int dtype, int num_kv_heads,
                                    int num_seqs, int max_q_len, cudaStream_t stream) {
  if (dtype == B200_DTYPE_BFLOAT16)
    return launch_tc_typed<__nv_bfloat16>(mk, mv, p, num_kv_heads, num_seqs, max_q_len, stream);
  return launch_tc_typed<__half>(mk, mv, p, num_kv_heads, num_seqs, max_q_len, stream);
}

}  // namespace b200
