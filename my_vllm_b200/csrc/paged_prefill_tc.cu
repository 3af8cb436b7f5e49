// paged_prefill_tc.cu — paged prefill / chunked-prefill attention on the
// 5th-generation tensor cores (tcgen05 + TMEM) for sm_100a.
//
// Semantics (tests/test_attention_backend.py:660-699): sequence s has
// q_len = query_start_loc[s+1] - query_start_loc[s] new query tokens and
// seq_len = seq_lens[s] KV tokens in the paged cache (prefix-cache hits plus
// the new chunk, already appended). Query token i sits at KV position
// seq_len - q_len + i and attends to positions <= that one.
//
// Design (one CTA per (sequence, KV head, block of 256 packed rows)):
//   * A row is a (query token, q head of the GQA group) pair; the CTA's rows
//     form two UMMA M = 128 tiles, A and B, that share every K/V tile.
//   * warps 0-3 / 4-7: two softmax warpgroups, one per Q tile; thread t of a
//     group owns row t = TMEM lane t, so row max and row sum need no shuffles.
//     Q reaches shared memory (K-major, 128-byte swizzle) by TMA, issued by
//     the producer before its first K tile, when the GQA group divides 128
//     (then a tile's rows are one box of the q tensor; FP8 caches convert
//     the landed rows to fp16 in place); otherwise these warps stage it.
//     Either way an mbarrier hands it to the MMA warp, and K/V streaming
//     does not wait for it.
//   * warp 8: TMA producer streaming 128-token K and V tiles of the paged
//     cache (8 x 16-token sub-tiles, one lane each; page ids read from the
//     block table four tiles at a time, a group ahead) into separate rings: K
//     (3 stages) is released as soon as a tile's S MMAs retire and so runs two
//     tiles ahead; V (2 stages) is released after the PV MMAs.
//   * warp 9: allocates all 512 TMEM columns (S_A | O_A | S_B | O_B) and one
//     thread issues every tcgen05.mma. The order
//        PV_A(j), S_A(j+1), PV_B(j), S_B(j+1), PV_A(j+1), ...
//     keeps the tensor core on one tile's MMAs while the other warpgroup runs
//     its softmax (ping-pong), and because MMAs of one thread complete in
//     order, "S_X(j) done" also means "PV_X(j-1) done": the softmax may then
//     rescale O_X and overwrite S_X with P_X without further waits. P is
//     handed over in two 64-token halves, so the first four PV MMAs run while
//     the softmax still exponentiates the second half.
//   * S = Q K^T with A = Q, B = K both K-major from shared memory. The softmax
//     writes P (16-bit) over S in TMEM and O += P V reads A = P from tensor
//     memory and B = V N-major straight from the TMA tile.
//   * Online softmax in the exp2 domain with a lazy rescale: the running
//     maximum only moves when a tile's maximum exceeds it by more than 2^8, so
//     O (in TMEM) is rarely rescaled; O / l is independent of that choice.
//   * Epilogue: O / l packed to T; a tile whose rows all belong to the
//     sequence is written into its freed Q region and stored by TMA, other
//     tiles row by row.
//   * The bottom-right causal mask and the sequence end are applied in
//     registers; V rows past the sequence end are zeroed in shared memory
//     before the last PV MMAs (never-written cache slots may hold NaN).
//   * Every mbarrier wait is bounded; on a timeout the CTA reports
//     B200_STATUS_WAIT_TIMEOUT, drains its TMA loads and MMAs with bounded
//     waits, frees its tensor memory and exits.
//   * FP8 E4M3 caches (kFp8): the producer warp TMA-loads each 128-token K or
//     V tile as 16 KiB of FP8 into a 2-slot staging ring (one tile ahead)
//     and converts it, exactly, into the same fp16 K-major / N-major tile
//     layout the MMAs read (E4M3 values are all representable in fp16), then
//     signals the tile full. Q is converted to fp16 and P packed as fp16, so the
//     MMAs run kind::f16 on fp16 operands; the K scale folds into the softmax
//     scale and the V scale into the final normalisation. The K ring has 2
//     stages instead of 3 to make room for the staging ring.
#include <cuda_runtime.h>
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "paged_decode.cuh"
#include "paged_prefill.cuh"
#include "tcgen05.cuh"

namespace b200 {

constexpr int kTcRows = 128;   // UMMA M (rows of one Q tile)
constexpr int kTcTiles = 2;    // Q tiles per CTA
constexpr int kTcKv = 128;     // KV tokens per tile (N of QK^T, K of PV)
constexpr int kTcProducerWarp = 8;
constexpr int kTcMmaWarp = 9;
constexpr int kTcConvWarp0 = 10;  // FP8 only: warps 10 and 11 convert staged tiles
constexpr int kTcConvWarps = 2;
template <bool kFp8>
constexpr int tc_threads() { return (kFp8 ? 12 : 10) * 32; }
constexpr int kTcHalf = kTcRows * 128;          // [128 rows x 64 elements] = 16 KiB
constexpr int kTcQ = 0;                         // Q_A, Q_B: 2 x 32 KiB
constexpr int kTcTileBytes = 2 * kTcHalf;       // one K or V tile (lo/hi halves) = 32 KiB
constexpr int kTcVStages = 2;                   // V is freed after the PV MMAs
constexpr int kTcK0 = kTcTiles * kTcTileBytes;
constexpr int kTcRawTileBytes = kTcKv * 128;    // one FP8 K or V tile = 16 KiB
// Shared-memory map per cache type: Q_A | Q_B | K ring | V ring | [FP8 staging] | barriers.
// K is freed after the S MMAs, so a deeper ring lets it run further ahead.
template <bool kFp8>
struct TcLayout {
  static constexpr int kKStages = kFp8 ? 2 : 3;
  static constexpr int kV0 = kTcK0 + kKStages * kTcTileBytes;
  static constexpr int kRaw0 = kV0 + kTcVStages * kTcTileBytes;  // FP8 staging, 2 slots
  static constexpr int kBars = kRaw0 + (kFp8 ? 2 * kTcRawTileBytes : 0);
  static constexpr int kSmemBytes = 1024 + kBars + 256;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};
constexpr uint32_t kTcTmemCols = 512;           // per tile X: S_X at 256X, O_X at 256X+128
constexpr float kRescaleThreshold = 8.0f;       // log2 units

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return Elem<T>::pack(lo, hi);
}

// 16-bit pair of T -> fp16 pair (exact for fp16; bf16 values round to
// nearest fp16, exact for |x| in [2^-14, 65504] with <= 8 significant bits)
__device__ __forceinline__ uint32_t pair_to_f16(uint32_t w, __half) { return w; }
__device__ __forceinline__ uint32_t pair_to_f16(uint32_t w, __nv_bfloat16) {
  return Elem<__half>::pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Work units are (sequence, row block, KV head). A unit's cost is the number
// of 128-token KV tiles it streams, which grows with the sequence's cached
// prefix and, under the causal mask, with the row block. The 1-D grid lists
// the units longest first (ties by (sequence, row block) id, then KV head),
// so the hardware's in-order block dispatch is greedy longest-processing-
// time-first scheduling: without it, whole sequences with long prefixes can
// land in the last wave. Every CTA recomputes the same order from the
// metadata (no host sort, no workspace): a histogram of the (sequence,
// row block) costs, the cost bucket holding its grid position, then the
// position's rank inside that bucket in id order.
constexpr int kTcCostKeys = 2048;  // cost keys are clamped here: order only, never results

// Cost of row block rb of a sequence with q_len new tokens and seq_len keys.
__device__ __forceinline__ int tc_cost_of(const PrefillParams& p, int q_len, int seq_len, int rb) {
  const int tpc = (kTcTiles * kTcRows) / p.group;
  const int tok_begin = rb * tpc;
  if (tok_begin >= q_len || seq_len <= 0) return 0;
  const int last_tok = min(q_len - 1, tok_begin + (min(kTcTiles * kTcRows, tpc * p.group) - 1) /
                                                      p.group);
  const int kv_limit = min(seq_len, max(1, seq_len - q_len + last_tok + 1));
  return min((kv_limit + kTcKv - 1) / kTcKv, kTcCostKeys - 1);
}

__device__ __forceinline__ int tc_unit_cost(const PrefillParams& p, int s, int rb) {
  const int q_len = __ldg(p.query_start_loc + s + 1) - __ldg(p.query_start_loc + s);
  return tc_cost_of(p, q_len, __ldg(p.seq_lens + s), rb);
}

// Pair costs kept in shared memory by tc_decode_unit (beyond this many pairs
// the rank search recomputes them from the metadata).
constexpr int kTcCachedPairs = 8192;
// The histogram is padded by 4 ints after every 64 keys, so the 32 lanes that
// each sum one 64-key chunk with 16-byte loads spread over the banks.
constexpr int kTcHistInts = kTcCostKeys + kTcCostKeys / 16;
__device__ __forceinline__ int tc_hist_slot(int key) { return key + (key >> 6) * 4; }
// The persistent kernel also keeps (first query row, new tokens, keys) of the
// first kTcSeqCache sequences in its scratch, after the pair costs.
constexpr int kTcSeqCache = 1024;
constexpr int kTcScratchInts = kTcHistInts + 4 + kTcCachedPairs + 3 * kTcSeqCache;
static_assert(kTcScratchInts * 4 <= kTcTiles * 2 * kTcHalf, "scratch lives in the Q tiles");

// Histogram of the (sequence, row block) pair costs, plus a cache of the
// first kTcCachedPairs costs, in `scratch` (kTcScratchInts ints of 16-byte
// aligned shared memory). Call with all threads of the CTA.
__device__ __forceinline__ void tc_build_hist(const PrefillParams& p, int* scratch) {
  int* hist = scratch;                        // [kTcHistInts], key k at tc_hist_slot(k)
  int* cost = scratch + kTcHistInts + 4;      // [kTcCachedPairs]
  const int pairs = p.num_seqs * p.blocks_per_seq;
  for (int i = threadIdx.x; i < kTcHistInts / 4; i += blockDim.x)
    reinterpret_cast<int4*>(hist)[i] = make_int4(0, 0, 0, 0);
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int c = tc_unit_cost(p, i / p.blocks_per_seq, i % p.blocks_per_seq);
    if (i < kTcCachedPairs) cost[i] = c;
    atomicAdd(&hist[tc_hist_slot(c)], 1);
  }
  __syncthreads();
}

// The pair (sequence * blocks_per_seq + row block) at position `pair_pos` of
// the longest-first order (ties in id order), from the histogram that
// tc_build_hist left in `scratch`. Warp-collective; the result is the same
// in every lane.
__device__ __forceinline__ int tc_pair_at(const PrefillParams& p, const int* scratch,
                                          int pair_pos, int lane) {
  const int* hist = scratch;
  const int* cost = scratch + kTcHistInts + 4;
  const int pairs = p.num_seqs * p.blocks_per_seq;
  const unsigned full = 0xffffffffu;
  // Keys in descending order: lane l owns the chunk of keys
  // [2048 - 64(l+1), 2048 - 64l), so lower lanes hold larger costs.
  constexpr int kPerLane = kTcCostKeys / 32;
  const int chunk_lo = kTcCostKeys - kPerLane * (lane + 1);
  int chunk = 0;
#pragma unroll
  for (int k = 0; k < kPerLane / 4; ++k) {
    const int4 h = reinterpret_cast<const int4*>(hist + tc_hist_slot(chunk_lo))[k];
    chunk += (h.x + h.y) + (h.z + h.w);
  }
  // pairs in the chunks of lower lanes (larger keys): exclusive prefix sum
  int incl = chunk;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(full, incl, d);
    if (lane >= d) incl += v;
  }
  const unsigned own = __ballot_sync(full, pair_pos >= incl - chunk && pair_pos < incl);
  const int o = own ? __ffs(own) - 1 : 0;
  const int before_o = __shfl_sync(full, incl - chunk, o);
  // inside chunk o, lane l takes keys hi = top - 2l and hi - 1 (descending)
  const int hi = kTcCostKeys - 1 - kPerLane * o - 2 * lane;
  const int h0 = hist[tc_hist_slot(hi)], h1 = hist[tc_hist_slot(hi - 1)];
  int incl2 = h0 + h1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(full, incl2, d);
    if (lane >= d) incl2 += v;
  }
  const int first = before_o + incl2 - (h0 + h1);  // pairs before key hi
  int key = -1, rank = 0;
  if (pair_pos >= first && pair_pos < first + h0) {
    key = hi;
    rank = pair_pos - first;
  } else if (pair_pos >= first + h0 && pair_pos < first + h0 + h1) {
    key = hi - 1;
    rank = pair_pos - first - h0;
  }
  const unsigned owner = __ballot_sync(full, key >= 0);
  const int src = owner ? __ffs(owner) - 1 : 0;
  key = __shfl_sync(full, key, src);
  rank = __shfl_sync(full, rank, src);
  // the rank-th pair (in id order) whose cost key is `key`
  int found = 0;
  for (int base = 0; base < pairs; base += 32) {
    const int id = base + lane;
    int c = -1;
    if (id < pairs)
      c = id < kTcCachedPairs ? cost[id]
                              : tc_unit_cost(p, id / p.blocks_per_seq, id % p.blocks_per_seq);
    const unsigned m = __ballot_sync(full, c == key);
    const int n = __popc(m);
    if (rank < n) {
      unsigned mm = m;
      for (int r = 0; r < rank; ++r) mm &= mm - 1;  // drop the lower set bits
      found = base + __ffs(mm) - 1;
      break;
    }
    rank -= n;
  }
  return found;
}

// (sequence, row block, KV head) of grid position `pos`; `scratch` holds
// kTcScratchInts ints of 16-byte aligned shared memory. Call with all
// threads of the CTA. One round of metadata loads, then shared memory and
// shuffles only: the whole CTA waits on this before any load is issued.
__device__ __forceinline__ void tc_decode_unit(const PrefillParams& p, int pos, int* scratch,
                                               int& s, int& rb, int& kvh) {
  int* result = scratch + kTcHistInts;        // [2]
  tc_build_hist(p, scratch);
  if (threadIdx.x < 32) {
    const int found = tc_pair_at(p, scratch, pos / p.num_kv_heads, threadIdx.x);
    if (threadIdx.x == 0) {
      result[0] = found;
      result[1] = pos % p.num_kv_heads;
    }
  }
  __syncthreads();
  const int pair = result[0];
  kvh = result[1];
  s = pair / p.blocks_per_seq;
  rb = pair % p.blocks_per_seq;
  __syncthreads();  // scratch is reused as the Q tiles
}

// Page ids of the producer warp's 128-token KV tiles, read from the block
// table four tiles at a time (one page slot per lane) and a group ahead of
// use, so that no TMA issue waits on a dependent global load: lane l holds
// the page of sub-tile l % 8 of tile 4g + l / 8 of group g, even and odd
// groups in two registers. Indices past the sequence end read its last page.
struct TilePages {
  const int32_t* bt_row;
  int max_page_idx, block_size, lane;
  int even, odd;
  int g0 = 0;  // first group: tile g0 * 4 is the first the caller streams (KV parts)

  __device__ __forceinline__ int fetch(int g) const {
    const int tok = (g * 4 + (lane >> 3)) * kTcKv + (lane & 7) * kTileTokens;
    return __ldg(bt_row + min(tok / block_size, max_page_idx));
  }
  // g0 is warp-uniform: a branch, not a select, so no instruction waits on
  // the loads until a page id is used
  __device__ __forceinline__ void init() {
    if (g0 & 1) {
      odd = fetch(g0);
      even = fetch(g0 + 1);
    } else {
      even = fetch(g0);
      odd = fetch(g0 + 1);
    }
  }
  // Call before tile j's V load (the K loads run ahead, in tile j / 4 or
  // later): group j / 4 - 1 is dead, so group j / 4 + 1 takes its register.
  __device__ __forceinline__ void advance(int j) {
    if ((j & 3) != 0 || (j >> 2) <= g0) return;
    const int g = j / 4 + 1;
    if (g & 1)
      odd = fetch(g);
    else
      even = fetch(g);
  }
  // Page of sub-tile `lane % 8` of tile j (warp-collective).
  __device__ __forceinline__ int page(int j) const {
    return __shfl_sync(0xffffffffu, ((j >> 2) & 1) ? odd : even, (j & 3) * 8 + (lane & 7));
  }
};

template <typename T, bool kFp8>
__global__ void __launch_bounds__(tc_threads<kFp8>(), 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_k,
                            const __grid_constant__ CUtensorMap tmap_v,
                            const __grid_constant__ CUtensorMap tmap_q,
                            const __grid_constant__ CUtensorMap tmap_o,
                            const PrefillParams p) {
  using L = TcLayout<kFp8>;
  using M = typename std::conditional<kFp8, __half, T>::type;  // MMA operand type
  constexpr int kTcKStages = L::kKStages;
  constexpr int kTcV0 = L::kV0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* k_full = bars + 0;     // [<=3] TMA (FP8: the converter) -> MMA
  uint64_t* k_empty = bars + 3;    // [<=3] MMA (commit after the S MMAs) -> TMA
  uint64_t* v_full = bars + 6;     // [2] TMA -> MMA
  uint64_t* v_empty = bars + 8;    // [2] MMA (commit after the PV MMAs) -> TMA
  uint64_t* s_full = bars + 10;    // [2] per Q tile: MMA (commit) -> softmax
  uint64_t* p_ready = bars + 12;   // [2] per Q tile: P tokens 0-63 written (128 arrivals) -> MMA
  uint64_t* o_done = bars + 14;    // [2] per Q tile: MMA (commit) -> epilogue
  uint64_t* mma_drain = bars + 16; // MMA (commit) -> MMA, before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  uint64_t* raw_full = bars + 18;   // [2] FP8 staging: TMA -> converter warps
  uint64_t* raw_empty = bars + 20;  // [2] FP8 staging: converter warps -> TMA
  uint64_t* q_full = bars + 22;     // Q staged (TMA bytes, or 256 softmax arrivals) -> MMA
  uint64_t* p_ready_hi = bars + 23; // [2] per Q tile: P tokens 64-127 written -> MMA
  uint64_t* q_raw = bars + 25;      // FP8 caches: 16-bit Q landed by TMA -> softmax warps
  uint64_t* o_staged = bars + 26;   // [2] per Q tile (128 arrivals): output rows in smem

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int s, rb, kvh;
  tc_decode_unit(p, blockIdx.x, reinterpret_cast<int*>(smem + kTcQ), s, rb, kvh);

  const int q_start = p.query_start_loc[s];
  const int q_len = p.query_start_loc[s + 1] - q_start;
  const int seq_len = p.seq_lens[s];
  const int group = p.group;
  const int tpc = (kTcTiles * kTcRows) / group;  // query tokens per CTA
  const int tok_begin = rb * tpc;
  if (tok_begin >= q_len || seq_len <= 0) return;  // CTA-uniform, before any sync
  const int ctx = seq_len - q_len;

  // KV tiles each Q tile needs: up to its last valid row's causal limit.
  auto tiles_for = [&](int x) {
    const int first_row = x * kTcRows;
    if (first_row / group >= tpc || tok_begin + first_row / group >= q_len) return 0;
    const int last_row = min((x + 1) * kTcRows, tpc * group) - 1;
    const int last_tok = min(q_len - 1, tok_begin + last_row / group);
    const int kv_limit = min(seq_len, max(1, ctx + last_tok + 1));
    return (kv_limit + kTcKv - 1) / kTcKv;
  };
  const int n_a = tiles_for(0);
  const int n_b = tiles_for(1);
  const int n_total = max(n_a, n_b);  // tiles the producer streams

  const uint32_t sbase = smem_u32(smem);
  if (threadIdx.x == 0) {
    // FP8: a K/V tile is full when both converter warps have written their rows
    const uint32_t fills = kFp8 ? kTcConvWarps : 1;
    for (int i = 0; i < kTcKStages; ++i) {
      mbar_init(smem_u32(&k_full[i]), fills);
      mbar_init(smem_u32(&k_empty[i]), 1);
    }
    for (int i = 0; i < kTcVStages; ++i) {
      mbar_init(smem_u32(&v_full[i]), fills);
      mbar_init(smem_u32(&v_empty[i]), 1);
    }
    for (int x = 0; x < kTcTiles; ++x) {
      mbar_init(smem_u32(&s_full[x]), 1);
      mbar_init(smem_u32(&p_ready[x]), kTcRows);
      mbar_init(smem_u32(&p_ready_hi[x]), kTcRows);
      mbar_init(smem_u32(&o_done[x]), 1);
    }
    mbar_init(smem_u32(mma_drain), 1);
    // 16-bit caches: the Q TMA bytes complete q_full; FP8 caches: the softmax
    // warps' 256 arrivals do, after converting (a TMA-landed) Q to fp16
    mbar_init(smem_u32(q_full), (p.q_tma && !kFp8) ? 1 : 2 * kTcRows);
    mbar_init(smem_u32(q_raw), 1);
    for (int x = 0; x < kTcTiles; ++x) mbar_init(smem_u32(&o_staged[x]), kTcRows);
    if (kFp8) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(smem_u32(&raw_full[i]), 1);
        mbar_init(smem_u32(&raw_empty[i]), kTcConvWarps);
      }
    }
    mbar_init_fence();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }

  // Barriers and the TMEM address are visible after this; the producer
  // starts streaming K/V while the softmax warps still stage Q.
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();

  // ---- softmax warps: this thread's row and its Q into shared memory ----
  const int x_tile = warp >> 2;       // Q tile of a softmax warp (0 or 1)
  const int t = threadIdx.x & 127;    // row within the Q tile = TMEM lane
  int row_token = -1, row_head = 0, qpos = -1;
  if (warp < 8) {
    const int r = x_tile * kTcRows + t;  // rows are (token, q head of the group) pairs
    const int tl = r / group;
    if (tl < tpc && tok_begin + tl < q_len) {
      row_token = tok_begin + tl;
      row_head = kvh * group + (r - tl * group);
      qpos = ctx + row_token;
    }
  }
  if (kFp8 && warp < 8 && p.q_tma) {
    // FP8 caches run the MMAs on fp16 operands: convert this row of the
    // TMA-landed 16-bit Q in place (same size, same swizzled positions)
    if (!mbar_wait(smem_u32(q_raw), 0) && lane == 0)
      report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
    uint8_t* qtile = smem + kTcQ + x_tile * 2 * kTcHalf;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4* ptr = reinterpret_cast<uint4*>(qtile + (c >> 3) * kTcHalf + swz128(t, c & 7));
      uint4 v = *ptr;
      v.x = pair_to_f16(v.x, T());
      v.y = pair_to_f16(v.y, T());
      v.z = pair_to_f16(v.z, T());
      v.w = pair_to_f16(v.w, T());
      *ptr = v;
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(q_full));
  }
  if (warp < 8 && !p.q_tma) {
    const uint4* src = reinterpret_cast<const uint4*>(
        reinterpret_cast<const T*>(p.q) + (int64_t)(q_start + max(row_token, 0)) * p.q_token_stride +
        (int64_t)row_head * p.q_head_stride);
    uint8_t* qtile = smem + kTcQ + x_tile * 2 * kTcHalf;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      uint4 v = row_token >= 0 ? __ldg(src + c) : make_uint4(0, 0, 0, 0);
      if (kFp8) {  // the MMAs run on fp16 operands
        v.x = pair_to_f16(v.x, T());
        v.y = pair_to_f16(v.y, T());
        v.z = pair_to_f16(v.z, T());
        v.w = pair_to_f16(v.w, T());
      }
      *reinterpret_cast<uint4*>(qtile + (c >> 3) * kTcHalf + swz128(t, c & 7)) = v;
    }
    // generic-proxy writes -> the MMAs' async-proxy reads, then hand off
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(q_full));
  }
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  // FP8 items in the 16-bit producer's order: K0, K1, then (V_m, K_{m+2}),
  // then the last V tiles. Item i is TMA-loaded into staging slot i % 2 by
  // the producer warp and converted into its fp16 K or V stage by warps 10-11.
  const int k_first = min(2, n_total);
  const int kv_pairs = max(0, n_total - 2);
  auto item_at = [&](int i, bool& is_v, int& j) {
    if (i < k_first) {
      is_v = false;
      j = i;
    } else if (i - k_first < 2 * kv_pairs) {
      const int m = i - k_first;
      is_v = (m & 1) == 0;
      j = is_v ? m / 2 : m / 2 + 2;
    } else {
      is_v = true;
      j = kv_pairs + (i - k_first - 2 * kv_pairs);
    }
  };
  const int n_items = 2 * n_total;

  // Q by TMA (producer lane 0): per tile and d half one box of group heads x
  // 128 / group tokens, which is the tile's 128 (token, head) rows in order;
  // tokens past the query's end load the next sequence's rows or zeros, and
  // those rows are never written out.
  auto load_q = [&](uint64_t* bar) {
    const int tpt = kTcRows / group;
    mbar_arrive_expect_tx(smem_u32(bar), kTcTiles * kTcTileBytes);
    for (int x = 0; x < kTcTiles; ++x)
      for (int h = 0; h < 2; ++h)
        tma_load_3d(sbase + kTcQ + x * kTcTileBytes + h * kTcHalf, &tmap_q, smem_u32(bar),
                    h * 64, kvh * group, q_start + tok_begin + x * tpt);
  };
  if (warp == kTcProducerWarp && kFp8) {
    // ------------------------------------------------------- FP8 producer --
    if (p.q_tma && lane == 0) load_q(q_raw);
    __syncwarp();
    const int max_page_idx = (seq_len - 1) / p.block_size;
    TilePages pages{p.block_tables + (int64_t)s * p.block_table_stride, max_page_idx,
                    p.block_size, lane, 0, 0};
    pages.init();
    const uint32_t raw0 = sbase + L::kRaw0;
    int issued = 0;
    for (int i = 0; i < n_items && ok; ++i) {
      if (i >= 2) {  // slot i % 2 is free once both converters have read item i - 2
        const bool got = mbar_wait(smem_u32(&raw_empty[i & 1]), ((i >> 1) - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
      }
      bool is_v;
      int j;
      item_at(i, is_v, j);
      if (is_v) pages.advance(j);
      const uint32_t bar = smem_u32(&raw_full[i & 1]);
      if (lane == 0) mbar_arrive_expect_tx(bar, kTcRawTileBytes);
      __syncwarp();
      const int page = pages.page(j);
      if (lane < kTcKv / kTileTokens) {
        const int tok = j * kTcKv + lane * kTileTokens;
        // past the sequence end: the last page (any valid one), masked later
        const int row = tok / p.block_size > max_page_idx ? 0 : tok % p.block_size;
        if (page < 0 || page >= p.num_blocks)
          report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
        tma_load_4d(raw0 + (i & 1) * kTcRawTileBytes + lane * kFp8TileBytes,
                    is_v ? &tmap_v : &tmap_k, bar, 0, kvh, row, page);
      }
      issued = i + 1;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      for (int i = max(0, issued - 2); i < issued; ++i)  // loads still in flight
        mbar_wait(smem_u32(&raw_full[i & 1]), (i >> 1) & 1);
    }
  } else if (kFp8 && warp >= kTcConvWarp0) {
    // ----------------------------------------------- FP8 converter warps --
    // Warp 10 converts rows 0-63 of every staged tile, warp 11 rows 64-127:
    // chunk c of a row (E4M3 d = 16c .. 16c + 15) -> fp16 chunks 2c', 2c'+1
    // of half c / 4 (c' = c % 4), all 128-byte swizzled like the TMA tiles.
    const int row0 = (warp - kTcConvWarp0) * (kTcKv / kTcConvWarps);
    const int c = lane & 7;
    const int h = c >> 2;
    const int c2 = (c & 3) * 2;
    for (int i = 0; i < n_items; ++i) {
      bool is_v;
      int j;
      item_at(i, is_v, j);
      const int nst = is_v ? kTcVStages : kTcKStages;
      const int st = j % nst;
      bool got = true;
      if (j >= nst)  // the fp16 stage is free once the MMAs that read it retired
        got = mbar_wait(smem_u32(&(is_v ? v_empty : k_empty)[st]), ((j / nst) - 1) & 1);
      if (got) got = mbar_wait(smem_u32(&raw_full[i & 1]), (i >> 1) & 1);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const uint8_t* raw = smem + L::kRaw0 + (i & 1) * kTcRawTileBytes;
      uint8_t* dst = smem + (is_v ? kTcV0 : kTcK0) + st * kTcTileBytes + h * kTcHalf;
#pragma unroll 4
      for (int it = 0; it < kTcKv / kTcConvWarps / 4; ++it) {
        const int r = row0 + it * 4 + (lane >> 3);
        const uint4 w = *reinterpret_cast<const uint4*>(raw + swz128(r, c));
        uint4 lo, hi;
        e4m3x4_to_f16(w.x, lo.x, lo.y);
        e4m3x4_to_f16(w.y, lo.z, lo.w);
        e4m3x4_to_f16(w.z, hi.x, hi.y);
        e4m3x4_to_f16(w.w, hi.z, hi.w);
        *reinterpret_cast<uint4*>(dst + swz128(r, c2)) = lo;
        *reinterpret_cast<uint4*>(dst + swz128(r, c2 + 1)) = hi;
      }
      // generic-proxy reads of the staging slot (refilled by TMA) and writes
      // of the fp16 tile (read by the MMAs) -> async proxy, then hand off
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&raw_empty[i & 1]));
        mbar_arrive(smem_u32(is_v ? &v_full[st] : &k_full[st]));
      }
    }
    if (!ok && lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
  } else if (warp == kTcProducerWarp) {
    // ------------------------------------------------------------ producer --
    // Issue order K0, K1, then (V_j, K_{j+2}) for j = 0, 1, ...: K runs two
    // tiles ahead (its stage frees as soon as the S MMAs of a tile retire),
    // V one to two tiles ahead.
    const int max_page_idx = (seq_len - 1) / p.block_size;
    TilePages pages{p.block_tables + (int64_t)s * p.block_table_stride, max_page_idx,
                    p.block_size, lane, 0, 0};
    pages.init();
    int issued_k = 0, issued_v = 0;
    auto load = [&](bool is_v, int j) -> bool {
      const int nst = is_v ? kTcVStages : kTcKStages;
      const int st = j % nst;
      uint64_t* empty = is_v ? v_empty : k_empty;
      if (j >= nst) {
        const bool got = mbar_wait(smem_u32(&empty[st]), ((j / nst) - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) return false;
      }
      const uint32_t bar = smem_u32(is_v ? &v_full[st] : &k_full[st]);
      if (lane == 0) mbar_arrive_expect_tx(bar, kTcTileBytes);
      __syncwarp();
      const int page = pages.page(j);
      if (lane < kTcKv / kTileTokens) {
        const int tok = j * kTcKv + lane * kTileTokens;
        // past the sequence end: the last page (any valid one), masked later
        const int row = tok / p.block_size > max_page_idx ? 0 : tok % p.block_size;
        if (page < 0 || page >= p.num_blocks)
          report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
        const uint32_t dst =
            sbase + (is_v ? kTcV0 : kTcK0) + st * kTcTileBytes + lane * kHalfTileBytes;
        const CUtensorMap* map = is_v ? &tmap_v : &tmap_k;
        tma_load_4d(dst, map, bar, 0, kvh, row, page);
        tma_load_4d(dst + kTcHalf, map, bar, 64, kvh, row, page);
      }
      if (is_v) issued_v = j + 1; else issued_k = j + 1;
      return true;
    };
    if (p.q_tma && lane == 0) load_q(q_full);
    __syncwarp();
    for (int j = 0; j < min(2, n_total) && ok; ++j) ok = load(false, j);
    for (int j = 0; j < n_total && ok; ++j) {
      pages.advance(j);
      ok = load(true, j);
      if (ok && j + 2 < n_total) ok = load(false, j + 2);
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      for (int j = max(0, issued_k - kTcKStages); j < issued_k; ++j)
        mbar_wait(smem_u32(&k_full[j % kTcKStages]), (j / kTcKStages) & 1);
      for (int j = max(0, issued_v - kTcVStages); j < issued_v; ++j)
        mbar_wait(smem_u32(&v_full[j % kTcVStages]), (j / kTcVStages) & 1);
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr bool kBf16 = Elem<M>::kDtype == B200_DTYPE_BFLOAT16;
      const uint32_t idesc_s = f16_instr_desc(kTcRows, kTcKv, kBf16, false);
      const uint32_t idesc_pv = f16_instr_desc(kTcRows, kHeadDim, kBf16, true);
      auto kmajor = [&](uint32_t addr, int k) {  // K-major, 16-element k-step k
        return smem_desc(addr + (k >> 2) * kTcHalf + (k & 3) * 32, 16, 1024);
      };
      auto issue_s = [&](int x, int j) {
        const uint32_t qbase = sbase + kTcQ + x * 2 * kTcHalf;
        const uint32_t kbase = sbase + kTcK0 + (j % kTcKStages) * kTcTileBytes;
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k)
          umma_f16(tmem_base + x * 256, kmajor(qbase, k), kmajor(kbase, k), idesc_s,
                   k > 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[x]));
      };
      // PV k-steps [k0, k0 + 4): the 64 KV tokens of one half of P
      auto issue_pv = [&](int x, int j, int k0) {
        const uint32_t vbase = sbase + kTcV0 + (j % kTcVStages) * kTcTileBytes;
        const uint32_t tP = tmem_base + x * 256;  // P (16-bit, packed) over S
#pragma unroll
        for (int k = k0; k < k0 + kTcKv / 32; ++k)
          umma_f16_ts(tmem_base + x * 256 + 128, tP + k * 8,
                      smem_desc(vbase + k * 16 * 128, kTcHalf, 1024), idesc_pv,
                      (j > 0 || k > 0) ? 1u : 0u);
      };
      // K/V tiles arrive through the async proxy (TMA, or the FP8 converters'
      // proxy fence before their arrival): the mbarrier wait alone orders the
      // MMAs' shared-memory reads after them, no tcgen05 fence.
      int k_ready = -1, v_ready = -1;  // highest tiles whose full phase was observed
      auto wait_k = [&](int j) {
        if (j <= k_ready) return true;
        if (!mbar_wait(smem_u32(&k_full[j % kTcKStages]), (j / kTcKStages) & 1)) return false;
        k_ready = j;
        return true;
      };
      auto wait_v = [&](int j) {
        if (j <= v_ready) return true;
        if (!mbar_wait(smem_u32(&v_full[j % kTcVStages]), (j / kTcVStages) & 1)) return false;
        v_ready = j;
        return true;
      };
      // One Q tile's step j: PV of tile j, then S of tile j + 1.
      auto step = [&](int x, int n_x, int j) {
        if (j >= n_x) return true;
        if (!mbar_wait(smem_u32(&p_ready[x]), j & 1)) return false;
        tc_fence_after_sync();
        if (!wait_v(j)) return false;
        issue_pv(x, j, 0);
        if (!mbar_wait(smem_u32(&p_ready_hi[x]), j & 1)) return false;
        tc_fence_after_sync();
        issue_pv(x, j, kTcKv / 32);
        if (j == n_x - 1) umma_commit(smem_u32(&o_done[x]));
        if (j + 1 < n_x) {
          if (!wait_k(j + 1)) return false;
          issue_s(x, j + 1);
        }
        return true;
      };
      // prologue: S of tile 0 for both Q tiles, once Q is staged
      if (!mbar_wait(smem_u32(q_full), 0)) ok = false;
      if (ok && !wait_k(0)) ok = false;
      if (ok && n_a > 0) issue_s(0, 0);
      if (ok && n_b > 0) issue_s(1, 0);
      if (ok) umma_commit(smem_u32(&k_empty[0]));  // after every S of tile 0
      for (int j = 0; j < n_total && ok; ++j) {
        if (!step(0, n_a, j) || !step(1, n_b, j)) {
          ok = false;
          break;
        }
        umma_commit(smem_u32(&v_empty[j % kTcVStages]));  // after every PV of tile j
        if (j + 1 < n_total)
          umma_commit(smem_u32(&k_empty[(j + 1) % kTcKStages]));  // every S of tile j+1
      }
      if (!ok) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(smem_u32(mma_drain));
      mbar_wait(smem_u32(mma_drain), 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------- softmax warps --
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + x_tile * 256 + lane_off;
    const uint32_t tO = tS + 128;
    const int my_tiles = x_tile ? n_b : n_a;
    const float kNegInf = -INFINITY;
    float m_used = kNegInf, l = 0.f;
    float scale = p.scale_log2;  // FP8: times the K dequantisation scale
    float out_scale = 1.f;       // FP8: the V dequantisation scale
    if (kFp8) {
      if (p.k_scale != nullptr) scale *= __ldg(p.k_scale);
      if (p.v_scale != nullptr) out_scale = __ldg(p.v_scale);
    }
    for (int j = 0; j < my_tiles; ++j) {
      const bool got = mbar_wait(smem_u32(&s_full[x_tile]), j & 1);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      // S_X(j) done implies PV_X(j-1) done (in-order MMAs): O_X is stable and
      // the P_X(j-1) columns may be overwritten. Two passes over the row in
      // 32-column chunks (max, then exp2 + pack) keep register use low enough
      // for 10 warps per SM; independent accumulators keep the few warps per
      // SM sub-partition busy instead of waiting on one dependency chain.
      const int kbase = j * kTcKv;
      // columns [0, lim) of this tile are visible to this row
      const int lim = min(qpos - kbase + 1, seq_len - kbase);
      const bool need_mask = lim < kTcKv;
      float mk[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mk[k] = kNegInf;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float sv[64];
        tmem_ld64(tS + c * 64, sv);
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            mk[i & 7] = fmaxf(mk[i & 7], c * 64 + i < lim ? sv[i] : kNegInf);
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) mk[i & 7] = fmaxf(mk[i & 7], sv[i]);
        }
      }
      // the softmax scale is positive, so it commutes with the maximum
      const float m_raw = fmaxf(fmaxf(fmaxf(mk[0], mk[1]), fmaxf(mk[2], mk[3])),
                                fmaxf(fmaxf(mk[4], mk[5]), fmaxf(mk[6], mk[7])));
      const float m_tile = m_raw == kNegInf ? kNegInf : m_raw * scale;
      float alpha = 1.f;
      bool rescale = false;
      if (m_tile > m_used + kRescaleThreshold) {
        alpha = fast_exp2(m_used - m_tile);
        m_used = m_tile;
        rescale = true;
      }
      // O_X is stable (S_X(j) done implies PV_X(j-1) done): rescale it before
      // any of P_X(j) is handed to the PV MMAs.
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tO + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(tO + c * 32, ov);
        }
      }
      if (kbase + kTcKv > seq_len) {
        // Last KV tile: V rows past the sequence end may hold never-written
        // cache slots (possibly NaN) and P = 0 does not cancel NaN. Both
        // warpgroups write the same zeros, each before its own PV.
        const bool landed = mbar_wait(smem_u32(&v_full[j % kTcVStages]), (j / kTcVStages) & 1);
        if (!__all_sync(0xffffffffu, landed)) {
          ok = false;
          break;
        }
        if (kbase + t >= seq_len) {
          uint8_t* vrow = smem + kTcV0 + (j % kTcVStages) * kTcTileBytes + t * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + kTcHalf + c * 16) = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
      }
      const float neg_base = m_used == kNegInf ? 0.f : -m_used;
      // exponent arguments and row sums two columns at a time (f32x2); each
      // 64-token half of P is handed to the MMA warp as soon as it is written
      const uint64_t scale2 = f2(scale, scale), base2 = f2(neg_base, neg_base);
      uint64_t sk2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float sv[32];
        tmem_ld32(tS + c * 32, sv);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0, x1;
          f2_split(f2_fma(f2(sv[2 * i], sv[2 * i + 1]), scale2, base2), x0, x1);
          float p0 = ex2_approx(x0);
          float p1 = ex2_approx(x1);
          if (need_mask) {
            p0 = c * 32 + 2 * i < lim ? p0 : 0.f;
            p1 = c * 32 + 2 * i + 1 < lim ? p1 : 0.f;
          }
          sk2[i & 1] = f2_add(sk2[i & 1], f2(p0, p1));
          pk[i] = pack2<M>(p0, p1);
        }
        // P over S: chunk c's 32 values -> 16 columns at 16c, which only
        // overlap S columns this row has already read
        tmem_st16(tS + c * 16, pk);
        if (c == 1 || c == 3) {
          tmem_wait_st();
          tc_fence_before_sync();
          mbar_arrive(smem_u32(c == 1 ? &p_ready[x_tile] : &p_ready_hi[x_tile]));
        }
      }
      float s0, s1, s2, s3;
      f2_split(sk2[0], s0, s1);
      f2_split(sk2[1], s2, s3);
      const float sum = (s0 + s1) + (s2 + s3);
      l = l * alpha + sum;
    }
    if (ok && my_tiles > 0) {
      const bool done = mbar_wait(smem_u32(&o_done[x_tile]), 0);
      if (!__all_sync(0xffffffffu, done)) ok = false;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
    } else if (my_tiles > 0) {
      tc_fence_after_sync();
      const float inv_l = l > 0.f ? out_scale / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.out) +
                (int64_t)(q_start + max(row_token, 0)) * p.out_token_stride +
                (int64_t)row_head * p.out_head_stride;
      // the row's 128 O columns in four loads under one wait (the softmax
      // registers are free by now)
      uint32_t ob[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_issue(tO + c * 32, ob[c]);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_wait_ld32(ob[c]);
      // A tile whose 128 rows all belong to the sequence (group divides 128)
      // is one box of the out tensor: its rows go to the tile's Q region
      // (free: every MMA of this tile has completed) in the 128-byte swizzled
      // layout, and one thread stores the box with TMA. Other tiles, whose
      // trailing rows would fall on the next sequence, store row by row.
      const int tpt = kTcRows / group;
      const bool box_out = p.o_tma && tok_begin + (x_tile + 1) * tpt <= q_len;
      uint8_t* otile = smem + kTcQ + x_tile * kTcTileBytes;
      if (box_out || row_token >= 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float* ov = reinterpret_cast<const float*>(ob[c]);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 pk;
            pk.x = pack2<T>(ov[q8 * 8 + 0] * inv_l, ov[q8 * 8 + 1] * inv_l);
            pk.y = pack2<T>(ov[q8 * 8 + 2] * inv_l, ov[q8 * 8 + 3] * inv_l);
            pk.z = pack2<T>(ov[q8 * 8 + 4] * inv_l, ov[q8 * 8 + 5] * inv_l);
            pk.w = pack2<T>(ov[q8 * 8 + 6] * inv_l, ov[q8 * 8 + 7] * inv_l);
            const int chunk = c * 4 + q8;  // 16-byte chunk of the 256-byte row
            if (box_out)
              *reinterpret_cast<uint4*>(otile + (chunk >> 3) * kTcHalf + swz128(t, chunk & 7)) = pk;
            else
              *reinterpret_cast<uint4*>(orow + c * 32 + q8 * 8) = pk;
          }
        }
      }
      if (box_out) {
        fence_proxy_async_smem();  // generic writes -> the TMA's async-proxy reads
        mbar_arrive(smem_u32(&o_staged[x_tile]));
        if (t == 0) {
          if (mbar_wait(smem_u32(&o_staged[x_tile]), 0)) {
            const int tok0 = q_start + tok_begin + x_tile * tpt;
            tma_store_3d(&tmap_o, smem_u32(otile), 0, kvh * group, tok0);
            tma_store_3d(&tmap_o, smem_u32(otile + kTcHalf), 64, kvh * group, tok0);
            bulk_commit_group();
            bulk_wait_group_all();  // shared memory is read and out written before exit
          } else {
            report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Persistent variant (16-bit caches, Q by TMA): one CTA per SM walks a list
// of units instead of one CTA per unit. The per-CTA work of the one-unit
// kernel — tensor-memory allocation, barrier set-up, the unit decode, the
// first Q/K/V loads, the last MMAs' drain and the epilogue — was a fixed
// cost of about 10 us per unit, paid again for every short unit; here it is
// paid once per CTA, and a unit's tail overlaps the next unit's start:
//   * the producer loads the next unit's Q as soon as the current unit's
//     last S MMAs have retired (q_empty), then keeps streaming K/V tiles of
//     the next unit into the same rings (global stage counters);
//   * the MMA warp issues the next unit's first S MMAs right after the
//     current unit's last PV MMAs; before a Q tile's first PV MMA of a new
//     unit it waits until that tile's epilogue has read O (o_free);
//   * the softmax warps write a tile's output rows (epilogue) while the
//     tensor core already computes the next unit's scores.
// The units are the one-unit kernel's (sequence, row block, KV head), dealt
// to the CTAs from the longest-first order in snake order: position
// r * G + c on even rounds r and r * G + (G - 1 - c) on odd rounds for CTA c
// of G, so a CTA that drew a long unit in one round draws a short one in the
// next. Each CTA decodes its whole list once, before it starts.
constexpr int kTcMaxUnitsPerCta = 64;
// per list entry: item id, record base, ticket | parts << 24, and the
// sequence's first query row, new tokens and keys (read at set-up, so that no
// role waits on a global load when it moves to its next unit: under the
// streaming of every SM one such round trip took microseconds)
constexpr int kTcUnitInts = 6;
constexpr int kTcPersistSmem =
    TcLayout<false>::kSmemBytes + kTcMaxUnitsPerCta * kTcUnitInts * 4;  // + the unit list
static_assert(kTcPersistSmem <= 227 * 1024, "shared memory budget");
// Split-KV: a unit of more than twice the launch's average work per SM is cut
// into at most kTcMaxParts KV parts of at least kTcMinPartTiles tiles each
// (a unit only a little above the average gains less than its merge costs).
constexpr int kTcMaxParts = 8;
constexpr int kTcMinPartTiles = 4;
// A part record per Q tile is column-major, [130][128 rows]: O columns 0-127,
// then m, then l, so a warp's rows are consecutive floats (coalesced).
constexpr int kTcRecordFloats = 130 * kTcRows;

__device__ __forceinline__ int tc_snake_pos(int k, int cta, int grid) {
  return k * grid + ((k & 1) ? grid - 1 - cta : cta);
}

// KV parts of a unit of `cost` tiles under the split target (0: no split).
__device__ __forceinline__ int tc_parts(int cost, int target) {
  if (target <= 0 || cost <= 2 * target) return 1;
  return min(kTcMaxParts, (cost + target - 1) / target);
}

__device__ __forceinline__ int tc_cached_cost(const PrefillParams& p, const int* cost, int id) {
  return id < kTcCachedPairs ? cost[id] : tc_unit_cost(p, id / p.blocks_per_seq, id % p.blocks_per_seq);
}

// The launch's split target, the same in every CTA: the average work per SM
// (every unit's KV tiles / SMs, at least kTcMinPartTiles), raised until the
// split units' parts fit the workspace's records; 0 without a workspace.
// Then the histogram of item cost keys: a unit of cost c in P parts is P
// items of key ceil(c / P); the number of items is left in scratch int
// kTcHistInts + 3. Call with all threads of the CTA; `scratch` as for
// tc_build_hist (its 4 result ints serve as reduction slots).
__device__ __forceinline__ int tc_build_split_hist(const PrefillParams& p, int* scratch) {
  int* hist = scratch;
  int* red = scratch + kTcHistInts;  // [0] total tiles, [1] split parts, [2] split pairs, [3] items
  int* cost = scratch + kTcHistInts + 4;
  int* seqc = cost + kTcCachedPairs;  // [kTcSeqCache][3]
  const int pairs = p.num_seqs * p.blocks_per_seq;
  for (int s = threadIdx.x; s < min(p.num_seqs, kTcSeqCache); s += blockDim.x) {
    const int q0 = __ldg(p.query_start_loc + s);
    seqc[3 * s] = q0;
    seqc[3 * s + 1] = __ldg(p.query_start_loc + s + 1) - q0;
    seqc[3 * s + 2] = __ldg(p.seq_lens + s);
  }
  for (int i = threadIdx.x; i < kTcHistInts / 4; i += blockDim.x)
    reinterpret_cast<int4*>(hist)[i] = make_int4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    red[0] = 0;
    red[3] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int s = i / p.blocks_per_seq;
    const int c = s < kTcSeqCache ? tc_cost_of(p, seqc[3 * s + 1], seqc[3 * s + 2], i % p.blocks_per_seq)
                                  : tc_unit_cost(p, s, i % p.blocks_per_seq);
    if (i < kTcCachedPairs) cost[i] = c;
    atomicAdd(&red[0], c);
  }
  __syncthreads();
  int target = 0;
  if (p.split_cap > 0 && p.num_sms > 0) {
    const int64_t total = (int64_t)red[0] * p.num_kv_heads;
    const int64_t avg = (total + p.num_sms - 1) / p.num_sms;
    const bool one_wave = (int64_t)pairs * p.num_kv_heads <= p.num_sms;
    target = avg > kTcMinPartTiles ? (int)avg : kTcMinPartTiles;
    for (int round = 0; round < 64; ++round) {
      __syncthreads();
      if (threadIdx.x == 0) {
        red[1] = 0;
        red[2] = 0;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
        const int parts = tc_parts(tc_cached_cost(p, cost, i), target);
        if (parts > 1) {
          atomicAdd(&red[1], parts);
          atomicAdd(&red[2], 1);  // split pairs
        }
      }
      __syncthreads();
      // the parts fit the records, and when every unit has its own SM the
      // items still do (a part in a second wave costs more than it saves)
      const int64_t items = (int64_t)(pairs + red[1] - red[2]) * p.num_kv_heads;
      if ((int64_t)red[1] * p.num_kv_heads <= p.split_cap && (!one_wave || items <= p.num_sms))
        break;
      target += target / 4 + 1;
    }
    const int64_t items = (int64_t)(pairs + red[1] - red[2]) * p.num_kv_heads;
    if ((int64_t)red[1] * p.num_kv_heads > p.split_cap || (one_wave && items > p.num_sms))
      target = 0;  // never split then
  }
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int c = tc_cached_cost(p, cost, i);
    const int parts = tc_parts(c, target);
    atomicAdd(&hist[tc_hist_slot((c + parts - 1) / parts)], parts);
    atomicAdd(&red[3], parts);  // items
  }
  __syncthreads();
  return target;
}

// The item (pair, part) at position `item_pos` of the longest-first item
// order (ties by pair id, then part), from tc_build_split_hist's histogram.
// Warp-collective; the result is the same in every lane.
__device__ __forceinline__ void tc_item_at(const PrefillParams& p, const int* scratch, int target,
                                           int item_pos, int lane, int& pair, int& part) {
  const int* hist = scratch;
  const int* cost = scratch + kTcHistInts + 4;
  const int pairs = p.num_seqs * p.blocks_per_seq;
  const unsigned full = 0xffffffffu;
  constexpr int kPerLane = kTcCostKeys / 32;
  const int chunk_lo = kTcCostKeys - kPerLane * (lane + 1);
  int chunk = 0;
#pragma unroll
  for (int k = 0; k < kPerLane / 4; ++k) {
    const int4 h = reinterpret_cast<const int4*>(hist + tc_hist_slot(chunk_lo))[k];
    chunk += (h.x + h.y) + (h.z + h.w);
  }
  int incl = chunk;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(full, incl, d);
    if (lane >= d) incl += v;
  }
  const unsigned own = __ballot_sync(full, item_pos >= incl - chunk && item_pos < incl);
  const int o = own ? __ffs(own) - 1 : 0;
  const int before_o = __shfl_sync(full, incl - chunk, o);
  const int hi = kTcCostKeys - 1 - kPerLane * o - 2 * lane;
  const int h0 = hist[tc_hist_slot(hi)], h1 = hist[tc_hist_slot(hi - 1)];
  int incl2 = h0 + h1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int v = __shfl_up_sync(full, incl2, d);
    if (lane >= d) incl2 += v;
  }
  const int first = before_o + incl2 - (h0 + h1);
  int key = -1, rank = 0;
  if (item_pos >= first && item_pos < first + h0) {
    key = hi;
    rank = item_pos - first;
  } else if (item_pos >= first + h0 && item_pos < first + h0 + h1) {
    key = hi - 1;
    rank = item_pos - first - h0;
  }
  const unsigned owner = __ballot_sync(full, key >= 0);
  const int src = owner ? __ffs(owner) - 1 : 0;
  key = __shfl_sync(full, key, src);
  rank = __shfl_sync(full, rank, src);
  // the rank-th item of key `key`: pairs in id order, each with its parts
  pair = 0;
  part = 0;
  for (int base = 0; base < pairs; base += 32) {
    const int id = base + lane;
    int w = 0;
    if (id < pairs) {
      const int c = tc_cached_cost(p, cost, id);
      const int parts = tc_parts(c, target);
      w = (c + parts - 1) / parts == key ? parts : 0;
    }
    int wincl = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(full, wincl, d);
      if (lane >= d) wincl += v;
    }
    const int chunk_items = __shfl_sync(full, wincl, 31);
    if (rank < chunk_items) {
      const unsigned hit = __ballot_sync(full, wincl > rank);
      const int l = __ffs(hit) - 1;
      pair = base + l;
      part = rank - (__shfl_sync(full, wincl, l) - __shfl_sync(full, w, l));
      break;
    }
    rank -= chunk_items;
  }
}

// For a split pair: (split pairs, their parts) before it in id order.
// Warp-collective.
__device__ __forceinline__ void tc_split_prefix(const PrefillParams& p, const int* scratch,
                                                int target, int pair, int lane, int& n_before,
                                                int& parts_before) {
  const int* cost = scratch + kTcHistInts + 4;
  n_before = 0;
  parts_before = 0;
  for (int base = 0; base < pair; base += 32) {
    const int id = base + lane;
    int parts = 1;
    if (id < pair) parts = tc_parts(tc_cached_cost(p, cost, id), target);
    int a = (id < pair && parts > 1) ? 1 : 0;
    int b = a ? parts : 0;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, d);
      b += __shfl_xor_sync(0xffffffffu, b, d);
    }
    n_before += a;
    parts_before += b;
  }
}

struct TcUnit {
  int s, kvh, q_start, q_len, seq_len, ctx, tok_begin, n_a, n_b, n_total;
  // KV part: tiles [lo, lo + n) of the unit's n_total; parts == 1 unless split
  int part, parts, lo, n, rec, ticket;
};

// Everything a role needs about list entry `e` (item id = (pair *
// num_kv_heads + KV head) * kTcMaxParts + part, record base, ticket | parts
// << 24, the sequence's metadata), from shared memory only; n = 0 for a row
// block past the sequence's chunk.
__device__ __forceinline__ TcUnit tc_unit(const PrefillParams& p, const int* e) {
  TcUnit u;
  const int id = e[0];
  u.part = id % kTcMaxParts;
  const int unit = id / kTcMaxParts;
  const int pair = unit / p.num_kv_heads;
  u.kvh = unit - pair * p.num_kv_heads;
  u.rec = e[1];
  u.ticket = e[2] & 0xffffff;
  u.parts = e[2] >> 24;
  u.s = pair / p.blocks_per_seq;
  const int rb = pair - u.s * p.blocks_per_seq;
  u.q_start = e[3];
  u.q_len = e[4];
  u.seq_len = e[5];
  u.ctx = u.seq_len - u.q_len;
  const int tpc = (kTcTiles * kTcRows) / p.group;
  u.tok_begin = rb * tpc;
  u.n_a = u.n_b = u.n_total = 0;
  u.lo = u.n = 0;
  if (u.tok_begin >= u.q_len || u.seq_len <= 0) return u;
  int n[kTcTiles];
#pragma unroll
  for (int x = 0; x < kTcTiles; ++x) {
    n[x] = 0;
    const int first_row = x * kTcRows;
    if (first_row / p.group >= tpc || u.tok_begin + first_row / p.group >= u.q_len) continue;
    const int last_row = min((x + 1) * kTcRows, tpc * p.group) - 1;
    const int last_tok = min(u.q_len - 1, u.tok_begin + last_row / p.group);
    const int kv_limit = min(u.seq_len, max(1, u.ctx + last_tok + 1));
    n[x] = (kv_limit + kTcKv - 1) / kTcKv;
  }
  u.n_total = max(n[0], n[1]);
  // part `part` of `parts`: tiles [part * n / parts, (part + 1) * n / parts),
  // never empty because parts <= n
  u.lo = u.part * u.n_total / u.parts;
  const int hi = (u.part + 1) * u.n_total / u.parts;
  u.n = hi - u.lo;
  // this part's tiles of each Q tile (a Q tile with fewer tiles may have none)
  u.n_a = max(0, min(hi, n[0]) - u.lo);
  u.n_b = max(0, min(hi, n[1]) - u.lo);
  return u;
}

template <typename T>
__global__ void __launch_bounds__(tc_threads<false>(), 1)
    paged_prefill_tc_persistent_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                       const __grid_constant__ CUtensorMap tmap_v,
                                       const __grid_constant__ CUtensorMap tmap_q,
                                       const PrefillParams p) {
  using L = TcLayout<false>;
  constexpr int kKSt = L::kKStages;
  constexpr int kTcV0 = L::kV0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* k_full = bars + 0;      // [3] TMA -> MMA
  uint64_t* k_empty = bars + 3;     // [3] MMA (commit after the S MMAs) -> TMA
  uint64_t* v_full = bars + 6;      // [2] TMA -> MMA
  uint64_t* v_empty = bars + 8;     // [2] MMA (commit after the PV MMAs) -> TMA
  uint64_t* s_full = bars + 10;     // [2] per Q tile: MMA (commit) -> softmax
  uint64_t* p_ready = bars + 12;    // [2] per Q tile: P tokens 0-63 written -> MMA
  uint64_t* o_done = bars + 14;     // [2] per Q tile: a unit's last PV retired -> epilogue
  uint64_t* mma_drain = bars + 16;  // MMA (commit) -> MMA, before TMEM is freed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  uint64_t* q_full = bars + 18;     // a unit's Q landed (TMA bytes) -> MMA
  uint64_t* p_ready_hi = bars + 19; // [2] per Q tile: P tokens 64-127 written -> MMA
  uint64_t* q_empty = bars + 21;    // a unit's last S MMAs retired -> producer (next Q)
  uint64_t* o_free = bars + 22;     // [2] per Q tile: epilogue read O (128 arrivals) -> MMA
  uint64_t* pv0_done = bars + 24;   // [2] per Q tile: a tile's first-half PV MMAs retired
  uint64_t* merge_bar = bars + 26;  // [2] per Q tile: split records written / ticket known
  int* merge_ticket = reinterpret_cast<int*>(bars + 28);  // [2] per Q tile
  int* units = reinterpret_cast<int*>(bars + 32);  // [kTcMaxUnitsPerCta][kTcUnitInts]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- this CTA's unit list, from the longest-first order (Q region as scratch) ----
  int* scratch = reinterpret_cast<int*>(smem + kTcQ);
  const int target = tc_build_split_hist(p, scratch);
  const int total = scratch[kTcHistInts + 3] * p.num_kv_heads;  // items x KV heads
  int n_units = 0;
  while (n_units < kTcMaxUnitsPerCta && tc_snake_pos(n_units, blockIdx.x, gridDim.x) < total)
    ++n_units;
  const int n_warps = blockDim.x / 32;
  const int* seqc = scratch + kTcHistInts + 4 + kTcCachedPairs;
  // the producer decodes unit 0, so it can fetch that unit's first page ids
  // while the barriers and tensor memory are set up
  for (int k = (warp + n_warps - kTcProducerWarp) % n_warps; k < n_units; k += n_warps) {
    const int pos = tc_snake_pos(k, blockIdx.x, gridDim.x);
    const int kvh = pos % p.num_kv_heads;
    int pair, part;
    tc_item_at(p, scratch, target, pos / p.num_kv_heads, lane, pair, part);
    const int parts =
        tc_parts(tc_cached_cost(p, scratch + kTcHistInts + 4, pair), target);
    int n_before = 0, parts_before = 0;
    if (parts > 1) tc_split_prefix(p, scratch, target, pair, lane, n_before, parts_before);
    if (lane == 0) {
      int* e = units + k * kTcUnitInts;
      e[0] = (pair * p.num_kv_heads + kvh) * kTcMaxParts + part;
      e[1] = parts_before * p.num_kv_heads + kvh * parts;           // first record of the unit
      e[2] = (n_before * p.num_kv_heads + kvh) | (parts << 24);     // its ticket, parts
      const int s = pair / p.blocks_per_seq;
      if (s < kTcSeqCache) {
        e[3] = seqc[3 * s];
        e[4] = seqc[3 * s + 1];
        e[5] = seqc[3 * s + 2];
      } else {
        e[3] = __ldg(p.query_start_loc + s);
        e[4] = __ldg(p.query_start_loc + s + 1) - e[3];
        e[5] = __ldg(p.seq_lens + s);
      }
    }
  }
  // producer: unit 0 and the page ids of its first two tile groups (the loads
  // stay in flight across the set-up below)
  __syncwarp();
  TcUnit pu{};
  TilePages ppages{};
  if (warp == kTcProducerWarp && n_units > 0) {
    pu = tc_unit(p, units);
    if (pu.n > 0) {
      ppages = TilePages{p.block_tables + (int64_t)pu.s * p.block_table_stride,
                         (pu.seq_len - 1) / p.block_size, p.block_size, lane, 0, 0, pu.lo >> 2};
      ppages.init();
    }
  }

  const uint32_t sbase = smem_u32(smem);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kKSt; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
    }
    for (int i = 0; i < kTcVStages; ++i) {
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_empty[i]), 1);
    }
    for (int x = 0; x < kTcTiles; ++x) {
      mbar_init(smem_u32(&s_full[x]), 1);
      mbar_init(smem_u32(&p_ready[x]), kTcRows);
      mbar_init(smem_u32(&p_ready_hi[x]), kTcRows);
      mbar_init(smem_u32(&o_done[x]), 1);
      mbar_init(smem_u32(&o_free[x]), kTcRows);
      mbar_init(smem_u32(&pv0_done[x]), 1);
      mbar_init(smem_u32(&merge_bar[x]), kTcRows);
    }
    mbar_init(smem_u32(mma_drain), 1);
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);
    mbar_init_fence();
  }
  if (warp == kTcMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }
  // the unit list, barriers and TMEM address are visible after this; the
  // scratch (Q region) is free for the first unit's Q
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  bool ok = true;

  if (warp == kTcProducerWarp) {
    // ------------------------------------------------------------ producer --
    // Per unit: its Q (once the previous unit's S MMAs retired), then K0, K1,
    // (V_j, K_{j+2}) ... as in the one-unit kernel; stages and phases count
    // the K and V tiles of all units in order. The next unit's first page ids
    // are read when a unit starts, a whole unit ahead of their use.
    int issued_k = 0, issued_v = 0, units_q = 0;
    int gk = 0, gv = 0;  // first global K / V tile index of the current unit
    TcUnit U = pu;
    TilePages pages = ppages;
    for (int k = 0; k < n_units && ok; ++k) {
      TcUnit un{};
      TilePages next_pages{};
      if (k + 1 < n_units) {
        un = tc_unit(p, units + (k + 1) * kTcUnitInts);
        if (un.n > 0) {
          next_pages = TilePages{p.block_tables + (int64_t)un.s * p.block_table_stride,
                                 (un.seq_len - 1) / p.block_size, p.block_size, lane, 0, 0,
                                 un.lo >> 2};
          next_pages.init();
        }
      }
      if (U.n == 0) {
        U = un;
        pages = next_pages;
        continue;
      }
      const int max_page_idx = (U.seq_len - 1) / p.block_size;
      // jj: tile of this part (0 .. n - 1); the unit's tile is U.lo + jj
      auto load = [&](bool is_v, int jj) -> bool {
        const int g = (is_v ? gv : gk) + jj;
        const int j = U.lo + jj;
        const int nst = is_v ? kTcVStages : kKSt;
        const int st = g % nst;
        uint64_t* empty = is_v ? v_empty : k_empty;
        if (g >= nst) {
          const bool got = mbar_wait(smem_u32(&empty[st]), ((g / nst) - 1) & 1);
          if (!__all_sync(0xffffffffu, got)) return false;
        }
        const uint32_t bar = smem_u32(is_v ? &v_full[st] : &k_full[st]);
        if (lane == 0) mbar_arrive_expect_tx(bar, kTcTileBytes);
        __syncwarp();
        const int page = pages.page(j);
        if (lane < kTcKv / kTileTokens) {
          const int tok = j * kTcKv + lane * kTileTokens;
          // past the sequence end: the last page (any valid one), masked later
          const int row = tok / p.block_size > max_page_idx ? 0 : tok % p.block_size;
          if (page < 0 || page >= p.num_blocks)
            report_status(p.status, B200_STATUS_PAGE_OUT_OF_RANGE);
          const uint32_t dst =
              sbase + (is_v ? kTcV0 : kTcK0) + st * kTcTileBytes + lane * kHalfTileBytes;
          const CUtensorMap* map = is_v ? &tmap_v : &tmap_k;
          tma_load_4d(dst, map, bar, 0, U.kvh, row, page);
          tma_load_4d(dst + kTcHalf, map, bar, 64, U.kvh, row, page);
        }
        if (is_v) issued_v = g + 1; else issued_k = g + 1;
        return true;
      };
      // the Q tiles are free once every S MMA of the previous unit retired
      if (units_q > 0) {
        const bool got = mbar_wait(smem_u32(q_empty), (units_q - 1) & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
      }
      if (lane == 0) {
        // per tile and d half one box of group heads x 128 / group tokens,
        // which is the tile's 128 (token, head) rows in order
        const int tpt = kTcRows / p.group;
        mbar_arrive_expect_tx(smem_u32(q_full), kTcTiles * kTcTileBytes);
        for (int x = 0; x < kTcTiles; ++x)
          for (int h = 0; h < 2; ++h)
            tma_load_3d(sbase + kTcQ + x * kTcTileBytes + h * kTcHalf, &tmap_q,
                        smem_u32(q_full), h * 64, U.kvh * p.group,
                        U.q_start + U.tok_begin + x * tpt);
      }
      __syncwarp();
      ++units_q;
      const int n = U.n;
      for (int jj = 0; jj < min(2, n) && ok; ++jj) ok = load(false, jj);
      for (int jj = 0; jj < n && ok; ++jj) {
        pages.advance(U.lo + jj);
        ok = load(true, jj);
        if (ok && jj + 2 < n) ok = load(false, jj + 2);
      }
      gk += n;
      gv += n;
      U = un;
      pages = next_pages;
    }
    if (!ok) {
      if (lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      // loads still in flight land before the CTA exits (bounded waits)
      for (int g = max(0, issued_k - kKSt); g < issued_k; ++g)
        mbar_wait(smem_u32(&k_full[g % kKSt]), (g / kKSt) & 1);
      for (int g = max(0, issued_v - kTcVStages); g < issued_v; ++g)
        mbar_wait(smem_u32(&v_full[g % kTcVStages]), (g / kTcVStages) & 1);
      if (units_q > 0) mbar_wait(smem_u32(q_full), (units_q - 1) & 1);
    }
  } else if (warp == kTcMmaWarp) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr bool kBf16 = Elem<T>::kDtype == B200_DTYPE_BFLOAT16;
      const uint32_t idesc_s = f16_instr_desc(kTcRows, kTcKv, kBf16, false);
      const uint32_t idesc_pv = f16_instr_desc(kTcRows, kHeadDim, kBf16, true);
      // Shared-memory descriptors are built once: a k-step or a ring stage
      // only moves the start-address field (bits 0-13, address / 16, no carry
      // below 256 KiB), so each MMA adds a constant to a precomputed base
      // instead of rebuilding the descriptor (the single issuing thread is
      // the pipeline's serial resource).
      uint64_t qdesc[kTcTiles], kdesc[kKSt], vdesc[kTcVStages];
#pragma unroll
      for (int x = 0; x < kTcTiles; ++x) qdesc[x] = smem_desc(sbase + kTcQ + x * 2 * kTcHalf, 16, 1024);
#pragma unroll
      for (int st = 0; st < kKSt; ++st) kdesc[st] = smem_desc(sbase + kTcK0 + st * kTcTileBytes, 16, 1024);
#pragma unroll
      for (int st = 0; st < kTcVStages; ++st)
        vdesc[st] = smem_desc(sbase + kTcV0 + st * kTcTileBytes, kTcHalf, 1024);
      // K-major operand, 16-element k-step k: (k / 4) 64-element halves + (k % 4) 32-byte steps
      auto kstep = [](int k) -> uint64_t {
        return static_cast<uint64_t>(((k >> 2) * kTcHalf + (k & 3) * 32) >> 4);
      };
      auto issue_s = [&](int x, int g) {  // S_X = Q_X K(g)^T
        const uint64_t kd = kdesc[g % kKSt];
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k)
          umma_f16(tmem_base + x * 256, qdesc[x] + kstep(k), kd + kstep(k), idesc_s,
                   k > 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[x]));
      };
      // O_X (+)= P_X V(g), k-steps [k0, k0 + 4): the 64 KV tokens of one half of P
      auto issue_pv = [&](int x, int g, int k0, bool first_of_unit) {
        const uint64_t vd = vdesc[g % kTcVStages];
        const uint32_t tP = tmem_base + x * 256;  // P (16-bit, packed) over S
#pragma unroll
        for (int k = k0; k < k0 + kTcKv / 32; ++k)
          umma_f16_ts(tmem_base + x * 256 + 128, tP + k * 8,
                      vd + static_cast<uint64_t>((k * 16 * 128) >> 4), idesc_pv,
                      (!first_of_unit || k > 0) ? 1u : 0u);
      };
      int k_ready = -1, v_ready = -1;  // highest global tiles whose full phase was observed
      auto wait_k = [&](int g) {
        if (g <= k_ready) return true;
        if (!mbar_wait(smem_u32(&k_full[g % kKSt]), (g / kKSt) & 1)) return false;
        k_ready = g;
        return true;
      };
      auto wait_v = [&](int g) {
        if (g <= v_ready) return true;
        if (!mbar_wait(smem_u32(&v_full[g % kTcVStages]), (g / kTcVStages) & 1)) return false;
        v_ready = g;
        return true;
      };
      int gk = 0, gv = 0, units_q = 0;
      int ts[kTcTiles] = {0, 0};  // tile steps per Q tile (s_full / p_ready phases)
      int ep[kTcTiles] = {0, 0};  // units with rows per Q tile (o_done / o_free phases)
      for (int k = 0; k < n_units && ok; ++k) {
        const TcUnit U = tc_unit(p, units + k * kTcUnitInts);
        if (U.n == 0) continue;
        const int nx[kTcTiles] = {U.n_a, U.n_b};  // this part's tiles per Q tile
        const int n = U.n;
        // S of tile 0 for both Q tiles, once this unit's Q landed
        if (!mbar_wait(smem_u32(q_full), units_q & 1) || !wait_k(gk)) {
          ok = false;
          break;
        }
        ++units_q;
        for (int x = 0; x < kTcTiles; ++x)
          if (nx[x] > 0) issue_s(x, gk);
        umma_commit(smem_u32(&k_empty[gk % kKSt]));  // after every S of tile 0
        if (n == 1) umma_commit(smem_u32(q_empty));   // the unit's last S MMAs
        for (int j = 0; j < n && ok; ++j) {
          for (int x = 0; x < kTcTiles && ok; ++x) {
            if (j >= nx[x]) continue;
            if (!mbar_wait(smem_u32(&p_ready[x]), ts[x] & 1)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            if (j == 0 && ep[x] > 0) {
              // the first PV of a unit overwrites O_X: the previous unit's
              // epilogue must have read it
              if (!mbar_wait(smem_u32(&o_free[x]), (ep[x] - 1) & 1)) {
                ok = false;
                break;
              }
              tc_fence_after_sync();
            }
            if (!wait_v(gv + j)) {
              ok = false;
              break;
            }
            issue_pv(x, gv + j, 0, j == 0);
            umma_commit(smem_u32(&pv0_done[x]));  // for a softmax that must rescale O
            if (!mbar_wait(smem_u32(&p_ready_hi[x]), ts[x] & 1)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            issue_pv(x, gv + j, kTcKv / 32, false);
            if (j == nx[x] - 1) umma_commit(smem_u32(&o_done[x]));
            if (j + 1 < nx[x]) {
              if (!wait_k(gk + j + 1)) {
                ok = false;
                break;
              }
              issue_s(x, gk + j + 1);
            }
            ++ts[x];
          }
          if (!ok) break;
          umma_commit(smem_u32(&v_empty[(gv + j) % kTcVStages]));  // after every PV of tile j
          if (j + 1 < n) umma_commit(smem_u32(&k_empty[(gk + j + 1) % kKSt]));
          if (j + 2 == n) umma_commit(smem_u32(q_empty));  // S of the last tile issued above
        }
        for (int x = 0; x < kTcTiles; ++x) ep[x] += nx[x] > 0 ? 1 : 0;
        gk += n;
        gv += n;
      }
      if (!ok) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
      // every MMA this thread issued has completed before TMEM is released
      umma_commit(smem_u32(mma_drain));
      mbar_wait(smem_u32(mma_drain), 0);
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------- softmax warps --
    const int x_tile = warp >> 2;       // Q tile of this warpgroup
    const int t = threadIdx.x & 127;    // row within the Q tile = TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + x_tile * 256 + lane_off;
    const uint32_t tO = tS + 128;
    const float kNegInf = -INFINITY;
    const float scale = p.scale_log2;
    const int group = p.group;
    const int tpc = (kTcTiles * kTcRows) / group;
    int ts = 0, ep = 0, gv = 0, mp = 0;
    for (int k = 0; k < n_units && ok; ++k) {
      const TcUnit U = tc_unit(p, units + k * kTcUnitInts);
      const int my_tiles = x_tile ? U.n_b : U.n_a;  // this part's tiles of this Q tile
      // a Q tile with no tiles in a part of a split unit still hands in an
      // (empty) record and takes its ticket
      if (my_tiles == 0 && U.parts == 1) {
        gv += U.n;
        continue;
      }
      const int seq_len = U.seq_len;
      int row_token = -1, row_head = 0, qpos = -1;
      {
        const int r = x_tile * kTcRows + t;  // rows are (token, q head of the group) pairs
        const int tl = r / group;
        if (tl < tpc && U.tok_begin + tl < U.q_len) {
          row_token = U.tok_begin + tl;
          row_head = U.kvh * group + (r - tl * group);
          qpos = U.ctx + row_token;
        }
      }
      float m_used = kNegInf, l = 0.f;
      // P of the 64 columns [64h, 64h + 64) with exponent base -neg_base:
      // packed 16-bit pairs, their sum and the raw maximum of the visible scores
      auto exp_half = [&](auto masked, int h, float neg_base, int lim, uint32_t (&pk)[2][16],
                          float& sum, float& mraw) {
        constexpr bool kMasked = decltype(masked)::value;
        const uint64_t scale2 = f2(scale, scale), base2 = f2(neg_base, neg_base);
        uint64_t sk2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
        float mk[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = 2 * h + cc;
          float sv[32];
          tmem_ld32(tS + c * 32, sv);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const bool v0 = !kMasked || c * 32 + 2 * i < lim;
            const bool v1 = !kMasked || c * 32 + 2 * i + 1 < lim;
            mk[(2 * i) & 3] = fmaxf(mk[(2 * i) & 3], v0 ? sv[2 * i] : kNegInf);
            mk[(2 * i + 1) & 3] = fmaxf(mk[(2 * i + 1) & 3], v1 ? sv[2 * i + 1] : kNegInf);
            float x0, x1;
            f2_split(f2_fma(f2(sv[2 * i], sv[2 * i + 1]), scale2, base2), x0, x1);
            float p0 = ex2_approx(x0);
            float p1 = ex2_approx(x1);
            if (kMasked) {
              p0 = v0 ? p0 : 0.f;
              p1 = v1 ? p1 : 0.f;
            }
            sk2[i & 1] = f2_add(sk2[i & 1], f2(p0, p1));
            pk[cc][i] = pack2<T>(p0, p1);
          }
        }
        float s0, s1, s2, s3;
        f2_split(sk2[0], s0, s1);
        f2_split(sk2[1], s2, s3);
        sum = (s0 + s1) + (s2 + s3);
        mraw = fmaxf(fmaxf(mk[0], mk[1]), fmaxf(mk[2], mk[3]));
      };
      auto rescale_o = [&](float a) {  // warp-collective; a = 1 leaves a row as it is
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tO + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= a;
          tmem_st32(tO + c * 32, ov);
        }
      };
      for (int j = 0; j < my_tiles; ++j) {
        const bool got = mbar_wait(smem_u32(&s_full[x_tile]), ts & 1);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        tc_fence_after_sync();
        const int kbase = (U.lo + j) * kTcKv;  // j counts this part's tiles
        // columns [0, lim) of this tile are visible to this row
        const int lim = min(qpos - kbase + 1, seq_len - kbase);
        const bool need_mask = lim < kTcKv;
        // exp_half holds warp-collective tensor-memory loads: the masked or
        // unmasked variant is chosen for the whole warp (a row without a mask
        // has lim >= 128, so masking leaves it unchanged)
        const bool warp_mask = __any_sync(0xffffffffu, need_mask);
        if (kbase + kTcKv > seq_len) {
          // Last KV tile: V rows past the sequence end may hold never-written
          // cache slots (possibly NaN) and P = 0 does not cancel NaN. Both
          // warpgroups write the same zeros, each before its own PV.
          const int g = gv + j;
          const bool landed = mbar_wait(smem_u32(&v_full[g % kTcVStages]), (g / kTcVStages) & 1);
          if (!__all_sync(0xffffffffu, landed)) {
            ok = false;
            break;
          }
          if (kbase + t >= seq_len) {
            uint8_t* vrow = smem + kTcV0 + (g % kTcVStages) * kTcTileBytes + t * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0, 0, 0, 0);
              *reinterpret_cast<uint4*>(vrow + kTcHalf + c * 16) = make_uint4(0, 0, 0, 0);
            }
          }
          fence_proxy_async_smem();
        }
        if (j == 0) {
          // ---- a unit's first tile: the exact maximum first (there is no
          // running base yet), then the exponentials ----
          float mk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mk[i] = kNegInf;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            float sv[64];
            tmem_ld64(tS + c * 64, sv);
            if (need_mask) {
#pragma unroll
              for (int i = 0; i < 64; ++i)
                mk[i & 7] = fmaxf(mk[i & 7], c * 64 + i < lim ? sv[i] : kNegInf);
            } else {
#pragma unroll
              for (int i = 0; i < 64; ++i) mk[i & 7] = fmaxf(mk[i & 7], sv[i]);
            }
          }
          // the softmax scale is positive, so it commutes with the maximum
          const float m_raw = fmaxf(fmaxf(fmaxf(mk[0], mk[1]), fmaxf(mk[2], mk[3])),
                                    fmaxf(fmaxf(mk[4], mk[5]), fmaxf(mk[6], mk[7])));
          m_used = m_raw == kNegInf ? kNegInf : m_raw * scale;
          const float nb = m_used == kNegInf ? 0.f : -m_used;
          float tile_sum = 0.f;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t pk[2][16];
            float sh, mr;
            if (warp_mask) exp_half(std::true_type{}, h, nb, lim, pk, sh, mr);
            else exp_half(std::false_type{}, h, nb, lim, pk, sh, mr);
            tile_sum += sh;
            // P over S: the half's 64 values -> 32 columns at 32h, which only
            // overlap S columns this row has already read
            tmem_st16(tS + (2 * h) * 16, pk[0]);
            tmem_st16(tS + (2 * h + 1) * 16, pk[1]);
            tmem_wait_st();
            tc_fence_before_sync();
            mbar_arrive(smem_u32(h == 0 ? &p_ready[x_tile] : &p_ready_hi[x_tile]));
          }
          l = tile_sum;
        } else {
          // ---- later tiles: one pass with the running base, keeping each
          // half's maximum; only a half whose maximum exceeds the base by
          // more than the threshold (rare) is done again with a new base ----
          float tile_sum = 0.f;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t pk[2][16];
            float sh, mr;
            const float nb = m_used == kNegInf ? 0.f : -m_used;
            if (warp_mask) exp_half(std::true_type{}, h, nb, lim, pk, sh, mr);
            else exp_half(std::false_type{}, h, nb, lim, pk, sh, mr);
            const float mh = mr == kNegInf ? kNegInf : mr * scale;
            const bool need = mh > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, need)) {
              const float m_new = need ? mh : m_used;
              const float a = need ? fast_exp2(m_used - m_new) : 1.f;
              if (h == 1) {
                // half 0 of this tile is with the MMA warp: O must hold it
                // before it is rescaled
                const bool got0 = mbar_wait(smem_u32(&pv0_done[x_tile]), ts & 1);
                if (!__all_sync(0xffffffffu, got0)) {
                  ok = false;
                  break;
                }
                tc_fence_after_sync();
              }
              // O_X holds every earlier contribution (S_X(j) done implies
              // PV_X(j-1) done; for h = 1 also half 0 of this tile)
              rescale_o(a);
              l *= a;
              tile_sum *= a;
              m_used = m_new;
              const float nb2 = m_used == kNegInf ? 0.f : -m_used;
              if (warp_mask) exp_half(std::true_type{}, h, nb2, lim, pk, sh, mr);
              else exp_half(std::false_type{}, h, nb2, lim, pk, sh, mr);
            }
            tile_sum += sh;
            tmem_st16(tS + (2 * h) * 16, pk[0]);
            tmem_st16(tS + (2 * h + 1) * 16, pk[1]);
            tmem_wait_st();
            tc_fence_before_sync();
            mbar_arrive(smem_u32(h == 0 ? &p_ready[x_tile] : &p_ready_hi[x_tile]));
          }
          if (!ok) break;
          l += tile_sum;
        }
        ++ts;
      }
      if (!ok) break;
      if (U.parts > 1) {
        // ---- split unit: this part's record (O, m, l per row); the part
        // that takes the last ticket merges every part into the output ----
        const int64_t part_floats = (int64_t)kTcTiles * kTcRecordFloats;
        float* rec0 = p.split_records + (int64_t)U.rec * part_floats +
                      (int64_t)x_tile * kTcRecordFloats + t;  // this row of part 0
        float* rec = rec0 + (int64_t)U.part * part_floats;
        if (my_tiles > 0) {
          const bool done = mbar_wait(smem_u32(&o_done[x_tile]), ep & 1);
          if (!__all_sync(0xffffffffu, done)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t ob[2][32];
            tmem_ld32_issue(tO + h * 64, ob[0]);
            tmem_ld32_issue(tO + h * 64 + 32, ob[1]);
            tmem_wait_ld32(ob[0]);
            tmem_wait_ld32(ob[1]);
#pragma unroll
            for (int c = 0; c < 2; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i)
                rec[(h * 64 + c * 32 + i) * kTcRows] = __uint_as_float(ob[c][i]);
          }
          tc_fence_before_sync();
          mbar_arrive(smem_u32(&o_free[x_tile]));
          ++ep;
        }
        rec[128 * kTcRows] = my_tiles > 0 ? m_used : kNegInf;
        rec[129 * kTcRows] = my_tiles > 0 ? l : 0.f;
        __threadfence();  // the record is visible before the ticket is taken
        mbar_arrive(smem_u32(&merge_bar[x_tile]));
        bool got = mbar_wait(smem_u32(&merge_bar[x_tile]), mp & 1);
        ++mp;
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (t == 0)
          merge_ticket[x_tile] = atomicAdd(p.split_tickets + U.ticket * kTcTiles + x_tile, 1);
        mbar_arrive(smem_u32(&merge_bar[x_tile]));
        got = mbar_wait(smem_u32(&merge_bar[x_tile]), mp & 1);
        ++mp;
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        // the last part puts the ticket back to 0: a launch leaves its tickets
        // as it found them (zero), so none is cleared before a launch
        if (t == 0 && merge_ticket[x_tile] == U.parts - 1)
          p.split_tickets[U.ticket * kTcTiles + x_tile] = 0;
        if (merge_ticket[x_tile] == U.parts - 1 && row_token >= 0) {
          __threadfence();  // every other part's record, seen through L2
          // Every load below is issued for all parts at once (parts past
          // U.parts read part 0 and get weight 0), so the merge costs a few
          // L2 round trips instead of one per part and column chunk.
          float w[kTcMaxParts], lq[kTcMaxParts];
#pragma unroll
          for (int q = 0; q < kTcMaxParts; ++q) {
            const float* src = rec0 + (q < U.parts ? q : 0) * part_floats;
            w[q] = __ldcg(src + 128 * kTcRows);
            lq[q] = __ldcg(src + 129 * kTcRows);
          }
          float m = kNegInf;
#pragma unroll
          for (int q = 0; q < kTcMaxParts; ++q)
            if (q < U.parts) m = fmaxf(m, w[q]);
          float lsum = 0.f;
#pragma unroll
          for (int q = 0; q < kTcMaxParts; ++q) {
            // a part that saw no key of the row (m = -inf), or no part, weighs 0
            w[q] = (q < U.parts && w[q] != kNegInf) ? fast_exp2(w[q] - m) : 0.f;
            lsum += w[q] > 0.f ? w[q] * lq[q] : 0.f;
          }
          const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
          uint4* orow = reinterpret_cast<uint4*>(
              reinterpret_cast<T*>(p.out) + (int64_t)(U.q_start + row_token) * p.out_token_stride +
              (int64_t)row_head * p.out_head_stride);
#pragma unroll 1
          for (int c8 = 0; c8 < kHeadDim / 8; ++c8) {
            float v[kTcMaxParts][8];
#pragma unroll
            for (int q = 0; q < kTcMaxParts; ++q) {
              const float* src = rec0 + (q < U.parts ? q : 0) * part_floats + c8 * 8 * kTcRows;
#pragma unroll
              for (int i = 0; i < 8; ++i) v[q][i] = __ldcg(src + i * kTcRows);
            }
            float acc[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[i] = 0.f;
#pragma unroll
              for (int q = 0; q < kTcMaxParts; ++q)
                acc[i] += w[q] > 0.f ? w[q] * v[q][i] : 0.f;  // never 0 * garbage
            }
            uint4 pk;
            pk.x = pack2<T>(acc[0] * inv, acc[1] * inv);
            pk.y = pack2<T>(acc[2] * inv, acc[3] * inv);
            pk.z = pack2<T>(acc[4] * inv, acc[5] * inv);
            pk.w = pack2<T>(acc[6] * inv, acc[7] * inv);
            orow[c8] = pk;
          }
        }
        gv += U.n;
        continue;
      }
      // ---- epilogue: O / l to the output rows, then O_X is free ----
      const bool done = mbar_wait(smem_u32(&o_done[x_tile]), ep & 1);
      if (!__all_sync(0xffffffffu, done)) {
        ok = false;
        break;
      }
      tc_fence_after_sync();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      // O / l packed to T in two 64-column halves (bounded register use);
      // the row's output stays in registers until O_X is released
      uint4 packed[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t ob[2][32];
        tmem_ld32_issue(tO + h * 64, ob[0]);
        tmem_ld32_issue(tO + h * 64 + 32, ob[1]);
        tmem_wait_ld32(ob[0]);
        tmem_wait_ld32(ob[1]);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float* ov = reinterpret_cast<const float*>(ob[c]);
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8) {
            uint4 pk;
            pk.x = pack2<T>(ov[q8 * 8 + 0] * inv_l, ov[q8 * 8 + 1] * inv_l);
            pk.y = pack2<T>(ov[q8 * 8 + 2] * inv_l, ov[q8 * 8 + 3] * inv_l);
            pk.z = pack2<T>(ov[q8 * 8 + 4] * inv_l, ov[q8 * 8 + 5] * inv_l);
            pk.w = pack2<T>(ov[q8 * 8 + 6] * inv_l, ov[q8 * 8 + 7] * inv_l);
            packed[(h * 2 + c) * 4 + q8] = pk;
          }
        }
      }
      // every read of O_X has landed in registers: the next unit may overwrite it
      tc_fence_before_sync();
      mbar_arrive(smem_u32(&o_free[x_tile]));
      if (row_token >= 0) {
        uint4* orow = reinterpret_cast<uint4*>(
            reinterpret_cast<T*>(p.out) + (int64_t)(U.q_start + row_token) * p.out_token_stride +
            (int64_t)row_head * p.out_head_stride);
        if (p.out_v8) {
#pragma unroll
          for (int i = 0; i < 8; ++i) st_global_v8(orow + 2 * i, packed[2 * i], packed[2 * i + 1]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) orow[i] = packed[i];
        }
      }
      ++ep;
      gv += U.n;
    }
    if (!ok && lane == 0) report_status(p.status, B200_STATUS_WAIT_TIMEOUT);
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

template <typename T, bool kFp8>
static cudaError_t launch_tc_typed(const CUtensorMap& mk, const CUtensorMap& mv,
                                   const CUtensorMap& mq, const CUtensorMap& mo,
                                   const PrefillParams& p, int num_kv_heads, int num_seqs,
                                   int max_q_len, cudaStream_t stream) {
  auto kernel = paged_prefill_tc_kernel<T, kFp8>;
  constexpr int kSmem = TcLayout<kFp8>::kSmemBytes;
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kernel), kSmem);
  if (e != cudaSuccess) return e;
  const int tpc = (kTcTiles * kTcRows) / p.group;
  const int blocks = (max_q_len + tpc - 1) / tpc;
  if (blocks <= 0) return cudaSuccess;
  PrefillParams q = p;
  q.num_seqs = num_seqs;
  q.num_kv_heads = num_kv_heads;
  q.blocks_per_seq = blocks;
  const int64_t units = (int64_t)blocks * num_kv_heads * num_seqs;
  if (units > 0x7fffffff) return cudaErrorInvalidConfiguration;
  if constexpr (!kFp8) {
    int dev = 0, sms = 0;
    if (q.q_tma) {
      if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    }
    // The persistent kernel where it pays: more than two units per SM (its per-CTA
    // set-up is paid once, not per unit), or at most half an SM wave of units with
    // a split-KV workspace (a few long units cut into parts on the idle SMs: one
    // 64-token chunk on an 8k prefix, 158 -> 50 us). Otherwise the one-unit kernel
    // is faster: the hardware hands second-wave units to the SMs that finish first,
    // whole output tiles leave by TMA store, and nothing is set up per list (L2
    // cold: 128 units 56 vs 64 us, config 3's 256 units 68.6 vs 72.7 us).
    const bool persistent = q.q_tma && sms > 0 &&
                            (units > 2 * (int64_t)sms || (q.split_cap > 0 && 2 * units <= sms));
    if (persistent) {
      // persistent: one CTA per SM (at most kTcMaxUnitsPerCta units each)
      auto pkernel = paged_prefill_tc_persistent_kernel<T>;
      e = ensure_smem_attr(reinterpret_cast<const void*>(pkernel), kTcPersistSmem);
      if (e != cudaSuccess) return e;
      q.num_sms = sms;
      // split parts add at most split_cap items to the units
      const int64_t items = units + (q.split_cap > 0 ? q.split_cap : 0);
      int64_t grid = items < sms ? items : sms;
      const int64_t min_grid = (items + kTcMaxUnitsPerCta - 1) / kTcMaxUnitsPerCta;
      if (grid < min_grid) grid = min_grid;
      pkernel<<<(unsigned)grid, tc_threads<false>(), kTcPersistSmem, stream>>>(mk, mv, mq, q);
      return cudaGetLastError();
    }
  }
  kernel<<<(unsigned)units, tc_threads<kFp8>(), kSmem, stream>>>(mk, mv, mq, mo, q);
  return cudaGetLastError();
}

cudaError_t launch_paged_prefill_tc(const CUtensorMap& mk, const CUtensorMap& mv,
                                    const CUtensorMap& mq, const CUtensorMap& mo,
                                    const PrefillParams& p, int dtype, bool kv_fp8,
                                    int num_kv_heads, int num_seqs, int max_q_len,
                                    cudaStream_t stream) {
  if (dtype == B200_DTYPE_BFLOAT16)
    return kv_fp8 ? launch_tc_typed<__nv_bfloat16, true>(mk, mv, mq, mo, p, num_kv_heads, num_seqs,
                                                         max_q_len, stream)
                  : launch_tc_typed<__nv_bfloat16, false>(mk, mv, mq, mo, p, num_kv_heads, num_seqs,
                                                          max_q_len, stream);
  return kv_fp8 ? launch_tc_typed<__half, true>(mk, mv, mq, mo, p, num_kv_heads, num_seqs, max_q_len,
                                                stream)
                : launch_tc_typed<__half, false>(mk, mv, mq, mo, p, num_kv_heads, num_seqs, max_q_len,
                                                 stream);
}

}  // namespace b200
