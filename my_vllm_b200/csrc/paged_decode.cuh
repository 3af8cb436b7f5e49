// paged_decode.cuh — parameters and tile geometry of the decode kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

constexpr int kHeadDim = 128;       // Qwen3 head_dim; the kernels are built for it
constexpr int kTileTokens = 16;     // KV tokens per tile (one MMA k-step of PV)
constexpr int kHalfTileBytes = kTileTokens * 128;  // 16 rows x 64 elements x 2 B
constexpr int kDecodeWarps = 4;
constexpr int kDecodeStages = 3;
constexpr int kDecodeStageBytes = 4 * kHalfTileBytes;  // K lo/hi + V lo/hi = 8 KiB
constexpr int kDecodeStageArenaBytes = kDecodeWarps * kDecodeStages * kDecodeStageBytes;
// FP8 E4M3 caches: a 16-token tile of K (or V) is 16 rows x 128 bytes, one TMA
// box. Per-token work is the same as for 16-bit caches but the bytes halve,
// so the FP8 kernel runs 4 CTAs per SM (more warps to hide MMA and convert
// latency; 3 for groups of more than 8 q heads, whose registers allow no
// more) with 3 stages of 4 KiB per warp: 192 KiB in flight per SM, as the
// 16-bit kernel's 2 CTAs x 4 warps x 3 x 8 KiB.
constexpr int kFp8TileBytes = kTileTokens * 128;
constexpr int kFp8Stages = 3;
constexpr int kFp8StageBytes = 2 * kFp8TileBytes;  // K + V = 4 KiB
constexpr int kFp8StageArenaBytes = kDecodeWarps * kFp8Stages * kFp8StageBytes;
// Longest KV partition one CTA takes; the planner splits longer contexts.
constexpr int kMaxPartTokens = 8192;
constexpr int kMaxPartPages = kMaxPartTokens / kTileTokens + 8;
constexpr int kMergeStride = kHeadDim + 4;  // padded fp32 row in the merge area
constexpr int decode_smem_bytes(bool fp8) {
  return 1024 /* alignment slack */ + (fp8 ? kFp8StageArenaBytes : kDecodeStageArenaBytes) +
         kDecodeWarps * (fp8 ? kFp8Stages : kDecodeStages) * 8 + kMaxPartPages * 4;
}
static_assert(kDecodeWarps * (32 + 16 * kMergeStride) * 4 <= kFp8StageArenaBytes,
              "merge area must fit in the stage arena");
static_assert(4 * (decode_smem_bytes(true) + 1024) <= 228 * 1024, "4 FP8 CTAs per SM");

struct DecodeParams {
  const void* q;
  int64_t q_seq_stride;
  int64_t q_head_stride;
  const int32_t* block_tables;
  int64_t block_table_stride;
  const int32_t* seq_lens;
  void* out;
  int64_t out_seq_stride;
  int64_t out_head_stride;
  float* part_o;    // [num_seqs, num_q_heads, num_parts, head_dim]
  float* part_lse;  // [num_seqs, num_q_heads, num_parts], log2 domain
  int num_parts;
  int part_tokens;
  int block_size;
  int group;  // q heads per KV head
  int num_q_heads;
  int64_t num_blocks;
  float scale_log2;  // softmax_scale * log2(e)
  const float* k_scale;  // FP8 caches: dequantisation scales (nullptr = 1)
  const float* v_scale;
  int32_t* status;
};

cudaError_t launch_paged_decode(const CUtensorMap& mk, const CUtensorMap& mv,
                                const DecodeParams& p, int dtype, bool kv_fp8,
                                int num_kv_heads, int num_seqs, cudaStream_t stream);

cudaError_t launch_kv_append(const void* key, int64_t key_row_stride,
                             const void* value, int64_t value_row_stride,
                             void* k_cache, void* v_cache, int64_t cache_slot_stride,
                             const void* slot_mapping, bool slot64, int64_t num_tokens,
                             int64_t row_elems, int32_t elem_bytes, int64_t num_slots,
                             int32_t* status, cudaStream_t stream);

cudaError_t launch_kv_append_fp8(const void* key, int64_t key_row_stride, const void* value,
                                 int64_t value_row_stride, int src_dtype, void* k_cache,
                                 void* v_cache, int64_t cache_slot_stride,
                                 const int32_t* slot_mapping, int64_t num_tokens,
                                 int64_t row_elems, const float* k_scale, const float* v_scale,
                                 int64_t num_slots, int32_t* status, cudaStream_t stream);

cudaError_t launch_build_slot_mapping(const int32_t* block_tables, int64_t bt_stride,
                                      int max_blocks, int64_t num_blocks,
                                      const int32_t* seq_lens, const int32_t* query_start_loc,
                                      int num_seqs, int num_tokens, int block_size,
                                      int32_t* slots, int32_t* status, cudaStream_t stream);

cudaError_t launch_build_block_tables(const int32_t* block_ids, const int32_t* offsets,
                                      int num_seqs, int max_blocks, int32_t* tables,
                                      int64_t stride, int32_t* status, cudaStream_t stream);

}  // namespace b200
