// paged_prefill.cuh — parameters of the paged prefill / chunked-prefill kernel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace b200 {

struct PrefillParams {
  const void* q;
  int64_t q_token_stride;
  int64_t q_head_stride;
  const int32_t* block_tables;
  int64_t block_table_stride;
  const int32_t* seq_lens;
  const int32_t* query_start_loc;
  void* out;
  int64_t out_token_stride;
  int64_t out_head_stride;
  int block_size;
  int group;  // q heads per KV head
  int num_q_heads;
  int64_t num_blocks;
  float scale_log2;  // softmax_scale * log2(e)
  const float* k_scale;  // FP8 caches: dequantisation scales (nullptr = 1)
  const float* v_scale;
  int num_seqs;
  int num_kv_heads;
  int blocks_per_seq;  // row blocks of the longest query chunk
  int q_tma;           // 1: Q arrives by TMA through the q tensor map (group divides
                       // 128); 0: the softmax warps stage it
  int o_tma;           // 1: Q tiles whose rows all belong to the sequence leave by a
                       // TMA store through the out tensor map; 0: per-thread stores
  int out_v8;          // 1: out is 32-byte aligned with strides that are multiples of
                       // 16 elements (rows leave in 32-byte stores)
  int32_t* status;
  // Split-KV (persistent kernel, 16-bit caches): a unit costlier than the
  // average per-SM work is cut into KV parts on different CTAs; the part
  // that finishes last merges the others' partial records. Off when
  // split_cap == 0 (no workspace).
  float* split_records;  // [split_cap][2 Q tiles][130][128 rows]: O columns, m, l
  int* split_tickets;    // [split_cap][2 Q tiles], zeroed before each launch
  int split_cap;         // part records the workspace holds
  int num_sms;
};

// Part records of the prefill split-KV workspace and its size.
constexpr int kPrefillSplitCap = 256;
constexpr int64_t kPrefillRecordFloats = 2 * 130 * 128;
constexpr int64_t prefill_split_ticket_bytes() { return (kPrefillSplitCap * 2 * 4 + 255) / 256 * 256; }
constexpr int64_t prefill_workspace_bytes() {
  return prefill_split_ticket_bytes() + kPrefillSplitCap * kPrefillRecordFloats * 4;
}

// tcgen05 / TMEM prefill: 128 packed (query token, q head of the group) rows
// per CTA on UMMA M = 128 tiles, so the GQA heads of a KV head share every
// K/V tile the CTA loads.
// mq / mo: tensor maps over q / out viewed as (head_dim, q head, token), box
// 64 x group x 128 / group, 128-byte swizzle; used only when p.q_tma / p.o_tma
// is set.
cudaError_t launch_paged_prefill_tc(const CUtensorMap& mk, const CUtensorMap& mv,
                                    const CUtensorMap& mq, const CUtensorMap& mo,
                                    const PrefillParams& p, int dtype, bool kv_fp8,
                                    int num_kv_heads, int num_seqs, int max_q_len,
                                    cudaStream_t stream);

}  // namespace b200
