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
  int32_t* status;
};

// Rows of one CTA: (query token, q head of the group) pairs, packed so the
// GQA heads of a KV head share every K/V tile the CTA loads.
int prefill_rows_per_cta();

cudaError_t launch_paged_prefill(const CUtensorMap& mk, const CUtensorMap& mv,
                                 const PrefillParams& p, int dtype, int num_kv_heads,
                                 int num_seqs, int max_q_len, cudaStream_t stream);

// tcgen05 / TMEM version: 128 packed rows per CTA on UMMA M = 128 tiles.
cudaError_t launch_paged_prefill_tc(const CUtensorMap& mk, const CUtensorMap& mv,
                                    const PrefillParams& p, int dtype, int num_kv_heads,
                                    int num_seqs, int max_q_len, cudaStream_t stream);

}  // namespace b200
