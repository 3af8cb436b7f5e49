/*
 * b200_paged_attn.h — C ABI of the B200 (sm_100a) paged-KV attention path.
 *
 * The path has three kernels and a reduce pass:
 *   1. KV append   — scatters new K/V rows into the paged cache by slot.
 *   2. paged decode — one query token per sequence, GQA heads grouped per
 *      KV head, TMA-staged 16-token tiles, split-KV with an LSE reduce.
 *   3. paged prefill — chunked prefill over prefix-cached plus new tokens
 *      with a bottom-right causal mask, tcgen05/TMEM tensor-core tiles.
 *
 * Conventions shared by every entry point:
 *   - Pointers are device pointers; sizes and strides are in ELEMENTS unless
 *     the name ends in _bytes.
 *   - The paged cache is NHD: [num_blocks, block_size, num_kv_heads, head_dim]
 *     (nanovllm/engine/model_runner.py:346), one tensor for K and one for V.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every call is
 *     asynchronous on that stream; nothing here synchronises the device.
 *   - `status` is an optional device int32 word. Kernels OR error bits into
 *     it (B200_STATUS_*) instead of trapping; the host reads it when it
 *     chooses to synchronise. Pass NULL to skip the reporting.
 *   - Return value: B200_OK, or an error code with a message available from
 *     b200_last_error() (thread-local).
 */
#ifndef B200_PAGED_ATTN_H_
#define B200_PAGED_ATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1
#define B200_ERR_UNSUPPORTED 2
#define B200_ERR_CUDA 3

/* device status bits (OR-ed into *status by the kernels) */
#define B200_STATUS_SLOT_OUT_OF_RANGE 0x1
#define B200_STATUS_PAGE_OUT_OF_RANGE 0x2
#define B200_STATUS_WAIT_TIMEOUT 0x4
#define B200_STATUS_TMEM_ALLOC_FAILED 0x8
#define B200_STATUS_PLAN_EXCEEDED 0x10 /* a sequence is longer than the decode plan covers */
#define B200_STATUS_POSITION_OUT_OF_RANGE 0x20 /* a RoPE position beyond the cos/sin table */

/* element types of Q / K / V / O */
#define B200_DTYPE_FLOAT16 0
#define B200_DTYPE_BFLOAT16 1
/* FP8 E4M3 (1 sign, 4 exponent bits of bias 7, 3 mantissa bits; finite
 * values up to +-448, no infinities): a KV-cache storage type only. */
#define B200_DTYPE_FP8_E4M3 2

/* Version of this ABI (major * 100 + minor). */
B200_API int b200_abi_version(void);

/* Message of the last failing call on this host thread ("" if none). */
B200_API const char* b200_last_error(void);

/*
 * KV append. Replaces the Triton `store_kvcache` launcher and kernel
 * (nanovllm/layers/attention.py:11-41; CPU semantics in
 * KVCacheStore.forward_native, attention.py:69-85).
 *
 * For every token i with slot_mapping[i] != -1, copies the row of
 * `row_elems` (= num_kv_heads * head_dim) contiguous elements at
 * key + i * key_row_stride to k_cache + slot * cache_slot_stride, and the
 * value row likewise into v_cache. Slots of -1 are skipped. The copy is
 * byte-exact for any element size. A slot outside [0, num_slots) is
 * skipped and reported as B200_STATUS_SLOT_OUT_OF_RANGE.
 *
 *   slot_is_int64: 0 -> slot_mapping is int32 (the engine's layout,
 *                  model_runner.py:451), 1 -> int64.
 */
B200_API int b200_store_kvcache(const void* key, int64_t key_row_stride,
                       const void* value, int64_t value_row_stride,
                       void* k_cache, void* v_cache, int64_t cache_slot_stride,
                       const void* slot_mapping, int32_t slot_is_int64,
                       int64_t num_tokens, int64_t row_elems,
                       int32_t elem_bytes, int64_t num_slots,
                       int32_t* status, void* stream);

/*
 * KV append into an FP8 E4M3 cache (see b200_paged_cache.kv_fp8). No
 * counterpart in the reference. For every token i with a slot s != -1:
 *   k_cache[s][e] = fp8(key[i][e] * rk), v_cache[s][e] = fp8(value[i][e] * rv)
 * for e < row_elems, where rk = 1 / *k_scale and rv = 1 / *v_scale are
 * correctly rounded to fp32 once (scale NULL = 1), each product is one fp32
 * multiply, and fp8() rounds to nearest even, saturating to +-448 (NaN
 * stays NaN).
 * key/value: 16-bit rows of `src_dtype` with row strides in elements;
 * caches: one byte per element, cache_slot_stride bytes between slots.
 * row_elems must be a multiple of 16; rows, strides and caches 16-byte
 * aligned. Slots outside [0, num_slots) other than -1 are skipped and
 * reported as B200_STATUS_SLOT_OUT_OF_RANGE.
 */
B200_API int b200_store_kvcache_fp8(const void* key, int64_t key_row_stride,
                                    const void* value, int64_t value_row_stride,
                                    int32_t src_dtype, void* k_cache, void* v_cache,
                                    int64_t cache_slot_stride, const int32_t* slot_mapping,
                                    int64_t num_tokens, int64_t row_elems,
                                    const float* k_scale, const float* v_scale,
                                    int64_t num_slots, int32_t* status, void* stream);

/*
 * Fused q/k RMSNorm + rotary embedding + KV append: the step before attention
 * of Qwen3Attention.forward (nanovllm/models/qwen3.py:96-100: q_norm, k_norm
 * from layers/layernorm.py:30-41, the neox rotary embedding of
 * layers/rotary_embedding.py:7-15,40-51) fused with the KV append of
 * Attention.forward (layers/attention.py:139-141). For every token t:
 *   q_out[t, h] = rope(rmsnorm(q[t, h]) * q_weight, positions[t])   (all q heads)
 *   k_cache[slot_mapping[t], h] = rope(rmsnorm(k[t, h]) * k_weight, positions[t])
 *   v_cache[slot_mapping[t], h] = v[t, h]
 * RMSNorm is x / sqrt(mean(x^2) + eps) in fp32 rounded to the element type,
 * times the element-type weight and rounded; rope rotates pairs (i, i + 64)
 * in fp32 with cos = cos_sin_cache[pos][i], sin = cos_sin_cache[pos][64 + i]
 * and rounds. Slots of -1 skip the cache writes (q is still produced).
 * head_dim must be 128; q/k/v rows may be strided views of the fused qkv
 * projection (heads packed within a row); q_out may alias q. Every pointer
 * (weights and cos_sin_cache included) must be 16-byte aligned and every
 * stride a multiple of 8 elements. Positions outside [0, max_position) set
 * B200_STATUS_POSITION_OUT_OF_RANGE and leave that token's q and k unwritten.
 */
B200_API int b200_qk_norm_rope_append(
    const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
    int64_t k_token_stride, const void* v, int64_t v_token_stride, void* q_out,
    int64_t q_out_token_stride, int64_t q_out_head_stride, const void* q_weight,
    const void* k_weight, float eps, const int64_t* positions, const float* cos_sin_cache,
    int64_t max_position, void* k_cache, void* v_cache, int64_t cache_slot_stride,
    const int32_t* slot_mapping, int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype, int64_t num_slots, int32_t* status, void* stream);

/*
 * The same fused step into an FP8 E4M3 pool (see b200_paged_cache.kv_fp8).
 * No counterpart in the reference. q_out is produced as above; the rotated k
 * row, rounded to `dtype`, and the v row are quantised exactly as
 * b200_store_kvcache_fp8 quantises 16-bit rows (scales NULL = 1). k_cache / v_cache hold one byte per
 * element and cache_slot_stride counts bytes (a multiple of 16).
 */
B200_API int b200_qk_norm_rope_append_fp8(
    const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
    int64_t k_token_stride, const void* v, int64_t v_token_stride, void* q_out,
    int64_t q_out_token_stride, int64_t q_out_head_stride, const void* q_weight,
    const void* k_weight, float eps, const int64_t* positions, const float* cos_sin_cache,
    int64_t max_position, void* k_cache, void* v_cache, int64_t cache_slot_stride,
    const int32_t* slot_mapping, int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype, const float* k_scale, const float* v_scale,
    int64_t num_slots, int32_t* status, void* stream);

/*
 * Slot mapping of the new tokens, built on the device. Replaces the host loop
 * of ModelRunner.prepare_model_input (nanovllm/engine/model_runner.py:414-425).
 * Token t of sequence s (rows [query_start_loc[s], query_start_loc[s+1]))
 * sits at KV position seq_lens[s] - q_len + (t - query_start_loc[s]) and is
 * stored in slot block_tables[s][pos / block_size] * block_size
 * + pos % block_size; a block-table entry of -1 (no cache) gives slot -1.
 * max_blocks is the number of valid columns of block_tables (<= its row
 * stride) and num_blocks the pool size: a position past a row's max_blocks
 * columns, or a page id >= num_blocks, gives slot -1 and sets
 * B200_STATUS_SLOT_OUT_OF_RANGE in *status (NULL = no report), so malformed
 * metadata never reads past a table row.
 * slot_mapping: int32 [num_tokens] output.
 */
B200_API int b200_build_slot_mapping(const int32_t* block_tables, int64_t block_table_stride,
                                     int32_t max_blocks, int64_t num_blocks,
                                     const int32_t* seq_lens, const int32_t* query_start_loc,
                                     int32_t num_seqs, int32_t num_tokens, int32_t block_size,
                                     int32_t* slot_mapping, int32_t* status, void* stream);

/*
 * Padded block tables, built on the device from the per-sequence block lists.
 * Replaces ModelRunner.prepare_block_tables
 * (nanovllm/engine/model_runner.py:354-358), which pads every
 * seq.block_table with -1 to the longest one on the host and copies the
 * [num_seqs, max_len] table. Here the caller uploads the lists once, packed:
 * block_ids int32 [offsets[num_seqs]] holds the lists back to back and
 * offsets int32 [num_seqs + 1] their boundaries (offsets[0] = 0). Row s of
 * block_tables (int32, row stride block_table_stride >= max_blocks) receives
 * block_ids[offsets[s] .. offsets[s+1]) followed by -1 up to max_blocks
 * columns. A list longer than max_blocks is cut there and reported with
 * B200_STATUS_PAGE_OUT_OF_RANGE.
 */
B200_API int b200_build_block_tables(const int32_t* block_ids, const int32_t* offsets,
                                     int32_t num_seqs, int32_t max_blocks,
                                     int32_t* block_tables, int64_t block_table_stride,
                                     int32_t* status, void* stream);

/*
 * Paged KV cache description (NHD). Strides are in elements of the cache's
 * storage type; the innermost (head_dim) stride is 1. Every stride must be a
 * multiple of 16 bytes and both base pointers 16-byte aligned (TMA rules).
 *
 * kv_fp8 = 0: K and V are stored in `dtype`, the type of Q and O.
 * kv_fp8 = 1: K and V are stored as FP8 E4M3 (one byte per element), written
 *   by b200_store_kvcache_fp8; the real values are stored x *k_scale and
 *   stored x *v_scale (device fp32 scalars, NULL = 1). Q and O stay in
 *   `dtype`. No counterpart in the reference, whose contract accepts only
 *   16-bit caches (nanovllm/layers/attention_backend.py:516-519); the layout
 *   is its [num_blocks, block_size, num_kv_heads, head_dim]
 *   (nanovllm/engine/model_runner.py:346) with one byte per element.
 */
typedef struct b200_paged_cache {
  const void* k_cache;
  const void* v_cache;
  int64_t num_blocks;
  int32_t block_size;   /* multiple of 16 */
  int32_t num_kv_heads;
  int32_t head_dim;     /* 128 */
  int32_t dtype;        /* B200_DTYPE_FLOAT16 / B200_DTYPE_BFLOAT16: Q, O (and K, V unless kv_fp8) */
  int64_t block_stride; /* elements between consecutive blocks */
  int64_t slot_stride;  /* elements between consecutive slots of a block */
  int64_t head_stride;  /* elements between consecutive KV heads */
  int32_t kv_fp8;       /* 1: K/V stored as B200_DTYPE_FP8_E4M3 */
  const float* k_scale; /* kv_fp8 only: dequantisation scales (device), NULL = 1 */
  const float* v_scale;
} b200_paged_cache;

/*
 * Decode work partition, computed once per scheduled batch (the engine calls
 * build_plan once per step, model_runner.py:502) and reused by every layer.
 *   num_parts       — KV partitions per (sequence, KV head); 1 = no split.
 *   part_tokens     — tokens per partition (multiple of 16).
 *   workspace_bytes — fp32 partial outputs + LSE the caller must provide
 *                     to b200_paged_decode (0 when num_parts == 1).
 */
typedef struct b200_decode_plan {
  int32_t num_parts;
  int32_t part_tokens;
  int64_t workspace_bytes;
} b200_decode_plan;

/*
 * Plan the decode split for `num_seqs` sequences of at most `max_kv_len`
 * tokens and `total_kv_tokens` tokens in all (0 = unknown: every sequence
 * is assumed to be max_kv_len long) on the current device. Host-only: the
 * engine knows both from its per-step block counts. `force_num_parts` > 0
 * pins the split count (tests); 0 lets the planner fill the SMs and cut the
 * longest sequences into pieces small enough to balance. `kv_fp8` = 1 plans
 * for an FP8 E4M3 cache (its kernel holds twice as many CTAs per SM, so
 * small batches split sooner). Replaces the decode half of
 * FlashInferBackend.build_plan (nanovllm/layers/attention_backend.py:827-839).
 */
B200_API int b200_paged_decode_plan(int32_t num_seqs, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, int32_t max_kv_len,
                           int64_t total_kv_tokens, int32_t force_num_parts,
                           int32_t kv_fp8, b200_decode_plan* plan);

/*
 * Paged decode attention: one query token per sequence.
 * q:   [num_seqs, num_q_heads, head_dim] with strides (q_seq_stride,
 *      q_head_stride, 1); q head h reads KV head h / (num_q_heads/num_kv_heads).
 * out: same shape, strides (out_seq_stride, out_head_stride, 1).
 * block_tables: int32 [num_seqs, >= ceil(seq_len/block_size)] row stride
 *      block_table_stride; seq_lens: int32 [num_seqs], each >= 1 and
 *      including the token being decoded (model_runner.py:404-406).
 * workspace: plan->workspace_bytes of device memory (may be NULL when 0).
 * The kernel is launched as a programmatic dependent of the kernel before it
 * on `stream`: it may start while that kernel runs, and it holds its cache
 * reads until that kernel has completed. q, the metadata and the workspace
 * must therefore be written before the previous kernel STARTS (an earlier
 * launch or copy); the cache may be written by the previous kernel itself
 * (the KV append of the same step, b200_store_kvcache).
 * Replaces BatchDecodeWithPagedKVCacheWrapper.run as called from
 * FlashInferBackend.forward (attention_backend.py:995-997, 1020-1025).
 */
B200_API int b200_paged_decode(const void* q, int64_t q_seq_stride, int64_t q_head_stride,
                      const b200_paged_cache* cache,
                      const int32_t* block_tables, int64_t block_table_stride,
                      const int32_t* seq_lens, int32_t num_seqs,
                      int32_t num_q_heads, void* out, int64_t out_seq_stride,
                      int64_t out_head_stride, float softmax_scale,
                      const b200_decode_plan* plan, void* workspace,
                      int64_t workspace_bytes, int32_t* status, void* stream);

/*
 * Split-KV paged decode that allocates nothing. No counterpart in the
 * reference: it exists for callers that cannot allocate device memory, such
 * as a serving process that reserved nearly all of HBM for its KV pool at
 * start-up and forbids later cudaMalloc calls, or a plugin host that owns
 * every device allocation through its own pool and exposes no allocator
 * across this ABI. Same arguments and result as b200_paged_decode without
 * the workspace: the split-KV partials live in a fixed scratch array built
 * into the library, B200_NOALLOC_DECODE_SCRATCH_BYTES per device, held by
 * every GPU that loads the library until the process exits.
 *   - A batch whose partials need more than that (num_seqs * num_q_heads *
 *     plan->num_parts * 516 bytes, rounded up) is rejected with
 *     B200_ERR_INVALID_ARGUMENT before anything is launched.
 *   - The first call on a device looks up that device's scratch address
 *     (cudaGetSymbolAddress, with the device current); make that first call
 *     before any stream capture. The address is remembered per device and
 *     per CUDA context: a call from another context on the same device (a
 *     host with its own driver context, or the primary context recreated
 *     after a device reset) looks it up again, so that call is again a
 *     first call.
 *   - Every call on a device shares the one scratch array, which keeps the
 *     last call's contents. Calls that overlap on the GPU (other streams,
 *     other host threads) race on it: serialise them.
 *   - No cudaMalloc, cudaFree or other allocating routine is called.
 */
#define B200_NOALLOC_DECODE_SCRATCH_BYTES (16u << 20) /* 16 MiB */
B200_API int b200_paged_decode_noalloc(const void* q, int64_t q_seq_stride,
                                       int64_t q_head_stride, const b200_paged_cache* cache,
                                       const int32_t* block_tables,
                                       int64_t block_table_stride, const int32_t* seq_lens,
                                       int32_t num_seqs, int32_t num_q_heads, void* out,
                                       int64_t out_seq_stride, int64_t out_head_stride,
                                       float softmax_scale, const b200_decode_plan* plan,
                                       int32_t* status, void* stream);

/*
 * Paged prefill / chunked-prefill attention over prefix-cached plus new
 * tokens. Sequence s owns query rows [query_start_loc[s], query_start_loc[s+1])
 * of q/out and seq_lens[s] KV tokens (the new ones included, already
 * appended to the cache). Query row i of a q_len-row chunk attends to KV
 * positions < seq_len - q_len + i + 1 (bottom-right causal mask,
 * tests/test_attention_backend.py:660-699).
 * max_q_len bounds the chunk length (host value from the metadata).
 * num_q_tokens is the number of rows q holds: Q tiles may be fetched, and
 * output tiles stored, as whole boxes through tensor maps bounded by it, so
 * both q and out must hold at least num_q_tokens rows.
 * workspace (optional, NULL = none): b200_paged_prefill_workspace_bytes()
 * of device memory, 256-byte aligned. With it, 16-bit caches whose GQA group
 * divides 128 split the KV range of units much longer than the batch's
 * average work per SM over several CTAs (partial results merged in the
 * workspace), when the launch has at most half as many (sequence, row
 * block, KV head) units as SMs or more than two per SM: a short chunk on a
 * long cached prefix then uses the whole GPU.
 * Zero the workspace once before its first use; a launch leaves its
 * counters zero again, unless it reports an error in *status, after which
 * the workspace must be zeroed again. Launches that share one workspace
 * must not overlap on the GPU.
 * Replaces BatchPrefillWithPagedKVCacheWrapper.run as called from
 * FlashInferBackend.forward (attention_backend.py:992-994, 1014-1019).
 */
B200_API int b200_paged_prefill(const void* q, int64_t q_token_stride,
                       int64_t q_head_stride, const b200_paged_cache* cache,
                       const int32_t* block_tables, int64_t block_table_stride,
                       const int32_t* seq_lens, const int32_t* query_start_loc,
                       int32_t num_seqs, int32_t num_q_tokens, int32_t max_q_len,
                       int32_t num_q_heads, void* out, int64_t out_token_stride,
                       int64_t out_head_stride, float softmax_scale, void* workspace,
                       int64_t workspace_bytes, int32_t* status, void* stream);

/* Bytes of the optional b200_paged_prefill workspace (split-KV partial
 * results). No counterpart in the reference (FlashInfer keeps its own). */
B200_API int64_t b200_paged_prefill_workspace_bytes(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* B200_PAGED_ATTN_H_ */
