// Kernel parameter blocks shared by the launchers and the C ABI layer.
#pragma once

#include <stdint.h>

namespace mi {

struct StoreParams {
  char *key_cache;
  char *value_cache;
  const char *keys;
  const char *values;
  const void *idx0;
  const void *idx1;
  int64_t num_blocks;
  int64_t num_tokens;
  int64_t key_stride_bytes;
  int64_t value_stride_bytes;
  int32_t block_size;
  int32_t row_bytes;
  int32_t *status;
};
struct GatherParams {
  char *out_keys;
  char *out_values;
  const char *key_cache;
  const char *value_cache;
  const int32_t *block_tables;
  const int32_t *cu_seqlens_k;
  int64_t block_table_stride;
  int64_t num_blocks;
  int32_t block_size;
  int32_t row_bytes;
  int32_t rows_per_cta;
  int64_t out_rows;  // rows of out_keys/out_values; never written past
  int32_t *status;
};
struct CowParams {
  char *key_pool;
  char *value_pool;
  const int32_t *pairs;
  int64_t layer_stride_bytes;
  int64_t num_blocks;
  int64_t block_bytes;
  int32_t chunk_bytes;
  int32_t *status;
};
struct AttnParams {
  void *out;
  const void *query;
  const char *key_base;
  const char *value_base;
  int64_t kv_token_stride;  // dense mode: elements between K/V token rows
  int64_t kv_rows;          // dense mode: rows in keys/values (bounds check)
  const int32_t *block_tables;
  int64_t bt_stride;  // entries per block-table row; never read past
  int64_t num_blocks;
  int32_t block_size;
  const int32_t *cu_q;
  const int32_t *cu_k;
  const int32_t *context_lens;
  int64_t num_seqs;
  int64_t num_tokens;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  float scale_log2;
  int32_t *status;
  // 1: the tensor-core prefill kernel leaves sequences with one query token to
  // the decode kernel launched after it (mixed batches), and lets that launch
  // start as soon as all its CTAs are running.
  int32_t mixed_decode;
};
struct DecodeParams {
  void *out;
  const void *query;
  const char *key_cache;
  const char *value_cache;
  const int32_t *block_tables;
  const int32_t *context_lens;
  // Split-K workspace (nsplit > 1): states and self-resetting arrival counters.
  float *ws_acc;
  float *ws_ml;
  int32_t *ws_count;
  int64_t bt_stride;
  int64_t num_blocks;
  int32_t block_size;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  float scale_log2;
  int32_t *status;
  // Fused store_kvcache of this step's token (k_new == nullptr: no store).
  const char *k_new;  // [num_seqs, Hkv, D] rows at new_token_stride_bytes
  const char *v_new;
  const int32_t *slot_mapping;  // int32 [num_seqs]; -1 = padding row, no store
  int64_t new_token_stride_bytes;
  // 1: read the block table, context lengths and cached pages before waiting
  // on the preceding kernel (programmatic dependent launch), so this layer's
  // page loads overlap the previous kernel's tail.  Only q and this step's
  // token are treated as produced by the preceding kernel; the caller
  // guarantees that kernel does not write the pool, tables or lengths.
  int32_t early_kv;
  // Decode rows of a mixed prefill batch (cu_q != nullptr): sequence s is handled
  // only if cu_q[s+1] - cu_q[s] == 1 (the prefill kernel skips exactly those); its
  // query and output row is token cu_q[s] and its context cu_k[s+1] - cu_k[s]
  // (context_lens unused).  This launch follows the prefill kernel as its
  // programmatic dependent and starts once every prefill CTA has passed its own
  // dependency wait, so everything it reads is complete: it does not wait before
  // working.  Block (0, 0, 0) waits for the prefill grid before exiting, so this
  // grid completes only after the prefill grid (the next kernel's wait covers both).
  const int32_t *cu_q;
  const int32_t *cu_k;
};

// Attention prologue (qk_prologue.cu): q/k RMSNorm + RoPE, k/v store.
struct QkPrologueParams {
  const char *qkv;  // [T, (Hq + 2 Hkv) * D] rows qkv_stride_bytes apart
  int64_t qkv_stride_bytes;
  const void *q_weight;  // [D] activation dtype
  const void *k_weight;
  float eps;
  const void *positions;  // [T] int32 or int64
  int32_t positions_int64;
  const float *cos_table;  // [max_positions, D/2]
  const float *sin_table;
  int64_t max_positions;
  int32_t interleaved;
  const int32_t *slot_mapping;  // [T], -1: no store
  char *key_cache;              // [num_slots, Hkv, D]
  char *value_cache;
  int64_t num_slots;
  char *q_out;  // [T, Hq, D] rows q_out_stride_bytes apart
  int64_t q_out_stride_bytes;
  int64_t num_tokens;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t *status;
};

// Per-step runner metadata from the device page table (runner_meta.cu).
struct RunnerMetaParams {
  int32_t *page_table;  // [max_rows, max_pages]
  int32_t max_rows;
  int32_t max_pages;
  const int32_t *records;  // [num_seqs, 6]
  int32_t num_seqs;
  const int32_t *updates;  // [num_updates, 2]: column, page
  int32_t num_updates;
  const int32_t *token_ids;  // prefill: scheduled tokens, concatenated
  int64_t num_tokens;
  int32_t block_size;
  int64_t num_blocks;
  int32_t table_width;
  int64_t *input_ids;
  int64_t *positions;
  int32_t *slot_mapping;
  int32_t *context_lens;   // decode
  int32_t *cu_seqlens_q;   // prefill
  int32_t *cu_seqlens_k;   // prefill
  int32_t *block_tables;   // [num_seqs, table_width], prefill: may be null
  int32_t *status;
};

}  // namespace mi
