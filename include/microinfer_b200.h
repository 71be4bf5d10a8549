/*
 * microinfer_b200.h - C ABI of the B200 (sm_100a) paged KV-cache hot path.
 *
 * Every entry point takes raw device pointers, element counts and a
 * cudaStream_t passed as `void*`; none allocates or frees memory.  Callers
 * own the KV pool, the outputs and any workspace.  All work is enqueued on
 * the given stream with no host synchronisation, so every entry point can be
 * captured into a CUDA graph.
 *
 * Return value: 0 on success, a negative MI_ERR_* code when an argument is
 * rejected (nothing was launched; mi_last_error() has the reason), or a
 * positive cudaError_t value when a launch failed.
 *
 * Device status word: most kernels take an optional `int32_t *dev_status`
 * (device memory, may be NULL).  A kernel that meets a block id outside the
 * pool, a slot outside the cache, or a bounded wait that ran out ORs one of
 * the MI_DEV_* bits into it and skips the offending access instead of
 * touching memory it does not own.
 *
 * Layouts (row-major, innermost last):
 *   key_cache / value_cache  [num_blocks, block_size, num_kv_heads, head_dim]
 *   query / out              [tokens, num_q_heads, head_dim]
 *   block_tables             int32 [num_seqs, block_table_stride], -1 padded;
 *                            kernels never read past a row's stride
 *   context_lens             int32 [num_seqs], includes the token just stored
 *   cu_seqlens_q/k           int32 [num_seqs + 1], cumulative (k: contexts)
 */
#ifndef MICROINFER_B200_H
#define MICROINFER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MI_ABI_VERSION 1

#if defined(__GNUC__)
#define MI_API __attribute__((visibility("default")))
#else
#define MI_API
#endif

/* element dtypes */
#define MI_DTYPE_FLOAT32 0
#define MI_DTYPE_FLOAT16 1
#define MI_DTYPE_BFLOAT16 2

/* index dtypes for slot / block / offset vectors */
#define MI_INDEX_INT32 0
#define MI_INDEX_INT64 1

/* host-side status codes */
#define MI_OK 0
#define MI_ERR_INVALID (-1)     /* shape, dtype, stride or range violation  */
#define MI_ERR_UNSUPPORTED (-2) /* valid input this build has no kernel for */
#define MI_ERR_ALIGNMENT (-3)   /* pointer or stride not 16-byte aligned    */

/* device status bits */
#define MI_DEV_BAD_BLOCK 1 /* block id outside [0, num_blocks)     */
#define MI_DEV_BAD_SLOT 2  /* slot outside [-1, num_blocks*bs)      */
#define MI_DEV_TIMEOUT 4   /* a bounded mbarrier/flag wait ran out  */
#define MI_DEV_BAD_POSITION 8 /* rotary position outside the cos/sin table */
#define MI_DEV_BAD_ROW 16     /* runner record: row, page count or range invalid */

/* Version of this ABI (MI_ABI_VERSION). */
MI_API int mi_abi_version(void);

/* Reason for the last negative status returned on this host thread. */
MI_API const char *mi_last_error(void);

/* Number of SMs of `device` (used by the split policy), or a negative status. */
MI_API int mi_device_sm_count(int device);

/*
 * store_kvcache: cache[blocks[t], offsets[t], h, :] = keys[t, h, :] (same
 * for values) for every token t.  Replaces the Triton `store_kv` launcher,
 * microinfer/worker/triton_kv_store.py:45-78 (kernel :17-41), as called by
 * LayerKVCache.write_fast, microinfer/worker/kv_cache.py:52-79.
 * keys/values rows may have any token stride (in elements) but each
 * [num_kv_heads, head_dim] row must be contiguous.  Caller guarantees
 * unique destinations (the reference's fast-path contract); ids outside the
 * pool are skipped and flagged with MI_DEV_BAD_SLOT.
 */
MI_API int mi_store_kv(void *key_cache, void *value_cache, int64_t num_blocks,
                int32_t block_size, int32_t num_kv_heads, int32_t head_dim,
                int32_t dtype, const void *blocks, const void *offsets,
                int32_t index_dtype, const void *keys, const void *values,
                int64_t key_token_stride, int64_t value_token_stride,
                int64_t num_tokens, int32_t *dev_status, void *stream);

/*
 * Per-step runner metadata from a device-resident page table
 * `page_table` [max_rows, max_pages] int32 (one row per running sequence,
 * entries past a row's page count are ignored).  Replaces the reference
 * runner's host-side assembly (microinfer/runner.py:160-188 _fill_decode_rows,
 * :348-384 prepare_decode, :298-346 prepare_block_tables / prepare_prefill):
 * the host sends `records` (int32 x 6 per sequence, in batch order) and only
 * the page-table entries that changed, `updates` (int32 x 2: column, page id);
 * one launch writes them into the table and produces the metadata tensors.
 * Rows must be distinct within a call.  Records:
 *   decode : row, num_tokens, last_token, num_pages, update_begin, update_count
 *   prefill: row, start, end, num_pages, update_begin, update_count
 * (update_begin/count index `updates`).  Decode writes, per sequence,
 * input_ids = last_token, positions = num_tokens - 1, its slot, context_lens
 * = num_tokens and the -1 padded block-table row [table_width]; prefill
 * writes, per scheduled token (positions start..end-1, `token_ids` holding
 * the scheduled tokens of all sequences concatenated), the id, position and
 * slot, plus cu_seqlens_q/k [num_seqs + 1] and, when table_width > 0, the
 * block tables.  Invalid records are flagged MI_DEV_BAD_ROW, invalid pages
 * MI_DEV_BAD_BLOCK (slot -1).  All buffers are device memory.
 */
MI_API int mi_build_decode_metadata(int32_t *page_table, int32_t max_rows, int32_t max_pages,
                                    const int32_t *records, int32_t num_seqs,
                                    const int32_t *updates, int32_t num_updates,
                                    int32_t block_size, int64_t num_blocks, int32_t table_width,
                                    int64_t *input_ids, int64_t *positions, int32_t *slot_mapping,
                                    int32_t *context_lens, int32_t *block_tables,
                                    int32_t *dev_status, void *stream);
MI_API int mi_build_prefill_metadata(int32_t *page_table, int32_t max_rows, int32_t max_pages,
                                     const int32_t *records, int32_t num_seqs,
                                     const int32_t *updates, int32_t num_updates,
                                     const int32_t *token_ids, int64_t num_tokens,
                                     int32_t block_size, int64_t num_blocks, int32_t table_width,
                                     int64_t *input_ids, int64_t *positions,
                                     int32_t *slot_mapping, int32_t *cu_seqlens_q,
                                     int32_t *cu_seqlens_k, int32_t *block_tables,
                                     int32_t *dev_status, void *stream);

/*
 * Attention prologue in one launch: per-head RMSNorm of q and k
 * (y = x / sqrt(mean(x^2) + eps) * weight, fp32, one rounding), rotary
 * position embedding of q and k (split-half, or interleaved when
 * `interleaved` != 0) with the caller's fp32 cos/sin tables
 * [max_positions, head_dim / 2] indexed by positions[t], then k and v stored
 * to slot_mapping[t] (-1 stores nothing) of the pool and q written to q_out.
 * Replaces, before paged attention, q_norm / k_norm and RotaryCache.apply on
 * q and k (microinfer/layer/transformer.py:222-225, layer/norm.py,
 * layer/rope.py:6-21) and the store of k/v (layer/cached_attention.py:76-85),
 * with the reference's rounding points.  qkv is the packed projection
 * output, rows of [num_q_heads + 2 * num_kv_heads, head_dim] `qkv_token_stride`
 * elements apart; q_out rows are [num_q_heads, head_dim], `q_out_token_stride`
 * apart.  head_dim 64 or 128; dtype f32/f16/bf16 (weights in the same
 * dtype); positions int32 or int64 (MI_INDEX_*).  Pointers and token strides
 * must be 16-byte aligned.  Slots outside the pool are skipped
 * (MI_DEV_BAD_SLOT), positions outside the table give zero rows
 * (MI_DEV_BAD_POSITION).
 */
MI_API int mi_qk_norm_rope_store(void *q_out, int64_t q_out_token_stride, const void *qkv,
                          int64_t qkv_token_stride, const void *q_weight,
                          const void *k_weight, float eps, const void *positions,
                          int32_t positions_dtype, const float *cos_table,
                          const float *sin_table, int64_t max_positions,
                          int32_t interleaved, const int32_t *slot_mapping,
                          void *key_cache, void *value_cache, int64_t num_blocks,
                          int32_t block_size, int64_t num_tokens, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                          int32_t *dev_status, void *stream);

/*
 * store_kvcache from flat slot ids (block * block_size + offset), splitting
 * the slot on the device; slot -1 is padding and writes nothing.  Replaces
 * the write in LayerKVCache.write_checked (microinfer/worker/kv_cache.py:30-50,
 * host validation stays in the caller) together with the per-step slot split
 * AttentionMetadata.slot_indices (microinfer/layer/metadata.py:75-84).
 */
MI_API int mi_store_kv_slots(void *key_cache, void *value_cache, int64_t num_blocks,
                      int32_t block_size, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype, const void *slots,
                      int32_t index_dtype, const void *keys, const void *values,
                      int64_t key_token_stride, int64_t value_token_stride,
                      int64_t num_tokens, int32_t *dev_status, void *stream);

/*
 * Split-K decode workspace size in bytes for `num_splits` splits (0 when
 * num_splits == 1: the single-split kernel writes `out` directly):
 * 64 KiB of arrival counters, then num_seqs * num_q_heads * num_splits
 * states of (head_dim + 2) floats.  The splits of one (sequence, kv head)
 * store their softmax states and the last to finish merges them, then sets
 * its counter back to zero: zero-fill a workspace once, before its first
 * use, and it stays valid for every later launch of any shape.  Launches
 * that can run at the same time (two streams) need separate workspaces.
 * Split-K takes at most 16384 (sequence, kv head) pairs per launch.
 */
MI_API size_t mi_paged_decode_workspace_bytes(int64_t num_seqs, int32_t num_q_heads,
                                       int32_t head_dim, int32_t num_splits);

/*
 * Split count the decode launcher uses when the caller passes num_splits=0
 * (the mma kernel differs for larger batches, see mi_paged_decode_plan).
 * When num_seqs * num_kv_heads fits in half the SMs, the layer's CTAs stay
 * within that half (one CTA per SM), so the next layer's CTAs fit beside
 * them and request their pages early; with `max_context_hint` > 0 each split
 * keeps >= 384 keys.  Larger batches fill every SM with two CTAs, each split
 * keeping >= 2 chunks of 8 keys per warp.
 */
MI_API int mi_paged_decode_default_splits(int64_t num_seqs, int32_t num_kv_heads,
                                   int32_t max_context_hint, int device);

/*
 * Paged decode attention, one query token per sequence:
 *   out[s, h] = softmax(scale * K_s q[s, h]) V_s
 * over the context_lens[s] cached positions found through block_tables[s],
 * with GQA kv head h / (num_q_heads / num_kv_heads).  Replaces
 * triton_paged_decode + _paged_decode_kernel + _paged_decode_reduce_kernel,
 * microinfer/layer/triton_paged_attention.py:352-457 (:39-131, :235-257).
 * num_splits > 1 needs `workspace` (mi_paged_decode_workspace_bytes,
 * zero-filled before its first use); the last split of each (sequence,
 * kv head) merges the states in the same launch.  num_splits == 0 picks
 * the split count of mi_paged_decode_plan.
 * Query and out are contiguous [num_seqs, num_q_heads, head_dim].
 */
MI_API int mi_paged_decode(void *out, const void *query, const void *key_cache,
                    const void *value_cache, int64_t num_blocks,
                    int32_t block_size, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                    const int32_t *block_tables, int64_t block_table_stride,
                    const int32_t *context_lens, int64_t num_seqs, float scale,
                    int32_t num_splits, void *workspace,
                    size_t workspace_bytes, int32_t *dev_status, void *stream);

/*
 * 1 when mi_paged_decode needs a workspace for `num_splits` splits (any
 * split count above 1), else 0.
 */
MI_API int mi_paged_decode_uses_workspace(int32_t num_splits);

/*
 * Launch plan of mi_paged_decode / mi_paged_decode_store for a shape with
 * 16-byte aligned tensors: returns the kernel (1 generic, 2 SIMT bulk-copy,
 * 4 warp-level mma tensor-core) and writes the split
 * count it will use for `num_splits` (0 = automatic) and the workspace bytes
 * the caller must pass.  The mma kernel runs bf16/fp16 with head_dim 64 or
 * 128, a GQA group of 1, 2, 4 or 8 and block_size a multiple of 16; other
 * fast shapes run the SIMT kernel; MICROINFER_B200_DECODE=simt|mma pins
 * one.  Automatic splits are mi_paged_decode_default_splits, except that the
 * mma kernel (one CTA per SM) takes one split once num_seqs * num_kv_heads
 * exceeds half the SMs.
 */
MI_API int mi_paged_decode_plan(int64_t num_seqs, int32_t num_q_heads,
                         int32_t num_kv_heads, int32_t head_dim,
                         int32_t dtype, int32_t block_size,
                         int64_t block_table_stride, int32_t num_splits,
                         int device, int32_t *splits_out,
                         size_t *workspace_bytes_out);

/*
 * Paged decode with this step's store_kvcache fused in: for each sequence s
 * with slot_mapping[s] >= 0, k_new/v_new row s ([num_kv_heads, head_dim],
 * rows new_token_stride elements apart) is written to that slot of the pool,
 * then decode runs exactly as mi_paged_decode.  slot_mapping[s] must address
 * position context_lens[s]-1 of sequence s (the reference's decode contract,
 * microinfer/runner.py:160-177).  Replaces the LayerKVCache.write_fast +
 * paged_attention_meta pair of CachedAttention.forward for decode
 * (microinfer/layer/cached_attention.py:76-85) with one launch.  The result
 * is that of storing first and attending second, but position
 * context_lens[s]-1 is taken from k_new/v_new directly, so no cached page
 * waits on the store.
 *
 * flags: MI_DECODE_EARLY_KV lets the kernel read the block table, context
 * lengths and cached pages before it waits on the preceding kernel in the
 * stream (programmatic dependent launch), so page loads overlap that
 * kernel's tail; only query and k_new/v_new are taken to be produced by it.
 * Set it only when the preceding kernel does not write the pool, the tables
 * or the lengths (e.g. a QKV projection, or the previous layer's decode).
 */
#define MI_DECODE_EARLY_KV 1
MI_API int mi_paged_decode_store(void *out, const void *query, void *key_cache,
                          void *value_cache, int64_t num_blocks,
                          int32_t block_size, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                          const int32_t *block_tables,
                          int64_t block_table_stride,
                          const int32_t *context_lens, int64_t num_seqs,
                          const void *k_new, const void *v_new,
                          int64_t new_token_stride,
                          const int32_t *slot_mapping, float scale,
                          int32_t num_splits, int32_t flags,
                          void *workspace, size_t workspace_bytes,
                          int32_t *dev_status, void *stream);

/*
 * Allocation-free paged decode.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory on the call path (a serving
 * loop that reserved nearly all HBM for the KV pool up front, or an FFI host
 * that owns only the buffers it was given).  Same arguments and results as
 * mi_paged_decode without the workspace: split-K states go to a 2 MiB scratch
 * array built into the library (held by every GPU that loads it until exit).
 * Limit: 64 KiB + num_seqs * num_q_heads * num_splits * (head_dim + 2) * 4
 * bytes must fit in 2 MiB; an explicit num_splits that does not fit gives
 * MI_ERR_INVALID, num_splits = 0 takes the default split count capped to what
 * fits (one split needs no scratch).  The first call on a device looks up the
 * array's device address (make it outside stream capture; a failed lookup is
 * retried on the next call).  Calls share the
 * array, so calls that overlap on the GPU race; serialise them.  Calls no
 * cudaMalloc/cudaFree.
 */
MI_API int mi_paged_decode_noalloc(void *out, const void *query,
                            const void *key_cache, const void *value_cache,
                            int64_t num_blocks, int32_t block_size,
                            int32_t num_q_heads, int32_t num_kv_heads,
                            int32_t head_dim, int32_t dtype,
                            const int32_t *block_tables,
                            int64_t block_table_stride,
                            const int32_t *context_lens, int64_t num_seqs,
                            float scale, int32_t num_splits,
                            int32_t *dev_status, void *stream);

/*
 * Paged chunked-prefill attention (also mixed prefill + decode batches): the
 * q_len = cu_seqlens_q[s+1]-cu_seqlens_q[s] query rows of sequence s sit at
 * absolute positions prefix+i, prefix = context - q_len, context =
 * cu_seqlens_k[s+1]-cu_seqlens_k[s]; row i attends causally to cached keys
 * 0..prefix+i.  Replaces triton_paged_prefill + _paged_prefill_kernel,
 * microinfer/layer/triton_paged_attention.py:260-339 (:133-233), and the
 * torch reference _paged_attention_reference, paged_attention.py:22-67.
 * `max_seqlen_q` bounds the per-sequence tile count (static launch shape).
 */
MI_API int mi_paged_prefill(void *out, const void *query, const void *key_cache,
                     const void *value_cache, int64_t num_blocks,
                     int32_t block_size, int32_t num_q_heads,
                     int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                     const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                     const int32_t *block_tables, int64_t block_table_stride,
                     int64_t num_seqs, int64_t num_tokens, int32_t max_seqlen_q,
                     float scale, int32_t *dev_status, void *stream);

/*
 * Which kernel mi_paged_prefill / mi_varlen_prefill dispatch to for a shape
 * with 16-byte aligned tensors: 2 = tcgen05 tensor-core kernel, 1 = generic
 * CUDA-core kernel, negative = invalid shape.  block_size 0 asks for the
 * dense (varlen) mode.
 */
MI_API int mi_prefill_kernel_for(int32_t dtype, int32_t head_dim,
                          int32_t num_q_heads, int32_t num_kv_heads,
                          int32_t block_size);

/*
 * Dense varlen causal prefill on this step's contiguous K/V (no cached
 * prefix): keys/values [num_kv_tokens, num_kv_heads, head_dim] with row
 * stride `kv_token_stride` (elements), cu_seqlens_q == cu_seqlens_k in the
 * reference's use; K/V rows at or past `num_kv_tokens` are never read.
 * Replaces _direct_prefill_flash / _direct_prefill_sdpa,
 * microinfer/layer/cached_attention.py:17-55 (called at :87-101).
 */
MI_API int mi_varlen_prefill(void *out, const void *query, const void *keys,
                      const void *values, int64_t kv_token_stride,
                      int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype,
                      const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                      int64_t num_seqs, int64_t num_tokens,
                      int64_t num_kv_tokens, int32_t max_seqlen_q, float scale,
                      int32_t *dev_status, void *stream);

/*
 * Block-table gather: out_keys[cu_seqlens_k[s] + t] = key_cache row of
 * logical position t of sequence s, for t < context_s (same for values), in
 * request-major order.  Replaces _gather_paged_kv,
 * microinfer/layer/paged_attention.py:76-101 (test twin
 * tests/support/kv.py:8-24).  `max_context` bounds the launch shape;
 * `out_rows` is the row capacity of out_keys/out_values (never written past).
 */
MI_API int mi_gather_paged_kv(void *out_keys, void *out_values, const void *key_cache,
                       const void *value_cache, int64_t num_blocks,
                       int32_t block_size, int32_t num_kv_heads,
                       int32_t head_dim, int32_t dtype,
                       const int32_t *block_tables, int64_t block_table_stride,
                       const int32_t *cu_seqlens_k, int64_t num_seqs,
                       int64_t out_rows, int32_t max_context,
                       int32_t *dev_status, void *stream);

/*
 * Device-side copy-on-write of KV pages: for each pair p, copy block
 * pairs[2p] -> pairs[2p+1] in every layer of a whole pool, for K and V.
 * Pools are [num_layers, num_blocks, block_size, num_kv_heads, head_dim];
 * `layer_stride_bytes` is the distance between layers and `block_bytes` the
 * size of one block (block_size * num_kv_heads * head_dim * elem).  No
 * destination may also be a source and destinations must be unique; ids
 * outside the pool are skipped and flagged with MI_DEV_BAD_BLOCK.  The
 * reference has no copy-on-write (prefix sharing only, never of a partial
 * block: microinfer/engine/blockmanager.py:144-201); this entry point is
 * what lets a sequence write into a private copy of a shared block.
 */
MI_API int mi_copy_blocks(void *key_pool, void *value_pool, int32_t num_layers,
                   int64_t layer_stride_bytes, int64_t num_blocks,
                   int64_t block_bytes, const int32_t *pairs,
                   int64_t num_pairs, int32_t *dev_status, void *stream);

/*
 * Bounded-wait self test: one thread spins on `flag` (device int32) until it
 * becomes non-zero or `timeout_ns` passes, then ORs MI_DEV_TIMEOUT into
 * dev_status if it ran out.  Exercises the same bounded-wait helper every
 * pipelined kernel uses, so timeouts can be tested without hanging a GPU.
 */
MI_API int mi_wait_flag_selftest(const int32_t *flag, int64_t timeout_ns,
                          int32_t *dev_status, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MICROINFER_B200_H */
