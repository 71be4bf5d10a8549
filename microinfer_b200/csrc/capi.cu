// extern "C" entry points of libmicroinfer_b200.so: argument validation,
// kernel selection and launch.  Nothing here allocates or synchronises.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "split_merge.cuh"

namespace mi {

cudaError_t launch_store_kv(const StoreParams &p, int index_dtype, bool slots, int elem_bytes,
                            bool vec16, cudaStream_t stream);
cudaError_t launch_gather(const GatherParams &p, int64_t num_seqs, int32_t max_context, bool vec16,
                          cudaStream_t stream);
cudaError_t launch_cow(const CowParams &p, int32_t num_layers, int64_t num_pairs, bool vec16,
                       cudaStream_t stream);
cudaError_t launch_wait_flag(const int32_t *flag, int64_t timeout_ns, int32_t *status,
                             cudaStream_t stream);
cudaError_t launch_attn_generic(const AttnParams &p, int dtype, bool paged, cudaStream_t stream);
bool decode_fast_supported(int dtype, int D, int G);
bool decode_mma_supported(int dtype, int D, int G, int block_size);
cudaError_t launch_qk_prologue(const QkPrologueParams &p, int dtype, int D, cudaStream_t stream);
cudaError_t launch_decode_meta(const RunnerMetaParams &p, cudaStream_t stream);
cudaError_t launch_prefill_meta(const RunnerMetaParams &p, cudaStream_t stream);
cudaError_t launch_decode_mma(const DecodeParams &d, int dtype, int D, int G, int64_t num_seqs,
                              int nsplit, bool pair, cudaStream_t stream);
cudaError_t launch_decode_fast(const DecodeParams &p, int dtype, int D, int G, int64_t num_seqs,
                               int nsplit, bool wide, cudaStream_t stream);
bool decode_wide_supported(int dtype, int D, int G);
bool prefill_tc_supported(int dtype, int D, int G, int block_size);
cudaError_t launch_prefill_tc(const AttnParams &p, int dtype, int G, int32_t max_seqlen_q,
                              bool paged, cudaStream_t stream);

// Keys one 16-warp SIMT decode CTA holds in flight (16 warps x 3 stages x 8).
constexpr int64_t kDecodeKeysPerCta = 384;

static int sm_counts[64];
static std::once_flag sm_once[64];

int sm_count_of(int device) {
  if (device < 0 || device >= 64) return 148;
  std::call_once(sm_once[device], [device] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    sm_counts[device] = n;
  });
  return sm_counts[device];
}

int sm_count_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  return sm_count_of(dev);
}

bool pdl_enabled() {
  static const bool enabled = [] {
    const char *v = std::getenv("MICROINFER_B200_PDL");
    return !(v != nullptr && std::strcmp(v, "0") == 0);
  }();
  return enabled;
}

}  // namespace mi

using namespace mi;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string &msg) {
  g_last_error = msg;
  return code;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return MI_OK;
  g_last_error = std::string("CUDA launch failed: ") + cudaGetErrorString(e);
  return static_cast<int>(e);
}

int elem_size(int32_t dtype) {
  switch (dtype) {
    case MI_DTYPE_FLOAT32: return 4;
    case MI_DTYPE_FLOAT16: return 2;
    case MI_DTYPE_BFLOAT16: return 2;
  }
  return 0;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// This library carries its own (static) CUDA runtime, whose current device
// is independent of the caller's.  Make the device that owns `p` current
// before launching; a pointer that is not device memory is rejected here
// instead of faulting inside a kernel.
int select_device(const void *p) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    cudaGetLastError();
    return fail(MI_ERR_INVALID, "pointer is not known to the CUDA driver");
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(MI_ERR_INVALID, "expected device memory, got a host pointer");
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != attr.device) {
    const cudaError_t e = cudaSetDevice(attr.device);
    if (e != cudaSuccess) return fail(static_cast<int>(e), "cudaSetDevice failed");
  }
  return MI_OK;
}

constexpr float kLog2eHost = 1.4426950408889634f;

}  // namespace

// Error reporting and device selection for entry points defined in other
// translation units (their messages surface through mi_last_error()).
namespace mi {
int capi_fail(int code, const char *msg) { return fail(code, msg); }
int capi_select_device(const void *p) { return select_device(p); }
}  // namespace mi

extern "C" {

int mi_abi_version(void) { return MI_ABI_VERSION; }

const char *mi_last_error(void) { return g_last_error.c_str(); }

int mi_device_sm_count(int device) {
  int count = 0;
  if (device < 0) return fail(MI_ERR_INVALID, "device must be >= 0");
  if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count)
    return fail(MI_ERR_INVALID, "no such CUDA device");
  return sm_count_of(device);
}

static int store_common(void *key_cache, void *value_cache, int64_t num_blocks, int32_t block_size,
                        int32_t num_kv_heads, int32_t head_dim, int32_t dtype, const void *idx0,
                        const void *idx1, int32_t index_dtype, const void *keys, const void *values,
                        int64_t key_token_stride, int64_t value_token_stride, int64_t num_tokens,
                        int32_t *dev_status, void *stream, bool slots) {
  const int e = elem_size(dtype);
  if (e == 0) return fail(MI_ERR_INVALID, "unknown dtype");
  if (index_dtype != MI_INDEX_INT32 && index_dtype != MI_INDEX_INT64)
    return fail(MI_ERR_INVALID, "index dtype must be int32 or int64");
  if (num_tokens < 0) return fail(MI_ERR_INVALID, "num_tokens must be >= 0");
  if (num_blocks <= 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(MI_ERR_INVALID, "cache dimensions must be positive");
  if (key_token_stride < 0 || value_token_stride < 0)
    return fail(MI_ERR_INVALID, "token strides must be >= 0");
  if (num_tokens == 0) return MI_OK;
  if (!key_cache || !value_cache || !keys || !values || !idx0 || (!slots && !idx1))
    return fail(MI_ERR_INVALID, "null pointer");
  if (const int s = select_device(key_cache)) return s;
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * e;
  if (row_bytes > (1 << 30)) return fail(MI_ERR_INVALID, "token row too large");
  StoreParams p;
  p.key_cache = static_cast<char *>(key_cache);
  p.value_cache = static_cast<char *>(value_cache);
  p.keys = static_cast<const char *>(keys);
  p.values = static_cast<const char *>(values);
  p.idx0 = idx0;
  p.idx1 = idx1;
  p.num_blocks = num_blocks;
  p.num_tokens = num_tokens;
  p.key_stride_bytes = key_token_stride * e;
  p.value_stride_bytes = value_token_stride * e;
  p.block_size = block_size;
  p.row_bytes = static_cast<int32_t>(row_bytes);
  p.status = dev_status;
  const bool vec16 = (row_bytes % 16 == 0) && aligned16(key_cache) && aligned16(value_cache) &&
                     aligned16(keys) && aligned16(values) && (p.key_stride_bytes % 16 == 0) &&
                     (p.value_stride_bytes % 16 == 0);
  return cuda_status(
      launch_store_kv(p, index_dtype, slots, e, vec16, static_cast<cudaStream_t>(stream)));
}

int mi_store_kv(void *key_cache, void *value_cache, int64_t num_blocks, int32_t block_size,
                int32_t num_kv_heads, int32_t head_dim, int32_t dtype, const void *blocks,
                const void *offsets, int32_t index_dtype, const void *keys, const void *values,
                int64_t key_token_stride, int64_t value_token_stride, int64_t num_tokens,
                int32_t *dev_status, void *stream) {
  return store_common(key_cache, value_cache, num_blocks, block_size, num_kv_heads, head_dim, dtype,
                      blocks, offsets, index_dtype, keys, values, key_token_stride,
                      value_token_stride, num_tokens, dev_status, stream, false);
}

int mi_store_kv_slots(void *key_cache, void *value_cache, int64_t num_blocks, int32_t block_size,
                      int32_t num_kv_heads, int32_t head_dim, int32_t dtype, const void *slots,
                      int32_t index_dtype, const void *keys, const void *values,
                      int64_t key_token_stride, int64_t value_token_stride, int64_t num_tokens,
                      int32_t *dev_status, void *stream) {
  return store_common(key_cache, value_cache, num_blocks, block_size, num_kv_heads, head_dim, dtype,
                      slots, nullptr, index_dtype, keys, values, key_token_stride,
                      value_token_stride, num_tokens, dev_status, stream, true);
}

int mi_qk_norm_rope_store(void *q_out, int64_t q_out_token_stride, const void *qkv,
                          int64_t qkv_token_stride, const void *q_weight, const void *k_weight,
                          float eps, const void *positions, int32_t positions_dtype,
                          const float *cos_table, const float *sin_table, int64_t max_positions,
                          int32_t interleaved, const int32_t *slot_mapping, void *key_cache,
                          void *value_cache, int64_t num_blocks, int32_t block_size,
                          int64_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                          int32_t head_dim, int32_t dtype, int32_t *dev_status, void *stream) {
  const int e = elem_size(dtype);
  if (e == 0) return fail(MI_ERR_INVALID, "unknown dtype");
  if (num_tokens < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      num_blocks <= 0 || block_size <= 0)
    return fail(MI_ERR_INVALID, "sizes must be positive (num_tokens >= 0)");
  if (head_dim != 64 && head_dim != 128) return fail(MI_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (positions_dtype != MI_INDEX_INT32 && positions_dtype != MI_INDEX_INT64)
    return fail(MI_ERR_INVALID, "positions must be int32 or int64");
  if (!(eps >= 0.f)) return fail(MI_ERR_INVALID, "eps must be >= 0");
  if (num_tokens == 0) return MI_OK;
  if (!q_out || !qkv || !q_weight || !k_weight || !positions || !cos_table || !sin_table ||
      !slot_mapping || !key_cache || !value_cache)
    return fail(MI_ERR_INVALID, "null pointer");
  if (max_positions <= 0) return fail(MI_ERR_INVALID, "max_positions must be positive");
  const int64_t heads = num_q_heads + 2 * static_cast<int64_t>(num_kv_heads);
  if (qkv_token_stride < heads * head_dim || q_out_token_stride < num_q_heads * int64_t{head_dim})
    return fail(MI_ERR_INVALID, "token stride shorter than a row");
  if (!aligned16(q_out) || !aligned16(qkv) || !aligned16(key_cache) || !aligned16(value_cache) ||
      !aligned16(q_weight) || !aligned16(k_weight) || !aligned16(cos_table) ||
      !aligned16(sin_table) || (qkv_token_stride * e) % 16 != 0 || (q_out_token_stride * e) % 16 != 0)
    return fail(MI_ERR_ALIGNMENT, "pointers and token strides must be 16-byte aligned");
  if (const int s = select_device(key_cache)) return s;
  QkPrologueParams p = {};
  p.qkv = static_cast<const char *>(qkv);
  p.qkv_stride_bytes = qkv_token_stride * e;
  p.q_weight = q_weight;
  p.k_weight = k_weight;
  p.eps = eps;
  p.positions = positions;
  p.positions_int64 = positions_dtype == MI_INDEX_INT64 ? 1 : 0;
  p.cos_table = cos_table;
  p.sin_table = sin_table;
  p.max_positions = max_positions;
  p.interleaved = interleaved ? 1 : 0;
  p.slot_mapping = slot_mapping;
  p.key_cache = static_cast<char *>(key_cache);
  p.value_cache = static_cast<char *>(value_cache);
  p.num_slots = num_blocks * block_size;
  p.q_out = static_cast<char *>(q_out);
  p.q_out_stride_bytes = q_out_token_stride * e;
  p.num_tokens = num_tokens;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.status = dev_status;
  return cuda_status(launch_qk_prologue(p, dtype, head_dim, static_cast<cudaStream_t>(stream)));
}

static int check_runner_meta(const int32_t *page_table, int32_t max_rows, int32_t max_pages,
                             const int32_t *records, int32_t num_seqs, const int32_t *updates,
                             int32_t num_updates, int32_t block_size, int64_t num_blocks,
                             int32_t table_width) {
  if (max_rows <= 0 || max_pages <= 0 || num_seqs < 0 || num_updates < 0 || block_size <= 0 ||
      num_blocks <= 0 || table_width < 0 || table_width > max_pages)
    return fail(MI_ERR_INVALID, "bad page-table or batch sizes");
  if (num_blocks * static_cast<int64_t>(block_size) > INT32_MAX)
    return fail(MI_ERR_INVALID, "slots must fit int32");
  if (num_seqs > 0 && (!page_table || !records)) return fail(MI_ERR_INVALID, "null pointer");
  if (num_updates > 0 && !updates) return fail(MI_ERR_INVALID, "null updates");
  return MI_OK;
}

static RunnerMetaParams runner_meta_params(int32_t *page_table, int32_t max_rows, int32_t max_pages,
                                           const int32_t *records, int32_t num_seqs,
                                           const int32_t *updates, int32_t num_updates,
                                           int32_t block_size, int64_t num_blocks,
                                           int32_t table_width, int32_t *dev_status) {
  RunnerMetaParams p = {};
  p.page_table = page_table;
  p.max_rows = max_rows;
  p.max_pages = max_pages;
  p.records = records;
  p.num_seqs = num_seqs;
  p.updates = updates;
  p.num_updates = num_updates;
  p.block_size = block_size;
  p.num_blocks = num_blocks;
  p.table_width = table_width;
  p.status = dev_status;
  return p;
}

int mi_build_decode_metadata(int32_t *page_table, int32_t max_rows, int32_t max_pages,
                             const int32_t *records, int32_t num_seqs, const int32_t *updates,
                             int32_t num_updates, int32_t block_size, int64_t num_blocks,
                             int32_t table_width, int64_t *input_ids, int64_t *positions,
                             int32_t *slot_mapping, int32_t *context_lens, int32_t *block_tables,
                             int32_t *dev_status, void *stream) {
  if (const int s = check_runner_meta(page_table, max_rows, max_pages, records, num_seqs, updates,
                                      num_updates, block_size, num_blocks, table_width))
    return s;
  if (num_seqs == 0) return MI_OK;
  if (!input_ids || !positions || !slot_mapping || !context_lens ||
      (table_width > 0 && !block_tables))
    return fail(MI_ERR_INVALID, "null output");
  if (const int s = select_device(page_table)) return s;
  RunnerMetaParams p = runner_meta_params(page_table, max_rows, max_pages, records, num_seqs,
                                          updates, num_updates, block_size, num_blocks,
                                          table_width, dev_status);
  p.input_ids = input_ids;
  p.positions = positions;
  p.slot_mapping = slot_mapping;
  p.context_lens = context_lens;
  p.block_tables = block_tables;
  return cuda_status(launch_decode_meta(p, static_cast<cudaStream_t>(stream)));
}

int mi_build_prefill_metadata(int32_t *page_table, int32_t max_rows, int32_t max_pages,
                              const int32_t *records, int32_t num_seqs, const int32_t *updates,
                              int32_t num_updates, const int32_t *token_ids, int64_t num_tokens,
                              int32_t block_size, int64_t num_blocks, int32_t table_width,
                              int64_t *input_ids, int64_t *positions, int32_t *slot_mapping,
                              int32_t *cu_seqlens_q, int32_t *cu_seqlens_k,
                              int32_t *block_tables, int32_t *dev_status, void *stream) {
  if (const int s = check_runner_meta(page_table, max_rows, max_pages, records, num_seqs, updates,
                                      num_updates, block_size, num_blocks, table_width))
    return s;
  if (num_tokens < 0 || num_tokens > INT32_MAX) return fail(MI_ERR_INVALID, "bad num_tokens");
  if (num_seqs == 0) return MI_OK;
  if (!cu_seqlens_q || !cu_seqlens_k || (num_tokens > 0 && (!token_ids || !input_ids ||
                                                            !positions || !slot_mapping)) ||
      (table_width > 0 && !block_tables))
    return fail(MI_ERR_INVALID, "null pointer");
  if (const int s = select_device(page_table)) return s;
  RunnerMetaParams p = runner_meta_params(page_table, max_rows, max_pages, records, num_seqs,
                                          updates, num_updates, block_size, num_blocks,
                                          table_width, dev_status);
  p.token_ids = token_ids;
  p.num_tokens = num_tokens;
  p.input_ids = input_ids;
  p.positions = positions;
  p.slot_mapping = slot_mapping;
  p.cu_seqlens_q = cu_seqlens_q;
  p.cu_seqlens_k = cu_seqlens_k;
  p.block_tables = table_width > 0 ? block_tables : nullptr;
  return cuda_status(launch_prefill_meta(p, static_cast<cudaStream_t>(stream)));
}

size_t mi_paged_decode_workspace_bytes(int64_t num_seqs, int32_t num_q_heads, int32_t head_dim,
                                       int32_t num_splits) {
  if (num_seqs <= 0 || num_q_heads <= 0 || head_dim <= 0 || num_splits <= 1) return 0;
  const size_t states = static_cast<size_t>(num_seqs) * num_q_heads * num_splits;
  return kSplitCounterBytes + states * (static_cast<size_t>(head_dim) + 2) * sizeof(float);
}

int mi_paged_decode_default_splits(int64_t num_seqs, int32_t num_kv_heads, int32_t max_context_hint,
                                   int device) {
  if (num_seqs <= 0 || num_kv_heads <= 0) return 1;
  const int64_t sms = sm_count_of(device < 0 ? 0 : device);
  const int64_t base = num_seqs * num_kv_heads;
  int64_t s;
  if (2 * base <= sms) {
    // Small batch: the layer's CTAs stay within half the SMs (one CTA per SM),
    // so the next layer's CTAs fit beside them and request their pages while
    // this layer runs (programmatic dependent launch); splitting further would
    // take that room away.  Each split gets at least kDecodeKeysPerCta keys.
    s = (sms / 2) / base;
    if (max_context_hint > 0) {
      const int64_t need = (static_cast<int64_t>(max_context_hint) + kDecodeKeysPerCta - 1) /
                           kDecodeKeysPerCta;
      if (need > 2 * s)
        // Long contexts stream for longer than a launch: spread over all but an
        // eighth of the SMs, which the next layer's CTAs take to start their
        // page loads early (batch 1 x 32K, 8 kv heads: 16 splits 4700 GB/s,
        // 18 splits 4386).
        s = (sms - sms / 8) / base;
      else if (s > need)
        s = need;
    }
  } else {
    // Larger batch: one wave of two CTAs per SM.
    s = (2 * sms) / base;
    if (max_context_hint > 0) {
      const int64_t chunks = (static_cast<int64_t>(max_context_hint) + 15) / 16;
      const int64_t cap = chunks / 8;  // keep >= 2 chunks per warp
      if (s > cap) s = cap;
    }
  }
  if (s < 1) s = 1;
  if (s > 256) s = 256;
  return static_cast<int>(s);
}

}  // extern "C"

namespace mi {
// SIMT decode CTA shape: 16 warps (one CTA per SM) when the whole grid fits
// one per SM, else 8 warps (two per SM).
bool decode_simt_wide(int dtype, int D, int G, int64_t ctas, int dev) {
  return decode_wide_supported(dtype, D, G) && ctas <= sm_count_of(dev);
}
}  // namespace mi

namespace {

// Split-K merges through the workspace (last-arriver, split_merge.cuh).
bool decode_uses_workspace(int nsplit) { return nsplit > 1; }

// Decode kernels, in order of preference: warp-level tensor-core MMA
// (mma.sync, bf16/fp16, D 64/128, block size a multiple of 16), SIMT
// (TMA-staged, CUDA cores, every fast shape), generic (any shape).
// MICROINFER_B200_DECODE=simt|mma pins one of the fast kernels.  Plan code 5
// is the mma kernel in cluster pairs (decode_pair_for).
constexpr int kDecodeGeneric = 1, kDecodeSimt = 2, kDecodeMma = 4, kDecodeMmaPair = 5;

int decode_kernel_for(int dtype, int D, int G, int block_size, bool aligned, int64_t max_context) {
  (void)max_context;
  static const int mode = [] {
    const char *v = std::getenv("MICROINFER_B200_DECODE");
    if (v != nullptr && std::strcmp(v, "simt") == 0) return 1;
    if (v != nullptr && std::strcmp(v, "mma") == 0) return 3;
    return 0;
  }();
  if (!aligned || !decode_fast_supported(dtype, D, G)) return kDecodeGeneric;
  if (mode == 1) return kDecodeSimt;
  if (decode_mma_supported(dtype, D, G, block_size)) return kDecodeMma;
  return kDecodeSimt;
}

// Split count: the caller's, else enough CTAs for one wave (the mma kernel
// holds one CTA per SM, the SIMT kernel two).
int decode_splits_for(int kernel, int64_t num_seqs, int num_kv_heads, int num_splits, int dev,
                      int64_t ctx_bound) {
  if (num_splits > 0) return num_splits;
  if (kernel == kDecodeGeneric) return 1;
  if (kernel == kDecodeMma && 2 * num_seqs * num_kv_heads > sm_count_of(dev)) {
    // The mma kernel holds one CTA per SM: once the (sequence, kv head) pairs
    // fill more than half the SMs, a second split only adds a merge through
    // global memory and a second wave (batch 16, Qwen3-0.6B heads: 1 split
    // 6.2-45 us per layer for contexts 512-4096, 2 splits 13-52 us).
    return 1;
  }
  const int64_t hint = ctx_bound > INT32_MAX ? INT32_MAX : ctx_bound;
  return mi_paged_decode_default_splits(num_seqs, num_kv_heads, static_cast<int32_t>(hint), dev);
}

// Automatic splits of the mma kernel for small batches: instead of one CTA per
// (sequence, kv head) on at most half the SMs, a cluster of two CTAs per pair
// takes every other 16-key chunk and merges through distributed shared memory
// (no workspace, no global round trips), so each pair streams through two SMs.
// Taken when the pairs fill at most half the SMs and the automatic split count
// is at most 2; MICROINFER_B200_DECODE_PAIR=0 turns it off.
bool decode_pair_for(int kernel, int64_t num_seqs, int num_kv_heads, int num_splits, int dev,
                     int64_t ctx_bound) {
  static const bool enabled = [] {
    const char *v = std::getenv("MICROINFER_B200_DECODE_PAIR");
    return !(v != nullptr && std::strcmp(v, "0") == 0);
  }();
  if (!enabled || num_splits != 0 || kernel != kDecodeMma) return false;
  if (2 * num_seqs * num_kv_heads > sm_count_of(dev)) return false;
  return decode_splits_for(kernel, num_seqs, num_kv_heads, 0, dev, ctx_bound) <= 2;
}

struct NewToken {
  const void *k_new;
  const void *v_new;
  int64_t stride;  // elements between sequences' rows
  const int32_t *slots;
};

int decode_impl(void *out, const void *query, const void *key_cache, const void *value_cache,
                int64_t num_blocks, int32_t block_size, int32_t num_q_heads, int32_t num_kv_heads,
                int32_t head_dim, int32_t dtype, const int32_t *block_tables,
                int64_t block_table_stride, const int32_t *context_lens, int64_t num_seqs,
                const NewToken *nt, float scale, int32_t num_splits, int32_t flags, void *workspace,
                size_t workspace_bytes, int32_t *dev_status, void *stream) {
  const int e = elem_size(dtype);
  if (e == 0) return fail(MI_ERR_INVALID, "unknown dtype");
  if (num_seqs < 0) return fail(MI_ERR_INVALID, "num_seqs must be >= 0");
  if (num_blocks <= 0 || block_size <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(MI_ERR_INVALID, "cache dimensions must be positive");
  if (num_q_heads % num_kv_heads != 0)
    return fail(MI_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads");
  if (head_dim > 256) return fail(MI_ERR_UNSUPPORTED, "head_dim > 256");
  if (block_table_stride < 0) return fail(MI_ERR_INVALID, "block_table_stride must be >= 0");
  if (num_splits < 0 || num_splits > 1024) return fail(MI_ERR_INVALID, "num_splits out of range");
  if (num_seqs > 65535) return fail(MI_ERR_UNSUPPORTED, "more than 65535 sequences in one call");
  if (num_seqs == 0) return MI_OK;
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return fail(MI_ERR_INVALID, "null pointer");
  if (nt != nullptr && (!nt->k_new || !nt->v_new || !nt->slots || nt->stride < 0))
    return fail(MI_ERR_INVALID, "fused store needs k_new, v_new, slot_mapping and a stride >= 0");
  const int G = num_q_heads / num_kv_heads;
  const bool aligned = aligned16(key_cache) && aligned16(value_cache) && aligned16(query);
  // A sequence's context cannot exceed its block-table row.
  const int kernel =
      decode_kernel_for(dtype, head_dim, G, block_size, aligned, block_table_stride * block_size);
  const bool fast = kernel != kDecodeGeneric;
  if (fast && num_splits > 0 && decode_uses_workspace(num_splits) &&
      (workspace == nullptr ||
       workspace_bytes < mi_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, num_splits)))
    return fail(MI_ERR_INVALID, "workspace too small for num_splits (see "
                                "mi_paged_decode_workspace_bytes)");
  if (const int s = select_device(key_cache)) return s;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaGetDevice(&dev);
  // The fused store reads k_new/v_new rows with 16-byte loads.
  const bool fuse_store = nt != nullptr && fast && aligned16(nt->k_new) && aligned16(nt->v_new) &&
                          (nt->stride * e) % 16 == 0;
  if (nt != nullptr && !fuse_store) {  // store first, as its own launch
    StoreParams sp;
    sp.key_cache = static_cast<char *>(const_cast<void *>(key_cache));
    sp.value_cache = static_cast<char *>(const_cast<void *>(value_cache));
    sp.keys = static_cast<const char *>(nt->k_new);
    sp.values = static_cast<const char *>(nt->v_new);
    sp.idx0 = nt->slots;
    sp.idx1 = nullptr;
    sp.num_blocks = num_blocks;
    sp.num_tokens = num_seqs;
    sp.key_stride_bytes = nt->stride * e;
    sp.value_stride_bytes = nt->stride * e;
    sp.block_size = block_size;
    sp.row_bytes = num_kv_heads * head_dim * e;
    sp.status = dev_status;
    const bool vec16 = sp.row_bytes % 16 == 0 && aligned16(key_cache) && aligned16(value_cache) &&
                       aligned16(nt->k_new) && aligned16(nt->v_new) && sp.key_stride_bytes % 16 == 0;
    const cudaError_t se = launch_store_kv(sp, MI_INDEX_INT32, true, e, vec16, st);
    if (se != cudaSuccess) return cuda_status(se);
  }
  if (!fast) {
    AttnParams p = {};
    p.out = out;
    p.query = query;
    p.key_base = static_cast<const char *>(key_cache);
    p.value_base = static_cast<const char *>(value_cache);
    p.block_tables = block_tables;
    p.bt_stride = block_table_stride;
    p.num_blocks = num_blocks;
    p.block_size = block_size;
    p.context_lens = context_lens;
    p.num_seqs = num_seqs;
    p.num_tokens = num_seqs;
    p.num_q_heads = num_q_heads;
    p.num_kv_heads = num_kv_heads;
    p.head_dim = head_dim;
    p.scale_log2 = scale * kLog2eHost;
    p.status = dev_status;
    return cuda_status(launch_attn_generic(p, dtype, true, st));
  }
  const bool pair = decode_pair_for(kernel, num_seqs, num_kv_heads, num_splits, dev,
                                    block_table_stride * block_size);
  const int nsplit = pair ? 2
                          : decode_splits_for(kernel, num_seqs, num_kv_heads, num_splits, dev,
                                              block_table_stride * block_size);
  DecodeParams p = {};
  p.out = out;
  p.query = query;
  p.key_cache = static_cast<const char *>(key_cache);
  p.value_cache = static_cast<const char *>(value_cache);
  p.block_tables = block_tables;
  p.context_lens = context_lens;
  p.bt_stride = block_table_stride;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.scale_log2 = scale * kLog2eHost;
  p.status = dev_status;
  if (fuse_store) {
    p.k_new = static_cast<const char *>(nt->k_new);
    p.v_new = static_cast<const char *>(nt->v_new);
    p.slot_mapping = nt->slots;
    p.new_token_stride_bytes = nt->stride * e;
  }
  if (!pair && decode_uses_workspace(nsplit)) {
    if (num_seqs * num_kv_heads > kSplitCounters)
      return fail(MI_ERR_UNSUPPORTED, "split-K decode takes at most 16384 (sequence, kv head) "
                                      "pairs per launch; use num_splits=1 or smaller batches");
    const size_t need = mi_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, nsplit);
    if (workspace == nullptr || workspace_bytes < need)
      return fail(MI_ERR_INVALID, "workspace too small for num_splits (see "
                                  "mi_paged_decode_workspace_bytes)");
    if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
      return fail(MI_ERR_ALIGNMENT, "workspace must be 16-byte aligned");
    set_split_workspace(p, workspace, num_seqs, num_q_heads, head_dim, nsplit);
  }
  if (flags & MI_DECODE_EARLY_KV) {
    p.early_kv = 1;
  }
  if (kernel == kDecodeMma) {
    const cudaError_t me = launch_decode_mma(p, dtype, head_dim, G, num_seqs, nsplit, pair, st);
    if (me != cudaErrorNotSupported) return cuda_status(me);
  }
  return cuda_status(launch_decode_fast(p, dtype, head_dim, G, num_seqs, nsplit,
                                        decode_simt_wide(dtype, head_dim, G, num_seqs * num_kv_heads * nsplit, dev),
                                        st));
}

}  // namespace

extern "C" {

int mi_paged_decode_uses_workspace(int32_t num_splits) {
  return decode_uses_workspace(num_splits) ? 1 : 0;
}

int mi_paged_decode_plan(int64_t num_seqs, int32_t num_q_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t dtype, int32_t block_size,
                         int64_t block_table_stride, int32_t num_splits, int device,
                         int32_t *splits_out, size_t *workspace_bytes_out) {
  if (elem_size(dtype) == 0 || num_seqs < 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      head_dim <= 0 || head_dim > 256 || num_q_heads % num_kv_heads != 0 || block_size <= 0 ||
      block_table_stride < 0 || num_splits < 0 || num_splits > 1024)
    return fail(MI_ERR_INVALID, "invalid decode shape");
  const int kernel = decode_kernel_for(dtype, head_dim, num_q_heads / num_kv_heads, block_size, true,
                                       block_table_stride * block_size);
  const int dev = device < 0 ? 0 : device;
  if (decode_pair_for(kernel, num_seqs, num_kv_heads, num_splits, dev,
                      block_table_stride * block_size)) {
    if (splits_out) *splits_out = 2;
    if (workspace_bytes_out) *workspace_bytes_out = 0;
    return kDecodeMmaPair;
  }
  const int s = decode_splits_for(kernel, num_seqs, num_kv_heads, num_splits, dev,
                                  block_table_stride * block_size);
  if (splits_out) *splits_out = s;
  if (workspace_bytes_out)
    *workspace_bytes_out = (kernel != kDecodeGeneric && decode_uses_workspace(s))
                               ? mi_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, s)
                               : 0;
  return kernel;
}

int mi_paged_decode(void *out, const void *query, const void *key_cache, const void *value_cache,
                    int64_t num_blocks, int32_t block_size, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                    const int32_t *block_tables, int64_t block_table_stride,
                    const int32_t *context_lens, int64_t num_seqs, float scale, int32_t num_splits,
                    void *workspace, size_t workspace_bytes, int32_t *dev_status, void *stream) {
  return decode_impl(out, query, key_cache, value_cache, num_blocks, block_size, num_q_heads,
                     num_kv_heads, head_dim, dtype, block_tables, block_table_stride, context_lens,
                     num_seqs, nullptr, scale, num_splits, 0, workspace, workspace_bytes, dev_status,
                     stream);
}

int mi_paged_decode_store(void *out, const void *query, void *key_cache, void *value_cache,
                          int64_t num_blocks, int32_t block_size, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                          const int32_t *block_tables, int64_t block_table_stride,
                          const int32_t *context_lens, int64_t num_seqs, const void *k_new,
                          const void *v_new, int64_t new_token_stride,
                          const int32_t *slot_mapping, float scale, int32_t num_splits,
                          int32_t flags, void *workspace, size_t workspace_bytes,
                          int32_t *dev_status, void *stream) {
  if (flags & ~MI_DECODE_EARLY_KV) return fail(MI_ERR_INVALID, "unknown decode flags");
  const NewToken nt{k_new, v_new, new_token_stride, slot_mapping};
  return decode_impl(out, query, key_cache, value_cache, num_blocks, block_size, num_q_heads,
                     num_kv_heads, head_dim, dtype, block_tables, block_table_stride, context_lens,
                     num_seqs, &nt, scale, num_splits, flags, workspace, workspace_bytes, dev_status,
                     stream);
}

static int prefill_common(void *out, const void *query, const void *kbase, const void *vbase,
                          int64_t kv_token_stride, int64_t num_blocks, int32_t block_size,
                          int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                          int32_t dtype, const int32_t *cu_q, const int32_t *cu_k,
                          const int32_t *block_tables, int64_t bt_stride, int64_t num_seqs,
                          int64_t num_tokens, int64_t num_kv_tokens, int32_t max_seqlen_q,
                          float scale, int32_t *dev_status, void *stream, bool paged) {
  const int e = elem_size(dtype);
  if (e == 0) return fail(MI_ERR_INVALID, "unknown dtype");
  if (num_seqs < 0 || num_tokens < 0) return fail(MI_ERR_INVALID, "negative sizes");
  if (num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(MI_ERR_INVALID, "head counts and head_dim must be positive");
  if (num_q_heads % num_kv_heads != 0)
    return fail(MI_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads");
  if (head_dim > 256) return fail(MI_ERR_UNSUPPORTED, "head_dim > 256");
  if (paged && (num_blocks <= 0 || block_size <= 0 || bt_stride < 0))
    return fail(MI_ERR_INVALID, "paged cache dimensions must be positive");
  if (!paged && kv_token_stride < static_cast<int64_t>(num_kv_heads) * head_dim)
    return fail(MI_ERR_INVALID, "kv_token_stride smaller than one K/V row");
  if (num_tokens == 0 || num_seqs == 0) return MI_OK;
  if (max_seqlen_q <= 0) return fail(MI_ERR_INVALID, "max_seqlen_q must be positive");
  if (!out || !query || !kbase || !vbase || !cu_q || !cu_k || (paged && !block_tables))
    return fail(MI_ERR_INVALID, "null pointer");
  if (const int s = select_device(kbase)) return s;
  AttnParams p = {};
  p.out = out;
  p.query = query;
  p.key_base = static_cast<const char *>(kbase);
  p.value_base = static_cast<const char *>(vbase);
  p.kv_token_stride = kv_token_stride;
  p.kv_rows = num_kv_tokens;
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.cu_q = cu_q;
  p.cu_k = cu_k;
  p.num_seqs = num_seqs;
  p.num_tokens = num_tokens;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.head_dim = head_dim;
  p.scale_log2 = scale * kLog2eHost;
  p.status = dev_status;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = num_q_heads / num_kv_heads;
  const bool tc = prefill_tc_supported(dtype, head_dim, G, paged ? block_size : 16) &&
                  aligned16(kbase) && aligned16(vbase) && aligned16(query) && aligned16(out) &&
                  (paged || (kv_token_stride * e) % 16 == 0);
  if (tc) {
    // Mixed batch (some sequences have one query token, detectable on the host
    // when the tokens are fewer than num_seqs * max_seqlen_q, or all of them when
    // max_seqlen_q == 1): those rows go to the mma decode kernel, launched right
    // after the prefill kernel as its programmatic dependent, so its CTAs take
    // the SMs the prefill tail leaves free instead of running M=128 tensor tiles
    // for one token each.
    const bool mixed = paged && decode_mma_supported(dtype, head_dim, G, block_size) &&
                       num_seqs <= 65535 &&
                       static_cast<uint64_t>(num_blocks) * block_size < (1ull << 31) &&
                       (max_seqlen_q == 1 || num_tokens < num_seqs * static_cast<int64_t>(max_seqlen_q));
    p.mixed_decode = mixed ? 1 : 0;
    const cudaError_t te = launch_prefill_tc(p, dtype, G, max_seqlen_q, paged, st);
    if (te == cudaErrorNotSupported) {  // shape outside its grid limits: generic for every row
      p.mixed_decode = 0;
      return cuda_status(launch_attn_generic(p, dtype, paged, st));
    }
    if (te != cudaSuccess || !mixed) return cuda_status(te);
    DecodeParams d = {};
    d.out = out;
    d.query = query;
    d.key_cache = static_cast<const char *>(kbase);
    d.value_cache = static_cast<const char *>(vbase);
    d.block_tables = block_tables;
    d.bt_stride = bt_stride;
    d.num_blocks = num_blocks;
    d.block_size = block_size;
    d.num_q_heads = num_q_heads;
    d.num_kv_heads = num_kv_heads;
    d.scale_log2 = p.scale_log2;
    d.status = dev_status;
    d.cu_q = cu_q;
    d.cu_k = cu_k;
    return cuda_status(launch_decode_mma(d, dtype, head_dim, G, num_seqs, 1, false, st));
  }
  return cuda_status(launch_attn_generic(p, dtype, paged, st));
}

int mi_prefill_kernel_for(int32_t dtype, int32_t head_dim, int32_t num_q_heads,
                          int32_t num_kv_heads, int32_t block_size) {
  if (elem_size(dtype) == 0 || head_dim <= 0 || head_dim > 256 || num_q_heads <= 0 ||
      num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || block_size < 0)
    return fail(MI_ERR_INVALID, "invalid shape");
  const int G = num_q_heads / num_kv_heads;
  return prefill_tc_supported(dtype, head_dim, G, block_size == 0 ? 16 : block_size) ? 2 : 1;
}

int mi_paged_prefill(void *out, const void *query, const void *key_cache, const void *value_cache,
                     int64_t num_blocks, int32_t block_size, int32_t num_q_heads,
                     int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                     const int32_t *cu_seqlens_q, const int32_t *cu_seqlens_k,
                     const int32_t *block_tables, int64_t block_table_stride, int64_t num_seqs,
                     int64_t num_tokens, int32_t max_seqlen_q, float scale, int32_t *dev_status,
                     void *stream) {
  return prefill_common(out, query, key_cache, value_cache, 0, num_blocks, block_size, num_q_heads,
                        num_kv_heads, head_dim, dtype, cu_seqlens_q, cu_seqlens_k, block_tables,
                        block_table_stride, num_seqs, num_tokens, 0, max_seqlen_q, scale,
                        dev_status, stream, true);
}

int mi_varlen_prefill(void *out, const void *query, const void *keys, const void *values,
                      int64_t kv_token_stride, int32_t num_q_heads, int32_t num_kv_heads,
                      int32_t head_dim, int32_t dtype, const int32_t *cu_seqlens_q,
                      const int32_t *cu_seqlens_k, int64_t num_seqs, int64_t num_tokens,
                      int64_t num_kv_tokens, int32_t max_seqlen_q, float scale,
                      int32_t *dev_status, void *stream) {
  if (num_kv_tokens < 0) return fail(MI_ERR_INVALID, "num_kv_tokens must be >= 0");
  return prefill_common(out, query, keys, values, kv_token_stride, 0, 0, num_q_heads, num_kv_heads,
                        head_dim, dtype, cu_seqlens_q, cu_seqlens_k, nullptr, 0, num_seqs,
                        num_tokens, num_kv_tokens, max_seqlen_q, scale, dev_status, stream, false);
}

int mi_gather_paged_kv(void *out_keys, void *out_values, const void *key_cache,
                       const void *value_cache, int64_t num_blocks, int32_t block_size,
                       int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                       const int32_t *block_tables, int64_t block_table_stride,
                       const int32_t *cu_seqlens_k, int64_t num_seqs, int64_t out_rows,
                       int32_t max_context, int32_t *dev_status, void *stream) {
  const int e = elem_size(dtype);
  if (e == 0) return fail(MI_ERR_INVALID, "unknown dtype");
  if (num_blocks <= 0 || block_size <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(MI_ERR_INVALID, "cache dimensions must be positive");
  if (num_seqs < 0 || max_context < 0 || block_table_stride < 0 || out_rows < 0)
    return fail(MI_ERR_INVALID, "negative sizes");
  if (num_seqs > 65535) return fail(MI_ERR_UNSUPPORTED, "more than 65535 sequences in one call");
  if (num_seqs == 0 || max_context == 0) return MI_OK;
  if (!out_keys || !out_values || !key_cache || !value_cache || !block_tables || !cu_seqlens_k)
    return fail(MI_ERR_INVALID, "null pointer");
  if (const int s = select_device(key_cache)) return s;
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * e;
  GatherParams p;
  p.out_keys = static_cast<char *>(out_keys);
  p.out_values = static_cast<char *>(out_values);
  p.key_cache = static_cast<const char *>(key_cache);
  p.value_cache = static_cast<const char *>(value_cache);
  p.block_tables = block_tables;
  p.cu_seqlens_k = cu_seqlens_k;
  p.block_table_stride = block_table_stride;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.row_bytes = static_cast<int32_t>(row_bytes);
  // ~16 KB of rows per CTA per tensor.
  int64_t rows = 16384 / row_bytes;
  p.rows_per_cta = static_cast<int32_t>(rows < 1 ? 1 : rows);
  p.out_rows = out_rows;
  p.status = dev_status;
  const bool vec16 = row_bytes % 16 == 0 && aligned16(out_keys) && aligned16(out_values) &&
                     aligned16(key_cache) && aligned16(value_cache);
  return cuda_status(
      launch_gather(p, num_seqs, max_context, vec16, static_cast<cudaStream_t>(stream)));
}

int mi_copy_blocks(void *key_pool, void *value_pool, int32_t num_layers, int64_t layer_stride_bytes,
                   int64_t num_blocks, int64_t block_bytes, const int32_t *pairs, int64_t num_pairs,
                   int32_t *dev_status, void *stream) {
  if (num_layers <= 0 || num_blocks <= 0 || block_bytes <= 0)
    return fail(MI_ERR_INVALID, "pool dimensions must be positive");
  if (layer_stride_bytes < num_blocks * block_bytes)
    return fail(MI_ERR_INVALID, "layer_stride_bytes smaller than one layer");
  if (num_pairs < 0 || num_pairs > 2147483647) return fail(MI_ERR_INVALID, "num_pairs out of range");
  if (num_layers > 65535) return fail(MI_ERR_UNSUPPORTED, "more than 65535 layers");
  if (num_pairs == 0) return MI_OK;
  if (!key_pool || !value_pool || !pairs) return fail(MI_ERR_INVALID, "null pointer");
  if (const int s = select_device(key_pool)) return s;
  CowParams p;
  p.key_pool = static_cast<char *>(key_pool);
  p.value_pool = static_cast<char *>(value_pool);
  p.pairs = pairs;
  p.layer_stride_bytes = layer_stride_bytes;
  p.num_blocks = num_blocks;
  p.block_bytes = block_bytes;
  p.chunk_bytes = 8192;
  p.status = dev_status;
  const bool vec16 = aligned16(key_pool) && aligned16(value_pool) && block_bytes % 16 == 0 &&
                     layer_stride_bytes % 16 == 0;
  return cuda_status(launch_cow(p, num_layers, num_pairs, vec16, static_cast<cudaStream_t>(stream)));
}

int mi_wait_flag_selftest(const int32_t *flag, int64_t timeout_ns, int32_t *dev_status,
                          void *stream) {
  if (!flag || !dev_status) return fail(MI_ERR_INVALID, "null pointer");
  if (timeout_ns <= 0 || timeout_ns > 10000000000ll)
    return fail(MI_ERR_INVALID, "timeout_ns must be in (0, 10 s]");
  if (const int s = select_device(flag)) return s;
  return cuda_status(launch_wait_flag(flag, timeout_ns, dev_status, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
