// Allocation-free split-K paged decode.
//
// Some callers cannot allocate device memory on the call path: a serving
// loop that reserved nearly all of HBM for the KV pool up front and forbids
// allocation afterwards, or a host runtime reaching this library through an
// FFI that only owns the buffers it was handed and has no device allocator to
// ask for a workspace.  mi_paged_decode_noalloc serves them: it runs the same
// decode kernels as mi_paged_decode, but the split-K partial states live in a
// fixed scratch array compiled into this library instead of a caller-provided
// workspace.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes (2 MiB)
// that every GPU loading the library holds until the process exits.  Host
// code cannot use the array's name as a device address, so on the first call
// on each device (with that device current) its address is looked up with
// cudaGetSymbolAddress and cached; make that first call outside any stream
// capture.  A failed lookup is not cached: the next call tries again.  With
// num_splits = 0 the split count is the library default capped to what the
// scratch holds (down to one split, which needs no scratch); an explicit
// split count that does not fit is rejected.  All calls share the one array.
// It starts zeroed (static storage), the split-K arrival counters at its start
// are left at zero by every launch, and every split state is written before it
// is read, so nothing needs clearing between calls; calls that overlap on the
// GPU (two streams, or two threads) race on the array and must be serialised
// by the caller.
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "split_merge.cuh"

namespace mi {

int capi_fail(int code, const char *msg);
int capi_select_device(const void *p);
bool decode_fast_supported(int dtype, int D, int G);
cudaError_t launch_decode_fast(const DecodeParams &p, int dtype, int D, int G, int64_t num_seqs,
                               int nsplit, bool wide, cudaStream_t stream);
bool decode_simt_wide(int dtype, int D, int G, int64_t ctas, int dev);
cudaError_t launch_attn_generic(const AttnParams &p, int dtype, bool paged, cudaStream_t stream);

constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;

static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {

constexpr int kMaxDevices = 64;
float *g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device.  Only a
// successful lookup is kept; a failed one (for instance made while a stream
// capture was active) clears its non-sticky error and is retried next call.
int scratch_address(float **out) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return capi_fail(static_cast<int>(e), "cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return capi_fail(MI_ERR_UNSUPPORTED, "device index >= 64");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t se = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (se != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return capi_fail(static_cast<int>(se != cudaSuccess ? se : cudaErrorInvalidSymbol),
                       "cudaGetSymbolAddress of the decode scratch array failed");
    }
    g_scratch_ptr[dev] = static_cast<float *>(ptr);
  }
  *out = g_scratch_ptr[dev];
  return MI_OK;
}

}  // namespace
}  // namespace mi

using namespace mi;

extern "C" int mi_paged_decode_noalloc(void *out, const void *query, const void *key_cache,
                                       const void *value_cache, int64_t num_blocks,
                                       int32_t block_size, int32_t num_q_heads,
                                       int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
                                       const int32_t *block_tables, int64_t block_table_stride,
                                       const int32_t *context_lens, int64_t num_seqs, float scale,
                                       int32_t num_splits, int32_t *dev_status, void *stream) {
  if (dtype != MI_DTYPE_FLOAT32 && dtype != MI_DTYPE_FLOAT16 && dtype != MI_DTYPE_BFLOAT16)
    return capi_fail(MI_ERR_INVALID, "unknown dtype");
  if (num_seqs < 0) return capi_fail(MI_ERR_INVALID, "num_seqs must be >= 0");
  if (num_blocks <= 0 || block_size <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return capi_fail(MI_ERR_INVALID, "cache dimensions must be positive");
  if (num_q_heads % num_kv_heads != 0)
    return capi_fail(MI_ERR_INVALID, "num_q_heads must be divisible by num_kv_heads");
  if (head_dim > 256) return capi_fail(MI_ERR_UNSUPPORTED, "head_dim > 256");
  if (block_table_stride < 0) return capi_fail(MI_ERR_INVALID, "block_table_stride must be >= 0");
  if (num_splits < 0 || num_splits > 1024)
    return capi_fail(MI_ERR_INVALID, "num_splits out of range");
  if (num_seqs > 65535) return capi_fail(MI_ERR_UNSUPPORTED, "more than 65535 sequences in one call");
  if (num_seqs == 0) return MI_OK;
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return capi_fail(MI_ERR_INVALID, "null pointer");
  if (const int s = capi_select_device(key_cache)) return s;

  const int G = num_q_heads / num_kv_heads;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float scale_log2 = scale * 1.4426950408889634f;
  const bool fast = decode_fast_supported(dtype, head_dim, G) &&
                    (reinterpret_cast<uintptr_t>(key_cache) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(value_cache) & 15u) == 0 &&
                    (reinterpret_cast<uintptr_t>(query) & 15u) == 0;
  if (!fast) {  // the generic kernel needs no scratch at all
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
    p.scale_log2 = scale_log2;
    p.status = dev_status;
    const cudaError_t e = launch_attn_generic(p, dtype, true, st);
    return e == cudaSuccess ? MI_OK : capi_fail(static_cast<int>(e), cudaGetErrorString(e));
  }

  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t ctx_bound = block_table_stride * block_size;
  int nsplit = num_splits;
  if (nsplit == 0) {
    nsplit = mi_paged_decode_default_splits(
        num_seqs, num_kv_heads, static_cast<int32_t>(ctx_bound > INT32_MAX ? INT32_MAX : ctx_bound),
        dev);
    // Cap the default to the split states the scratch holds.
    const int64_t per_split = num_seqs * num_q_heads * (static_cast<int64_t>(head_dim) + 2) *
                              static_cast<int64_t>(sizeof(float));
    const int64_t fit = (static_cast<int64_t>(kNoAllocScratchBytes) - kSplitCounterBytes) / per_split;
    if (nsplit > fit) nsplit = fit > 1 ? static_cast<int>(fit) : 1;
  }
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
  p.scale_log2 = scale_log2;
  p.status = dev_status;
  if (nsplit > 1) {
    if (num_seqs * num_kv_heads > kSplitCounters)
      return capi_fail(MI_ERR_UNSUPPORTED, "split-K decode takes at most 16384 (sequence, kv "
                                           "head) pairs per launch; use num_splits=1");
    const size_t need = mi_paged_decode_workspace_bytes(num_seqs, num_q_heads, head_dim, nsplit);
    if (need > kNoAllocScratchBytes)
      return capi_fail(MI_ERR_INVALID,
                       "split-K state exceeds the 2 MiB built-in scratch of "
                       "mi_paged_decode_noalloc (64 KiB + num_seqs * num_q_heads * "
                       "num_splits * (head_dim + 2) * 4 bytes); use fewer splits or "
                       "mi_paged_decode");
    float *scratch = nullptr;
    if (const int s = scratch_address(&scratch)) return s;
    set_split_workspace(p, scratch, num_seqs, num_q_heads, head_dim, nsplit);
  }
  const cudaError_t e =
      launch_decode_fast(p, dtype, head_dim, G, num_seqs, nsplit,
                         decode_simt_wide(dtype, head_dim, G, num_seqs * num_kv_heads * nsplit, dev), st);
  return e == cudaSuccess ? MI_OK : capi_fail(static_cast<int>(e), cudaGetErrorString(e));
}
