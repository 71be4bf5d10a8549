// Data-movement kernels of the paged KV-cache path: store_kvcache (append
// this step's K/V into pool slots), the block-table gather into contiguous
// request-major K/V, and device-side copy-on-write of whole pages across all
// layers.  All are HBM-bound byte copies: 16-byte vector loads/stores when
// every row and base pointer is 16-byte aligned, element copies otherwise.
// Block / slot ids are range-checked on the device; a bad id is skipped and
// reported in the status word, never dereferenced.
#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

// ---------------------------------------------------------------------------
// store_kvcache
// ---------------------------------------------------------------------------
// Resolve token t to a destination row (block * bs + offset) or -1 to skip.
template <typename I, bool SLOTS>
__device__ __forceinline__ int64_t store_dest_row(const StoreParams &p, int64_t t) {
  if (SLOTS) {
    const int64_t slot = static_cast<int64_t>(static_cast<const I *>(p.idx0)[t]);
    if (slot == -1) return -1;  // padding row
    if (slot < -1 || slot >= p.num_blocks * p.block_size) {
      flag_status(p.status, MI_DEV_BAD_SLOT);
      return -1;
    }
    return slot;
  } else {
    const int64_t blk = static_cast<int64_t>(static_cast<const I *>(p.idx0)[t]);
    const int64_t off = static_cast<int64_t>(static_cast<const I *>(p.idx1)[t]);
    if (blk < 0 || blk >= p.num_blocks || off < 0 || off >= p.block_size) {
      flag_status(p.status, MI_DEV_BAD_SLOT);
      return -1;
    }
    return blk * p.block_size + off;
  }
}

// One CTA per group of tokens; each thread moves 16-byte vectors of K and V.
template <typename I, bool SLOTS>
__global__ void __launch_bounds__(256) store_kv_vec16_kernel(StoreParams p) {
  pdl_wait();
  const int vecs_per_row = p.row_bytes >> 4;
  const int64_t total = p.num_tokens * vecs_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vecs_per_row;
    const int v = static_cast<int>(i - t * vecs_per_row);
    const int64_t row = store_dest_row<I, SLOTS>(p, t);
    if (row < 0) continue;
    const uint4 kv = *reinterpret_cast<const uint4 *>(p.keys + t * p.key_stride_bytes + v * 16);
    const uint4 vv = *reinterpret_cast<const uint4 *>(p.values + t * p.value_stride_bytes + v * 16);
    *reinterpret_cast<uint4 *>(p.key_cache + row * p.row_bytes + v * 16) = kv;
    *reinterpret_cast<uint4 *>(p.value_cache + row * p.row_bytes + v * 16) = vv;
  }
  pdl_launch_dependents();
}

// Unaligned fallback: element-size copies (2 or 4 bytes).
template <typename I, bool SLOTS, typename W>
__global__ void __launch_bounds__(256) store_kv_scalar_kernel(StoreParams p) {
  pdl_wait();
  const int per_row = p.row_bytes / static_cast<int>(sizeof(W));
  const int64_t total = p.num_tokens * per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / per_row;
    const int e = static_cast<int>(i - t * per_row);
    const int64_t row = store_dest_row<I, SLOTS>(p, t);
    if (row < 0) continue;
    const W k = reinterpret_cast<const W *>(p.keys + t * p.key_stride_bytes)[e];
    const W v = reinterpret_cast<const W *>(p.values + t * p.value_stride_bytes)[e];
    reinterpret_cast<W *>(p.key_cache + row * p.row_bytes)[e] = k;
    reinterpret_cast<W *>(p.value_cache + row * p.row_bytes)[e] = v;
  }
  pdl_launch_dependents();
}

template <typename I, bool SLOTS>
static cudaError_t launch_store_typed(const StoreParams &p, int elem_bytes, bool vec16,
                                      cudaStream_t stream) {
  const int threads = 256;
  const int64_t per_row = vec16 ? (p.row_bytes >> 4) : (p.row_bytes / elem_bytes);
  const int64_t total = p.num_tokens * per_row;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count_current()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (vec16)
    return launch_pdl(store_kv_vec16_kernel<I, SLOTS>, dim3((unsigned)blocks), dim3(threads), 0,
                      stream, p);
  if (elem_bytes == 4)
    return launch_pdl(store_kv_scalar_kernel<I, SLOTS, uint32_t>, dim3((unsigned)blocks),
                      dim3(threads), 0, stream, p);
  return launch_pdl(store_kv_scalar_kernel<I, SLOTS, uint16_t>, dim3((unsigned)blocks),
                    dim3(threads), 0, stream, p);
}

cudaError_t launch_store_kv(const StoreParams &p, int index_dtype, bool slots, int elem_bytes,
                            bool vec16, cudaStream_t stream) {
  if (index_dtype == MI_INDEX_INT32)
    return slots ? launch_store_typed<int32_t, true>(p, elem_bytes, vec16, stream)
                 : launch_store_typed<int32_t, false>(p, elem_bytes, vec16, stream);
  return slots ? launch_store_typed<int64_t, true>(p, elem_bytes, vec16, stream)
               : launch_store_typed<int64_t, false>(p, elem_bytes, vec16, stream);
}

// ---------------------------------------------------------------------------
// block-table gather
// ---------------------------------------------------------------------------
// grid (ceil(max_context / rows_per_cta), num_seqs): CTA copies a run of
// logical rows of one sequence, 16 bytes per thread per step.
template <bool VEC16>
__global__ void __launch_bounds__(256) gather_kernel(GatherParams p) {
  pdl_wait();
  const int64_t seq = blockIdx.y;
  const int64_t base = p.cu_seqlens_k[seq];
  const int64_t ctx = p.cu_seqlens_k[seq + 1] - base;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * p.rows_per_cta;
  if (row0 >= ctx) return;
  const int64_t nrows = min(static_cast<int64_t>(p.rows_per_cta), ctx - row0);
  const int unit = VEC16 ? 16 : 1;
  const int per_row = p.row_bytes / unit;
  const int64_t total = nrows * per_row;
  const int32_t *table = p.block_tables + seq * p.block_table_stride;
  for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
    const int64_t r = i / per_row;
    const int e = static_cast<int>(i - r * per_row);
    const int64_t pos = row0 + r;
    const int64_t col = pos / p.block_size;
    const int64_t blk = col < p.block_table_stride ? table[col] : -1;
    if (blk < 0 || blk >= p.num_blocks) {
      flag_status(p.status, MI_DEV_BAD_BLOCK);
      continue;
    }
    const int64_t src_row = blk * p.block_size + pos % p.block_size;
    const int64_t dst_row = base + pos;
    if (dst_row < 0 || dst_row >= p.out_rows) {
      flag_status(p.status, MI_DEV_BAD_SLOT);
      continue;
    }
    if (VEC16) {
      const uint4 k = *reinterpret_cast<const uint4 *>(p.key_cache + src_row * p.row_bytes + e * 16);
      const uint4 v = *reinterpret_cast<const uint4 *>(p.value_cache + src_row * p.row_bytes + e * 16);
      *reinterpret_cast<uint4 *>(p.out_keys + dst_row * p.row_bytes + e * 16) = k;
      *reinterpret_cast<uint4 *>(p.out_values + dst_row * p.row_bytes + e * 16) = v;
    } else {
      p.out_keys[dst_row * p.row_bytes + e] = p.key_cache[src_row * p.row_bytes + e];
      p.out_values[dst_row * p.row_bytes + e] = p.value_cache[src_row * p.row_bytes + e];
    }
  }
  pdl_launch_dependents();
}

cudaError_t launch_gather(const GatherParams &p, int64_t num_seqs, int32_t max_context, bool vec16,
                          cudaStream_t stream) {
  const int64_t gx = (static_cast<int64_t>(max_context) + p.rows_per_cta - 1) / p.rows_per_cta;
  if (gx <= 0 || num_seqs <= 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(num_seqs));
  if (vec16) return launch_pdl(gather_kernel<true>, grid, dim3(256), 0, stream, p);
  return launch_pdl(gather_kernel<false>, grid, dim3(256), 0, stream, p);
}

// ---------------------------------------------------------------------------
// copy-on-write of whole pages across every layer of a pool
// ---------------------------------------------------------------------------
// grid (num_pairs, num_layers, 2 * chunks): z selects K/V and the chunk.
template <bool VEC16>
__global__ void __launch_bounds__(256) cow_kernel(CowParams p) {
  pdl_wait();
  const int64_t pair = blockIdx.x;
  const int64_t layer = blockIdx.y;
  const int kv = blockIdx.z & 1;
  const int64_t chunk = blockIdx.z >> 1;
  const int64_t src = p.pairs[2 * pair];
  const int64_t dst = p.pairs[2 * pair + 1];
  if (src < 0 || src >= p.num_blocks || dst < 0 || dst >= p.num_blocks) {
    if (threadIdx.x == 0 && layer == 0 && blockIdx.z == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    return;
  }
  char *pool = kv ? p.value_pool : p.key_pool;
  const char *s = pool + layer * p.layer_stride_bytes + src * p.block_bytes;
  char *d = pool + layer * p.layer_stride_bytes + dst * p.block_bytes;
  const int64_t begin = chunk * p.chunk_bytes;
  const int64_t end = min(begin + p.chunk_bytes, p.block_bytes);
  if (VEC16) {
    for (int64_t o = begin + threadIdx.x * 16; o < end; o += blockDim.x * 16)
      *reinterpret_cast<uint4 *>(d + o) = *reinterpret_cast<const uint4 *>(s + o);
  } else {
    for (int64_t o = begin + threadIdx.x; o < end; o += blockDim.x) d[o] = s[o];
  }
  pdl_launch_dependents();
}

cudaError_t launch_cow(const CowParams &p, int32_t num_layers, int64_t num_pairs, bool vec16,
                       cudaStream_t stream) {
  if (num_pairs <= 0 || num_layers <= 0) return cudaSuccess;
  const int64_t chunks = (p.block_bytes + p.chunk_bytes - 1) / p.chunk_bytes;
  dim3 grid(static_cast<unsigned>(num_pairs), static_cast<unsigned>(num_layers),
            static_cast<unsigned>(2 * chunks));
  if (vec16) return launch_pdl(cow_kernel<true>, grid, dim3(256), 0, stream, p);
  return launch_pdl(cow_kernel<false>, grid, dim3(256), 0, stream, p);
}

// ---------------------------------------------------------------------------
// bounded-wait self test
// ---------------------------------------------------------------------------
__global__ void wait_flag_kernel(const int32_t *flag, int64_t timeout_ns, int32_t *status) {
  if (threadIdx.x != 0) return;
  const uint64_t start = global_ns();
  const volatile int32_t *f = flag;
  while (*f == 0) {
    if (global_ns() - start > static_cast<uint64_t>(timeout_ns)) {
      flag_status(status, MI_DEV_TIMEOUT);
      return;
    }
    __nanosleep(1000);
  }
}

cudaError_t launch_wait_flag(const int32_t *flag, int64_t timeout_ns, int32_t *status,
                             cudaStream_t stream) {
  wait_flag_kernel<<<1, 32, 0, stream>>>(flag, timeout_ns, status);
  return cudaGetLastError();
}

}  // namespace mi
