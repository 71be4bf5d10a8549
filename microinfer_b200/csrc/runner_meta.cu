// Per-step attention metadata built on the device from a device-resident page
// table.  Replaces the reference runner's host-side assembly:
//   prepare_decode + _fill_decode_rows   microinfer/runner.py:160-188, 348-384
//   prepare_prefill + prepare_block_tables                  runner.py:298-346
// which walk every scheduled sequence in Python each step, build the block
// tables row by row and copy five tensors to the device.  Here the page table
// lives in HBM ([max_rows, max_pages] int32, one row per running sequence);
// each step the host sends one small int32 buffer -- a record per sequence and
// only the page-table entries that changed since the last step -- and one
// launch applies the changes and writes every metadata tensor.
//
// Record layout (int32 x 6 per sequence):
//   decode : row, num_tokens, last_token, num_pages, update_begin, update_count
//   prefill: row, start,      end,        num_pages, update_begin, update_count
// Update layout (int32 x 2): page-table column, page id.
//
// A sequence's row is owned by the warp (decode) or CTA (prefill) that handles
// the sequence, so its updates are ordered before its reads by __syncwarp /
// __syncthreads; rows are distinct within a step (checked by the host).  Bad
// rows, columns and page ids are flagged (MI_DEV_BAD_ROW / MI_DEV_BAD_BLOCK)
// and skipped; a token whose page is missing gets slot -1.
#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

namespace {

constexpr int kMetaRecord = 6;
constexpr int kDecodeWarps = 8;
constexpr int kPrefillThreads = 256;

struct RowRecord {
  int row, a, b, num_pages, upd_begin, upd_count;
};

__device__ __forceinline__ RowRecord load_record(const int32_t *records, int i) {
  const int32_t *r = records + static_cast<int64_t>(i) * kMetaRecord;
  return {r[0], r[1], r[2], r[3], r[4], r[5]};
}

__device__ __forceinline__ bool record_ok(const RowRecord &r, const RunnerMetaParams &p) {
  return r.row >= 0 && r.row < p.max_rows && r.num_pages >= 0 && r.num_pages <= p.max_pages &&
         r.upd_begin >= 0 && r.upd_count >= 0 && r.upd_begin <= p.num_updates - r.upd_count;
}

// Apply the record's page-table changes; threads [t0, t0 + stride) share the work.
__device__ __forceinline__ void apply_updates(const RowRecord &r, int32_t *trow,
                                              const RunnerMetaParams &p, int t0, int stride) {
  for (int u = t0; u < r.upd_count; u += stride) {
    const int32_t *e = p.updates + 2 * static_cast<int64_t>(r.upd_begin + u);
    const int col = e[0], page = e[1];
    if (col < 0 || col >= p.max_pages || page < 0 || page >= p.num_blocks) {
      flag_status(p.status, MI_DEV_BAD_BLOCK);
      continue;
    }
    trow[col] = page;
  }
}

__device__ __forceinline__ int32_t slot_at(const int32_t *trow, int num_pages, int64_t pos,
                                           const RunnerMetaParams &p) {
  const int64_t index = pos / p.block_size;
  if (pos < 0 || index >= num_pages) {
    flag_status(p.status, MI_DEV_BAD_BLOCK);
    return -1;
  }
  const int page = trow[index];
  if (page < 0 || page >= p.num_blocks) {
    flag_status(p.status, MI_DEV_BAD_BLOCK);
    return -1;
  }
  return static_cast<int32_t>(page * static_cast<int64_t>(p.block_size) + pos % p.block_size);
}

}  // namespace

// One warp per sequence.
__global__ void __launch_bounds__(kDecodeWarps * 32) decode_meta_kernel(const RunnerMetaParams p) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * kDecodeWarps + (threadIdx.x >> 5);
  if (i < p.num_seqs) {
    const RowRecord r = load_record(p.records, i);
    int32_t *bt = p.block_tables + static_cast<int64_t>(i) * p.table_width;
    if (!record_ok(r, p)) {
      if (lane == 0) {
        flag_status(p.status, MI_DEV_BAD_ROW);
        p.input_ids[i] = 0;
        p.positions[i] = 0;
        p.slot_mapping[i] = -1;
        p.context_lens[i] = 0;
      }
      for (int j = lane; j < p.table_width; j += 32) bt[j] = -1;
    } else {
      int32_t *trow = p.page_table + static_cast<int64_t>(r.row) * p.max_pages;
      apply_updates(r, trow, p, lane, 32);
      __syncwarp();
      if (lane == 0) {
        const int64_t pos = static_cast<int64_t>(r.a) - 1;  // num_tokens - 1
        p.input_ids[i] = r.b;
        p.positions[i] = pos;
        p.slot_mapping[i] = slot_at(trow, r.num_pages, pos, p);
        p.context_lens[i] = r.a;
      }
      for (int j = lane; j < p.table_width; j += 32) bt[j] = j < r.num_pages ? trow[j] : -1;
    }
  }
  pdl_launch_dependents();
}

// One CTA per sequence; the cumulative offsets of the sequences before it are
// summed by the CTA itself (a step schedules at most a few thousand sequences).
__global__ void __launch_bounds__(kPrefillThreads) prefill_meta_kernel(const RunnerMetaParams p) {
  __shared__ long long red[2][kPrefillThreads / 32];
  pdl_wait();
  const int i = blockIdx.x, tid = threadIdx.x;
  long long q_before = 0, k_before = 0;
  for (int j = tid; j < i; j += kPrefillThreads) {
    const int32_t *r = p.records + static_cast<int64_t>(j) * kMetaRecord;
    q_before += r[2] - r[1];
    k_before += r[2];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    q_before += __shfl_xor_sync(0xffffffffu, q_before, off);
    k_before += __shfl_xor_sync(0xffffffffu, k_before, off);
  }
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = q_before;
    red[1][tid >> 5] = k_before;
  }
  const RowRecord r = load_record(p.records, i);
  const bool ok = record_ok(r, p) && r.a >= 0 && r.b > r.a;
  int32_t *trow = ok ? p.page_table + static_cast<int64_t>(r.row) * p.max_pages : nullptr;
  if (ok) apply_updates(r, trow, p, tid, kPrefillThreads);
  __syncthreads();
  q_before = k_before = 0;
#pragma unroll
  for (int w = 0; w < kPrefillThreads / 32; ++w) {
    q_before += red[0][w];
    k_before += red[1][w];
  }
  if (tid == 0) {
    if (!ok) flag_status(p.status, MI_DEV_BAD_ROW);
    if (i == 0) {
      p.cu_seqlens_q[0] = 0;
      p.cu_seqlens_k[0] = 0;
    }
    p.cu_seqlens_q[i + 1] = static_cast<int32_t>(q_before + (r.b - r.a));
    p.cu_seqlens_k[i + 1] = static_cast<int32_t>(k_before + r.b);
  }
  const int n = ok ? r.b - r.a : 0;
  const int64_t q_end = q_before + n;
  if (ok && q_end <= p.num_tokens) {
    for (int t = tid; t < n; t += kPrefillThreads) {
      const int64_t o = q_before + t, pos = static_cast<int64_t>(r.a) + t;
      p.input_ids[o] = p.token_ids[o];
      p.positions[o] = pos;
      p.slot_mapping[o] = slot_at(trow, r.num_pages, pos, p);
    }
  } else if (ok && tid == 0) {
    flag_status(p.status, MI_DEV_BAD_ROW);  // ranges longer than the token buffer
  }
  if (p.block_tables) {
    int32_t *bt = p.block_tables + static_cast<int64_t>(i) * p.table_width;
    for (int j = tid; j < p.table_width; j += kPrefillThreads)
      bt[j] = ok && j < r.num_pages ? trow[j] : -1;
  }
  pdl_launch_dependents();
}

cudaError_t launch_decode_meta(const RunnerMetaParams &p, cudaStream_t stream) {
  if (p.num_seqs == 0) return cudaSuccess;
  const dim3 grid((p.num_seqs + kDecodeWarps - 1) / kDecodeWarps), block(kDecodeWarps * 32);
  return launch_pdl(decode_meta_kernel, grid, block, 0, stream, p);
}

cudaError_t launch_prefill_meta(const RunnerMetaParams &p, cudaStream_t stream) {
  if (p.num_seqs == 0) return cudaSuccess;
  return launch_pdl(prefill_meta_kernel, dim3(p.num_seqs), dim3(kPrefillThreads), 0, stream, p);
}

}  // namespace mi
