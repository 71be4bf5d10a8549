// Generic paged / dense attention kernel (sm_100a).
//
// attn_generic_kernel: one warp per (query token, q head); walks the keys of
// its sequence one at a time with a warp-reduced dot product and an online
// softmax.  It covers every shape the reference accepts (any head_dim <= 256,
// any block size, fp32/fp16/bf16, paged or dense K/V, decode, chunked prefill
// and mixed batches) and is the path for shapes the specialised decode
// (decode.cu) and tensor-core prefill (prefill_tc.cu) kernels do not take.
#include <float.h>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

namespace {
constexpr unsigned kFull = 0xffffffffu;
}

template <typename T, bool PAGED, int EPL>
__global__ void __launch_bounds__(128) attn_generic_kernel(AttnParams p) {
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (item >= p.num_tokens * p.num_q_heads) return;
  const int64_t t = item / p.num_q_heads;
  const int h = static_cast<int>(item - t * p.num_q_heads);
  const int D = p.head_dim;

  int64_t seq, q_start, q_len, ctx;
  if (p.cu_q == nullptr) {
    seq = t;
    q_start = t;
    q_len = 1;
  } else {
    int64_t lo = 0, hi = p.num_seqs - 1;  // largest s with cu_q[s] <= t
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (p.cu_q[mid] <= t) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    q_start = p.cu_q[seq];
    q_len = p.cu_q[seq + 1] - q_start;
  }
  int64_t kv_row0 = 0;
  if (p.cu_k != nullptr) {
    kv_row0 = p.cu_k[seq];
    ctx = p.cu_k[seq + 1] - kv_row0;
  } else {
    ctx = p.context_lens[seq];
  }
  const int64_t pos = ctx - q_len + (t - q_start);  // absolute position of this query row
  int64_t nkeys = min(pos + 1, ctx);
  if (PAGED && nkeys > p.bt_stride * p.block_size) {  // beyond what the table row addresses
    if (lane == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    nkeys = p.bt_stride * p.block_size;
  }
  const int kvh = h / (p.num_q_heads / p.num_kv_heads);

  const T *q = static_cast<const T *>(p.query) + (t * p.num_q_heads + h) * D;
  float qv[EPL], acc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < D ? Elem<T>::to_float(q[d]) * p.scale_log2 : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int32_t *table = PAGED ? p.block_tables + seq * p.bt_stride : nullptr;
  for (int64_t j = 0; j < nkeys; ++j) {
    int64_t row;
    if (PAGED) {
      const int64_t col = j / p.block_size;
      const int64_t blk = col < p.bt_stride ? table[col] : -1;
      if (blk < 0 || blk >= p.num_blocks) {
        if (lane == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
        continue;
      }
      row = ((blk * p.block_size + j % p.block_size) * p.num_kv_heads + kvh) * D;
    } else {
      if (kv_row0 < 0 || kv_row0 + j >= p.kv_rows) {
        if (lane == 0) flag_status(p.status, MI_DEV_BAD_SLOT);
        break;
      }
      row = (kv_row0 + j) * p.kv_token_stride + static_cast<int64_t>(kvh) * D;
    }
    const T *kr = reinterpret_cast<const T *>(p.key_base) + row;
    const T *vr = reinterpret_cast<const T *>(p.value_base) + row;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int d = lane + 32 * i;
      if (d < D) s += qv[i] * Elem<T>::to_float(kr[d]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
    const float m_new = fmaxf(m, s);
    const float alpha = fast_exp2(m - m_new);  // exp2(-inf) = 0 on the first key
    const float pe = fast_exp2(s - m_new);
    l = l * alpha + pe;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int d = lane + 32 * i;
      const float v = d < D ? Elem<T>::to_float(vr[d]) : 0.f;
      acc[i] = acc[i] * alpha + pe * v;
    }
    m = m_new;
  }
  T *o = static_cast<T *>(p.out) + (t * p.num_q_heads + h) * D;
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int d = lane + 32 * i;
    if (d < D) o[d] = Elem<T>::from_float(acc[i] * inv);
  }
  pdl_launch_dependents();
}

template <typename T, bool PAGED>
static cudaError_t launch_generic_t(const AttnParams &p, cudaStream_t stream) {
  const int64_t items = p.num_tokens * p.num_q_heads;
  if (items == 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>((items + 3) / 4));
  const dim3 block(128);
  const int epl = (p.head_dim + 31) / 32;
  switch (epl) {
    case 1: return launch_pdl(attn_generic_kernel<T, PAGED, 1>, grid, block, 0, stream, p);
    case 2: return launch_pdl(attn_generic_kernel<T, PAGED, 2>, grid, block, 0, stream, p);
    case 3:
    case 4: return launch_pdl(attn_generic_kernel<T, PAGED, 4>, grid, block, 0, stream, p);
    default: return launch_pdl(attn_generic_kernel<T, PAGED, 8>, grid, block, 0, stream, p);
  }
}

cudaError_t launch_attn_generic(const AttnParams &p, int dtype, bool paged, cudaStream_t stream) {
  if (dtype == MI_DTYPE_FLOAT32)
    return paged ? launch_generic_t<float, true>(p, stream) : launch_generic_t<float, false>(p, stream);
  if (dtype == MI_DTYPE_FLOAT16)
    return paged ? launch_generic_t<__half, true>(p, stream) : launch_generic_t<__half, false>(p, stream);
  return paged ? launch_generic_t<__nv_bfloat16, true>(p, stream)
               : launch_generic_t<__nv_bfloat16, false>(p, stream);
}

}  // namespace mi
