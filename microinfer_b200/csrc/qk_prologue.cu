// Attention prologue in one launch: per-head RMSNorm of q and k, rotary
// position embedding of q and k, and the store of k and v into the paged
// cache.  It replaces, on the path into paged attention, the reference's
//   q, _ = self.q_norm(q); k, _ = self.k_norm(k)     microinfer/layer/transformer.py:222-223
//   q = self.rotary.apply(q, position); same for k   transformer.py:224-225, layer/rope.py:6-21
//   store_kv(k, v at slot_mapping)                   layer/cached_attention.py:76-85
// with the reference's rounding points, so the results match its eager ops:
//   norm: y = round(x * (1 / sqrt(mean(x^2) + eps)) * w), all in fp32, one
//         rounding to the activation dtype (torch's F.rms_norm);
//   rope: on the rounded y widened to fp32, split-half
//           out[i]      = y[i] * cos[j] - y[i + D/2] * sin[j]
//           out[i+D/2]  = y[i+D/2] * cos[j] + y[i] * sin[j]      (j = i < D/2)
//         or interleaved
//           out[2j]     = y[2j] * cos[j] - y[2j+1] * sin[j]
//           out[2j+1]   = y[2j] * sin[j] + y[2j+1] * cos[j]
//         with every product and sum rounded separately (no fused multiply-add,
//         as the reference's element-wise tensor ops), then rounded once more.
// The cos/sin tables are the caller's (the model's RotaryCache, fp32
// [max_positions, D/2]); nothing here evaluates a trigonometric function.
//
// One warp per (token, head) of the packed qkv row [Hq | Hkv | Hkv] x D: lane
// L holds elements [L*E, L*E + E) with E = D/32, so the split-half partner of
// an element sits in lane L ^ 16 and the interleaved partner in the same lane.
// HBM-bound: every element is read once and written once.
#include <type_traits>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

namespace {

constexpr int kPrologueWarps = 8;

// E consecutive elements of T as one aligned vector access.
template <typename T, int E>
struct RowVec {
  static constexpr int kBytes = E * static_cast<int>(sizeof(T));
  using V = typename std::conditional<kBytes == 16, uint4,
                                      typename std::conditional<kBytes == 8, uint2, uint32_t>::type>::type;
  __device__ __forceinline__ static void load(const void *src, float (&x)[E]) {
    const V v = *reinterpret_cast<const V *>(src);
    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = Elem<T>::to_float(e[i]);
  }
  __device__ __forceinline__ static void store(void *dst, const float (&x)[E]) {
    V v;
    T *e = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = Elem<T>::from_float(x[i]);
    *reinterpret_cast<V *>(dst) = v;
  }
  __device__ __forceinline__ static void copy(void *dst, const void *src) {
    *reinterpret_cast<V *>(dst) = *reinterpret_cast<const V *>(src);
  }
};

}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__(kPrologueWarps * 32) qk_prologue_kernel(const QkPrologueParams p) {
  constexpr int E = D / 32;  // elements per lane
  using RV = RowVec<T, E>;
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * kPrologueWarps + warp;
  if (item < p.num_tokens * heads) {
    const int64_t t = item / heads;
    const int h = static_cast<int>(item - t * heads);
    const int kind = h < p.num_q_heads ? 0 : (h < p.num_q_heads + p.num_kv_heads ? 1 : 2);
    const char *src = p.qkv + t * p.qkv_stride_bytes + (static_cast<int64_t>(h) * D + lane * E) * sizeof(T);
    int64_t slot = -1;
    if (kind != 0) {
      slot = p.slot_mapping[t];
      if (slot < -1 || slot >= p.num_slots) {
        if (lane == 0) flag_status(p.status, MI_DEV_BAD_SLOT);
        slot = -1;
      }
    }
    const int kvh = h - p.num_q_heads - (kind == 2 ? p.num_kv_heads : 0);
    const int64_t cache_off = (slot * p.num_kv_heads + kvh) * D * static_cast<int64_t>(sizeof(T)) +
                              lane * E * static_cast<int64_t>(sizeof(T));
    if (kind == 2) {
      if (slot >= 0) RV::copy(p.value_cache + cache_off, src);
    } else {
      float x[E];
      RV::load(src, x);
      // RMSNorm (fp32, one rounding to T, as F.rms_norm)
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = 1.f / sqrtf(ss / static_cast<float>(D) + p.eps);
      const T *w = static_cast<const T *>(kind == 0 ? p.q_weight : p.k_weight) + lane * E;
      float y[E];
#pragma unroll
      for (int i = 0; i < E; ++i)
        y[i] = Elem<T>::to_float(Elem<T>::from_float(__fmul_rn(__fmul_rn(x[i], inv), Elem<T>::to_float(w[i]))));
      // RoPE on the rounded values
      const int64_t pos = p.positions_int64 ? static_cast<const int64_t *>(p.positions)[t]
                                            : static_cast<const int32_t *>(p.positions)[t];
      float out[E];
      if (pos < 0 || pos >= p.max_positions) {
        if (lane == 0) flag_status(p.status, MI_DEV_BAD_POSITION);
#pragma unroll
        for (int i = 0; i < E; ++i) out[i] = 0.f;
      } else if (p.interleaved) {
        const float *cs = p.cos_table + pos * (D / 2) + lane * (E / 2);
        const float *sn = p.sin_table + pos * (D / 2) + lane * (E / 2);
#pragma unroll
        for (int j = 0; j < E / 2; ++j) {
          const float c = cs[j], s = sn[j], a = y[2 * j], b = y[2 * j + 1];
          out[2 * j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
          out[2 * j + 1] = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
        }
      } else {
        const bool upper = lane >= 16;  // elements D/2 .. D-1
        const int j0 = (lane & 15) * E;
        float partner[E];
#pragma unroll
        for (int i = 0; i < E; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
#pragma unroll
        for (int i = 0; i < E; ++i) {
          const float c = p.cos_table[pos * (D / 2) + j0 + i], s = p.sin_table[pos * (D / 2) + j0 + i];
          out[i] = upper ? __fadd_rn(__fmul_rn(y[i], c), __fmul_rn(partner[i], s))
                         : __fsub_rn(__fmul_rn(y[i], c), __fmul_rn(partner[i], s));
        }
      }
      if (kind == 0)
        RV::store(p.q_out + t * p.q_out_stride_bytes + (static_cast<int64_t>(h) * D + lane * E) * sizeof(T), out);
      else if (slot >= 0)
        RV::store(p.key_cache + cache_off, out);
    }
  }
  pdl_launch_dependents();
}

template <typename T>
static cudaError_t launch_prologue_t(const QkPrologueParams &p, int D, cudaStream_t stream) {
  const int64_t items = p.num_tokens * (p.num_q_heads + 2 * p.num_kv_heads);
  const int64_t blocks = (items + kPrologueWarps - 1) / kPrologueWarps;
  if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(blocks)), block(kPrologueWarps * 32);
  if (D == 128) return launch_pdl(qk_prologue_kernel<T, 128>, grid, block, 0, stream, p);
  return launch_pdl(qk_prologue_kernel<T, 64>, grid, block, 0, stream, p);
}

cudaError_t launch_qk_prologue(const QkPrologueParams &p, int dtype, int D, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  if (dtype == MI_DTYPE_BFLOAT16) return launch_prologue_t<__nv_bfloat16>(p, D, stream);
  if (dtype == MI_DTYPE_FLOAT16) return launch_prologue_t<__half>(p, D, stream);
  return launch_prologue_t<float>(p, D, stream);
}

}  // namespace mi
