// Attention prologue in one launch: per-head RMSNorm of q and k, rotary
// position embedding of q and k, and the store of k and v into the paged
// cache.  It replaces, on the path into paged attention, the reference's
//   q, _ = self.q_norm(q); k, _ = self.k_norm(k)     microinfer/layer/transformer.py:222-223
//   q = self.rotary.apply(q, position); same for k   transformer.py:224-225, layer/rope.py:6-21
//   store_kv(k, v at slot_mapping)                   layer/cached_attention.py:76-85
// with the reference's rounding points, so the results match its eager ops:
//   norm: y = round(x * rsqrt(mean(x^2) + eps) * w), all in fp32, one rounding
//         to the activation dtype (torch's F.rms_norm; the reciprocal square root
//         is the hardware one, within 2 ulp of 1/sqrt in fp32 as in torch's CUDA
//         kernel, so a 16-bit result can rarely differ by one unit from a CPU run);
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
// One CTA per token, 2 warps over the token's Hq + 2 Hkv head rows.  A head row
// spans a group of G = D / E lanes, E = 16 / sizeof(T) elements per lane (one
// 16-byte vector), so a warp covers 32 / G rows per instruction; each warp
// loads 8 such row groups before it processes any (4 KB in flight per warp for
// bf16).  The split-half partner of an element sits in lane ^ G/2 of its group,
// the interleaved partner in the same lane.  Position, slot, the cos/sin
// coefficients and the two weight vectors are read once per warp for all of
// the token's heads.  Products and sums use the packed f32x2 instructions
// with explicit round-to-nearest (each lane rounded exactly as __fmul_rn /
// __fadd_rn; a negated operand turns a sum into the reference's difference
// exactly).  HBM-bound: every element is read once and written once.
#include <type_traits>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

namespace {

constexpr int kPrologueThreads = 64;
constexpr int kPrologueWarps = kPrologueThreads / 32;
constexpr int kRowsPerWarp = 8;  // row groups per warp loaded ahead

// E consecutive elements of T as one aligned vector.
template <typename T, int E>
struct RowVec {
  static constexpr int kBytes = E * static_cast<int>(sizeof(T));
  using V = typename std::conditional<kBytes == 16, uint4,
                                      typename std::conditional<kBytes == 8, uint2, uint32_t>::type>::type;
  static constexpr int kWords = kBytes / 4;
  __device__ __forceinline__ static void to_float(const V &v, float (&x)[E]) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      // exact widening by bit placement (plain ALU ops)
      const uint32_t *w = reinterpret_cast<const uint32_t *>(&v);
#pragma unroll
      for (int i = 0; i < E / 2; ++i) {
        x[2 * i] = __uint_as_float(w[i] << 16);
        x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    } else {
      const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
      for (int i = 0; i < E; ++i) x[i] = Elem<T>::to_float(e[i]);
    }
  }
  __device__ __forceinline__ static V from_float(const float (&x)[E]) {
    V v;
    T *e = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = Elem<T>::from_float(x[i]);
    return v;
  }
  __device__ __forceinline__ static uint32_t word(const V &v, int i) {
    return reinterpret_cast<const uint32_t *>(&v)[i];
  }
  __device__ __forceinline__ static void set_word(V &v, int i, uint32_t w) {
    reinterpret_cast<uint32_t *>(&v)[i] = w;
  }
};

// Round E fp32 values to T and return them packed; `y` receives the rounded
// values widened back to fp32 (bf16: one packed conversion per pair, widened
// back by bit placement).
template <typename T, int E, typename V>
__device__ __forceinline__ V round_pack(const float (&x)[E], float (&y)[E]) {
  V v;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    uint32_t *w = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
    for (int i = 0; i < E; i += 2) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(x[i], x[i + 1]);
      w[i / 2] = *reinterpret_cast<const uint32_t *>(&b);
      y[i] = __uint_as_float(w[i / 2] << 16);
      y[i + 1] = __uint_as_float(w[i / 2] & 0xffff0000u);
    }
  } else {
    T *e = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      e[i] = Elem<T>::from_float(x[i]);
      y[i] = Elem<T>::to_float(e[i]);
    }
  }
  return v;
}

// n consecutive fp32 values as one vector load (n = 1, 2 or 4).
template <int N>
__device__ __forceinline__ void load_f32(const float *src, float (&dst)[N]) {
  if constexpr (N == 4) {
    const float4 v = *reinterpret_cast<const float4 *>(src);
    dst[0] = v.x, dst[1] = v.y, dst[2] = v.z, dst[3] = v.w;
  } else if constexpr (N == 2) {
    const float2 v = *reinterpret_cast<const float2 *>(src);
    dst[0] = v.x, dst[1] = v.y;
  } else {
    dst[0] = *src;
  }
}

}  // namespace

template <typename T, int D>
__global__ void __launch_bounds__(kPrologueThreads, 10) qk_prologue_kernel(const QkPrologueParams p) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));  // elements per lane: one 16-byte vector
  constexpr int G = D / E;                             // lanes per head row
  constexpr int R = 32 / G;                            // rows one warp instruction covers
  constexpr int kPass = kRowsPerWarp;                  // row groups loaded before any is used
  static_assert(G >= 2 && G <= 32 && 32 % G == 0, "a head row must span a power-of-two lane group");
  using RV = RowVec<T, E>;
  using V = typename RV::V;
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gl = lane & (G - 1), sub = lane / G;  // lane within its row, row within the warp
  const int64_t t = blockIdx.x;
  const int hq = p.num_q_heads, hkv = p.num_kv_heads, heads = hq + 2 * hkv;

  const int64_t pos = p.positions_int64 ? static_cast<const int64_t *>(p.positions)[t]
                                        : static_cast<const int32_t *>(p.positions)[t];
  const bool pos_ok = pos >= 0 && pos < p.max_positions;
  int64_t slot = p.slot_mapping[t];
  const bool slot_bad = slot < -1 || slot >= p.num_slots;
  if (slot_bad) slot = -1;
  if (threadIdx.x == 0) {
    if (!pos_ok) flag_status(p.status, MI_DEV_BAD_POSITION);
    if (slot_bad) flag_status(p.status, MI_DEV_BAD_SLOT);
  }

  // Rotation coefficients of this lane's elements (the same for every head).
  float cs[E], sn[E];
#pragma unroll
  for (int i = 0; i < E; ++i) cs[i] = sn[i] = 0.f;  // bad positions: rows are zeroed below
  if (pos_ok) {
    if (p.interleaved) {
      const int64_t off = pos * (D / 2) + gl * (E / 2);
#pragma unroll
      for (int j = 0; j < E / 2; j += 4) {
        float c4[4], s4[4];
        load_f32<(E / 2 < 4 ? E / 2 : 4)>(p.cos_table + off + j, reinterpret_cast<float(&)[(E / 2 < 4 ? E / 2 : 4)]>(c4));
        load_f32<(E / 2 < 4 ? E / 2 : 4)>(p.sin_table + off + j, reinterpret_cast<float(&)[(E / 2 < 4 ? E / 2 : 4)]>(s4));
#pragma unroll
        for (int u = 0; u < (E / 2 < 4 ? E / 2 : 4); ++u)
          cs[2 * (j + u)] = cs[2 * (j + u) + 1] = c4[u], sn[2 * (j + u)] = sn[2 * (j + u) + 1] = s4[u];
      }
    } else {
      const int64_t off = pos * (D / 2) + (gl & (G / 2 - 1)) * E;
#pragma unroll
      for (int j = 0; j < E; j += 4) {
        load_f32<4>(p.cos_table + off + j, reinterpret_cast<float(&)[4]>(cs[j]));
        load_f32<4>(p.sin_table + off + j, reinterpret_cast<float(&)[4]>(sn[j]));
      }
    }
  }
  // Norm weights of this lane's elements, kept packed.
  const V wq = *reinterpret_cast<const V *>(static_cast<const T *>(p.q_weight) + gl * E);
  const V wk = *reinterpret_cast<const V *>(static_cast<const T *>(p.k_weight) + gl * E);
  const bool upper = gl >= G / 2;  // split-half: elements D/2 .. D-1
  const int64_t lane_off = gl * E * static_cast<int64_t>(sizeof(T));
  const char *row0 = p.qkv + t * p.qkv_stride_bytes + lane_off;
  constexpr int kStep = kPrologueWarps * R * kPass;  // rows per CTA pass

  for (int base = 0; base < heads; base += kStep) {
    V raw[kPass];
#pragma unroll
    for (int j = 0; j < kPass; ++j) {
      const int h = base + (j * kPrologueWarps + warp) * R + sub;
      raw[j] = h < heads ? *reinterpret_cast<const V *>(row0 + static_cast<int64_t>(h) * D * sizeof(T)) : V{};
    }
#pragma unroll
    for (int j = 0; j < kPass; ++j) {
      const int h0 = base + (j * kPrologueWarps + warp) * R;
      if (h0 >= heads) break;  // warp-uniform
      const int h = h0 + sub;
      if (h0 >= hq + hkv) {  // every row of the group is a v row (warp-uniform): copy only
        if (h < heads && slot >= 0)
          *reinterpret_cast<V *>(p.value_cache + (slot * hkv + (h - hq - hkv)) * D * static_cast<int64_t>(sizeof(T)) +
                                 lane_off) = raw[j];
        continue;
      }
      // every lane runs the q/k math (v and out-of-range lanes of a mixed group
      // discard it), so the shuffles below see whole groups
      float x[E];
      RV::to_float(raw[j], x);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < E; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float inv = rsqrtf(ss / static_cast<float>(D) + p.eps);
      float w[E];
      RV::to_float(h < hq ? wq : wk, w);
      // RMSNorm: fp32, one rounding to T (F.rms_norm)
      float y[E];
#pragma unroll
      for (int i = 0; i < E; i += 2) {
        const float2 v2 = fmul2(fmul2(make_float2(x[i], x[i + 1]), make_float2(inv, inv)),
                                make_float2(w[i], w[i + 1]));
        y[i] = v2.x, y[i + 1] = v2.y;
      }
      const V yb = round_pack<T, E, V>(y, y);  // the rounded norm output, as the reference holds it
      float out[E];
      if (p.interleaved) {
        // out[2j] = a c - b s, out[2j+1] = a s + b c
#pragma unroll
        for (int i = 0; i < E; i += 2) {
          const float2 m1 = fmul2(make_float2(y[i], y[i]), make_float2(cs[i], sn[i]));
          const float2 m2 = fmul2(make_float2(y[i + 1], y[i + 1]), make_float2(sn[i], cs[i]));
          const float2 o = fadd2(m1, make_float2(-m2.x, m2.y));
          out[i] = o.x, out[i + 1] = o.y;
        }
      } else {
        // partner elements (i +- D/2) from lane ^ G/2, moved as packed T words
        V pb;
#pragma unroll
        for (int wd = 0; wd < RV::kWords; ++wd)
          RV::set_word(pb, wd, __shfl_xor_sync(0xffffffffu, RV::word(yb, wd), G / 2));
        float partner[E];
        RV::to_float(pb, partner);
        // lower: y c - partner s; upper: y c + partner s
#pragma unroll
        for (int i = 0; i < E; i += 2) {
          const float2 m1 = fmul2(make_float2(y[i], y[i + 1]), make_float2(cs[i], cs[i + 1]));
          float2 m2 = fmul2(make_float2(partner[i], partner[i + 1]), make_float2(sn[i], sn[i + 1]));
          if (!upper) m2 = make_float2(-m2.x, -m2.y);
          const float2 o = fadd2(m1, m2);
          out[i] = o.x, out[i + 1] = o.y;
        }
      }
      if (!pos_ok) {
#pragma unroll
        for (int i = 0; i < E; ++i) out[i] = 0.f;
      }
      float unused[E];
      const V ob = round_pack<T, E, V>(out, unused);
      if (h < hq) {
        *reinterpret_cast<V *>(p.q_out + t * p.q_out_stride_bytes + static_cast<int64_t>(h) * D * sizeof(T) +
                               lane_off) = ob;
      } else if (h < heads && slot >= 0) {
        const bool is_k = h < hq + hkv;
        char *cache = is_k ? p.key_cache : p.value_cache;
        const int kvh = is_k ? h - hq : h - hq - hkv;
        *reinterpret_cast<V *>(cache + (slot * hkv + kvh) * D * static_cast<int64_t>(sizeof(T)) + lane_off) =
            is_k ? ob : raw[j];
      }
    }
  }
  pdl_launch_dependents();
}

template <typename T>
static cudaError_t launch_prologue_t(const QkPrologueParams &p, int D, cudaStream_t stream) {
  if (p.num_tokens > 0x7fffffff) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(p.num_tokens)), block(kPrologueThreads);
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
