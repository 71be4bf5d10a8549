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
// Two forms share the per-row math (norm_rope).  The streaming form, used
// whenever a token's packed row fits its shared-memory stages: persistent CTAs
// of 4 consumer warps and one producer lane; the producer brings each token's
// whole [Hq | Hkv | Hkv] x D row and its cos/sin rows into a 3-stage ring with
// bulk copies (the TMA engine, completing on mbarriers), so the bytes in flight
// cost no registers, and the consumers write q, k and v straight to HBM.  The
// register form (one 64-thread CTA per token, 8 row groups loaded per warp
// before use) covers larger rows.  A head row spans a group of G = D / E lanes,
// E = 16 / sizeof(T) elements per lane (one 16-byte vector), so a warp covers
// 32 / G rows per instruction; the split-half partner of an element sits in
// lane ^ G/2 of its group, the interleaved partner in the same lane.  Products
// and sums use the packed f32x2 instructions with explicit round-to-nearest
// (each lane rounded exactly as __fmul_rn / __fadd_rn; a negated operand turns
// a sum into the reference's difference exactly).  Groups made only of v rows
// are copied without the math.  HBM-bound: every element is read once and
// written once.
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

// The rotation coefficients of lane-in-group `gl` for one position, from that
// position's cos/sin rows (global table or a shared-memory copy).
template <int D, int E, int G>
__device__ __forceinline__ void lane_coeffs(const float *cos_row, const float *sin_row, int gl,
                                            bool interleaved, float (&cs)[E], float (&sn)[E]) {
  if (interleaved) {
    constexpr int N = E / 2 < 4 ? E / 2 : 4;
#pragma unroll
    for (int j = 0; j < E / 2; j += 4) {
      float c4[4], s4[4];
      load_f32<N>(cos_row + gl * (E / 2) + j, reinterpret_cast<float(&)[N]>(c4));
      load_f32<N>(sin_row + gl * (E / 2) + j, reinterpret_cast<float(&)[N]>(s4));
#pragma unroll
      for (int u = 0; u < N; ++u)
        cs[2 * (j + u)] = cs[2 * (j + u) + 1] = c4[u], sn[2 * (j + u)] = sn[2 * (j + u) + 1] = s4[u];
    }
  } else {
    const int off = (gl & (G / 2 - 1)) * E;
#pragma unroll
    for (int j = 0; j < E; j += 4) {
      load_f32<4>(cos_row + off + j, reinterpret_cast<float(&)[4]>(cs[j]));
      load_f32<4>(sin_row + off + j, reinterpret_cast<float(&)[4]>(sn[j]));
    }
  }
}

// One row group of a q or k head: RMSNorm (fp32, one rounding to T, as
// F.rms_norm) then the rotation, packed back to T.  Every lane of the warp
// must call it (shuffles within each G-lane group); rows of a group that are
// not q/k just discard the result.
template <typename T, int D>
__device__ __forceinline__ typename RowVec<T, 16 / sizeof(T)>::V norm_rope(
    const typename RowVec<T, 16 / sizeof(T)>::V &raw, const typename RowVec<T, 16 / sizeof(T)>::V &wv,
    const float (&cs)[16 / sizeof(T)], const float (&sn)[16 / sizeof(T)], float eps, bool interleaved,
    bool upper, bool pos_ok) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));
  constexpr int G = D / E;
  using RV = RowVec<T, E>;
  using V = typename RV::V;
  float x[E];
  RV::to_float(raw, x);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
  float w[E];
  RV::to_float(wv, w);
  float y[E];
#pragma unroll
  for (int i = 0; i < E; i += 2) {
    const float2 v2 = fmul2(fmul2(make_float2(x[i], x[i + 1]), make_float2(inv, inv)),
                            make_float2(w[i], w[i + 1]));
    y[i] = v2.x, y[i + 1] = v2.y;
  }
  const V yb = round_pack<T, E, V>(y, y);  // the rounded norm output, as the reference holds it
  float out[E];
  if (interleaved) {
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
  return round_pack<T, E, V>(out, unused);
}

}  // namespace

// Register-staged form: one 64-thread CTA per token, each warp loading 8 row
// groups before it processes any.  Used when a token's row does not fit the
// shared-memory stages of the streaming form below.
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
  for (int i = 0; i < E; ++i) cs[i] = sn[i] = 0.f;  // bad positions: rows are zeroed
  if (pos_ok)
    lane_coeffs<D, E, G>(p.cos_table + pos * (D / 2), p.sin_table + pos * (D / 2), gl, p.interleaved,
                         cs, sn);
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
      const V ob = norm_rope<T, D>(raw[j], h < hq ? wq : wk, cs, sn, p.eps, p.interleaved, upper, pos_ok);
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

// Streaming form: a persistent CTA walks tokens blockIdx.x, + gridDim.x, ...
// A producer lane brings each token's whole packed row and its cos/sin rows
// into a ring of shared-memory stages with bulk copies (the TMA engine), so the
// bytes in flight cost no registers; 4 consumer warps take the row groups of
// the staged token from shared memory and write q, k and v straight to HBM.
constexpr int kStreamWarps = 4;
constexpr int kStreamThreads = (kStreamWarps + 1) * 32;
constexpr int kStreamStages = 3;

struct StageMeta {
  int64_t pos;
  int64_t slot;
};

__host__ __device__ constexpr int stream_stage_bytes(int row_bytes, int D) {
  return (row_bytes + D * 4 + static_cast<int>(sizeof(StageMeta)) + 127) / 128 * 128;
}

template <typename T, int D>
__global__ void __launch_bounds__(kStreamThreads) qk_prologue_stream_kernel(const QkPrologueParams p) {
  constexpr int E = 16 / static_cast<int>(sizeof(T));
  constexpr int G = D / E;
  constexpr int R = 32 / G;
  using RV = RowVec<T, E>;
  using V = typename RV::V;
  extern __shared__ __align__(128) uint8_t smem[];
  const int hq = p.num_q_heads, hkv = p.num_kv_heads, heads = hq + 2 * hkv;
  const int row_bytes = heads * D * static_cast<int>(sizeof(T));
  const int stage_bytes = stream_stage_bytes(row_bytes, D);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStreamStages * stage_bytes);
  uint64_t *empty = full + kStreamStages;
  int *abort_flag = reinterpret_cast<int *>(empty + kStreamStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStreamStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStreamWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();

  if (warp == kStreamWarps) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    int k = 0;
    for (int64_t t = blockIdx.x; t < p.num_tokens; t += gridDim.x, ++k) {
      const int st = k % kStreamStages;
      if (k >= kStreamStages &&
          !mbar_wait_bounded(&empty[st], ((k / kStreamStages) & 1) ^ 1, p.status)) {
        *(volatile int *)abort_flag = 1;
        break;
      }
      if (*(volatile int *)abort_flag) break;
      uint8_t *stage = smem + st * stage_bytes;
      StageMeta *meta = reinterpret_cast<StageMeta *>(stage + row_bytes + D * 4);
      const int64_t pos = p.positions_int64 ? static_cast<const int64_t *>(p.positions)[t]
                                            : static_cast<const int32_t *>(p.positions)[t];
      const bool pos_ok = pos >= 0 && pos < p.max_positions;
      meta->pos = pos;
      meta->slot = p.slot_mapping[t];
      mbar_arrive_expect_tx(&full[st], row_bytes + (pos_ok ? D * 4 : 0));
      bulk_g2s(stage, p.qkv + t * p.qkv_stride_bytes, row_bytes, &full[st]);
      if (pos_ok) {
        bulk_g2s(stage + row_bytes, p.cos_table + pos * (D / 2), D * 2, &full[st]);
        bulk_g2s(stage + row_bytes + D * 2, p.sin_table + pos * (D / 2), D * 2, &full[st]);
      }
    }
    if (*(volatile int *)abort_flag) {
      // the consumers gave up: wait (bounded) for this CTA's copies still in flight
      for (int kk = k > kStreamStages ? k - kStreamStages : 0; kk < k; ++kk)
        if (!mbar_wait_bounded(&full[kk % kStreamStages], (kk / kStreamStages) & 1, p.status)) break;
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int gl = lane & (G - 1), sub = lane / G;
  const V wq = *reinterpret_cast<const V *>(static_cast<const T *>(p.q_weight) + gl * E);
  const V wk = *reinterpret_cast<const V *>(static_cast<const T *>(p.k_weight) + gl * E);
  const bool upper = gl >= G / 2;
  const int64_t lane_off = gl * E * static_cast<int64_t>(sizeof(T));
  const int groups = (heads + R - 1) / R;
  int k = 0;
  for (int64_t t = blockIdx.x; t < p.num_tokens; t += gridDim.x, ++k) {
    const int st = k % kStreamStages;
    if (!mbar_wait_bounded(&full[st], (k / kStreamStages) & 1, p.status)) {
      *(volatile int *)abort_flag = 1;
      break;
    }
    const uint8_t *stage = smem + st * stage_bytes;
    const StageMeta meta = *reinterpret_cast<const StageMeta *>(stage + row_bytes + D * 4);
    const bool pos_ok = meta.pos >= 0 && meta.pos < p.max_positions;
    int64_t slot = meta.slot;
    const bool slot_bad = slot < -1 || slot >= p.num_slots;
    if (slot_bad) slot = -1;
    if (warp == 0 && lane == 0) {
      if (!pos_ok) flag_status(p.status, MI_DEV_BAD_POSITION);
      if (slot_bad) flag_status(p.status, MI_DEV_BAD_SLOT);
    }
    float cs[E], sn[E];
#pragma unroll
    for (int i = 0; i < E; ++i) cs[i] = sn[i] = 0.f;
    if (pos_ok)
      lane_coeffs<D, E, G>(reinterpret_cast<const float *>(stage + row_bytes),
                           reinterpret_cast<const float *>(stage + row_bytes + D * 2), gl, p.interleaved,
                           cs, sn);
    for (int grp = warp; grp < groups; grp += kStreamWarps) {
      const int h0 = grp * R, h = h0 + sub;
      const V raw = h < heads ? *reinterpret_cast<const V *>(stage + h * D * static_cast<int>(sizeof(T)) +
                                                               lane_off)
                              : V{};
      if (h0 >= hq + hkv) {  // a group of v rows only (warp-uniform): copy
        if (h < heads && slot >= 0)
          *reinterpret_cast<V *>(p.value_cache + (slot * hkv + (h - hq - hkv)) * D * static_cast<int64_t>(sizeof(T)) +
                                 lane_off) = raw;
        continue;
      }
      const V ob = norm_rope<T, D>(raw, h < hq ? wq : wk, cs, sn, p.eps, p.interleaved, upper, pos_ok);
      if (h < hq) {
        *reinterpret_cast<V *>(p.q_out + t * p.q_out_stride_bytes + static_cast<int64_t>(h) * D * sizeof(T) +
                               lane_off) = ob;
      } else if (h < heads && slot >= 0) {
        const bool is_k = h < hq + hkv;
        char *cache = is_k ? p.key_cache : p.value_cache;
        const int kvh = is_k ? h - hq : h - hq - hkv;
        *reinterpret_cast<V *>(cache + (slot * hkv + kvh) * D * static_cast<int64_t>(sizeof(T)) + lane_off) =
            is_k ? ob : raw;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  pdl_launch_dependents();
}

template <typename T>
static cudaError_t launch_prologue_t(const QkPrologueParams &p, int D, cudaStream_t stream) {
  if (p.num_tokens > 0x7fffffff) return cudaErrorInvalidValue;
  const int heads = p.num_q_heads + 2 * p.num_kv_heads;
  const int64_t row_bytes = static_cast<int64_t>(heads) * D * sizeof(T);
  const int64_t stage = stream_stage_bytes(static_cast<int>(row_bytes < (1 << 20) ? row_bytes : (1 << 20)), D);
  const int64_t smem = kStreamStages * stage + 2 * kStreamStages * 8 + 16;
  if (row_bytes < (1 << 20) && smem <= 100 * 1024) {
    // two or more streaming CTAs per SM (up to 6), each with 3 tokens in flight
    auto kern = D == 128 ? qk_prologue_stream_kernel<T, 128> : qk_prologue_stream_kernel<T, 64>;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
      const cudaError_t e = cudaFuncSetAttribute(qk_prologue_stream_kernel<T, 128>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
      if (e != cudaSuccess) return e;
      const cudaError_t e2 = cudaFuncSetAttribute(qk_prologue_stream_kernel<T, 64>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
      if (e2 != cudaSuccess) return e2;
      attr_set[dev] = true;
    }
    const int per_sm = static_cast<int>((220 * 1024) / smem) < 6 ? static_cast<int>((220 * 1024) / smem) : 6;
    const int64_t cap = static_cast<int64_t>(sm_count_current()) * per_sm;
    const dim3 grid(static_cast<unsigned>(p.num_tokens < cap ? p.num_tokens : cap));
    return launch_pdl(kern, grid, dim3(kStreamThreads), static_cast<size_t>(smem), stream, p);
  }
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
