// HBM-bound paged decode attention for sm_100a.
//
// paged_decode_kernel: one CTA per (split, kv head, sequence), so each K/V
// byte is read once for the whole GQA group.  Four warps each stream their
// own 16-key chunks (chunk ids strided over splits and warps, so a CTA knows
// them before the context length arrives) through a ring of shared-memory
// stages filled by cp.async.bulk row copies -- one row per lane, K rows on
// lanes 0-15 and V rows on 16-31 -- completing on an mbarrier.  The context
// length, the block-table entries of the first stages and the slot of this
// step's token are fetched in a single round trip.
//
// Q for the group lives in registers pre-scaled into the log2 domain; q.k
// uses packed fp32x2 FMAs and a transposed butterfly reduction that leaves
// each lane whole dot products; the online softmax rescales lazily (only when
// a score passes the running max by 2^8).  p.V accumulates in fp32x2 pairs.
//
// Optional fused store_kvcache: the warp that owns the chunk holding this
// step's token writes k_new/v_new into its slot, fences the async proxy and
// only then bulk-copies that chunk, so the attention sees the new token
// without a separate store launch.
//
// Split-K: with 2..8 splits the splits of one (seq, kv head) run as a thread
// block cluster and rank 0 merges their (m, l, acc) states through
// distributed shared memory; with more splits the states go to a workspace
// and decode_combine_kernel merges them.
#include <cooperative_groups.h>
#include <float.h>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace cg = cooperative_groups;

namespace mi {

namespace {
constexpr unsigned kFull = 0xffffffffu;
}

template <typename T, int D, int G>
struct DecCfg {
  static constexpr int kRowBytes = D * static_cast<int>(sizeof(T));
  static constexpr int kVec = 16 / static_cast<int>(sizeof(T));  // elements per 16 B
  static constexpr int kChunks = kRowBytes / 16;                  // 16 B chunks per row
  static constexpr int kCPL = kChunks > 32 ? kChunks / 32 : 1;    // chunks per lane per row
  static constexpr int kLPR = kChunks / kCPL;                     // lanes per row
  static constexpr int kRPS = 32 / kLPR;                          // lane groups (rows in flight)
  static constexpr int kKeys = 8;                                 // keys per stage
  static constexpr int kKPG = kKeys / kRPS;                       // keys per lane group
  static constexpr int kEPL = kCPL * kVec;                        // elements per lane per row
  static constexpr int kSub = (kKPG * G <= 32) ? kKPG : (32 / G > 0 ? 32 / G : 1);
  static constexpr int kNSub = kKPG / kSub;
  static constexpr int kV0 = kSub * G;                     // dots per lane before reduction
  static constexpr int kF = kV0 >= kLPR ? kV0 / kLPR : 1;    // reduced dots kept per lane
  static constexpr int kDup = kV0 >= kLPR ? 1 : kLPR / kV0;  // lanes holding the same dot
  static constexpr int kStageBytes = kKeys * 2 * kRowBytes;
  static constexpr int kStages = kStageBytes <= 4096 ? 3 : 2;
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kSmemStages = kWarps * kStages * kStageBytes;
  static constexpr int kSmemP = kWarps * kKeys * G * 4;
  static constexpr int kSmemBars = kWarps * kStages * 8;
  static constexpr int kSmemMerge = kWarps * G * (D + 2) * 4;
  static constexpr int kSmemFin = G * (D + 2) * 4;
  static constexpr int kSmem = kSmemStages + kSmemP + kSmemBars;
  static constexpr int kNewLanes = (2 * kChunks + 31) / 32;  // 16 B pieces per lane for the store
  static_assert(kSmemMerge + kSmemFin <= kSmemStages, "merge buffers alias the stage ring");
  static_assert(kRPS <= kKeys, "row too short for the lane mapping");
  static_assert(kKPG % kSub == 0, "sub-step must divide the group's keys");
};

// Reduce N per-lane values across the LPR lanes of a lane group so that each
// lane ends with max(N / LPR, 1) complete sums: at each butterfly level the
// lane sends the half it gives away and keeps the other half.  With N >= LPR
// lane c of the group holds values c*F .. c*F+F-1; with N < LPR it holds
// value c / (LPR / N), duplicated on LPR / N lanes.
template <int N, int LPR>
__device__ __forceinline__ void transpose_reduce(float (&v)[N], int c) {
  int n = N;
#pragma unroll
  for (int m = LPR / 2; m >= 1; m >>= 1) {
    if (n > 1) {
      const bool upper = (c & m) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < n / 2) {
          const float send = upper ? v[i] : v[i + n / 2];
          const float keep = upper ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(kFull, send, m);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(kFull, v[0], m);
    }
  }
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(256, G >= 8 ? 1 : 2) paged_decode_kernel(DecodeParams p) {
  using C = DecCfg<T, D, G>;
  extern __shared__ __align__(128) char smem[];
  char *stage_mem = smem;
  float *p_smem = reinterpret_cast<float *>(smem + C::kSmemStages);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemStages + C::kSmemP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int kvh = blockIdx.y;
  const int64_t seq = blockIdx.z;
  const int r = lane / C::kLPR, c = lane % C::kLPR;
  uint64_t *wbar = bars + warp * C::kStages;
  char *wstage = stage_mem + warp * C::kStages * C::kStageBytes;
  float *wp = p_smem + warp * C::kKeys * G;
  // Copies: lanes 0-7 fetch the chunk's K rows, lanes 8-15 its V rows.
  const int copy_key = lane & (C::kKeys - 1);
  const int copy_kind = (lane / C::kKeys) & 1;
  const bool copy_lane = lane < 2 * C::kKeys;
  const bool fused = p.k_new != nullptr;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < C::kStages; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Without early_kv everything below may come from the preceding kernel.
  if (!p.early_kv) pdl_wait();
  // ---- one round trip: context, first table entries, this step's slot ----
  const int32_t *table = p.block_tables + seq * p.bt_stride;
  auto chunk_of = [&](int it) { return split + nsplit * (warp + C::kWarps * it); };
  auto table_entry = [&](int ci) -> int64_t {  // this lane's row of chunk ci
    const int64_t col = (static_cast<int64_t>(ci) * C::kKeys + copy_key) / p.block_size;
    return col < p.bt_stride ? static_cast<int64_t>(__ldg(table + col)) : -1;
  };
  int64_t pre_blk[C::kStages];
#pragma unroll
  for (int s = 0; s < C::kStages; ++s) pre_blk[s] = table_entry(chunk_of(s));
  int ctx = __ldg(p.context_lens + seq);
  const int64_t slot = fused ? static_cast<int64_t>(__ldg(p.slot_mapping + seq)) : -1;

  const int64_t cap = p.bt_stride * p.block_size;  // keys the table row can address
  if (ctx > cap) {
    if (threadIdx.x == 0 && split == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    ctx = static_cast<int>(cap);
  }
  const int nchunks = ctx > 0 ? (ctx + C::kKeys - 1) / C::kKeys : 0;
  const int first = split + nsplit * warp;
  const int stride = nsplit * C::kWarps;
  const int my_n = first < nchunks ? (nchunks - first + stride - 1) / stride : 0;
  const int last_chunk = nchunks - 1;
  const bool own_last = fused && slot >= 0 && last_chunk >= 0 && last_chunk % nsplit == split &&
                        (last_chunk / nsplit) % C::kWarps == warp;

  const int64_t tok_bytes = static_cast<int64_t>(p.num_kv_heads) * C::kRowBytes;
  const char *kv_src_base = (copy_kind ? p.value_cache : p.key_cache) +
                            static_cast<int64_t>(kvh) * C::kRowBytes;

  // Validate a prefetched table entry for this lane's row of chunk ci.
  auto check_blk = [&](int ci, int64_t blk) -> int64_t {
    const int key = ci * C::kKeys + copy_key;
    if (!copy_lane || key >= ctx) return -1;
    if (blk < 0 || blk >= p.num_blocks) {
      flag_status(p.status, MI_DEV_BAD_BLOCK);
      return -1;
    }
    return blk;
  };
  // Fused store of this step's token (head kvh) before its chunk is copied.
  auto store_new_token = [&]() {
    if (slot >= p.num_blocks * p.block_size) {
      if (lane == 0) flag_status(p.status, MI_DEV_BAD_SLOT);
      return;
    }
#pragma unroll
    for (int i = 0; i < C::kNewLanes; ++i) {
      const int piece = lane + 32 * i;
      if (piece < 2 * C::kChunks) {
        const int kind = piece / C::kChunks, chunk = piece % C::kChunks;
        const char *src = (kind ? p.v_new : p.k_new) + seq * p.new_token_stride_bytes +
                          static_cast<int64_t>(kvh) * C::kRowBytes + chunk * 16;
        char *dst = const_cast<char *>(kind ? p.value_cache : p.key_cache) +
                    (slot * p.num_kv_heads + kvh) * C::kRowBytes + chunk * 16;
        *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
      }
    }
    // Order the generic-proxy stores before the bulk copy (async proxy) below.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
  };
  auto issue = [&](int ci, int st, int64_t blk) {
    if (own_last && ci == last_chunk) store_new_token();
    const int key = ci * C::kKeys + copy_key;
    const bool go = blk >= 0;
    const unsigned mask = __ballot_sync(kFull, go);
    if (lane == 0) mbar_arrive_expect_tx(&wbar[st], __popc(mask) * C::kRowBytes);
    if (go) {
      const char *src = kv_src_base + (blk * p.block_size + key % p.block_size) * tok_bytes;
      char *dst = wstage + st * C::kStageBytes + copy_kind * C::kKeys * C::kRowBytes +
                  copy_key * C::kRowBytes;
      bulk_g2s(dst, src, C::kRowBytes, &wbar[st]);
    }
  };

  // Prologue: fill the ring.  With early_kv the cached pages are requested
  // before waiting on the preceding kernel; the chunk that receives this
  // step's token (whose K/V that kernel may have produced) waits for it.
  int issued = 0;
  int deferred = -1;
  int64_t deferred_blk = -1;
#pragma unroll
  for (int s = 0; s < C::kStages; ++s) {
    if (s < my_n) {
      const int ci = chunk_of(s);
      if (p.early_kv && own_last && ci == last_chunk) {
        deferred = s;
        deferred_blk = pre_blk[s];
      } else {
        issue(ci, s, check_blk(ci, pre_blk[s]));
      }
      ++issued;
    }
  }
  if (p.early_kv) {
    pdl_launch_dependents();  // the next kernel may start its own prologue
    pdl_wait();
    if (deferred >= 0) {
      const int ci = chunk_of(deferred);
      issue(ci, deferred, check_blk(ci, deferred_blk));
    }
  }

  // Query rows of the GQA group, scaled into the log2 domain.
  float2 q2[G][C::kEPL / 2];
  {
    const T *qbase = static_cast<const T *>(p.query) +
                     (seq * p.num_q_heads + static_cast<int64_t>(kvh) * G) * D;
#pragma unroll
    for (int h = 0; h < G; ++h) {
#pragma unroll
      for (int cp = 0; cp < C::kCPL; ++cp) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(qbase + h * D + (cp * C::kLPR + c) * C::kVec);
        float2 f[C::kVec / 2];
        Vec16<T>::unpack(raw, f);
#pragma unroll
        for (int e = 0; e < C::kVec / 2; ++e)
          q2[h][cp * C::kVec / 2 + e] = make_float2(f[e].x * p.scale_log2, f[e].y * p.scale_log2);
      }
    }
  }

  // Slot j of this lane's reduced dots: which (key within sub-step, head).
  int slot_head[C::kF], slot_key[C::kF];
  bool slot_owner[C::kF];
#pragma unroll
  for (int j = 0; j < C::kF; ++j) {
    const int idx = (C::kV0 >= C::kLPR) ? c * C::kF + j : c / C::kDup;
    slot_head[j] = idx % G;
    slot_key[j] = idx / G;
    slot_owner[j] = c % C::kDup == 0;
  }

  float m_run[G];
  float2 acc2[G][C::kEPL / 2];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m_run[h] = -INFINITY;
#pragma unroll
    for (int e = 0; e < C::kEPL / 2; ++e) acc2[h][e] = make_float2(0.f, 0.f);
  }
  float l_part[C::kF];
  float m_mine[C::kF];
#pragma unroll
  for (int j = 0; j < C::kF; ++j) {
    l_part[j] = 0.f;
    m_mine[j] = -INFINITY;
  }

  bool timed_out = false;
  int consumed = 0;
#pragma unroll 1
  for (int it = 0; it < my_n; ++it) {
    const int st = it % C::kStages;
    const uint32_t parity = (it / C::kStages) & 1;
    const int ci = chunk_of(it);
    const bool has_next = it + C::kStages < my_n;
    const int nci = chunk_of(it + C::kStages);
    const int64_t nblk_raw = has_next ? table_entry(nci) : -1;
    if (!mbar_wait_bounded(&wbar[st], parity, p.status)) {
      timed_out = true;
      break;
    }
    consumed = it + 1;
    const char *kst = wstage + st * C::kStageBytes;
    const char *vst = kst + C::kKeys * C::kRowBytes;
    const int valid = ctx - ci * C::kKeys;  // keys of this chunk below ctx (>= 1)

    // ---- scores: q . k for the group's keys ----
    float sc[C::kNSub][C::kF];
#pragma unroll
    for (int u = 0; u < C::kNSub; ++u) {
      float2 part[C::kSub][G];
#pragma unroll
      for (int kk = 0; kk < C::kSub; ++kk)
#pragma unroll
        for (int h = 0; h < G; ++h) part[kk][h] = make_float2(0.f, 0.f);
#pragma unroll
      for (int kk = 0; kk < C::kSub; ++kk) {
        const int row = r * C::kKPG + u * C::kSub + kk;
#pragma unroll
        for (int cp = 0; cp < C::kCPL; ++cp) {
          const uint4 raw =
              *reinterpret_cast<const uint4 *>(kst + row * C::kRowBytes + (cp * C::kLPR + c) * 16);
          float2 f[C::kVec / 2];
          Vec16<T>::unpack(raw, f);
#pragma unroll
          for (int h = 0; h < G; ++h)
#pragma unroll
            for (int e = 0; e < C::kVec / 2; ++e)
              part[kk][h] = ffma2(f[e], q2[h][cp * C::kVec / 2 + e], part[kk][h]);
        }
      }
      float vals[C::kV0];
#pragma unroll
      for (int kk = 0; kk < C::kSub; ++kk)
#pragma unroll
        for (int h = 0; h < G; ++h) vals[kk * G + h] = part[kk][h].x + part[kk][h].y;
      transpose_reduce<C::kV0, C::kLPR>(vals, c);
#pragma unroll
      for (int j = 0; j < C::kF; ++j) {
        const int key_local = r * C::kKPG + u * C::kSub + slot_key[j];
        sc[u][j] = key_local < valid ? vals[j] : -INFINITY;
      }
    }

    // ---- online softmax with lazy rescale ----
    bool need = false;
#pragma unroll
    for (int u = 0; u < C::kNSub; ++u)
#pragma unroll
      for (int j = 0; j < C::kF; ++j) need |= sc[u][j] > m_mine[j] + 8.f;
    if (__any_sync(kFull, need)) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float x = -INFINITY;
#pragma unroll
        for (int u = 0; u < C::kNSub; ++u)
#pragma unroll
          for (int j = 0; j < C::kF; ++j)
            if (slot_head[j] == h) x = fmaxf(x, sc[u][j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
        const float m_new = fmaxf(m_run[h], x);
        const float alpha = (m_new == -INFINITY) ? 1.f : fast_exp2(m_run[h] - m_new);
        const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
        for (int e = 0; e < C::kEPL / 2; ++e) acc2[h][e] = fmul2(acc2[h][e], a2);
#pragma unroll
        for (int j = 0; j < C::kF; ++j)
          if (slot_head[j] == h) {
            l_part[j] *= alpha;
            m_mine[j] = m_new;
          }
        m_run[h] = m_new;
      }
    }
#pragma unroll
    for (int u = 0; u < C::kNSub; ++u)
#pragma unroll
      for (int j = 0; j < C::kF; ++j) {
        const float s = sc[u][j];
        const float pe = (s == -INFINITY) ? 0.f : fast_exp2(s - m_mine[j]);
        l_part[j] += pe;
        if (slot_owner[j])
          wp[(r * C::kKPG + u * C::kSub + slot_key[j]) * G + slot_head[j]] = pe;
      }
    __syncwarp();

    // ---- acc += p . V ----
#pragma unroll
    for (int kk = 0; kk < C::kKPG; ++kk) {
      const int row = r * C::kKPG + kk;
      if (row < valid) {
        float pv[G];
#pragma unroll
        for (int h = 0; h < G; ++h) pv[h] = wp[row * G + h];
#pragma unroll
        for (int cp = 0; cp < C::kCPL; ++cp) {
          const uint4 raw =
              *reinterpret_cast<const uint4 *>(vst + row * C::kRowBytes + (cp * C::kLPR + c) * 16);
          float2 f[C::kVec / 2];
          Vec16<T>::unpack(raw, f);
#pragma unroll
          for (int h = 0; h < G; ++h) {
            const float2 ph = make_float2(pv[h], pv[h]);
#pragma unroll
            for (int e = 0; e < C::kVec / 2; ++e)
              acc2[h][cp * C::kVec / 2 + e] = ffma2(f[e], ph, acc2[h][cp * C::kVec / 2 + e]);
          }
        }
      }
    }
    // Every lane has consumed its loads from this stage (their values fed the
    // FMAs above), so the stage can be refilled: no proxy fence needed.
    __syncwarp();
    if (has_next) {
      issue(nci, st, check_blk(nci, nblk_raw));
      ++issued;
    }
  }
  if (timed_out) {
    // Let every copy still in flight land before the stage memory is reused.
    for (int it = consumed + 1; it < issued; ++it)
      if (!mbar_wait_bounded(&wbar[it % C::kStages], (it / C::kStages) & 1, p.status)) break;
#pragma unroll
    for (int h = 0; h < G; ++h) m_run[h] = -INFINITY;
  }
  pdl_launch_dependents();

  // ---- merge lane groups inside the warp (they share m_run) ----
#pragma unroll
  for (int m = C::kLPR; m < 32; m <<= 1)
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int e = 0; e < C::kEPL / 2; ++e) {
        acc2[h][e].x += __shfl_xor_sync(kFull, acc2[h][e].x, m);
        acc2[h][e].y += __shfl_xor_sync(kFull, acc2[h][e].y, m);
      }
  float l_head[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float x = 0.f;
#pragma unroll
    for (int j = 0; j < C::kF; ++j)
      if (slot_owner[j] && slot_head[j] == h) x += l_part[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    l_head[h] = x;
  }

  // ---- merge the warps through shared memory (aliases the drained ring) ----
  __syncthreads();
  float *mg_acc = reinterpret_cast<float *>(stage_mem);  // [warps][G][D]
  float *mg_ml = mg_acc + C::kWarps * G * D;              // [warps][G][2]
  float *fin_acc = mg_ml + C::kWarps * G * 2;             // [G][D]   (cluster merge)
  float *fin_ml = fin_acc + G * D;                        // [G][2]
  if (r == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int cp = 0; cp < C::kCPL; ++cp)
#pragma unroll
        for (int e = 0; e < C::kVec / 2; ++e) {
          const int d = (cp * C::kLPR + c) * C::kVec + 2 * e;
          *reinterpret_cast<float2 *>(&mg_acc[(warp * G + h) * D + d]) = acc2[h][cp * C::kVec / 2 + e];
        }
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      mg_ml[(warp * G + h) * 2] = m_run[h];
      mg_ml[(warp * G + h) * 2 + 1] = l_head[h];
    }
  }
  __syncthreads();
  const bool cluster_merge = p.cluster_combine != 0 && nsplit > 1;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) M = fmaxf(M, mg_ml[(w * G + h) * 2]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < C::kWarps; ++w) {
      const float mw = mg_ml[(w * G + h) * 2];
      const float f = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
      L += f * mg_ml[(w * G + h) * 2 + 1];
      A += f * mg_acc[(w * G + h) * D + d];
    }
    const int qh = kvh * G + h;
    if (nsplit == 1) {
      T *o = static_cast<T *>(p.out) + (seq * p.num_q_heads + qh) * D;
      o[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
    } else if (cluster_merge) {
      fin_acc[h * D + d] = A;
      if (d == 0) {
        fin_ml[h * 2] = M;
        fin_ml[h * 2 + 1] = L;
      }
    } else {
      const int64_t state = (seq * p.num_q_heads + qh) * nsplit + split;
      p.ws_acc[state * D + d] = A;
      if (d == 0) {
        p.ws_ml[state * 2] = M;
        p.ws_ml[state * 2 + 1] = L;
      }
    }
  }
  if (cluster_merge) {
    // The splits of this (seq, kv head) are the CTAs of one cluster along x.
    // Each rank finalises a slice of the (head, dim) outputs, issuing all of
    // its remote (DSMEM) loads before using any of them.
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    for (int i = split * C::kThreads + threadIdx.x; i < G * D; i += nsplit * C::kThreads) {
      const int h = i / D, d = i % D;
      float ms[8], ls[8], as[8];
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < nsplit) {
          const float *rml = cluster.map_shared_rank(fin_ml, s);
          ms[s] = rml[h * 2];
          ls[s] = rml[h * 2 + 1];
          as[s] = cluster.map_shared_rank(fin_acc, s)[h * D + d];
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int s = 0; s < 8; ++s)
        if (s < nsplit) M = fmaxf(M, ms[s]);
      float L = 0.f, A = 0.f;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (s < nsplit) {
          const float f = (ms[s] == -INFINITY) ? 0.f : fast_exp2(ms[s] - M);
          L += f * ls[s];
          A += f * as[s];
        }
      }
      T *o = static_cast<T *>(p.out) + (seq * p.num_q_heads + kvh * G + h) * D;
      o[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
    }
    cluster.sync();  // keep every rank's shared memory alive until all reads are done
  }
}

// Merge split-K states: grid (Hq, N), one thread per output element.
template <typename T>
__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeParams p, int nsplit, int D) {
  pdl_wait();
  const int qh = blockIdx.x;
  const int64_t seq = blockIdx.y;
  const int64_t state0 = (seq * p.num_q_heads + qh) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, p.ws_ml[(state0 + s) * 2]);
  float L = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = p.ws_ml[(state0 + s) * 2];
    if (ms != -INFINITY) L += fast_exp2(ms - M) * p.ws_ml[(state0 + s) * 2 + 1];
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T *o = static_cast<T *>(p.out) + (seq * p.num_q_heads + qh) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float A = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ms = p.ws_ml[(state0 + s) * 2];
      if (ms != -INFINITY) A += fast_exp2(ms - M) * p.ws_acc[(state0 + s) * D + d];
    }
    o[d] = Elem<T>::from_float(A * inv);
  }
  pdl_launch_dependents();
}

template <typename T, int D, int G>
static cudaError_t launch_decode_tdg(const DecodeParams &p, int64_t num_seqs, int nsplit,
                                     cudaStream_t stream) {
  using C = DecCfg<T, D, G>;
  auto kern = paged_decode_kernel<T, D, G>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid(nsplit, p.num_kv_heads, static_cast<unsigned>(num_seqs));
  if (p.cluster_combine && nsplit > 1) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
  }
  cudaError_t e = launch_pdl(kern, grid, dim3(C::kThreads), C::kSmem, stream, p);
  if (e != cudaSuccess || nsplit == 1) return e;
  return launch_pdl(decode_combine_kernel<T>, dim3(p.num_q_heads, static_cast<unsigned>(num_seqs)),
                    dim3(128), 0, stream, p, nsplit, D);
}

template <typename T, int D>
static cudaError_t launch_decode_td(const DecodeParams &p, int G, int64_t n, int s, cudaStream_t st) {
  switch (G) {
    case 1: return launch_decode_tdg<T, D, 1>(p, n, s, st);
    case 2: return launch_decode_tdg<T, D, 2>(p, n, s, st);
    case 4: return launch_decode_tdg<T, D, 4>(p, n, s, st);
    case 8: return launch_decode_tdg<T, D, 8>(p, n, s, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode_combine(const DecodeParams &p, int dtype, int D, int64_t num_seqs,
                                  int nsplit, cudaStream_t stream) {
  const dim3 grid(p.num_q_heads, static_cast<unsigned>(num_seqs));
  if (dtype == MI_DTYPE_FLOAT32)
    return launch_pdl(decode_combine_kernel<float>, grid, dim3(128), 0, stream, p, nsplit, D);
  if (dtype == MI_DTYPE_FLOAT16)
    return launch_pdl(decode_combine_kernel<__half>, grid, dim3(128), 0, stream, p, nsplit, D);
  return launch_pdl(decode_combine_kernel<__nv_bfloat16>, grid, dim3(128), 0, stream, p, nsplit, D);
}

bool decode_fast_supported(int dtype, int D, int G) {
  if (G != 1 && G != 2 && G != 4 && G != 8) return false;
  if (dtype == MI_DTYPE_FLOAT32) return D == 64 || D == 128;
  return D == 64 || D == 128 || D == 256;
}

cudaError_t launch_decode_fast(const DecodeParams &p, int dtype, int D, int G, int64_t num_seqs,
                               int nsplit, cudaStream_t stream) {
  if (dtype == MI_DTYPE_FLOAT32) {
    if (D == 64) return launch_decode_td<float, 64>(p, G, num_seqs, nsplit, stream);
    return launch_decode_td<float, 128>(p, G, num_seqs, nsplit, stream);
  }
  if (dtype == MI_DTYPE_FLOAT16) {
    if (D == 64) return launch_decode_td<__half, 64>(p, G, num_seqs, nsplit, stream);
    if (D == 128) return launch_decode_td<__half, 128>(p, G, num_seqs, nsplit, stream);
    return launch_decode_td<__half, 256>(p, G, num_seqs, nsplit, stream);
  }
  if (D == 64) return launch_decode_td<__nv_bfloat16, 64>(p, G, num_seqs, nsplit, stream);
  if (D == 128) return launch_decode_td<__nv_bfloat16, 128>(p, G, num_seqs, nsplit, stream);
  return launch_decode_td<__nv_bfloat16, 256>(p, G, num_seqs, nsplit, stream);
}

}  // namespace mi
