// HBM-bound paged decode attention for sm_100a.
//
// paged_decode_kernel: one CTA per (split, kv head, sequence), so each K/V
// byte is read once for the whole GQA group.  Eight warps each stream their
// own 8-key chunks (chunk ids strided over splits and warps, so a CTA knows
// them before the context length arrives) through a ring of shared-memory
// stages filled by cp.async.bulk row copies -- one row per lane, K rows on
// lanes 0-7 and V rows on 8-15 -- completing on an mbarrier.  The context
// length, the block-table entries of the first stages and the slot of this
// step's token are fetched in a single round trip.
//
// Q for the group lives in registers pre-scaled into the log2 domain; q.k
// uses packed fp32x2 FMAs and a transposed butterfly reduction that leaves
// each lane whole dot products; the online softmax rescales lazily (only when
// a score passes the running max by 2^8).  p.V accumulates in fp32x2 pairs.
//
// Optional fused store_kvcache: this step's token (position ctx-1) is not
// read back from the pool.  Its k_new/v_new rows are loaded into registers by
// one warp, folded into that warp's softmax state after its chunks, and
// written to the token's slot; every cached page can therefore be requested
// before the preceding kernel finishes (early_kv), and nothing waits on the
// store.
//
// Split-K: the splits of one (seq, kv head) store their (m, l, acc) states
// in the workspace and the last one to finish merges them (split_merge.cuh).
#include <float.h>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "split_merge.cuh"
#include "tc_helpers.cuh"
#include "tmap.cuh"

namespace mi {

// Launch parameters: the decode arguments plus, when every 8-key chunk lies
// in one page (block_size % 8 == 0) and a row is at most 256 bytes, tensor
// maps over the K and V pools ([slots][Hkv][D], box {D, 1, 8}, no swizzle)
// so that a chunk's rows of one head arrive in one TMA copy each.
struct __align__(64) DecodeSimtParams {
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  DecodeParams d;
  int32_t use_tma;
};

namespace {
constexpr unsigned kFull = 0xffffffffu;
constexpr int kL2Ahead = 4;  // chunks per warp prefetched into L2 beyond the smem ring
}

template <typename T, int D, int G, int W>
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
  static constexpr int kWarps = W;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kSmemStages = kWarps * kStages * kStageBytes;
  static constexpr int kSmemP = kWarps * kKeys * G * 4;
  static constexpr int kSmemBars = kWarps * kStages * 8;
  static constexpr int kSmemMerge = kWarps * G * (D + 2) * 4;
  static constexpr int kSmem = kSmemStages + kSmemP + kSmemBars + 16;
  // 16 warps (one CTA per SM, 384 keys in flight) where 3 stages fit and the
  // group's registers stay within 128 per thread
  static constexpr bool kWideOk = kStageBytes <= 4096 && G <= 4;
  static_assert(kSmemMerge <= kSmemStages, "merge buffers alias the stage ring");
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

template <typename T, int D, int G, int W>
__global__ void __launch_bounds__(W * 32, (W == 8 && G < 8) ? 2 : 1)
    paged_decode_kernel(const __grid_constant__ DecodeSimtParams P) {
  using C = DecCfg<T, D, G, W>;
  const DecodeParams &p = P.d;
  const bool use_tma = P.use_tma != 0;
  extern __shared__ __align__(128) char smem[];
  char *stage_mem = smem;
  float *p_smem = reinterpret_cast<float *>(smem + C::kSmemStages);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemStages + C::kSmemP);
  int *last_flag = reinterpret_cast<int *>(bars + C::kWarps * C::kStages);

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
  // Block-table window: win[j] is this lane's entry for chunk it + j of the
  // warp's loop (entries are loaded kWin - kStages iterations before use).
  constexpr int kWin = C::kStages + kL2Ahead;
  int32_t win[kWin];  // block ids are int32 in the table
#pragma unroll
  for (int j = 0; j < kWin; ++j) win[j] = static_cast<int32_t>(table_entry(chunk_of(j)));
  int ctx = __ldg(p.context_lens + seq);
  const int64_t slot = fused ? static_cast<int64_t>(__ldg(p.slot_mapping + seq)) : -1;

  const int64_t cap = p.bt_stride * p.block_size;  // keys the table row can address
  if (ctx > cap) {
    if (threadIdx.x == 0 && split == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    ctx = static_cast<int>(cap);
  }
  // With the fused store, position ctx-1 is this step's token: it comes from
  // k_new/v_new (folded in by warp 0 of one split), not from the pool.
  const bool fold = fused && slot >= 0 && ctx > 0;
  const int ctx_kv = fold ? ctx - 1 : ctx;  // keys read from the pool
  const bool own_new = fold && warp == 0 && split == ((ctx - 1) / C::kKeys) % nsplit;
  const int nchunks = ctx_kv > 0 ? (ctx_kv + C::kKeys - 1) / C::kKeys : 0;
  const int first = split + nsplit * warp;
  const int stride = nsplit * C::kWarps;
  const int my_n = first < nchunks ? (nchunks - first + stride - 1) / stride : 0;

  const int64_t tok_bytes = static_cast<int64_t>(p.num_kv_heads) * C::kRowBytes;
  const char *kv_src_base = (copy_kind ? p.value_cache : p.key_cache) +
                            static_cast<int64_t>(kvh) * C::kRowBytes;

  // Validate a prefetched table entry for this lane's row of chunk ci.
  auto check_blk = [&](int ci, int64_t blk) -> int64_t {
    const int key = ci * C::kKeys + copy_key;
    if (!copy_lane || key >= ctx_kv) return -1;
    if (blk < 0 || blk >= p.num_blocks) {
      flag_status(p.status, MI_DEV_BAD_BLOCK);
      return -1;
    }
    return blk;
  };
  auto issue = [&](int ci, int st, int64_t blk) {
    if (use_tma) {  // one 8-row copy each for K and V (lane 0's entry is the chunk's page)
      if (lane == 0) {
        if (blk >= 0) {
          const int row = static_cast<int>(blk * p.block_size + (ci * C::kKeys) % p.block_size);
          char *dst = wstage + st * C::kStageBytes;
          mbar_arrive_expect_tx(&wbar[st], 2 * C::kKeys * C::kRowBytes);
          tc::tma_load_3d(dst, &P.tmap_k, 0, kvh, row, &wbar[st]);
          tc::tma_load_3d(dst + C::kKeys * C::kRowBytes, &P.tmap_v, 0, kvh, row, &wbar[st]);
        } else {
          mbar_arrive(&wbar[st]);
        }
      }
      return;
    }
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
  // before waiting on the preceding kernel.
  int issued = 0;
#pragma unroll
  for (int s = 0; s < C::kStages; ++s) {
    if (s < my_n) {
      const int ci = chunk_of(s);
      issue(ci, s, check_blk(ci, win[s]));
      ++issued;
    }
  }
  // Chunks beyond the ring: warm L2 with their rows now, so their copies come
  // from L2 once the ring drains (bad ids are only skipped here; the copy
  // itself flags them).
#pragma unroll
  for (int j = C::kStages; j < kWin; ++j) {
    const int ci = chunk_of(j);
    const int key = ci * C::kKeys + copy_key;
    const int64_t blk = win[j];
    if (j >= my_n || blk < 0 || blk >= p.num_blocks) continue;
    if (use_tma) {
      if (lane == 0) {
        const int row = static_cast<int>(blk * p.block_size + (ci * C::kKeys) % p.block_size);
        tc::tma_prefetch_l2_3d(&P.tmap_k, 0, kvh, row);
        tc::tma_prefetch_l2_3d(&P.tmap_v, 0, kvh, row);
      }
    } else if (copy_lane && key < ctx_kv) {
      prefetch_l2_bulk(kv_src_base + (blk * p.block_size + key % p.block_size) * tok_bytes,
                       C::kRowBytes);
    }
  }
  if (p.early_kv) {
    pdl_launch_dependents();  // the next kernel may start its own prologue
    pdl_wait();
  }
  // This step's token: this lane's 16-byte pieces of the K and V rows (lane
  // group r holds the same dimensions as its q and acc registers).
  uint4 knew[C::kCPL], vnew[C::kCPL];
  if (own_new) {
    const int64_t off = seq * p.new_token_stride_bytes + static_cast<int64_t>(kvh) * C::kRowBytes;
#pragma unroll
    for (int cp = 0; cp < C::kCPL; ++cp) {
      knew[cp] = *reinterpret_cast<const uint4 *>(p.k_new + off + (cp * C::kLPR + c) * 16);
      vnew[cp] = *reinterpret_cast<const uint4 *>(p.v_new + off + (cp * C::kLPR + c) * 16);
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
    if (!mbar_wait_bounded(&wbar[st], parity, p.status)) {
      timed_out = true;
      break;
    }
    consumed = it + 1;
    const char *kst = wstage + st * C::kStageBytes;
    const char *vst = kst + C::kKeys * C::kRowBytes;
    const int valid = ctx_kv - ci * C::kKeys;  // keys of this chunk read from the pool (>= 1)

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
      issue(nci, st, check_blk(nci, win[C::kStages]));
      ++issued;
    }
    // Slide the window one chunk on; the new entry is first used kL2Ahead
    // iterations from now.
#pragma unroll
    for (int j = 0; j < kWin - 1; ++j) win[j] = win[j + 1];
    win[kWin - 1] = it + kWin < my_n ? static_cast<int32_t>(table_entry(chunk_of(it + kWin))) : -1;
  }
  if (timed_out) {
    // Let every copy still in flight land before the stage memory is reused.
    for (int it = consumed + 1; it < issued; ++it)
      if (!mbar_wait_bounded(&wbar[it % C::kStages], (it / C::kStages) & 1, p.status)) break;
#pragma unroll
    for (int h = 0; h < G; ++h) m_run[h] = -INFINITY;
  }

  // ---- this step's token: fold into the warp's state, write it to its slot ----
  float l_new[G];
#pragma unroll
  for (int h = 0; h < G; ++h) l_new[h] = 0.f;
  if (own_new) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float2 part = make_float2(0.f, 0.f);
#pragma unroll
      for (int cp = 0; cp < C::kCPL; ++cp) {
        float2 f[C::kVec / 2];
        Vec16<T>::unpack(knew[cp], f);
#pragma unroll
        for (int e = 0; e < C::kVec / 2; ++e) part = ffma2(f[e], q2[h][cp * C::kVec / 2 + e], part);
      }
      float s = part.x + part.y;
#pragma unroll
      for (int m = C::kLPR / 2; m >= 1; m >>= 1) s += __shfl_xor_sync(kFull, s, m);
      const float m_new = fmaxf(m_run[h], s);
      const float alpha = m_run[h] == -INFINITY ? 0.f : fast_exp2(m_run[h] - m_new);
      const float pn = fast_exp2(s - m_new);
      const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
      for (int cp = 0; cp < C::kCPL; ++cp) {
        float2 f[C::kVec / 2];
        Vec16<T>::unpack(vnew[cp], f);
#pragma unroll
        for (int e = 0; e < C::kVec / 2; ++e) {
          float2 &a = acc2[h][cp * C::kVec / 2 + e];
          a = fmul2(a, a2);
          // lane groups are summed below: only group 0 adds the token
          if (r == 0) a = ffma2(f[e], make_float2(pn, pn), a);
        }
      }
#pragma unroll
      for (int j = 0; j < C::kF; ++j)
        if (slot_head[j] == h) l_part[j] *= alpha;
      m_run[h] = m_new;
      l_new[h] = pn;
    }
    if (slot < p.num_blocks * p.block_size) {
      if (r == 0) {
        const int64_t row = (slot * p.num_kv_heads + kvh) * C::kRowBytes;
#pragma unroll
        for (int cp = 0; cp < C::kCPL; ++cp) {
          *reinterpret_cast<uint4 *>(const_cast<char *>(p.key_cache) + row + (cp * C::kLPR + c) * 16) = knew[cp];
          *reinterpret_cast<uint4 *>(const_cast<char *>(p.value_cache) + row + (cp * C::kLPR + c) * 16) = vnew[cp];
        }
      }
    } else if (lane == 0) {
      flag_status(p.status, MI_DEV_BAD_SLOT);
    }
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
    l_head[h] = x + l_new[h];
  }

  // ---- merge the warps through shared memory (aliases the drained ring) ----
  __syncthreads();
  float *mg_acc = reinterpret_cast<float *>(stage_mem);  // [warps][G][D]
  float *mg_ml = mg_acc + C::kWarps * G * D;              // [warps][G][2]
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
    } else {
      split_store_state(p, seq, qh, nsplit, split, D, d, M, L, A);
    }
  }
  if (nsplit > 1) split_arrive_and_merge<T, G, D>(p, seq, kvh, nsplit, last_flag);
}

template <typename T>
constexpr CUtensorMapDataType tmap_dtype() {
  return Elem<T>::kDtype == MI_DTYPE_FLOAT32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : Elem<T>::kDtype == MI_DTYPE_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

template <typename T, int D, int G, int W>
static cudaError_t launch_decode_tdgw(const DecodeParams &p, int64_t num_seqs, int nsplit,
                                      cudaStream_t stream) {
  using C = DecCfg<T, D, G, W>;
  auto kern = paged_decode_kernel<T, D, G, W>;
  DecodeSimtParams P;
  memset(&P, 0, sizeof(P));
  P.d = p;
  const uint64_t rows = static_cast<uint64_t>(p.num_blocks) * p.block_size;
  if (C::kRowBytes <= 256 && p.block_size % C::kKeys == 0 && rows < (1ull << 31)) {
    const uint64_t row_stride = static_cast<uint64_t>(p.num_kv_heads) * C::kRowBytes;
    P.use_tma = encode_rows_map(&P.tmap_k, tmap_dtype<T>(), p.key_cache, D, p.num_kv_heads, rows,
                                C::kRowBytes, row_stride, D, 1, C::kKeys,
                                CU_TENSOR_MAP_SWIZZLE_NONE) &&
                encode_rows_map(&P.tmap_v, tmap_dtype<T>(), p.value_cache, D, p.num_kv_heads,
                                rows, C::kRowBytes, row_stride, D, 1, C::kKeys,
                                CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid(nsplit, p.num_kv_heads, static_cast<unsigned>(num_seqs));
  return launch_pdl(kern, grid, dim3(C::kThreads), C::kSmem, stream, P);
}

template <typename T, int D, int G>
static cudaError_t launch_decode_tdg(const DecodeParams &p, int64_t num_seqs, int nsplit, bool wide,
                                     cudaStream_t stream) {
  if constexpr (DecCfg<T, D, G, 16>::kWideOk) {
    if (wide) return launch_decode_tdgw<T, D, G, 16>(p, num_seqs, nsplit, stream);
  }
  return launch_decode_tdgw<T, D, G, 8>(p, num_seqs, nsplit, stream);
}

template <typename T, int D>
static cudaError_t launch_decode_td(const DecodeParams &p, int G, int64_t n, int s, bool wide,
                                    cudaStream_t st) {
  switch (G) {
    case 1: return launch_decode_tdg<T, D, 1>(p, n, s, wide, st);
    case 2: return launch_decode_tdg<T, D, 2>(p, n, s, wide, st);
    case 4: return launch_decode_tdg<T, D, 4>(p, n, s, wide, st);
    case 8: return launch_decode_tdg<T, D, 8>(p, n, s, wide, st);
  }
  return cudaErrorInvalidValue;
}

bool decode_fast_supported(int dtype, int D, int G) {
  if (G != 1 && G != 2 && G != 4 && G != 8) return false;
  if (dtype == MI_DTYPE_FLOAT32) return D == 64 || D == 128;
  return D == 64 || D == 128 || D == 256;
}

// 16-warp variant available: 3 stages of 8 rows fit (2-byte elements with
// D <= 128, or fp32 with D = 64) and the GQA group is at most 4.
bool decode_wide_supported(int dtype, int D, int G) {
  return G <= 4 && (dtype == MI_DTYPE_FLOAT32 ? D == 64 : D <= 128);
}

cudaError_t launch_decode_fast(const DecodeParams &p, int dtype, int D, int G, int64_t num_seqs,
                               int nsplit, bool wide, cudaStream_t stream) {
  if (dtype == MI_DTYPE_FLOAT32) {
    if (D == 64) return launch_decode_td<float, 64>(p, G, num_seqs, nsplit, wide, stream);
    return launch_decode_td<float, 128>(p, G, num_seqs, nsplit, wide, stream);
  }
  if (dtype == MI_DTYPE_FLOAT16) {
    if (D == 64) return launch_decode_td<__half, 64>(p, G, num_seqs, nsplit, wide, stream);
    if (D == 128) return launch_decode_td<__half, 128>(p, G, num_seqs, nsplit, wide, stream);
    return launch_decode_td<__half, 256>(p, G, num_seqs, nsplit, wide, stream);
  }
  if (D == 64) return launch_decode_td<__nv_bfloat16, 64>(p, G, num_seqs, nsplit, wide, stream);
  if (D == 128) return launch_decode_td<__nv_bfloat16, 128>(p, G, num_seqs, nsplit, wide, stream);
  return launch_decode_td<__nv_bfloat16, 256>(p, G, num_seqs, nsplit, wide, stream);
}

}  // namespace mi
