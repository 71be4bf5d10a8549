// Warp-level tensor-core paged decode (mma.sync m16n8k16, sm_100a).
//
// Decode has at most 8 query rows per kv head.  On this part a tcgen05.mma
// costs about the same time at N=16 as at N=256, so the swap-AB tcgen05
// kernel spends ~1 us of tensor time per 128-key tile; CUDA-core dot
// products cost ~26 warp instructions per key.  The warp-level m16n8k16 MMA
// does a 16-key chunk of a kv head in 16 MMAs + 17 ldmatrix, with the keys
// in the M dimension and the GQA group in N = 8:
//   S^T[16 keys x 8]  = K . Q^T            (columns >= G of Q^T are zero)
//   O^T[D x 8]       += V^T . P^T          (P^T through 256 B of shared memory)
// i.e. ~3 warp instructions per key, accumulators in registers.
//
// One CTA per (split, kv head, sequence), 8 warps.  Each warp streams its
// own 16-key chunks (ids strided over splits and warps) through a 3-stage
// ring: per chunk one TMA copy per 64-dim half for K and for V (3-D tensor
// map over [slots][Hkv][D], box {64, 1, 16}, 128-byte swizzle, so ldmatrix
// reads are bank-conflict free); with early_kv the ring fills before the
// dependency wait.  The block table is read in batches of 32 chunks loaded
// a batch ahead.  Online softmax in the log2 domain with
// lazy rescale; the warps merge in shared memory, the splits through the
// workspace (split_merge.cuh).  With the fused store, this step's token is
// folded in as a one-key chunk built from k_new/v_new (the last item of the
// warp with the fewest chunks, in one of its free ring stages, so the load of
// k_new/v_new hides behind the cached chunks) and written to its slot.
//
// V rows past the context in a partial chunk are zeroed before P.V, so stale
// pool contents (even non-finite) never reach the output.  Every wait is
// bounded.
#include <type_traits>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "split_merge.cuh"
#include "tc_helpers.cuh"
#include "tmap.cuh"

namespace mi {

struct __align__(64) DecodeMmaParams {
  CUtensorMap tmap_k;  // [slots][Hkv][D], box {64, 1, 16}, 128-byte swizzle
  CUtensorMap tmap_v;
  DecodeParams d;
};

namespace {

constexpr unsigned kAll = 0xffffffffu;
constexpr int kChunk = 16;  // keys per chunk
constexpr int kStagesM = 3;
constexpr int kWarpsM = 8;

template <int D>
struct MmaCfg {
  static constexpr int kHalves = D / 64;             // 128-byte swizzled column halves
  static constexpr int kTileBytes = kHalves * 2048;  // 16 rows x D of one operand
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kKSteps = D / 16;
  static constexpr int kSmemStages = kWarpsM * kStagesM * kStageBytes;
  static constexpr int kSmemPT = kWarpsM * 256;   // per warp: P^T of a chunk, [16 keys][8 queries]
  static constexpr int kSmemBars = kWarpsM * kStagesM * 8;
  static constexpr int kSmem = kSmemStages + kSmemPT + kSmemBars + 16 + 1024;  // + slack
  // cluster pair: + the second CTA's merged state, (m, l) then acc, for up to 8 heads
  static constexpr int kSmemX = 8 * (D + 2) * 4;
  static constexpr int kSmemPair = kSmem + kSmemX;
  static_assert(kWarpsM * 8 * (D + 2) * 4 <= kSmemStages, "merge buffers alias the ring");
};

// Byte address of 16-byte column chunk `cj` of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t swz(uint32_t tile, int row, int cj) {
  return tile + (cj >> 3) * 2048 + row * 128 + ((((cj & 7) ^ (row & 7))) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                          uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// d += A . B for m16n8k16 with fp32 accumulation; A rows 8-15 are zero here.
template <typename T>
__device__ __forceinline__ void mma_rows8(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                          uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t &r0, uint32_t &r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr)
               : "memory");
}

// d += A . B for m16n8k16 with fp32 accumulation, full A fragment.
template <typename T>
__device__ __forceinline__ void mma_full(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
        "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Two floats -> one register of T pairs (lo in the low half).
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace

// Cluster barrier halves (every thread of both CTAs of a pair executes each).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Store to the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ void st_cluster_f32(const float *local, uint32_t rank, float v) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(local)), "r"(rank));
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}

// kPair: the two CTAs of a (sequence, kv head) form a cluster of 2 (grid.x = 2,
// split = rank); each takes every other 16-key chunk, and rank 1 hands its
// merged state to rank 0 through distributed shared memory instead of the
// global workspace.  Two cluster barrier phases: the first (arrive at the start,
// wait before the first remote store) makes sure rank 0 is running; the second
// (rank 1 arrives after its stores) hands them over and keeps rank 0's shared
// memory alive until they have landed.  Neither barrier can be left waiting:
// every other wait in the kernel is bounded and every path reaches both.
template <typename T, int D, int G, bool kPair>
__global__ void __launch_bounds__(kWarpsM * 32, 1)
    paged_decode_mma_kernel(const __grid_constant__ DecodeMmaParams P) {
  using C = MmaCfg<D>;
  const DecodeParams &p = P.d;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *pt_smem = smem + C::kSmemStages;
  uint64_t *bars = reinterpret_cast<uint64_t *>(pt_smem + C::kSmemPT);
  int *last_flag = reinterpret_cast<int *>(bars + kWarpsM * kStagesM);
  float *xml = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(last_flag) + 16);  // [8][2]
  float *xacc = xml + 16;                                                              // [8][D]
  if constexpr (kPair) cluster_arrive_relaxed();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;  // fragment row / column pair
  const int kvh = blockIdx.y;
  uint64_t *wbar = bars + warp * kStagesM;
  uint8_t *wstage = smem + warp * kStagesM * C::kStageBytes;
  const bool fused = p.k_new != nullptr;

  if (lane == 0) {
    tc::prefetch_tmap(&P.tmap_k);
    tc::prefetch_tmap(&P.tmap_v);
  }

  // Without early_kv everything below may come from the preceding kernel (a
  // mixed-batch launch needs no wait: see DecodeParams::cu_q).
  const bool mixed = p.cu_q != nullptr;
  if (!p.early_kv && !mixed) pdl_wait();

  const int split = blockIdx.x, nsplit = gridDim.x;
  const int64_t seq = blockIdx.z;
  const bool waits_for_prefill = mixed && split == 0 && kvh == 0 && seq == 0;
  int64_t qo_row = seq;  // query / output row
  if (mixed) {
    const int q0 = __ldg(p.cu_q + seq);
    if (__ldg(p.cu_q + seq + 1) - q0 != 1) {  // uniform: a prefill sequence
      if (waits_for_prefill) pdl_wait();
      return;
    }
    qo_row = q0;
  }
  const int32_t *table = p.block_tables + seq * p.bt_stride;
  auto chunk_of = [&](int it) { return split + nsplit * (warp + kWarpsM * it); };
  auto table_entry = [&](int ci) -> int32_t {  // page of chunk ci (block_size % 16 == 0)
    const int64_t col = static_cast<int64_t>(ci) * kChunk / p.block_size;
    return col < p.bt_stride ? __ldg(table + col) : -1;
  };
  // Pages in batches of 32 loop iterations: lane L holds the page of
  // iteration 32 * batch + L; the next batch is loaded a whole batch ahead
  // and page(it) is a shuffle, so no register move waits on a recent load.
  int32_t pg_cur = table_entry(chunk_of(lane)), pg_nxt = table_entry(chunk_of(32 + lane));
  auto page = [&](int it_now, int idx) -> int32_t {  // page of iteration idx (idx >= it_now)
    const int32_t a = __shfl_sync(kAll, pg_cur, idx & 31), b = __shfl_sync(kAll, pg_nxt, idx & 31);
    return (idx >> 5) == (it_now >> 5) ? a : b;
  };
  int ctx = mixed ? __ldg(p.cu_k + seq + 1) - __ldg(p.cu_k + seq) : __ldg(p.context_lens + seq);
  const int64_t slot = fused ? static_cast<int64_t>(__ldg(p.slot_mapping + seq)) : -1;
  // The ring's barriers are set up while those reads (the kernel's first global
  // accesses: context length, slot, block-table entries) are in flight.
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStagesM; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int64_t cap = p.bt_stride * p.block_size;
  if (ctx > cap) {
    if (threadIdx.x == 0 && split == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    ctx = static_cast<int>(cap);
  }
  // With the fused store, position ctx-1 is this step's token: folded in from
  // k_new/v_new by one warp of one split, not read from the pool.
  const bool fold = fused && slot >= 0 && ctx > 0;
  const int ctx_kv = fold ? ctx - 1 : ctx;
  const int nchunks = ctx_kv > 0 ? (ctx_kv + kChunk - 1) / kChunk : 0;
  const int first = split + nsplit * warp;
  const int stride = nsplit * kWarpsM;
  const int my_n = first < nchunks ? (nchunks - first + stride - 1) / stride : 0;
  // The token goes to the split that owns its chunk and, within it, to the
  // first warp with one chunk fewer than warp 0 (the last warp if all tie).
  const int new_split = ((ctx - 1) / kChunk) % nsplit;
  const int split_chunks = split < nchunks ? (nchunks - split + nsplit - 1) / nsplit : 0;
  const int new_warp = split_chunks % kWarpsM == 0 ? kWarpsM - 1 : split_chunks % kWarpsM;
  const bool own_new = fold && split == new_split && warp == new_warp;

  auto checked = [&](int32_t blk) -> int32_t {
    if (blk < 0 || blk >= p.num_blocks) {
      if (lane == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
      return -1;
    }
    return blk;
  };
  auto row_of = [&](int ci, int32_t blk) {
    return static_cast<int>(static_cast<int64_t>(blk) * p.block_size + (ci * kChunk) % p.block_size);
  };
  auto issue = [&](int ci, int st, int32_t blk) {
    if (lane != 0) return;
    if (blk < 0) {
      mbar_arrive(&wbar[st]);
      return;
    }
    const int row = row_of(ci, blk);
    uint8_t *dst = wstage + st * C::kStageBytes;
    mbar_arrive_expect_tx(&wbar[st], C::kStageBytes);
#pragma unroll
    for (int h = 0; h < C::kHalves; ++h) {
      tc::tma_load_3d(dst + h * 2048, &P.tmap_k, h * 64, kvh, row, &wbar[st]);
      tc::tma_load_3d(dst + C::kTileBytes + h * 2048, &P.tmap_v, h * 64, kvh, row, &wbar[st]);
    }
  };

  // Prologue: fill the ring, then wait on the preceding kernel (early_kv) and
  // let the next one start its prologue.  (An L2 prefetch of the chunks past
  // the ring measured slower: 3848 vs 4131 GB/s at batch 1 x 32K.)
  int issued = 0;
#pragma unroll
  for (int s = 0; s < kStagesM; ++s) {
    if (s < my_n) {
      issue(chunk_of(s), s, checked(page(0, s)));
      ++issued;
    }
  }
  if (p.early_kv) {
    pdl_launch_dependents();
    pdl_wait();
  }

  // Q^T of the group as m16n8k16 B fragments (column n = query g of the
  // group, zero for g >= G): b0 holds dims ks*16 + 2t, +1, b1 dims
  // ks*16 + 8 + 2t, +1.
  uint32_t qa[C::kKSteps][2];
  {
    const T *qrow = static_cast<const T *>(p.query) +
                    (qo_row * p.num_q_heads + static_cast<int64_t>(kvh) * G + (g < G ? g : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < C::kKSteps; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * t) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 8 + 2 * t) : 0u;
    }
  }
  const float sl2 = p.scale_log2;
  const uint32_t pbuf = smem_addr(pt_smem + warp * 256);

  // O^T accumulators: o[db] = O^T[dims db*16 + g, + 8][queries 2t, 2t + 1]
  // as {(g, 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)}; softmax state per query.
  float o[D / 16][4];
#pragma unroll
  for (int db = 0; db < D / 16; ++db) o[db][0] = o[db][1] = o[db][2] = o[db][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // queries 2t, 2t+1

  // Zero V rows [valid, 16) of a chunk so P = 0 never meets stale values.
  auto zero_v_tail = [&](uint32_t vtile, int valid) {
    for (int i = lane; i < (kChunk - valid) * (D / 8); i += 32) {
      const int row = valid + i / (D / 8), cj = i % (D / 8);
      asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(swz(vtile, row, cj)), "r"(0u)
                   : "memory");
    }
  };

  // This step's token (fused store) is the owning warp's last item: its K/V
  // rows are loaded here and written to shared memory and to their slot only
  // when that item comes up, so the load latency hides behind the cached
  // chunks.  Its one-key chunk sits in ring stage my_n % kStagesM, which holds
  // no chunk still to be processed by then (no refill reaches chunk my_n).
  const uint32_t fold_k = smem_addr(wstage + (my_n % kStagesM) * C::kStageBytes);
  const uint32_t fold_v = fold_k + C::kTileBytes;
  const bool new_lane = own_new && lane < 2 * (D / 8);
  const int new_kind = lane / (D / 8), new_cj = lane % (D / 8);
  uint4 new_row = make_uint4(0u, 0u, 0u, 0u);
  if (new_lane) {
    const int64_t off = seq * p.new_token_stride_bytes + static_cast<int64_t>(kvh) * D * sizeof(T);
    new_row = *reinterpret_cast<const uint4 *>((new_kind ? p.v_new : p.k_new) + off + new_cj * 16);
  }
  const int n_items = my_n + (own_new ? 1 : 0);

  // One chunk in the "swapped" form: S^T = K . Q^T (keys in M, the group in
  // N = 8), online softmax per query column, O^T += V^T . P^T with P^T handed
  // from the accumulator layout to the B-operand layout through 256 bytes of
  // shared memory.  16 MMAs per 16-key chunk.  The V^T fragments are loaded
  // right after the S MMAs so their latency overlaps the softmax.
  auto process = [&](uint32_t ktile, uint32_t vtile, int valid) {
    const int mi = lane >> 3, rr = lane & 7;
    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};  // even / odd k-steps
#pragma unroll
    for (int ks = 0; ks < C::kKSteps; ++ks) {
      uint32_t a0, a1, a2, a3;  // (keys 0-7 | 8-15) x (dims lo 8 | hi 8 of the k-step)
      ldsm_x4(swz(ktile, (mi & 1) * 8 + rr, ks * 2 + (mi >> 1)), a0, a1, a2, a3);
      if (ks & 1)
        mma_full<T>(sb, a0, a1, a2, a3, qa[ks][0], qa[ks][1]);
      else
        mma_full<T>(sa, a0, a1, a2, a3, qa[ks][0], qa[ks][1]);
    }
    uint32_t va[D / 16][4];  // V^T: (dims lo 8 | hi 8 of the block) x (keys 0-7 | 8-15)
#pragma unroll
    for (int db = 0; db < D / 16; ++db)
      ldsm_x4_t(swz(vtile, (mi >> 1) * 8 + rr, db * 2 + (mi & 1)), va[db][0], va[db][1], va[db][2],
                va[db][3]);
    // x: (key g, query 2t), (g, 2t+1), (g+8, 2t), (g+8, 2t+1)
    const bool k0 = g < valid, k1 = g + 8 < valid;
    float x[4] = {k0 ? (sa[0] + sb[0]) * sl2 : -INFINITY, k0 ? (sa[1] + sb[1]) * sl2 : -INFINITY,
                  k1 ? (sa[2] + sb[2]) * sl2 : -INFINITY, k1 ? (sa[3] + sb[3]) * sl2 : -INFINITY};
    float mx[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx[0] = fmaxf(mx[0], __shfl_xor_sync(kAll, mx[0], off));
      mx[1] = fmaxf(mx[1], __shfl_xor_sync(kAll, mx[1], off));
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      if (mx[c] > m_run[c] + 8.f) {  // lazy rescale: the lanes of a query column agree
        const float alpha = m_run[c] == -INFINITY ? 0.f : fast_exp2(m_run[c] - mx[c]);
#pragma unroll
        for (int db = 0; db < D / 16; ++db) {
          o[db][c] *= alpha;
          o[db][c + 2] *= alpha;
        }
        l_run[c] *= alpha;
        m_run[c] = mx[c];
      }
    }
    float pr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) pr[j] = x[j] == -INFINITY ? 0.f : fast_exp2(x[j] - m_run[j & 1]);
    l_run[0] += pr[0] + pr[2];
    l_run[1] += pr[1] + pr[3];
    // P^T rows (keys) of 8 queries x 16 bits
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(pbuf + g * 16 + 4 * t), "r"(pack2<T>(pr[0], pr[1]))
                 : "memory");
    asm volatile("st.shared.b32 [%0], %1;" ::"r"(pbuf + (g + 8) * 16 + 4 * t),
                 "r"(pack2<T>(pr[2], pr[3]))
                 : "memory");
    __syncwarp();
    uint32_t pb0, pb1;
    ldsm_x2_t(pbuf + (lane & 15) * 16, pb0, pb1);
#pragma unroll
    for (int db = 0; db < D / 16; ++db)
      mma_full<T>(o[db], va[db][0], va[db][1], va[db][2], va[db][3], pb0, pb1);
    __syncwarp();  // every lane has read P^T before the next item rewrites it
  };

  bool timed_out = false;
  int consumed = 0;  // cached chunks whose copies have landed, in order
#pragma unroll 1
  for (int it = 0; it < n_items; ++it) {
    uint32_t kt, vt;
    int valid;
    if (it < my_n) {
      const int st = it % kStagesM;
      if (!mbar_wait_bounded(&wbar[st], (it / kStagesM) & 1, p.status)) {
        timed_out = true;
        break;
      }
      consumed = it + 1;
      kt = smem_addr(wstage + st * C::kStageBytes);
      vt = kt + C::kTileBytes;
      valid = min(kChunk, ctx_kv - chunk_of(it) * kChunk);
      if (valid < kChunk) {
        zero_v_tail(vt, valid);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
    } else {  // this step's token, as a one-key chunk
      kt = fold_k;
      vt = fold_v;
      valid = 1;
      zero_v_tail(fold_v, 1);
      if (new_lane) {
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(
                         swz(new_kind ? fold_v : fold_k, 0, new_cj)),
                     "r"(new_row.x), "r"(new_row.y), "r"(new_row.z), "r"(new_row.w)
                     : "memory");
        if (slot < p.num_blocks * p.block_size)
          *reinterpret_cast<uint4 *>(const_cast<char *>(new_kind ? p.value_cache : p.key_cache) +
                                     (slot * p.num_kv_heads + kvh) * D * sizeof(T) + new_cj * 16) =
              new_row;
      }
      if (lane == 0 && slot >= p.num_blocks * p.block_size) flag_status(p.status, MI_DEV_BAD_SLOT);
    }
    __syncwarp();  // zeroed rows and the token's row are visible to every lane
    process(kt, vt, valid);
    if (it + kStagesM < my_n) {  // refill the stage just consumed
      issue(chunk_of(it + kStagesM), it % kStagesM, checked(page(it, it + kStagesM)));
      ++issued;
    }
    if ((it & 31) == 31) {  // the next iteration starts batch (it + 1) / 32
      pg_cur = pg_nxt;
      pg_nxt = table_entry(chunk_of(it + 33 + lane));
    }
  }
  if (timed_out) {
    if (lane == 0)
      for (int it = consumed + 1; it < issued; ++it)
        if (!mbar_wait_bounded(&wbar[it % kStagesM], (it / kStagesM) & 1, p.status)) break;
    __syncwarp();
    m_run[0] = m_run[1] = -INFINITY;
  }

  pdl_launch_dependents();

#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) l_run[c] += __shfl_xor_sync(kAll, l_run[c], off);

  // ---- merge the warps (shared memory aliases the drained ring) ----
  __syncthreads();
  float *mg_acc = reinterpret_cast<float *>(smem);  // [warps][G][D]
  float *mg_ml = mg_acc + kWarpsM * G * D;          // [warps][G][2]
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int q = 2 * t + c;
    if (q < G) {
#pragma unroll
      for (int db = 0; db < D / 16; ++db) {
        mg_acc[(warp * G + q) * D + db * 16 + g] = o[db][c];
        mg_acc[(warp * G + q) * D + db * 16 + g + 8] = o[db][c + 2];
      }
      if (g == 0) {
        mg_ml[(warp * G + q) * 2] = m_run[c];
        mg_ml[(warp * G + q) * 2 + 1] = l_run[c];
      }
    }
  }
  __syncthreads();
  constexpr int kIter = (G * D + kWarpsM * 32 - 1) / (kWarpsM * 32);
  float keep_m[kIter], keep_l[kIter], keep_a[kIter];
  if constexpr (kPair) cluster_wait_acquire();  // phase 1: rank 0 is running
#pragma unroll
  for (int k = 0; k < kIter; ++k) {
    const int i = threadIdx.x + k * kWarpsM * 32;
    if (i >= G * D) break;
    const int h = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsM; ++w) M = fmaxf(M, mg_ml[(w * G + h) * 2]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kWarpsM; ++w) {
      const float mw = mg_ml[(w * G + h) * 2];
      const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
      L += f * mg_ml[(w * G + h) * 2 + 1];
      A += f * mg_acc[(w * G + h) * D + d];
    }
    const int qh = kvh * G + h;
    if constexpr (kPair) {
      if (split == 1) {
        st_cluster_f32(xacc + h * D + d, 0, A);
        if (d == 0) {
          st_cluster_f32(xml + h * 2, 0, M);
          st_cluster_f32(xml + h * 2 + 1, 0, L);
        }
      }
      keep_m[k] = M;
      keep_l[k] = L;
      keep_a[k] = A;
    } else if (nsplit == 1) {
      T *out = static_cast<T *>(p.out) + (qo_row * p.num_q_heads + qh) * D;
      out[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
    } else {
      split_store_state(p, seq, qh, nsplit, split, D, d, M, L, A);
    }
  }
  if constexpr (kPair) {
    cluster_arrive_release();  // phase 2: rank 1's state is in rank 0's shared memory
    cluster_wait_acquire();
    if (split == 0) {
#pragma unroll
      for (int k = 0; k < kIter; ++k) {
        const int i = threadIdx.x + k * kWarpsM * 32;
        if (i >= G * D) break;
        const int h = i / D, d = i % D;
        const float m1 = xml[h * 2], l1 = xml[h * 2 + 1], a1 = xacc[h * D + d];
        const float M = fmaxf(keep_m[k], m1);
        const float f0 = keep_m[k] == -INFINITY ? 0.f : fast_exp2(keep_m[k] - M);
        const float f1 = m1 == -INFINITY ? 0.f : fast_exp2(m1 - M);
        const float L = f0 * keep_l[k] + f1 * l1, A = f0 * keep_a[k] + f1 * a1;
        T *out = static_cast<T *>(p.out) + (qo_row * p.num_q_heads + kvh * G + h) * D;
        out[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
      }
    }
  } else if (nsplit > 1) {
    split_arrive_and_merge<T, G, D>(p, seq, kvh, nsplit, last_flag);
  }
  if (waits_for_prefill) pdl_wait();
}

namespace {

template <typename T, int D, int G, bool kPair>
cudaError_t launch_mma_tdgp(const DecodeMmaParams &P, int64_t num_seqs, int nsplit,
                            cudaStream_t stream) {
  using C = MmaCfg<D>;
  auto kern = paged_decode_mma_kernel<T, D, G, kPair>;
  constexpr int smem = kPair ? C::kSmemPair : C::kSmem;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid(kPair ? 2 : nsplit, P.d.num_kv_heads, static_cast<unsigned>(num_seqs));
  return launch_pdl(kern, grid, dim3(kWarpsM * 32), smem, stream, kPair ? 2u : 1u, P);
}

template <typename T, int D, int G>
cudaError_t launch_mma_tdg(const DecodeMmaParams &P, int64_t num_seqs, int nsplit, bool pair,
                           cudaStream_t stream) {
  return pair ? launch_mma_tdgp<T, D, G, true>(P, num_seqs, 2, stream)
              : launch_mma_tdgp<T, D, G, false>(P, num_seqs, nsplit, stream);
}

template <typename T, int D>
cudaError_t launch_mma_td(const DecodeMmaParams &P, int G, int64_t n, int s, bool pair,
                          cudaStream_t st) {
  switch (G) {
    case 1: return launch_mma_tdg<T, D, 1>(P, n, s, pair, st);
    case 2: return launch_mma_tdg<T, D, 2>(P, n, s, pair, st);
    case 4: return launch_mma_tdg<T, D, 4>(P, n, s, pair, st);
    case 8: return launch_mma_tdg<T, D, 8>(P, n, s, pair, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

// bf16/fp16, D 64 or 128, GQA group 1..8, every 16-key chunk within one page.
bool decode_mma_supported(int dtype, int D, int G, int block_size) {
  if (dtype != MI_DTYPE_BFLOAT16 && dtype != MI_DTYPE_FLOAT16) return false;
  if ((D != 64 && D != 128) || (G != 1 && G != 2 && G != 4 && G != 8)) return false;
  if (block_size < kChunk || block_size % kChunk != 0) return false;
  return tensor_map_encoder() != nullptr;
}

cudaError_t launch_decode_mma(const DecodeParams &d, int dtype, int D, int G, int64_t num_seqs,
                              int nsplit, bool pair, cudaStream_t stream) {
  if (pair && (d.cu_q != nullptr || nsplit != 2)) return cudaErrorInvalidValue;
  const uint64_t rows = static_cast<uint64_t>(d.num_blocks) * d.block_size;
  if (rows == 0 || rows >= (1ull << 31) || num_seqs > 65535 || nsplit > 65535)
    return cudaErrorNotSupported;
  DecodeMmaParams P;
  memset(&P, 0, sizeof(P));
  P.d = d;
  const CUtensorMapDataType dt =
      dtype == MI_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t row_bytes = static_cast<uint64_t>(D) * 2;
  const uint64_t row_stride = static_cast<uint64_t>(d.num_kv_heads) * row_bytes;
  if (!encode_rows_map(&P.tmap_k, dt, d.key_cache, D, d.num_kv_heads, rows, row_bytes, row_stride,
                       64, 1, kChunk, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_rows_map(&P.tmap_v, dt, d.value_cache, D, d.num_kv_heads, rows, row_bytes,
                       row_stride, 64, 1, kChunk, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorNotSupported;
  if (dtype == MI_DTYPE_BFLOAT16)
    return D == 64 ? launch_mma_td<__nv_bfloat16, 64>(P, G, num_seqs, nsplit, pair, stream)
                   : launch_mma_td<__nv_bfloat16, 128>(P, G, num_seqs, nsplit, pair, stream);
  return D == 64 ? launch_mma_td<__half, 64>(P, G, num_seqs, nsplit, pair, stream)
                 : launch_mma_td<__half, 128>(P, G, num_seqs, nsplit, pair, stream);
}

}  // namespace mi
