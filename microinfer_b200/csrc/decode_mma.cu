// Warp-level tensor-core paged decode (mma.sync m16n8k16, sm_100a).
//
// Decode has at most 8 query rows per kv head.  On this part a tcgen05.mma
// costs about the same time at N=16 as at N=256, so the swap-AB tcgen05
// kernel spends ~1 us of tensor time per 128-key tile; CUDA-core dot
// products cost ~26 warp instructions per key.  The warp-level m16n8k16 MMA
// does a 16-key chunk of a kv head in 32 MMAs + 16 ldmatrix:
//   S[16 x 16 keys]  = Q[16 x D] . K^T   (rows >= G of Q are zero)
//   O[16 x D]       += P[16 x 16] . V      (P re-packed from S's registers)
// i.e. ~5 warp instructions per key, with everything in registers.
//
// One CTA per (split, kv head, sequence), 8 warps.  Each warp streams its
// own 16-key chunks (ids strided over splits and warps) through a 3-stage
// ring: per chunk one TMA copy per 64-dim half for K and for V (3-D tensor
// map over [slots][Hkv][D], box {64, 1, 16}, 128-byte swizzle, so ldmatrix
// reads are bank-conflict free).  Pages beyond the ring are prefetched into
// L2 before the dependency wait (early_kv), the block table in batches of
// 32 chunks loaded a batch ahead.  Online softmax in the log2 domain with lazy rescale; the
// warps merge in shared memory, the splits through the workspace
// (split_merge.cuh).  With the fused store, this step's token is folded in as
// a one-key chunk built from k_new/v_new (by the warp with the fewest chunks,
// right after the dependency wait) and written to its slot.
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
constexpr int kAheadM = 4;  // chunks per warp prefetched into L2 beyond the ring

template <int D>
struct MmaCfg {
  static constexpr int kHalves = D / 64;             // 128-byte swizzled column halves
  static constexpr int kTileBytes = kHalves * 2048;  // 16 rows x D of one operand
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kKSteps = D / 16;
  static constexpr int kNBlocks = D / 8;
  static constexpr int kSmemStages = kWarpsM * kStagesM * kStageBytes;
  static constexpr int kSmemFold = kStageBytes;  // this step's token as a one-key chunk
  static constexpr int kSmemBars = kWarpsM * kStagesM * 8;
  static constexpr int kSmem = kSmemStages + kSmemFold + kSmemBars + 16 + 1024;  // + alignment slack
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

template <typename T, int D, int G>
__global__ void __launch_bounds__(kWarpsM * 32, 1)
    paged_decode_mma_kernel(const __grid_constant__ DecodeMmaParams P) {
  using C = MmaCfg<D>;
  const DecodeParams &p = P.d;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint8_t *fold_tile = smem + C::kSmemStages;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::kSmemStages + C::kSmemFold);
  int *last_flag = reinterpret_cast<int *>(bars + kWarpsM * kStagesM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;  // fragment row / column pair
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int kvh = blockIdx.y;
  const int64_t seq = blockIdx.z;
  uint64_t *wbar = bars + warp * kStagesM;
  uint8_t *wstage = smem + warp * kStagesM * C::kStageBytes;
  const bool fused = p.k_new != nullptr;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kStagesM; ++s) mbar_init(&wbar[s], 1);
    fence_mbar_init();
    tc::prefetch_tmap(&P.tmap_k);
    tc::prefetch_tmap(&P.tmap_v);
  }
  __syncwarp();

  // Without early_kv everything below may come from the preceding kernel.
  if (!p.early_kv) pdl_wait();
  const int32_t *table = p.block_tables + seq * p.bt_stride;
  auto chunk_of = [&](int it) { return split + nsplit * (warp + kWarpsM * it); };
  auto table_entry = [&](int ci) -> int32_t {  // page of chunk ci (block_size % 16 == 0)
    const int64_t col = static_cast<int64_t>(ci) * kChunk / p.block_size;
    return col < p.bt_stride ? __ldg(table + col) : -1;
  };
  constexpr int kWin = kStagesM + kAheadM;
  // Pages in batches of 32 loop iterations: lane L holds the page of
  // iteration 32 * batch + L; the next batch is loaded a whole batch ahead
  // and page(it) is a shuffle, so no register move waits on a recent load.
  int32_t pg_cur = table_entry(chunk_of(lane)), pg_nxt = table_entry(chunk_of(32 + lane));
  auto page = [&](int it_now, int idx) -> int32_t {  // page of iteration idx (idx >= it_now)
    const int32_t a = __shfl_sync(kAll, pg_cur, idx & 31), b = __shfl_sync(kAll, pg_nxt, idx & 31);
    return (idx >> 5) == (it_now >> 5) ? a : b;
  };
  int ctx = __ldg(p.context_lens + seq);
  const int64_t slot = fused ? static_cast<int64_t>(__ldg(p.slot_mapping + seq)) : -1;
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

  // Prologue: fill the ring, warm L2 with the next chunks, then wait on the
  // preceding kernel (early_kv) and let the next one start its prologue.
  int issued = 0;
#pragma unroll
  for (int s = 0; s < kStagesM; ++s) {
    if (s < my_n) {
      issue(chunk_of(s), s, checked(page(0, s)));
      ++issued;
    }
  }
#pragma unroll
  for (int j = kStagesM; j < kWin; ++j) {
    const int32_t blk = page(0, j);
    if (lane == 0 && j < my_n && blk >= 0 && blk < p.num_blocks) {
      const int row = row_of(chunk_of(j), blk);
#pragma unroll
      for (int h = 0; h < C::kHalves; ++h) {
        tc::tma_prefetch_l2_3d(&P.tmap_k, h * 64, kvh, row);
        tc::tma_prefetch_l2_3d(&P.tmap_v, h * 64, kvh, row);
      }
    }
  }
  if (p.early_kv) {
    pdl_launch_dependents();
    pdl_wait();
  }

  // Query rows of the group as m16n8k16 A fragments: row g < G is query head
  // kvh * G + g; a0 holds dims ks*16 + 2t, +1 and a2 dims ks*16 + 8 + 2t, +1.
  uint32_t qa[C::kKSteps][2];
  {
    const T *qrow = static_cast<const T *>(p.query) +
                    (seq * p.num_q_heads + static_cast<int64_t>(kvh) * G + (g < G ? g : 0)) * D;
#pragma unroll
    for (int ks = 0; ks < C::kKSteps; ++ks) {
      qa[ks][0] = g < G ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 2 * t) : 0u;
      qa[ks][1] = g < G ? *reinterpret_cast<const uint32_t *>(qrow + ks * 16 + 8 + 2 * t) : 0u;
    }
  }
  const float sl2 = p.scale_log2;

  float o[C::kNBlocks][4];
#pragma unroll
  for (int nb = 0; nb < C::kNBlocks; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;  // row g; l_run covers this lane's columns

  // Zero V rows [valid, 16) of a chunk so P = 0 never meets stale values.
  auto zero_v_tail = [&](uint32_t vtile, int valid) {
    for (int i = lane; i < (kChunk - valid) * (D / 8); i += 32) {
      const int row = valid + i / (D / 8), cj = i % (D / 8);
      asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(swz(vtile, row, cj)), "r"(0u)
                   : "memory");
    }
  };

  // One chunk: S = Q K^T, online softmax, O += P V.
  auto process = [&](uint32_t ktile, uint32_t vtile, int valid) {
    // two accumulator sets per key block (even / odd k-steps) halve the
    // dependent MMA chain
    float s0[2][4] = {}, s1[2][4] = {};
    const int mi = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int ks = 0; ks < C::kKSteps; ++ks) {
      uint32_t b00, b01, b10, b11;  // keys 0-7 / 8-15, dims lo / hi 8 of the k-step
      ldsm_x4(swz(ktile, (mi >> 1) * 8 + rr, ks * 2 + (mi & 1)), b00, b01, b10, b11);
      mma_rows8<T>(s0[ks & 1], qa[ks][0], qa[ks][1], b00, b01);
      mma_rows8<T>(s1[ks & 1], qa[ks][0], qa[ks][1], b10, b11);
    }
    // row g, keys 2t, 2t+1, 8+2t, 9+2t
    float x[4] = {s0[0][0] + s0[1][0], s0[0][1] + s0[1][1], s1[0][0] + s1[1][0],
                  s1[0][1] + s1[1][1]};
    const int kidx[4] = {2 * t, 2 * t + 1, 8 + 2 * t, 9 + 2 * t};
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[j] = kidx[j] < valid ? x[j] * sl2 : -INFINITY;
      mx = fmaxf(mx, x[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(kAll, mx, 2));
    if (mx > m_run + 8.f) {  // lazy rescale: the four lanes of a row agree
      const float alpha = m_run == -INFINITY ? 0.f : fast_exp2(m_run - mx);
#pragma unroll
      for (int nb = 0; nb < C::kNBlocks; ++nb) {
        o[nb][0] *= alpha;
        o[nb][1] *= alpha;
      }
      l_run *= alpha;
      m_run = mx;
    }
    float pr[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      pr[j] = x[j] == -INFINITY ? 0.f : fast_exp2(x[j] - m_run);
      l_run += pr[j];
    }
    const uint32_t pa0 = pack2<T>(pr[0], pr[1]), pa2 = pack2<T>(pr[2], pr[3]);
#pragma unroll
    for (int np = 0; np < C::kNBlocks / 2; ++np) {
      uint32_t v0, v1, v2, v3;  // (keys 0-7 | 8-15) x (dims np*16 + 0..7 | 8..15)
      ldsm_x4_t(swz(vtile, (mi & 1) * 8 + rr, np * 2 + (mi >> 1)), v0, v1, v2, v3);
      mma_rows8<T>(o[2 * np], pa0, pa2, v0, v1);
      mma_rows8<T>(o[2 * np + 1], pa0, pa2, v2, v3);
    }
  };

  // ---- this step's token, as a one-key chunk in its own buffer, first ----
  if (own_new) {
    const uint32_t kt = smem_addr(fold_tile), vt = kt + C::kTileBytes;
    zero_v_tail(vt, 1);
    const int64_t off = seq * p.new_token_stride_bytes + static_cast<int64_t>(kvh) * D * sizeof(T);
    const bool store = slot < p.num_blocks * p.block_size;
    if (lane < 2 * (D / 8)) {
      const int kind = lane / (D / 8), cj = lane % (D / 8);
      const uint4 v = *reinterpret_cast<const uint4 *>((kind ? p.v_new : p.k_new) + off + cj * 16);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(swz(kind ? vt : kt, 0, cj)),
                   "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                   : "memory");
      if (store)
        *reinterpret_cast<uint4 *>(const_cast<char *>(kind ? p.value_cache : p.key_cache) +
                                   (slot * p.num_kv_heads + kvh) * D * sizeof(T) + cj * 16) = v;
    }
    if (!store && lane == 0) flag_status(p.status, MI_DEV_BAD_SLOT);
    __syncwarp();
    process(kt, vt, 1);
  }

  bool timed_out = false;
  int consumed = 0;
#pragma unroll 1
  for (int it = 0; it < my_n; ++it) {
    const int st = it % kStagesM;
    const int ci = chunk_of(it);
    if (!mbar_wait_bounded(&wbar[st], (it / kStagesM) & 1, p.status)) {
      timed_out = true;
      break;
    }
    consumed = it + 1;
    const uint32_t kt = smem_addr(wstage + st * C::kStageBytes);
    const uint32_t vt = kt + C::kTileBytes;
    const int valid = min(kChunk, ctx_kv - ci * kChunk);
    if (valid < kChunk) {
      zero_v_tail(vt, valid);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
    }
    process(kt, vt, valid);
    __syncwarp();  // every lane's ldmatrix of this stage is done before it is refilled
    if (it + kStagesM < my_n) {
      issue(chunk_of(it + kStagesM), st, checked(page(it, it + kStagesM)));
      ++issued;
    }
    // Rolling L2 prefetch of the chunk kWin - 1 ahead (the prologue covered
    // the first kWin), so long contexts keep kWin chunks per warp in flight.
    const int32_t pf_blk = page(it, it + kWin - 1);
    if (it > 0 && lane == 0 && it + kWin - 1 < my_n) {
      const int32_t blk = pf_blk;
      if (blk >= 0 && blk < p.num_blocks) {
        const int row = row_of(chunk_of(it + kWin - 1), blk);
#pragma unroll
        for (int h = 0; h < C::kHalves; ++h) {
          tc::tma_prefetch_l2_3d(&P.tmap_k, h * 64, kvh, row);
          tc::tma_prefetch_l2_3d(&P.tmap_v, h * 64, kvh, row);
        }
      }
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
    m_run = -INFINITY;
  }

  pdl_launch_dependents();

  // ---- merge the warps (shared memory aliases the drained ring) ----
  l_run += __shfl_xor_sync(kAll, l_run, 1);
  l_run += __shfl_xor_sync(kAll, l_run, 2);
  __syncthreads();
  float *mg_acc = reinterpret_cast<float *>(smem);  // [warps][G][D]
  float *mg_ml = mg_acc + kWarpsM * G * D;          // [warps][G][2]
  if (g < G) {
#pragma unroll
    for (int nb = 0; nb < C::kNBlocks; ++nb)
      *reinterpret_cast<float2 *>(&mg_acc[(warp * G + g) * D + nb * 8 + 2 * t]) =
          make_float2(o[nb][0], o[nb][1]);
    if (t == 0) {
      mg_ml[(warp * G + g) * 2] = m_run;
      mg_ml[(warp * G + g) * 2 + 1] = l_run;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
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
    if (nsplit == 1) {
      T *out = static_cast<T *>(p.out) + (seq * p.num_q_heads + qh) * D;
      out[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
    } else {
      split_store_state(p, seq, qh, nsplit, split, D, d, M, L, A);
    }
  }
  if (nsplit > 1) split_arrive_and_merge<T, G, D>(p, seq, kvh, nsplit, last_flag);
}

namespace {

template <typename T, int D, int G>
cudaError_t launch_mma_tdg(const DecodeMmaParams &P, int64_t num_seqs, int nsplit,
                           cudaStream_t stream) {
  using C = MmaCfg<D>;
  auto kern = paged_decode_mma_kernel<T, D, G>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const dim3 grid(nsplit, P.d.num_kv_heads, static_cast<unsigned>(num_seqs));
  return launch_pdl(kern, grid, dim3(kWarpsM * 32), C::kSmem, stream, P);
}

template <typename T, int D>
cudaError_t launch_mma_td(const DecodeMmaParams &P, int G, int64_t n, int s, cudaStream_t st) {
  switch (G) {
    case 1: return launch_mma_tdg<T, D, 1>(P, n, s, st);
    case 2: return launch_mma_tdg<T, D, 2>(P, n, s, st);
    case 4: return launch_mma_tdg<T, D, 4>(P, n, s, st);
    case 8: return launch_mma_tdg<T, D, 8>(P, n, s, st);
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
                              int nsplit, cudaStream_t stream) {
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
    return D == 64 ? launch_mma_td<__nv_bfloat16, 64>(P, G, num_seqs, nsplit, stream)
                   : launch_mma_td<__nv_bfloat16, 128>(P, G, num_seqs, nsplit, stream);
  return D == 64 ? launch_mma_td<__half, 64>(P, G, num_seqs, nsplit, stream)
                 : launch_mma_td<__half, 128>(P, G, num_seqs, nsplit, stream);
}

}  // namespace mi
