// tcgen05 paged decode attention (sm_100a), "swap-AB" form.
//
// Decode has 1..8 query rows per kv head, far below the 128-row MMA tile, so
// the roles of keys and queries are swapped: per 128-key tile
//     S^T[128 keys x 16] = K_tile[128 x D] . Q^T[D x 16]     (M=128, N=16, K=D)
//     O^T[D x 16]       += V_tile^T[D x 128] . P^T[128 x 16] (M=D,  N=16, K=128)
// with the GQA group in the N dimension (padded to 16; the padding columns
// are never read).  The tensor core does all the multiply-adds, so the SMs
// only run a short softmax per tile and the kernel stays HBM-bound.
//
// One CTA per (split, kv head, sequence); split s owns key tiles s, s+S, ...
// 224 threads:
//   warp 0    K producer: TMA of 8 groups of 16 keys per tile (3-D map over
//             [slots, Hkv, D], slot from the block table, zero fill past the
//             context) into a 3-stage ring; the G query rows.
//   warp 6    V producer: the same for V, so K runs ahead of V (K frees after
//             the S MMA, V only after P.V).
//   warp 1    TMEM owner (64 columns) and single-thread MMA issuer, issuing
//             whichever of S(next) and P.V(next) is ready first.
//   warps 2-5 softmax, one key per thread: scores from TMEM, per-head tile
//             max (warp shuffle + a 128-thread barrier exchange), lazy rescale
//             of O^T (only when a head's max grows by more than 2^8), P^T
//             (double-buffered) written as the B operand of the next MMA;
//             epilogue with one head dimension per thread.
// With the fused store, this step's token (position ctx-1) is not read from
// the pool: the softmax warps of one split load its k_new/v_new rows, fold it
// into the final state and write it to its slot, so every cached tile can be
// requested before the preceding kernel finishes (early_kv).
// Splits store their states and the last one to finish merges them
// (split_merge.cuh).  Every wait is bounded; the softmax warps abort
// together (barrier.red.or), so no warp is ever left at a barrier.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "split_merge.cuh"
#include "tc_helpers.cuh"
#include "tmap.cuh"

namespace mi {

struct __align__(64) DecodeTcParams {
  CUtensorMap tmap_q;
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  DecodeParams d;
  int64_t kv_rows;  // extent of the K/V maps' row dimension (OOB coordinate)
};

namespace {

constexpr int kThreads = 224;
constexpr int kStages = 3;
constexpr int kTile = 32768;  // 128 keys x 128 dims x 2 bytes
constexpr int kHalf = 16384;
constexpr int kPBytes = 4096;  // P^T: 16 rows x 128 keys x 2 bytes
constexpr int kOffQ = 0;       // 16 rows x 128 dims: two 2 KB column halves
constexpr int kOffK = 4096;
constexpr int kOffV = kOffK + kStages * kTile;
constexpr int kOffP = kOffV + kStages * kTile;  // 2 buffers
constexpr int kOffRed = kOffP + 2 * kPBytes;    // [2][4 warps][8 heads] + [4][8]
constexpr int kOffBar = kOffRed + 1024;
constexpr int kSmemBytes = kOffBar + 256 + 1024;
constexpr uint32_t kTmemCols = 64;  // S^T x2 (16 each) + O^T (16)
constexpr unsigned kFull = 0xffffffffu;

enum {
  B_Q = 0,
  B_KFULL = 1,    // +stage (3)
  B_VFULL = 4,    // +stage
  B_KEMPTY = 7,   // +stage
  B_VEMPTY = 10,  // +stage
  B_SFULL = 13,   // +S buffer (2)
  B_SEMPTY = 15,  // +S buffer
  B_PFULL = 17,   // +P buffer (2)
  B_ODONE = 19,   // +P buffer: P.V of tiles with that parity done
  B_FIN = 21,
  B_COUNT = 22
};

__device__ __forceinline__ uint64_t k_desc(uint32_t tile, int kk) {  // K tile, K-major
  return tc::smem_desc_sw128(tile + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t small_desc(uint32_t base, int kk) {  // 16-row K-major (Q, P^T)
  return tc::smem_desc_sw128(base + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t v_desc(uint32_t tile, int kk) {  // V^T as MN-major A
  return tc::smem_desc_sw128(tile + kk * 2048, kHalf, 1024);
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

// Barrier over the 4 softmax warps (id 1, 128 threads) that also ORs `bad`.
__device__ __forceinline__ bool softmax_sync_any(bool bad) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pin, pout;\n\tsetp.ne.u32 pin, %1, 0;\n\t"
      "bar.red.or.pred pout, 1, 128, pin;\n\tselp.u32 %0, 1, 0, pout;\n\t}"
      : "=r"(r)
      : "r"(bad ? 1u : 0u)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

}  // namespace

template <typename T, int G>
__global__ void __launch_bounds__(kThreads, 1)
    paged_decode_tc_kernel(const __grid_constant__ DecodeTcParams P) {
  const DecodeParams &p = P.d;
  constexpr bool kBf16 = Elem<T>::kDtype == MI_DTYPE_BFLOAT16;
  constexpr uint32_t kIdescS = tc::idesc_f16(128, 16, kBf16 ? 1 : 0, false, false);
  constexpr uint32_t kIdescO = tc::idesc_f16(128, 16, kBf16 ? 1 : 0, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kOffBar);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + B_COUNT);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  float *red = reinterpret_cast<float *>(smem + kOffRed);  // [2][4][8] then [4][8]
  const uint32_t sQ = smem_addr(smem + kOffQ);
  const uint32_t sK = smem_addr(smem + kOffK);
  const uint32_t sV = smem_addr(smem + kOffV);
  const uint32_t sP = smem_addr(smem + kOffP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, nsplit = gridDim.x;
  const int kvh = blockIdx.y;
  const int64_t seq = blockIdx.z;

  if (threadIdx.x == 0) {
    mbar_init(&bar[B_Q], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bar[B_KFULL + s], 1);
      mbar_init(&bar[B_VFULL + s], 1);
      mbar_init(&bar[B_KEMPTY + s], 1);
      mbar_init(&bar[B_VEMPTY + s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar[B_SFULL + b], 1);
      mbar_init(&bar[B_SEMPTY + b], 128);
      mbar_init(&bar[B_PFULL + b], 128);
      mbar_init(&bar[B_ODONE + b], 1);
    }
    mbar_init(&bar[B_FIN], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tc::tmem_alloc(tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 32;

  // Without early_kv everything below may come from the preceding kernel.
  if (!p.early_kv) pdl_wait();
  int ctx = p.context_lens[seq];
  const int64_t cap = p.bt_stride * p.block_size;
  if (ctx > cap) {
    if (threadIdx.x == 0 && split == 0) flag_status(p.status, MI_DEV_BAD_BLOCK);
    ctx = static_cast<int>(cap);
  }
  const int64_t slot = p.k_new != nullptr ? static_cast<int64_t>(p.slot_mapping[seq]) : -1;
  // With the fused store, position ctx-1 is this step's token, folded in from
  // k_new/v_new by one split instead of being read back from the pool.
  const bool fold = slot >= 0 && ctx > 0;
  const int ctx_kv = fold ? ctx - 1 : ctx;  // keys read from the pool
  const bool own_new = fold && split == ((ctx - 1) / 128) % nsplit;
  const int ntiles = ctx_kv > 0 ? (ctx_kv + 127) / 128 : 0;
  const int my_n = split < ntiles ? (ntiles - split + nsplit - 1) / nsplit : 0;
  auto tile_of = [&](int it) { return split + nsplit * it; };

  if (warp == 0 || warp == 6) {
    // ------------------------------------------------------------ producers
    const bool is_v = warp == 6;
    const int32_t *table = p.block_tables + seq * p.bt_stride;
    const CUtensorMap *map = is_v ? &P.tmap_v : &P.tmap_k;
    uint8_t *ring = smem + (is_v ? kOffV : kOffK);
    uint64_t *full_b = &bar[is_v ? B_VFULL : B_KFULL];
    uint64_t *empty_b = &bar[is_v ? B_VEMPTY : B_KEMPTY];
    const int g = lane >> 1, dh = lane & 1;  // lanes 0..15: (16-key group, column half)
    auto row_of = [&](int it) -> int {
      if (lane >= 16 || it >= my_n) return 0;
      const int key0 = tile_of(it) * 128 + g * 16;
      if (key0 >= ctx_kv) return static_cast<int>(P.kv_rows);  // zero fill
      const int64_t col = key0 / p.block_size;
      const int64_t blk = col < p.bt_stride ? table[col] : -1;
      if (blk < 0 || blk >= p.num_blocks) {
        flag_status(p.status, MI_DEV_BAD_BLOCK);
        return static_cast<int>(P.kv_rows);
      }
      return static_cast<int>(blk * p.block_size + key0 % p.block_size);
    };
    auto load = [&](int it, int row) -> bool {
      const int s = it % kStages;
      int good = 1;
      if (lane == 0)
        good = mbar_wait_bounded(&empty_b[s], ((it / kStages) & 1) ^ 1, p.status) &&
               !*(volatile int *)abort_flag;
      if (!__shfl_sync(kFull, good, 0)) return false;
      if (lane == 0) mbar_arrive_expect_tx(&full_b[s], kTile);
      __syncwarp();
      if (lane < 16)
        tc::tma_load_3d(ring + s * kTile + dh * kHalf + g * 2048, map, dh * 64, kvh, row, &full_b[s]);
      return true;
    };
    if (lane == 0) tc::prefetch_tmap(map);
    bool ok = true;
    int row = row_of(0);
    int it = 0;
    for (; it < kStages && it < my_n && ok; ++it) {
      const int next_row = row_of(it + 1);
      ok = load(it, row);
      row = next_row;
    }
    if (p.early_kv) {
      if (!is_v) pdl_launch_dependents();
      pdl_wait();
    }
    if (!is_v && lane == 0) {
      mbar_arrive_expect_tx(&bar[B_Q], 2 * G * 128);
      for (int h2 = 0; h2 < 2; ++h2)
        tc::tma_load_3d(smem + kOffQ + h2 * 2048, &P.tmap_q, h2 * 64, kvh * G,
                        static_cast<int>(seq), &bar[B_Q]);
    }
    for (; it < my_n && ok; ++it) {
      const int next_row = row_of(it + 1);  // table lookup of the next tile overlaps the wait
      ok = load(it, row);
      row = next_row;
    }
    if (!ok && lane == 0) *(volatile int *)abort_flag = 1;
    // Every load this warp issued lands before the CTA can exit.
    if (lane == 0) {
      const int issued = ok ? my_n : it;
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait_bounded(&full_b[j % kStages], (j / kStages) & 1, p.status);
      if (!is_v) mbar_wait_bounded(&bar[B_Q], 0, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Polls (test_wait) for whichever of S(next) and P.V(next) is ready first.
    if (lane == 0) {
      bool ok = mbar_wait_bounded(&bar[B_Q], 0, p.status);
      int ns = 0, npv = 0;  // next S tile, next P.V tile
      // The timeout clock (%globaltimer) is read only every 256 idle polls and
      // restarts whenever an MMA is issued.
      uint32_t idle = 0;
      uint64_t idle_since = 0;
      while (ok && npv < my_n) {
        bool progress = false;
        if (ns < my_n) {
          const int s = ns % kStages, b = ns & 1;
          if (mbar_test(&bar[B_KFULL + s], (ns / kStages) & 1) &&
              mbar_test(&bar[B_SEMPTY + b], ((ns >> 1) & 1) ^ 1)) {
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              tc::umma_f16(tS + b * 16, k_desc(sK + s * kTile, kk), small_desc(sQ, kk), kIdescS,
                           kk > 0 ? 1u : 0u);
            tc::umma_commit(&bar[B_SFULL + b]);
            tc::umma_commit(&bar[B_KEMPTY + s]);
            ++ns;
            progress = true;
          }
        }
        if (npv < ns) {
          const int s = npv % kStages, pb = npv & 1;
          if (mbar_test(&bar[B_PFULL + pb], (npv >> 1) & 1) &&
              mbar_test(&bar[B_VFULL + s], (npv / kStages) & 1)) {
            tc::fence_after_sync();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              tc::umma_f16(tO, v_desc(sV + s * kTile, kk), small_desc(sP + pb * kPBytes, kk),
                           kIdescO, (npv > 0 || kk > 0) ? 1u : 0u);
            tc::umma_commit(&bar[B_ODONE + pb]);
            tc::umma_commit(&bar[B_VEMPTY + s]);
            ++npv;
            progress = true;
          }
        }
        if (progress) {
          idle = 0;
          idle_since = 0;
        } else if (*(volatile int *)abort_flag) {
          ok = false;
        } else if ((++idle & 255u) == 0) {
          const uint64_t now = global_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > kWaitLimitNs) {
            flag_status(p.status, MI_DEV_TIMEOUT);
            ok = false;
          }
        }
      }
      if (!ok) *(volatile int *)abort_flag = 1;
      tc::umma_commit(&bar[B_FIN]);
      mbar_wait_bounded(&bar[B_FIN], 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int k = q4 * 32 + lane;  // key of the tile (S^T lane) / dimension (O^T lane)
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    // This step's token: dimension k of its K and V rows (produced by the
    // preceding kernel, so read after the dependency wait).
    float kn = 0.f, vn = 0.f;
    if (own_new) {
      if (p.early_kv) pdl_wait();
      const int64_t off = seq * p.new_token_stride_bytes + static_cast<int64_t>(kvh) * 256 + k * 2;
      kn = Elem<T>::to_float(*reinterpret_cast<const T *>(p.k_new + off));
      vn = Elem<T>::to_float(*reinterpret_cast<const T *>(p.v_new + off));
    }
    float m[G], lp[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m[h] = -INFINITY;
      lp[h] = 0.f;
    }
    bool ok = true;
    for (int it = 0; it < my_n; ++it) {
      const int b = it & 1;
      const bool good = __all_sync(kFull, mbar_wait_bounded(&bar[B_SFULL + b], (it >> 1) & 1, p.status) &&
                                              !*(volatile int *)abort_flag);
      float sv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) sv[i] = 0.f;
      if (good) {
        tc::fence_after_sync();
        tc::tmem_ld16(tS + b * 16 + lane_off, sv);
        tc::tmem_wait_ld();
        tc::fence_before_sync();
      }
      mbar_arrive(&bar[B_SEMPTY + b]);

      const bool valid = tile_of(it) * 128 + k < ctx_kv;
      float x[G];
#pragma unroll
      for (int h = 0; h < G; ++h) x[h] = valid ? sv[h] * p.scale_log2 : -INFINITY;
      // per-head max of this tile over all 128 keys
      float *rb = red + b * 32;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float wm = warp_max(x[h]);
        if (lane == 0) rb[q4 * 8 + h] = wm;
      }
      if (softmax_sync_any(!good)) {  // also publishes rb to the other warps
        ok = false;
        break;
      }
      float mn[G], alpha[G];
      bool rescale = false;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float tm = fmaxf(fmaxf(rb[h], rb[8 + h]), fmaxf(rb[16 + h], rb[24 + h]));
        mn[h] = tm > m[h] + 8.f ? tm : m[h];
        alpha[h] = mn[h] == m[h] ? 1.f : (m[h] == -INFINITY ? 0.f : fast_exp2(m[h] - mn[h]));
        rescale |= mn[h] != m[h] && m[h] != -INFINITY;
      }
      float pv[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        pv[h] = x[h] == -INFINITY ? 0.f : fast_exp2(x[h] - mn[h]);
        lp[h] = lp[h] * alpha[h] + pv[h];
      }
      // Rescaling O^T needs the previous tile's P.V done; reusing P^T buffer b
      // needs the P.V two tiles back done.  Both decisions are CTA-uniform.
      const bool need_r = rescale && it >= 1, need_p = it >= 2;
      if (need_r || need_p) {
        bool w = true;
        if (need_r) w &= mbar_wait_bounded(&bar[B_ODONE + ((it - 1) & 1)], ((it - 1) >> 1) & 1, p.status);
        if (need_p) w &= mbar_wait_bounded(&bar[B_ODONE + b], ((it - 2) >> 1) & 1, p.status);
        if (softmax_sync_any(!__all_sync(kFull, w))) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        if (need_r) {
          float o[16];
          tc::tmem_ld16(tO + lane_off, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < G; ++h) o[h] *= alpha[h];
          tc::tmem_st16(tO + lane_off, o);
          tc::tmem_wait_st();
        }
      }
      const uint32_t pbase = sP + b * kPBytes;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const uint32_t addr = pbase + (k >> 6) * 2048 + h * 128 +
                              ((((k & 63) >> 3) ^ (h & 7)) << 4) + (k & 7) * 2;
        const T v = Elem<T>::from_float(pv[h]);
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr),
                     "h"(*reinterpret_cast<const unsigned short *>(&v))
                     : "memory");
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc::fence_before_sync();
      mbar_arrive(&bar[B_PFULL + b]);
#pragma unroll
      for (int h = 0; h < G; ++h) m[h] = mn[h];
    }
    // ---- epilogue: thread k holds head dimension d = k of O^T ----
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i] = 0.f;
    if (ok && my_n > 0) {
      const int last = my_n - 1;
      const bool w = __all_sync(kFull, mbar_wait_bounded(&bar[B_ODONE + (last & 1)], (last >> 1) & 1, p.status));
      ok = !softmax_sync_any(!w);
      if (ok) {
        tc::fence_after_sync();
        tc::tmem_ld16(tO + lane_off, o);
        tc::tmem_wait_ld();
      }
    }
    if (!ok) {
      if (lane == 0) *(volatile int *)abort_flag = 1;
#pragma unroll
      for (int h = 0; h < G; ++h) m[h] = -INFINITY;
    }
    float *lred = red + 64;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float s = warp_sum(lp[h]);
      if (lane == 0) lred[q4 * 8 + h] = s;
    }
    float snew[G];
    if (own_new) {
      // q_h . k_new over the 128 dimensions (thread k holds dimension k)
      if (my_n == 0) mbar_wait_bounded(&bar[B_Q], 0, p.status);
      float *dred = red + 96;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const uint32_t qaddr = sQ + (k >> 6) * 2048 + h * 128 + ((((k & 63) >> 3) ^ (h & 7)) << 4) +
                               (k & 7) * 2;
        unsigned short raw;
        asm volatile("ld.shared.b16 %0, [%1];" : "=h"(raw) : "r"(qaddr) : "memory");
        const float part = warp_sum(Elem<T>::to_float(*reinterpret_cast<const T *>(&raw)) * kn);
        if (lane == 0) dred[q4 * 8 + h] = part;
      }
      softmax_sync_any(false);
#pragma unroll
      for (int h = 0; h < G; ++h)
        snew[h] = (dred[h] + dred[8 + h] + dred[16 + h] + dred[24 + h]) * p.scale_log2;
    } else {
      softmax_sync_any(false);
    }
    const int d = k;
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float L = lred[h] + lred[8 + h] + lred[16 + h] + lred[24 + h];
      float M = m[h];
      float A = o[h];
      if (own_new) {
        const float mn = fmaxf(M, snew[h]);
        const float alpha = M == -INFINITY ? 0.f : fast_exp2(M - mn);
        const float pn = fast_exp2(snew[h] - mn);
        A = A * alpha + pn * vn;
        L = L * alpha + pn;
        M = mn;
      }
      const int qh = kvh * G + h;
      if (nsplit == 1) {
        T *orow = static_cast<T *>(p.out) + (seq * p.num_q_heads + qh) * 128;
        orow[d] = Elem<T>::from_float(L > 0.f ? A / L : 0.f);
      } else {
        split_store_state(p, seq, qh, nsplit, split, 128, d, M, L, A);
      }
    }
    if (own_new) {
      if (slot < p.num_blocks * p.block_size) {
        const int64_t off = (slot * p.num_kv_heads + kvh) * 256 + k * 2;
        *reinterpret_cast<T *>(const_cast<char *>(p.key_cache) + off) = Elem<T>::from_float(kn);
        *reinterpret_cast<T *>(const_cast<char *>(p.value_cache) + off) = Elem<T>::from_float(vn);
      } else if (k == 0) {
        flag_status(p.status, MI_DEV_BAD_SLOT);
      }
    }
  }

  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
  if (nsplit > 1) split_arrive_and_merge<T, G, 128>(p, seq, kvh, nsplit, abort_flag + 1);
}

namespace {

bool encode(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t heads,
            uint64_t rows, uint64_t row_stride_bytes, uint32_t box_y, uint32_t box_z) {
  return encode_rows_map(map, dt, base, 128, heads, rows, 256, row_stride_bytes, 64, box_y, box_z,
                         CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int G>
cudaError_t launch_tg(const DecodeTcParams &P, int64_t num_seqs, int nsplit, cudaStream_t stream) {
  auto kern = paged_decode_tc_kernel<T, G>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, P.d.num_kv_heads, static_cast<unsigned>(num_seqs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, P);
}

}  // namespace

bool decode_tc_supported(int dtype, int D, int G, int block_size) {
  if (dtype != MI_DTYPE_BFLOAT16 && dtype != MI_DTYPE_FLOAT16) return false;
  if (D != 128 || (G != 1 && G != 2 && G != 4 && G != 8)) return false;
  if (block_size < 16 || block_size % 16 != 0) return false;
  return tensor_map_encoder() != nullptr;
}

cudaError_t launch_decode_tc(const DecodeParams &d, int dtype, int G, int64_t num_seqs,
                             int64_t num_blocks, int nsplit, cudaStream_t stream) {
  if (num_seqs > 65535 || nsplit > 65535) return cudaErrorNotSupported;
  const CUtensorMapDataType dt =
      dtype == MI_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  DecodeTcParams P;
  memset(&P, 0, sizeof(P));
  const uint64_t rows = static_cast<uint64_t>(num_blocks) * d.block_size;
  if (rows == 0 || rows >= (1ull << 31)) return cudaErrorNotSupported;
  if (!encode(&P.tmap_q, dt, d.query, d.num_q_heads, num_seqs,
              static_cast<uint64_t>(d.num_q_heads) * 256, G, 1) ||
      !encode(&P.tmap_k, dt, d.key_cache, d.num_kv_heads, rows,
              static_cast<uint64_t>(d.num_kv_heads) * 256, 1, 16) ||
      !encode(&P.tmap_v, dt, d.value_cache, d.num_kv_heads, rows,
              static_cast<uint64_t>(d.num_kv_heads) * 256, 1, 16))
    return cudaErrorInvalidValue;
  P.d = d;
  P.kv_rows = static_cast<int64_t>(rows);
  cudaError_t e;
  if (dtype == MI_DTYPE_BFLOAT16) {
    switch (G) {
      case 1: e = launch_tg<__nv_bfloat16, 1>(P, num_seqs, nsplit, stream); break;
      case 2: e = launch_tg<__nv_bfloat16, 2>(P, num_seqs, nsplit, stream); break;
      case 4: e = launch_tg<__nv_bfloat16, 4>(P, num_seqs, nsplit, stream); break;
      default: e = launch_tg<__nv_bfloat16, 8>(P, num_seqs, nsplit, stream); break;
    }
  } else {
    switch (G) {
      case 1: e = launch_tg<__half, 1>(P, num_seqs, nsplit, stream); break;
      case 2: e = launch_tg<__half, 2>(P, num_seqs, nsplit, stream); break;
      case 4: e = launch_tg<__half, 4>(P, num_seqs, nsplit, stream); break;
      default: e = launch_tg<__half, 8>(P, num_seqs, nsplit, stream); break;
    }
  }
  return e;
}

}  // namespace mi
