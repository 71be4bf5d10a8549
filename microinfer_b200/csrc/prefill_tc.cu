// tcgen05 (UMMA + TMEM) paged chunked-prefill attention for sm_100a.
//
// Work unit: a pair of 128-row query tiles (each TQ = 128/G tokens x the G
// query heads of one kv head) against every cached key of the sequence up to
// the tile's last position, in 128-key tiles; K/V tiles are shared by both
// query tiles.  Roles, TMEM layout and the MMA order are described above
// prefill_tc2_kernel.
//
// Shared memory operands use the SWIZZLE_128B canonical layout (8 rows x 128
// bytes atoms); a 128x128 16-bit tile is two 16 KB column halves.  K/V groups
// of 16 keys come from a 3-D tensor map over [slots, Hkv, D]; each group's
// slot comes from the block table, groups past the context load from an
// out-of-range coordinate (zero fill), and the rows past the context inside
// the last, partial group are zeroed in shared memory before P.V reads them.
//
// Dense mode (no block table) reads K/V rows cu_seqlens_k[s] + key of a
// contiguous [tokens, Hkv, D] tensor: the no-prefix ("direct") prefill.
// Every mbarrier wait is bounded; a timeout flags MI_DEV_TIMEOUT, unwinds,
// waits for this CTA's own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"
#include "tc_helpers.cuh"
#include "tmap.cuh"

namespace mi {

struct __align__(64) PrefillTcParams {
  CUtensorMap tmap_q;
  CUtensorMap tmap_k;
  CUtensorMap tmap_v;
  void *out;
  const int32_t *cu_q;
  const int32_t *cu_k;
  const int32_t *block_tables;
  int64_t bt_stride;
  int64_t num_blocks;
  int64_t kv_rows;  // extent of the K/V maps' row dimension (OOB coordinate)
  int32_t block_size;
  int32_t num_q_heads;
  int32_t paged;
  float scale_log2;
  int32_t *status;
  // Mixed batches: sequences with one query token are left to the decode kernel
  // launched right after this one, which may start once every CTA here has passed
  // its dependency wait (so the trigger comes early).
  int32_t skip_single;
  // prefill_tc2_kernel's work items: units (seq, kv head, tile pair) in the
  // order tile pair, kv head, sequence; units from split_from on run as two
  // single-tile items each, so a last round that would be less than half full
  // of pairs becomes one round of single tiles.
  int32_t pairs_per_seq;
  int32_t num_kv_heads;
  int64_t split_from;
  int64_t num_items;  // pair units before split_from, single tiles from there on
};

namespace {

constexpr int kTileBytes = 32768;  // 128 x 128 x 16-bit
constexpr int kHalf = 16384;
constexpr int kKStages = 3;  // K is released after S (early), so it runs deeper than V
constexpr int kVStages = 2;
constexpr uint32_t kTmemCols = 512;


// K-major SW128 descriptor of 16-element K-step `kk` of a 128 x 128 tile.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int kk) {
  return tc::smem_desc_sw128(tile + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor (V as the B operand): K-step kk = 16 key rows.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int kk) {
  return tc::smem_desc_sw128(tile + kk * 2048, kHalf, 1024);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t *>(&h);
}

}  // namespace

// ---------------------------------------------------------------------------
// Two query tiles per work item, persistent CTAs (prefill_tc2_kernel).
//
// Work item = (tile pair, kv head, sequence): query tiles A (tokens t0 ..
// t0+TQ-1) and B (the next TQ tokens) of one kv head share every K/V tile, so
// each key tile crosses into the SM once for 256 query rows.  Items from
// split_from on are single tiles (halves of the last pairs), so the last round
// of items is not half empty.  One CTA per SM takes items blockIdx.x,
// blockIdx.x + gridDim.x, ...; barriers, TMEM and the rings stay up across
// items, so the next item's Q and K/V loads and its first S = Q.K^T products
// run while the previous item's last P.V and output are still in flight (a
// CTA per item paid ~10 us of setup, ramp and drain on every item).
// 352 threads:
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: one TMEM lane
//               (= query row) per thread, the whole 128-key row in registers;
//               then the item's output rows
//   warp 8      TMA: Q of both tiles (once the previous item's last S has
//               read Q), then the K tiles (3-stage ring)
//   warp 9      TMEM owner and single-thread MMA issuer
//   warp 10     TMA: the V tiles (2-stage ring)
// TMEM (512 columns): S_A at 0, S_B at 128, O_A at 256, O_B at 384.  The
// softmax writes P (16-bit pairs) over the first 64 columns of its S and P.V
// reads A from TMEM, so P never goes through shared memory.  The MMA issuer
// alternates the tiles,
//   S_A(0) S_B(0) | PV_A(0) S_A(1) | PV_B(0) S_B(1) | PV_A(1) S_A(2) | ...
// so one tile's softmax runs while the tensor core works for the other.
// tcgen05.mma ops of one thread run in issue order: S_X(j+1) overwrites P_X(j)
// only after PV_X(j) has read it, and once S_X(j+1) is complete PV_X(j) is
// too, so the softmax may rescale O_X right after S_X(j+1) is ready.  The
// first P.V of an item (which overwrites O_X) waits until the softmax warps
// of tile X have read the previous item's O_X.
//
// Every barrier phase is counted per role across items (ring slots, S/P/O
// handoffs per tile, Q, the V fix-up), so the parities agree without any
// per-item reset.
namespace {

constexpr int kThreads2 = 352;
constexpr int kOffQ2 = 0;  // Q_A, Q_B
constexpr int kOffK2 = kOffQ2 + 2 * kTileBytes;
constexpr int kOffV2 = kOffK2 + kKStages * kTileBytes;
constexpr int kOffBar2 = kOffV2 + kVStages * kTileBytes;
constexpr int kSmemBytes2 = kOffBar2 + 256 + 1024;

enum {
  C_Q = 0,       // Q of the current item landed
  C_QEMPTY = 1,  // the item's last S MMA completed: Q may be overwritten
  C_KFULL = 2,   // +K stage (3)
  C_KEMPTY = 5,  // +K stage
  C_VFULL = 8,   // +V stage (2)
  C_VEMPTY = 10, // +V stage
  C_SFULL = 12,  // +tile: S_X(j) (and everything issued before it) done
  C_PFULL = 14,  // +tile: P_X(j) in TMEM (128 softmax threads)
  C_ODONE = 16,  // +tile: the item's last MMA done, O_X final
  C_OEMPTY = 18, // +tile: the item's O_X read out (128 softmax threads)
  C_FIN = 20,
  // +V stage: rows past the context in the tile's last group zeroed (32 lanes of
  // warp 10).  One per ring slot: a slot is refilled only after the MMA issuer has
  // released it, so a slot's fix-ups never run two phases ahead of the issuer.
  C_VFIX = 21,
  C_COUNT = 23
};

// Warp-uniform: this lane's wait succeeded in every lane and nobody aborted.
__device__ __forceinline__ bool warp_all_ok(bool ok, const int *abort_flag) {
  return __all_sync(0xffffffffu, ok && !*(volatile const int *)abort_flag);
}

__device__ __forceinline__ bool aborted(const int *abort_flag) {
  return *(volatile const int *)abort_flag != 0;
}

// One work item, as every role sees it.
struct Item {
  int64_t seq;
  int kvh, t0, q_start, q_len, kv0, ctx, prefix;
  int nt[2], nkv_t[2], nkv;
  int fix_tile, fix_group, fix_valid;
  bool skip;  // nothing to do (a sequence with fewer tile pairs, or a decode row)
};

template <int G>
__device__ __forceinline__ Item item_at(const PrefillTcParams &p, int64_t idx) {
  constexpr int TQ = 128 / G;
  Item it;
  const bool single = idx >= p.split_from;
  const int64_t unit = single ? p.split_from + (idx - p.split_from) / 2 : idx;
  const int half = single ? static_cast<int>((idx - p.split_from) & 1) : 0;
  const int pair = static_cast<int>(unit % p.pairs_per_seq);
  it.kvh = static_cast<int>((unit / p.pairs_per_seq) % p.num_kv_heads);
  it.seq = unit / (static_cast<int64_t>(p.pairs_per_seq) * p.num_kv_heads);
  it.q_start = __ldg(p.cu_q + it.seq);
  it.q_len = __ldg(p.cu_q + it.seq + 1) - it.q_start;
  it.t0 = pair * 2 * TQ + half * TQ;
  it.skip = it.t0 >= it.q_len || (p.skip_single && it.q_len == 1);
  it.kv0 = __ldg(p.cu_k + it.seq);
  it.ctx = __ldg(p.cu_k + it.seq + 1) - it.kv0;
  it.prefix = it.ctx - it.q_len;
  it.nt[0] = it.skip ? 0 : min(TQ, it.q_len - it.t0);
  it.nt[1] = it.skip || single ? 0 : max(0, min(TQ, it.q_len - it.t0 - TQ));
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    const int maxpos = it.prefix + it.t0 + x * TQ + it.nt[x] - 1;
    it.nkv_t[x] = it.nt[x] > 0 && maxpos >= 0 ? maxpos / 128 + 1 : 0;
  }
  it.nkv = max(it.nkv_t[0], it.nkv_t[1]);
  // The last key tile may hold a partial 16-key group (rows ctx % 16 .. 15 of
  // it lie past the context and hold stale pool contents, or another
  // sequence's rows in dense mode).  They meet P = 0, but 0 * Inf or NaN is
  // NaN, so the V producer zeroes them before P.V reads that tile.
  it.fix_tile = (it.nkv > 0 && it.ctx % 16 != 0 && (it.ctx - 1) / 128 == it.nkv - 1) ? it.nkv - 1 : -1;
  it.fix_group = ((it.ctx - 1) % 128) / 16;
  it.fix_valid = it.ctx % 16;
  return it;
}

}  // namespace

template <typename T, int G>
__global__ void __launch_bounds__(kThreads2, 1)
    prefill_tc2_kernel(const __grid_constant__ PrefillTcParams p) {
  constexpr int TQ = 128 / G;  // tokens per tile
  constexpr bool kBf16 = sizeof(T) == 2 && Elem<T>::kDtype == MI_DTYPE_BFLOAT16;
  constexpr uint32_t kIdescQK = tc::idesc_f16(128, 128, kBf16 ? 1 : 0, false);
  constexpr uint32_t kIdescPV = tc::idesc_f16(128, 128, kBf16 ? 1 : 0, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~static_cast<uintptr_t>(1023));
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + kOffBar2);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar + C_COUNT);
  int *abort_flag = reinterpret_cast<int *>(tmem_slot + 1);
  const uint32_t sQ = smem_addr(smem + kOffQ2);
  const uint32_t sK = smem_addr(smem + kOffK2);
  const uint32_t sV = smem_addr(smem + kOffV2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  T *out = static_cast<T *>(p.out);

  if (threadIdx.x == 0) {
    mbar_init(&bar[C_Q], 1);
    mbar_init(&bar[C_QEMPTY], 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&bar[C_KFULL + s], 1);
      mbar_init(&bar[C_KEMPTY + s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&bar[C_VFULL + s], 1);
      mbar_init(&bar[C_VEMPTY + s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bar[C_SFULL + x], 1);
      mbar_init(&bar[C_PFULL + x], 128);
      mbar_init(&bar[C_ODONE + x], 1);
      mbar_init(&bar[C_OEMPTY + x], 128);
    }
    mbar_init(&bar[C_FIN], 1);
    for (int s = 0; s < kVStages; ++s) mbar_init(&bar[C_VFIX + s], 32);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) tc::tmem_alloc(tmem_slot, kTmemCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();
  if (p.skip_single) pdl_launch_dependents();
  const int64_t n_items = p.num_items;

  if (warp == 8 || warp == 10) {
    // ---------------------------------------------------------- producers
    // warp 8 loads Q and the K tiles, warp 10 the V tiles.  Block-table
    // lookups in batches of 4 tiles, one batch ahead.
    const bool is_v = warp == 10;
    const int nst = is_v ? kVStages : kKStages;
    const CUtensorMap *map = is_v ? &p.tmap_v : &p.tmap_k;
    uint8_t *ring = smem + (is_v ? kOffV2 : kOffK2);
    const int full0 = is_v ? C_VFULL : C_KFULL, empty0 = is_v ? C_VEMPTY : C_KEMPTY;
    const int g = lane >> 1, dh = lane & 1;
    const int bt = lane >> 3, bg = lane & 7;
    if (lane == 0) {
      tc::prefetch_tmap(map);
      if (!is_v) tc::prefetch_tmap(&p.tmap_q);
    }
    bool ok = true;
    uint32_t tiles = 0;  // tiles issued by this warp so far (ring position)
    uint32_t items_q = 0;
    for (int64_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
      const Item it = item_at<G>(p, idx);
      if (it.skip || it.nkv == 0) continue;
      const int32_t *table = p.block_tables + it.seq * p.bt_stride;
      auto kv_entry = [&](int key0) -> int {
        if (key0 >= it.ctx || !p.paged) return 0;
        const int64_t col = key0 / p.block_size;
        return col < p.bt_stride ? __ldg(table + col) : -1;
      };
      auto kv_row = [&](int key0, int entry) -> int {
        if (key0 >= it.ctx) return static_cast<int>(p.kv_rows);  // past the context: zero fill
        if (!p.paged) return it.kv0 + key0;
        if (entry < 0 || entry >= p.num_blocks) {
          flag_status(p.status, MI_DEV_BAD_BLOCK);
          return static_cast<int>(p.kv_rows);
        }
        return static_cast<int>(static_cast<int64_t>(entry) * p.block_size + key0 % p.block_size);
      };
      if (!is_v) {  // Q of both tiles, once the previous item's S products have read Q
        int good = 1;
        if (lane == 0)
          good = mbar_wait_bounded(&bar[C_QEMPTY], (items_q & 1) ^ 1, p.status) && !aborted(abort_flag);
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int ntiles = it.nt[1] > 0 ? 2 : 1;
          mbar_arrive_expect_tx(&bar[C_Q], ntiles * 2 * kHalf);
          for (int x = 0; x < ntiles; ++x)
            for (int h = 0; h < 2; ++h)
              tc::tma_load_3d(smem + kOffQ2 + x * kTileBytes + h * kHalf, &p.tmap_q, h * 64,
                              it.kvh * G, it.q_start + it.t0 + x * TQ, &bar[C_Q]);
        }
        ++items_q;
      }
      auto entry_for = [&](int tile) { return tile < it.nkv ? kv_entry(tile * 128 + bg * 16) : 0; };
      int cur = entry_for(bt), nxt = entry_for(4 + bt);
      for (int j = 0; j < it.nkv; ++j) {
        const uint32_t s = tiles % nst;
        const uint32_t empty_parity = ((tiles / nst) & 1) ^ 1;
        if (j > 0 && (j & 3) == 0) {
          cur = nxt;
          nxt = entry_for(j + 4 + bt);
        }
        const int entry = __shfl_sync(0xffffffffu, cur, ((j & 3) * 8 + g) & 31);
        const int row = lane < 16 ? kv_row(j * 128 + g * 16, entry) : 0;
        int good = 1;
        if (lane == 0)
          good = mbar_wait_bounded(&bar[empty0 + s], empty_parity, p.status) && !aborted(abort_flag);
        if (!__shfl_sync(0xffffffffu, good, 0)) {
          ok = false;
          break;
        }
        if (lane == 0) mbar_arrive_expect_tx(&bar[full0 + s], kTileBytes);
        __syncwarp();
        if (lane < 16)
          tc::tma_load_3d(ring + s * kTileBytes + dh * kHalf + g * 2048, map, dh * 64, it.kvh, row,
                          &bar[full0 + s]);
        if (is_v && j == it.fix_tile) {
          // Wait for the tile, zero the group's rows past the context (both 64-column
          // halves; whole 128-byte rows, so the swizzle does not matter), make the
          // writes visible to the tensor core and release the tile to the MMA issuer.
          int landed = 1;
          if (lane == 0) landed = mbar_wait_bounded(&bar[full0 + s], (tiles / nst) & 1, p.status);
          landed = __shfl_sync(0xffffffffu, landed, 0);
          if (landed) {
            uint8_t *grp = ring + s * kTileBytes + it.fix_group * 2048;
            for (int i = lane; i < (16 - it.fix_valid) * 16; i += 32) {
              const int rr = it.fix_valid + i / 16, c = i % 16;
              *reinterpret_cast<uint4 *>(grp + (c >> 3) * kHalf + rr * 128 + (c & 7) * 16) =
                  make_uint4(0u, 0u, 0u, 0u);
            }
          } else {
            ok = false;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          mbar_arrive(&bar[C_VFIX + s]);
        }
        ++tiles;
        if (!ok) break;
      }
    }
    if (!ok && lane == 0) {
      *(volatile int *)abort_flag = 1;
      // Let this CTA's own loads in flight land before its shared memory goes away.
      const uint32_t lo = tiles > static_cast<uint32_t>(nst) ? tiles - nst : 0;
      for (uint32_t t = lo; t < tiles; ++t)
        mbar_wait_bounded(&bar[full0 + t % nst], (t / nst) & 1, p.status);
      if (!is_v && items_q > 0) mbar_wait_bounded(&bar[C_Q], (items_q - 1) & 1, p.status);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t kt = 0, vt = 0;            // K / V tiles consumed (ring positions)
      uint32_t sc[2] = {0, 0};            // S_X products issued
      uint32_t uses[2] = {0, 0};          // items that used tile X
      uint32_t items_q = 0;
      uint32_t fixes[kVStages] = {0, 0};  // fix-ups consumed per V ring slot
      bool ok = true;
      // Descriptors are built once; a K step or a ring slot only moves the start
      // address field (bits 0-13, in 16-byte units), so each MMA's operands are a
      // base plus a constant: this lone thread shares its SM sub-partition with two
      // busy softmax warps, and every issue slot it spends delays the tensor pipe.
      const uint64_t qd0 = kmajor_desc(sQ, 0), kd0 = kmajor_desc(sK, 0), vd0 = mnmajor_desc(sV, 0);
      constexpr uint64_t kTile16 = kTileBytes >> 4;
      auto kstep = [](int kk) -> uint64_t {  // K-major offset of K step kk, 16-byte units
        return static_cast<uint64_t>(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4);
      };
      auto s_mma = [&](int x) {  // S_X = Q_X K^T with the K tile at ring position kt
        const uint64_t qd = qd0 + x * kTile16, kd = kd0 + (kt % kKStages) * kTile16;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::umma_f16(tmem + x * 128, qd + kstep(kk), kd + kstep(kk), kIdescQK, kk > 0 ? 1u : 0u);
        tc::umma_commit(&bar[C_SFULL + x]);
        ++sc[x];
      };
      auto pv_mma = [&](int x, int j) -> bool {  // O_X += P_X(j) V_j, P from TMEM
        if (!mbar_spin_bounded(&bar[C_PFULL + x], (sc[x] - 1) & 1, p.status)) return false;
        tc::fence_after_sync();
        const uint64_t vd = vd0 + (vt % kVStages) * kTile16;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc::umma_f16_tmem_a(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, vd + kk * (2048 >> 4),
                              kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        return true;
      };
      for (int64_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
        const Item it = item_at<G>(p, idx);
        if (it.skip || it.nkv == 0) continue;
        const bool use0 = it.nkv_t[0] > 0, use1 = it.nkv_t[1] > 0;
        ok = mbar_spin_bounded(&bar[C_Q], items_q & 1, p.status) &&
             mbar_spin_bounded(&bar[C_KFULL + kt % kKStages], (kt / kKStages) & 1, p.status) &&
             !aborted(abort_flag);
        ++items_q;
        if (!ok) break;
        tc::fence_after_sync();
        if (use0) s_mma(0);
        if (use1) s_mma(1);
        tc::umma_commit(&bar[C_KEMPTY + kt % kKStages]);
        ++kt;
        if (it.nkv == 1) tc::umma_commit(&bar[C_QEMPTY]);
        for (int j = 0; j < it.nkv && ok; ++j) {
          const bool nA = j + 1 < it.nkv_t[0], nB = j + 1 < it.nkv_t[1];
          ok = mbar_spin_bounded(&bar[C_VFULL + vt % kVStages], (vt / kVStages) & 1, p.status) &&
               (!(nA || nB) ||
                mbar_spin_bounded(&bar[C_KFULL + kt % kKStages], (kt / kKStages) & 1, p.status)) &&
               !aborted(abort_flag);
          if (ok && j == it.fix_tile) {
            const uint32_t vs = vt % kVStages;
            ok = mbar_spin_bounded(&bar[C_VFIX + vs], fixes[vs]++ & 1, p.status);
          }
          // The first P.V of a tile overwrites O_X: the previous item's O_X must be read out.
          if (ok && j == 0 && use0) ok = mbar_spin_bounded(&bar[C_OEMPTY], (uses[0] & 1) ^ 1, p.status);
          if (ok && j == 0 && use1) ok = mbar_spin_bounded(&bar[C_OEMPTY + 1], (uses[1] & 1) ^ 1, p.status);
          if (!ok) break;
          tc::fence_after_sync();
          if (j < it.nkv_t[0] && !(ok = pv_mma(0, j))) break;
          if (nA) s_mma(0);
          if (j < it.nkv_t[1] && !(ok = pv_mma(1, j))) break;
          if (nB) s_mma(1);
          if (nA || nB) {
            tc::umma_commit(&bar[C_KEMPTY + kt % kKStages]);
            ++kt;
            if (j + 2 == it.nkv) tc::umma_commit(&bar[C_QEMPTY]);  // the item's last S issued
          }
          tc::umma_commit(&bar[C_VEMPTY + vt % kVStages]);
          ++vt;
        }
        if (!ok) break;
        if (use0) tc::umma_commit(&bar[C_ODONE]);
        if (use1) tc::umma_commit(&bar[C_ODONE + 1]);
        uses[0] += use0 ? 1 : 0;
        uses[1] += use1 ? 1 : 0;
      }
      if (!ok) *(volatile int *)abort_flag = 1;
      // Every MMA issued by this thread completes before TMEM is released.
      tc::umma_commit(&bar[C_FIN]);
      mbar_spin_bounded(&bar[C_FIN], 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int x = warp >= 4 ? 1 : 0;  // query tile
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // TMEM lane = query row of the tile
    const int tok = r / G;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t tS = tmem + x * 128 + lane_off, tO = tmem + 256 + x * 128 + lane_off;
    const float sl2 = p.scale_log2;
    const bool pos_scale = sl2 >= 0.f;
    const float masked = pos_scale ? -INFINITY : INFINITY;
    uint32_t sc = 0, uses = 0;  // S_X tiles consumed, items that used tile X
    bool ok = true;
    for (int64_t idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x) {
      const Item it = item_at<G>(p, idx);
      if (it.skip || it.nt[x] == 0) continue;
      const bool rvalid = tok < it.nt[x];
      const int pos = it.prefix + it.t0 + x * TQ + tok;
      const int my_nkv = it.nkv_t[x];
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < my_nkv; ++j) {
        if (!warp_all_ok(mbar_wait_bounded(&bar[C_SFULL + x], sc & 1, p.status), abort_flag)) {
          ok = false;
          break;
        }
        ++sc;
        tc::fence_after_sync();
        // The whole row in registers: one TMEM round trip per tile.
        float sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tc::tmem_ld32(tS + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) sr[c * 32 + i] = v[i];
        }
        tc::tmem_wait_ld();
        // key c of the tile is visible iff c <= pos - j * 128: only diagonal
        // tiles (and rows past the chunk) mask anything.
        const int lim = rvalid ? pos - j * 128 : -1;
        if (lim < 127) {
#pragma unroll
          for (int c = 0; c < 128; ++c) sr[c] = c <= lim ? sr[c] : masked;
        }
        float r4[4] = {masked, masked, masked, masked};
        if (pos_scale) {
#pragma unroll
          for (int c = 0; c < 128; c += 2) r4[(c >> 1) & 3] = fmax3(r4[(c >> 1) & 3], sr[c], sr[c + 1]);
        } else {
#pragma unroll
          for (int c = 0; c < 128; c += 2) r4[(c >> 1) & 3] = fmin3(r4[(c >> 1) & 3], sr[c], sr[c + 1]);
        }
        const float best = pos_scale ? fmaxf(fmaxf(r4[0], r4[1]), fmaxf(r4[2], r4[3]))
                                     : fminf(fminf(r4[0], r4[1]), fminf(r4[2], r4[3]));
        const float mx = lim < 0 ? -INFINITY : best * sl2;  // row max, log2 domain
        float m_new = m, alpha = 1.f;
        bool rescale = false;
        if (mx > m + 8.f) {
          m_new = mx;
          rescale = m != -INFINITY;
          alpha = rescale ? fast_exp2(m - m_new) : 0.f;
        }
        // P = 2^(s * scale - m) as 16-bit pairs over the first 64 columns of S
        // (the row is already read back).
        const float nb = m_new == -INFINITY ? 0.f : -m_new;  // masked: ex2(-inf) = 0
        const float2 sc2 = make_float2(sl2, sl2), nb2 = make_float2(nb, nb);
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // keys 16q .. 16q+15 -> columns 8q .. 8q+7
          float pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 a2 = ffma2(make_float2(sr[q * 16 + 2 * i], sr[q * 16 + 2 * i + 1]), sc2, nb2);
            const float2 e = make_float2(fast_exp2(a2.x), fast_exp2(a2.y));
            sum2[i & 1] = fadd2(sum2[i & 1], e);
            pk[i] = __uint_as_float(pack2(e.x, e.y, kBf16));
          }
          tc::tmem_st8(tS + q * 8, pk);
        }
        // O_X is quiescent here (PV_X(j-1) completed before S_X(j) did) and
        // PV_X(j) waits for this thread's arrival below.
        if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
          const float ra = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tc::tmem_ld32(tO + c * 32, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= ra;
            tc::tmem_st32(tO + c * 32, o);
          }
        }
        tc::tmem_wait_st();
        tc::fence_before_sync();
        mbar_arrive(&bar[C_PFULL + x]);
        const float2 s01 = fadd2(sum2[0], sum2[1]);
        l = l * alpha + (s01.x + s01.y);
        m = m_new;
      }
      if (!ok) break;
      if (my_nkv > 0) {
        ok = warp_all_ok(mbar_wait_bounded(&bar[C_ODONE + x], uses & 1, p.status), abort_flag);
        if (!ok) break;
        tc::fence_after_sync();
      }
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T *orow = out + (static_cast<int64_t>(it.q_start + it.t0 + x * TQ + tok) * p.num_q_heads +
                       it.kvh * G + r % G) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (my_nkv > 0) {
          tc::tmem_ld32(tO + c * 32, o);
          tc::tmem_wait_ld();
        } else {  // no visible key (context shorter than the chunk): zeros
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (rvalid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack2(o[i] * inv, o[i + 1] * inv, kBf16);
            w.y = pack2(o[i + 2] * inv, o[i + 3] * inv, kBf16);
            w.z = pack2(o[i + 4] * inv, o[i + 5] * inv, kBf16);
            w.w = pack2(o[i + 6] * inv, o[i + 7] * inv, kBf16);
            *reinterpret_cast<uint4 *>(orow + c * 32 + i) = w;
          }
        }
      }
      if (my_nkv > 0) {  // O_X is read: the next item's first P.V may overwrite it
        tc::fence_before_sync();
        mbar_arrive(&bar[C_OEMPTY + x]);
        ++uses;
      }
    }
    if (!ok && lane == 0) *(volatile int *)abort_flag = 1;
  }

  pdl_launch_dependents();
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 9) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

namespace {

// 3-D map (x = D columns, y = heads, z = rows) with a {64, box_y, box_z} box.
bool encode_3d(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t d, uint64_t heads,
               uint64_t rows, uint64_t head_stride_bytes, uint64_t row_stride_bytes, uint32_t box_y,
               uint32_t box_z) {
  return encode_rows_map(map, dt, base, d, heads, rows, head_stride_bytes, row_stride_bytes, 64,
                         box_y, box_z, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename T, int G>
cudaError_t launch_tg2(PrefillTcParams &p, int num_kv_heads, int64_t num_seqs, int32_t max_seqlen_q,
                       cudaStream_t stream) {
  auto kern = prefill_tc2_kernel<T, G>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes2);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  constexpr int TQ = 128 / G;
  const int64_t pairs = (max_seqlen_q + 2 * TQ - 1) / (2 * TQ);
  const int64_t units = pairs * num_kv_heads * num_seqs;
  const int64_t sms = sm_count_current();
  const int64_t rem = units % sms;  // pair units of the last (partial) round
  const int64_t split = units > sms && rem > 0 && 2 * rem <= sms ? rem : 0;
  if (units + split > 0x7fffffff) return cudaErrorNotSupported;
  p.pairs_per_seq = static_cast<int32_t>(pairs);
  p.num_kv_heads = num_kv_heads;
  p.split_from = units - split;
  p.num_items = units + split;
  // one persistent CTA per SM (or per item, when there are fewer)
  const int64_t ctas = p.num_items < sms ? p.num_items : sms;
  return launch_pdl(kern, dim3(static_cast<unsigned>(ctas)), dim3(kThreads2), kSmemBytes2, stream, p);
}

}  // namespace

bool prefill_tc_supported(int dtype, int D, int G, int block_size) {
  if (dtype != MI_DTYPE_BFLOAT16 && dtype != MI_DTYPE_FLOAT16) return false;
  if (D != 128) return false;
  if (G != 1 && G != 2 && G != 4 && G != 8) return false;
  if (block_size < 16 || block_size % 16 != 0) return false;
  return tensor_map_encoder() != nullptr;
}

cudaError_t launch_prefill_tc(const AttnParams &a, int dtype, int G, int32_t max_seqlen_q, bool paged,
                              cudaStream_t stream) {
  if (a.num_seqs > 65535 || a.num_kv_heads > 65535) return cudaErrorNotSupported;
  const int e = 2;
  const CUtensorMapDataType dt =
      dtype == MI_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t D = 128;
  PrefillTcParams p;
  memset(&p, 0, sizeof(p));
  const uint32_t TQ = 128 / G;
  if (!encode_3d(&p.tmap_q, dt, a.query, D, a.num_q_heads, a.num_tokens, D * e,
                 static_cast<uint64_t>(a.num_q_heads) * D * e, G, TQ))
    return cudaErrorInvalidValue;
  uint64_t rows, row_stride;
  if (paged) {
    rows = static_cast<uint64_t>(a.num_blocks) * a.block_size;
    row_stride = static_cast<uint64_t>(a.num_kv_heads) * D * e;
  } else {
    rows = static_cast<uint64_t>(a.kv_rows);
    row_stride = static_cast<uint64_t>(a.kv_token_stride) * e;
  }
  if (rows == 0 || rows >= (1ull << 31)) return cudaErrorNotSupported;
  if (!encode_3d(&p.tmap_k, dt, a.key_base, D, a.num_kv_heads, rows, D * e, row_stride, 1, 16) ||
      !encode_3d(&p.tmap_v, dt, a.value_base, D, a.num_kv_heads, rows, D * e, row_stride, 1, 16))
    return cudaErrorInvalidValue;
  p.out = a.out;
  p.cu_q = a.cu_q;
  p.cu_k = a.cu_k;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.num_blocks = a.num_blocks;
  p.kv_rows = static_cast<int64_t>(rows);
  p.block_size = paged ? a.block_size : 16;
  p.num_q_heads = a.num_q_heads;
  p.paged = paged ? 1 : 0;
  p.scale_log2 = a.scale_log2;
  p.status = a.status;
  p.skip_single = paged && a.mixed_decode ? 1 : 0;
  const int64_t n = a.num_seqs;
  if (dtype == MI_DTYPE_BFLOAT16) {
    switch (G) {
      case 1: return launch_tg2<__nv_bfloat16, 1>(p, a.num_kv_heads, n, max_seqlen_q, stream);
      case 2: return launch_tg2<__nv_bfloat16, 2>(p, a.num_kv_heads, n, max_seqlen_q, stream);
      case 4: return launch_tg2<__nv_bfloat16, 4>(p, a.num_kv_heads, n, max_seqlen_q, stream);
      default: return launch_tg2<__nv_bfloat16, 8>(p, a.num_kv_heads, n, max_seqlen_q, stream);
    }
  }
  switch (G) {
    case 1: return launch_tg2<__half, 1>(p, a.num_kv_heads, n, max_seqlen_q, stream);
    case 2: return launch_tg2<__half, 2>(p, a.num_kv_heads, n, max_seqlen_q, stream);
    case 4: return launch_tg2<__half, 4>(p, a.num_kv_heads, n, max_seqlen_q, stream);
    default: return launch_tg2<__half, 8>(p, a.num_kv_heads, n, max_seqlen_q, stream);
  }
}

}  // namespace mi
