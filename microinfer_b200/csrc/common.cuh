// Shared device helpers for the sm_100a paged KV-cache kernels: element
// traits, 16-byte vector conversion, mbarrier + bulk-copy wrappers, bounded
// waits and the device status word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/microinfer_b200.h"

namespace mi {

// ---------------------------------------------------------------------------
// element traits
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kDtype = MI_DTYPE_FLOAT32;
  __device__ static float to_float(float x) { return x; }
  __device__ static float from_float(float x) { return x; }
};
template <> struct Elem<__half> {
  static constexpr int kDtype = MI_DTYPE_FLOAT16;
  __device__ static float to_float(__half x) { return __half2float(x); }
  __device__ static __half from_float(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kDtype = MI_DTYPE_BFLOAT16;
  __device__ static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// Unpack one 16-byte vector of T into float pairs (2 floats per float2).
// bf16 -> f32 is exact bit placement: low half << 16, high half & 0xffff0000.
template <typename T> struct Vec16;
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&f)[4]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[i].x = __uint_as_float(w[i] << 16);
      f[i].y = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Vec16<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&f)[4]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2 *>(&w[i]);
      f[i] = __half22float2(h);
    }
  }
};
template <> struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4 &v, float2 (&f)[2]) {
    f[0] = make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
    f[1] = make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
  }
};

// Packed fp32x2 FMA (sm_100 FFMA2): d = a * b + c on two lanes at once.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long ra = *reinterpret_cast<unsigned long long *>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long *>(&b);
  unsigned long long rc = *reinterpret_cast<unsigned long long *>(&c);
  unsigned long long rd;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  return *reinterpret_cast<float2 *>(&rd);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long ra = *reinterpret_cast<unsigned long long *>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long *>(&b);
  unsigned long long rd;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  return *reinterpret_cast<float2 *>(&rd);
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  unsigned long long ra = *reinterpret_cast<unsigned long long *>(&a);
  unsigned long long rb = *reinterpret_cast<unsigned long long *>(&b);
  unsigned long long rd;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  return *reinterpret_cast<float2 *>(&rd);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---------------------------------------------------------------------------
// device status word
// ---------------------------------------------------------------------------
__device__ __forceinline__ void flag_status(int32_t *status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every spin in these kernels gives up after this long and reports
// MI_DEV_TIMEOUT, so a lost arrival cannot hang the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (TMA engine, non-tensor form)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and flags
// MI_DEV_TIMEOUT) when the limit passes; callers then stop issuing work.
// Reading %globaltimer costs far more than a try_wait round, so the clock is
// read only after every 64 unsuccessful try_waits: a wait that succeeds soon
// never touches it, and the limit is still enforced to within one round.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  int32_t *status) {
  uint64_t start = 0;
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    const uint64_t now = global_ns();
    if (start == 0) {
      start = now;
    } else if (now - start > kWaitLimitNs) {
      flag_status(status, MI_DEV_TIMEOUT);
      return false;
    }
  }
}

// Non-suspending probe of a phase (mbarrier.test_wait).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_wait_bounded, but spinning on test_wait so the caller sees the
// phase flip at once instead of after a suspension; for a lone thread with
// nothing else to do (an MMA issuer), never for whole warpgroups.
__device__ __forceinline__ bool mbar_spin_bounded(uint64_t *bar, uint32_t parity, int32_t *status) {
  uint64_t start = 0;
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    const uint64_t now = global_ns();
    if (start == 0) {
      start = now;
    } else if (now - start > kWaitLimitNs) {
      flag_status(status, MI_DEV_TIMEOUT);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared, completing `bytes` on `bar`.  Both
// addresses and the size must be multiples of 16 bytes.
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) into L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace mi
