// common.cuh -- device helpers shared by the sm_100a paged-attention kernels:
// element conversions, mbarrier waits with a time limit, TMA tensor loads and
// the device status word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200_paged_attn.h"

namespace b200 {

// A pipeline wait gives up after this many nanoseconds of %globaltimer and
// reports B200_DEV_WAIT_TIMEOUT instead of spinning forever.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report(int32_t* status, int bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------- elements
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kPerChunk = 4;  // elements per 16-byte chunk
  __device__ __forceinline__ static void unpack(const uint4& c, float* f) {
    f[0] = __uint_as_float(c.x);
    f[1] = __uint_as_float(c.y);
    f[2] = __uint_as_float(c.z);
    f[3] = __uint_as_float(c.w);
  }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kPerChunk = 8;
  // bf16 -> f32 is exact: the bf16 bits are the high half of the f32 bits.
  __device__ __forceinline__ static void unpack(const uint4& c, float* f) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};

// Scalar load / store of a runtime-typed element (q, out, k_new ...).
__device__ __forceinline__ float load_elem(const void* base, int64_t idx, int dtype) {
  if (dtype == B200_DTYPE_F32) return static_cast<const float*>(base)[idx];
  if (dtype == B200_DTYPE_BF16)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(base)[idx]);
  return __half2float(static_cast<const __half*>(base)[idx]);
}

__device__ __forceinline__ void store_elem(void* base, int64_t idx, int dtype, float v) {
  if (dtype == B200_DTYPE_F32) {
    static_cast<float*>(base)[idx] = v;
  } else if (dtype == B200_DTYPE_BF16) {
    static_cast<__nv_bfloat16*>(base)[idx] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(base)[idx] = __float2half_rn(v);
  }
}

__device__ __forceinline__ int64_t load_index(const void* base, int64_t idx, int i64) {
  return i64 ? static_cast<const int64_t*>(base)[idx]
             : static_cast<int64_t>(static_cast<const int32_t*>(base)[idx]);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false
// (and never blocks much longer than limit_ns) when it does not.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(a, parity)) return true;
    if ((i & 31u) == 0 && global_timer_ns() - t0 > limit_ns) return false;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled TMA load into this CTA's own shared memory, completing
// `bytes` on the mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 2-D tiled TMA load (x = inner coordinate) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Orders this thread's earlier generic-proxy global stores before later
// async-proxy (TMA) reads of the same addresses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

// Packed fp32x2 fused multiply-add (one sm_100 instruction for two lanes of
// work): returns a * b + c element-wise, each with a single rounding.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// Exact bf16 pair (one 32-bit word, element 0 in the low half) -> float2.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

}  // namespace b200
