// Shared device helpers for the GDN kernels (sm_100a).
//
// - bf16 <-> fp32 vector loads/stores
// - mbarrier + 1-D bulk async copy (cp.async.bulk through the TMA engine, one CTA)
// - bounded waits: every spin has a time limit, after which the kernel records
//   an error bit in g_gdn_device_error and skips the dependent work instead of
//   hanging the GPU.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 128;  // d_k = d_v = 128 (the definition's head size)

// Device error bits (read by gdn_device_error()).
constexpr unsigned kDevErrWaitTimeout = 1u << 0;
constexpr unsigned kDevErrBadSeqlens = 1u << 1;
constexpr unsigned kDevErrBadIndex = 1u << 2;

// Bounded-wait limit: ~2 s of %globaltimer after the fast spin.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

extern __device__ unsigned int g_gdn_device_error;

__device__ __forceinline__ void raise_device_error(unsigned bits) { atomicOr(&g_gdn_device_error, bits); }

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test of the phase with the given parity (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Same test, but the thread may be suspended (instead of spinning and taking
// issue slots from working warps) until the phase completes or `hint_ns` passes.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar_addr, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete. Returns false (and
// records kDevErrWaitTimeout) if it does not complete within limit_ns
// (kWaitLimitNs unless a caller asks for less).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  const uint32_t addr = smem_u32(bar);
#pragma unroll 1
  for (int i = 0; i < 256; ++i)
    if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      raise_device_error(kDevErrWaitTimeout);
      return false;
    }
  }
}

// Same bounded wait, but the thread is suspended between tests (for waits of a
// microsecond or more, e.g. on a copy from HBM, where polling would only take
// issue slots and shared-memory bandwidth from the warps doing the work).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait_sleep(addr, parity, 1000000u)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(kDevErrWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- bulk copy
// 1-D bulk copy global -> shared through the TMA engine; completion is counted
// on `bar` in bytes. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 evict-first hint (data read exactly once).
__device__ __forceinline__ void bulk_g2s_evict_first(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                                     uint64_t* bar) {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- bf16 / fp32
__device__ __forceinline__ float4 load_bf16x4(const __nv_bfloat16* p) {
  const uint2 raw = *reinterpret_cast<const uint2*>(p);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ float bf16_to_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }

__device__ __forceinline__ float4 ld_nc_f4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// Streaming (evict-first) 16-byte store.
__device__ __forceinline__ void st_cs_f4(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

__device__ __forceinline__ float dot4(float4 a, float4 b) {
  return fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, a.w * b.w)));
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Two independent all-reduces interleaved for ILP.
__device__ __forceinline__ void warp_sum2(float& x, float& y) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    x += __shfl_xor_sync(0xffffffffu, x, o);
    y += __shfl_xor_sync(0xffffffffu, y, o);
  }
}

// ---------------------------------------------------------------- gates
// g = exp(-exp(A_log) * softplus(a + dt_bias)), softplus(x) = x for x > 20;
// beta = sigmoid(b).   (reference: solution/triton/kernel_decode.py:52-55)
__device__ __forceinline__ void gdn_gates(float A_log, float a, float dt_bias, float b, float& g, float& beta) {
  const float x = a + dt_bias;
  const float sp = x > 20.0f ? x : log1pf(expf(x));
  g = expf(-expf(A_log) * sp);
  beta = 1.0f / (1.0f + expf(-b));
}

// The same gates from the hardware exp2 / log2 approximations (relative error ~1e-7 against
// gdn_gates), for kernels where the per-call gate cost is on the issue budget.
__device__ __forceinline__ void gdn_gates_fast(float A_log, float a, float dt_bias, float b, float& g, float& beta) {
  constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;
  float e1, e2, l1, e3, e4;
  const float x = a + dt_bias;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(x * kLog2e));
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(l1) : "f"(1.0f + e1));
  const float sp = x > 20.0f ? x : kLn2 * l1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e2) : "f"(A_log * kLog2e));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e3) : "f"(-e2 * sp * kLog2e));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e4) : "f"(-b * kLog2e));
  g = e3;
  beta = __frcp_rn(1.0f + e4);
}

// log of the decay gate: -exp(A_log) * softplus(a + dt_bias) (kept in log space
// for chunked cumulative products).
__device__ __forceinline__ float gdn_log_decay(float A_log, float a, float dt_bias) {
  const float x = a + dt_bias;
  const float sp = x > 20.0f ? x : log1pf(expf(x));
  return -expf(A_log) * sp;
}

}  // namespace gdn
