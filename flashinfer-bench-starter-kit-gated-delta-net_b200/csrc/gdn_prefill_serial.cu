// Token-serial varlen GDN prefill (sm_100a, CUDA cores).
//
// Reference semantics: solution/triton/kernel_prefill.py:42-142 — for every
// (sequence, v-head) the decode step is applied token by token and each
// token's output is stored; the final state is written once; an empty
// sequence passes its initial state through (kernel_prefill.py:65-73).
//
// This kernel keeps the CTA's 32 state rows in registers for the whole
// sequence (4 warps x 8 rows, a lane holds 4 consecutive K elements of each
// row) and prefetches the next token's q/k/v/a/b while the current token is
// applied.  It is the short-sequence path and the cross-check for the chunked
// tensor-core kernel.
#include "gdn_common.cuh"
#include "gdn_kernels.h"

namespace gdn {

namespace {

constexpr int kSerialRows = 32;  // rows per CTA
constexpr int kSerialWarps = 4;
constexpr int kSerialRowsPerWarp = kSerialRows / kSerialWarps;

struct TokenLoads {
  uint2 k, q;  // 4 bf16 each
  float v;     // this lane's row value (lanes < rows per warp)
  float a, b;
};

__device__ __forceinline__ float4 bf16x4_to_f4(uint2 raw) {
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int i) {
  return p.cu_is_int64 ? reinterpret_cast<const int64_t*>(p.cu_seqlens)[i]
                       : (int64_t) reinterpret_cast<const int32_t*>(p.cu_seqlens)[i];
}

template <bool L2NORM>
__global__ void __launch_bounds__(128) prefill_serial_kernel(PrefillParams p) {
  const int blocks_per_head = kHeadDim / kSerialRows;
  const int h = blockIdx.x / blocks_per_head;
  const int row0 = (blockIdx.x % blocks_per_head) * kSerialRows;
  const int n = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int wrow0 = row0 + warp * kSerialRowsPerWarp;
  const int qh = h / p.ratio;

  const int64_t t0 = load_cu(p, n), t1 = load_cu(p, n + 1);
  const bool bad = t1 < t0 || t0 < 0 || t1 > p.T;
  if (bad && threadIdx.x == 0) raise_device_error(kDevErrBadSeqlens);

  float4 s[kSerialRowsPerWarp];
  const float* src = p.state ? p.state + (size_t)n * p.s_sn + (size_t)h * p.s_sh + (size_t)wrow0 * kHeadDim + lane * 4
                             : nullptr;
#pragma unroll
  for (int r = 0; r < kSerialRowsPerWarp; ++r)
    s[r] = src ? ld_nc_f4(src + r * kHeadDim) : make_float4(0.f, 0.f, 0.f, 0.f);

  const float A_log = p.A_log[h], dt_bias = p.dt_bias[h], scale = p.scale;
  auto load_token = [&](int64_t t) {
    TokenLoads L;
    L.k = *reinterpret_cast<const uint2*>(p.k + t * p.k_st + (int64_t)qh * p.k_sh + lane * 4);
    L.q = *reinterpret_cast<const uint2*>(p.q + t * p.q_st + (int64_t)qh * p.q_sh + lane * 4);
    L.v = lane < kSerialRowsPerWarp ? bf16_to_f32(p.v + t * p.v_st + (int64_t)h * p.v_sh + wrow0 + lane) : 0.f;
    L.a = bf16_to_f32(p.a + t * p.a_st + h);
    L.b = bf16_to_f32(p.b + t * p.b_st + h);
    return L;
  };

  if (!bad && t1 > t0) {
    TokenLoads cur = load_token(t0);
#pragma unroll 1
    for (int64_t t = t0; t < t1; ++t) {
      const TokenLoads nxt = load_token(t + 1 < t1 ? t + 1 : t);
      float4 kv = bf16x4_to_f4(cur.k), qv = bf16x4_to_f4(cur.q);
      if (L2NORM) {
        float kk = dot4(kv, kv), qq = dot4(qv, qv);
        warp_sum2(kk, qq);
        const float rk = rsqrtf(kk + 1e-6f), rq = rsqrtf(qq + 1e-6f);
        kv = make_float4(kv.x * rk, kv.y * rk, kv.z * rk, kv.w * rk);
        qv = make_float4(qv.x * rq, qv.y * rq, qv.z * rq, qv.w * rq);
      }
      const float kq = warp_sum(dot4(kv, qv));
      float g, beta;
      gdn_gates(A_log, cur.a, dt_bias, cur.b, g, beta);
      float o_mine = 0.f;
      float pk[kSerialRowsPerWarp], pq[kSerialRowsPerWarp];
#pragma unroll
      for (int r = 0; r < kSerialRowsPerWarp; ++r) {
        s[r].x *= g;
        s[r].y *= g;
        s[r].z *= g;
        s[r].w *= g;
        pk[r] = dot4(s[r], kv);
        pq[r] = dot4(s[r], qv);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int r = 0; r < kSerialRowsPerWarp; ++r) {
          pk[r] += __shfl_xor_sync(0xffffffffu, pk[r], o);
          pq[r] += __shfl_xor_sync(0xffffffffu, pq[r], o);
        }
      }
#pragma unroll
      for (int r = 0; r < kSerialRowsPerWarp; ++r) {
        const float vr = __shfl_sync(0xffffffffu, cur.v, r);
        const float delta = beta * (vr - pk[r]);
        s[r].x = fmaf(delta, kv.x, s[r].x);
        s[r].y = fmaf(delta, kv.y, s[r].y);
        s[r].z = fmaf(delta, kv.z, s[r].z);
        s[r].w = fmaf(delta, kv.w, s[r].w);
        if (lane == r) o_mine = scale * fmaf(delta, kq, pq[r]);
      }
      if (lane < kSerialRowsPerWarp)
        p.out[t * p.o_st + (int64_t)h * p.o_sh + wrow0 + lane] = __float2bfloat16_rn(o_mine);
      cur = nxt;
    }
  }

  float* dst = p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh + (size_t)wrow0 * kHeadDim + lane * 4;
#pragma unroll
  for (int r = 0; r < kSerialRowsPerWarp; ++r) *reinterpret_cast<float4*>(dst + r * kHeadDim) = s[r];
}

}  // namespace

cudaError_t launch_prefill_serial(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  const dim3 grid(p.HV * (kHeadDim / kSerialRows), p.N);
  if (p.flags & kFlagQkL2Norm)
    prefill_serial_kernel<true><<<grid, 128, 0, stream>>>(p);
  else
    prefill_serial_kernel<false><<<grid, 128, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace gdn
