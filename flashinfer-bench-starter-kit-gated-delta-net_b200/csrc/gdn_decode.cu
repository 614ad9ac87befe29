// Fused single-token GDN decode (sm_100a).
//
// One read-modify-write pass over each 64 KB fp32 head state (k-last,
// [B, HV, V=128, K=128]).  Reference semantics: solution/triton/kernel_decode.py:8-103
// (per state row v: S <- g*S; u = S.k; delta = beta*(v - u); S <- S + delta*k;
// o = scale * S.q).
//
// Design (HBM-bound, ~8 MiB of state traffic per sequence step):
//   * CTA = 4 warps, owns ROWS consecutive state rows of one (sequence, v-head).
//   * Thread 0 streams the CTA's rows HBM -> shared memory with 1-D bulk
//     copies (TMA engine, one mbarrier per warp slice), so each warp starts as
//     soon as its own rows land, and keeps ROWS*512 B in flight per CTA.
//   * Gates, q/k (optionally L2-normalised) and k.q are computed while the
//     copy is in flight.
//   * Per row a lane holds 4 consecutive K elements (one 16 B shared load);
//     both dot products S.k and S.q are reduced in one interleaved butterfly
//     using o = scale * (g*S.q + delta * k.q), which equals scale * (S'.q).
//   * The updated row is written straight from registers with 16 B streaming
//     stores; o is written as bf16 by the lanes that own each row.
//   * Pooled form (DecodeParams::indices): the same pass on slot indices[b] of a
//     state pool, the one-token case of gdn_decode_pooled.
#include "gdn_common.cuh"
#include "gdn_kernels.h"

namespace gdn {

template <int ROWS, bool L2NORM>
__global__ void __launch_bounds__(128) decode_kernel(DecodeParams p) {
  constexpr int kWarps = 4;
  constexpr int kRowsPerWarp = ROWS / kWarps;
  static_assert(kRowsPerWarp >= 1 && kRowsPerWarp <= 32, "rows per warp");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float* tile = reinterpret_cast<float*>(smem_raw);                                  // [ROWS][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + ROWS * kHeadDim * sizeof(float));  // [4]

  const int blocks_per_head = kHeadDim / ROWS;
  const int h = blockIdx.x / blocks_per_head;
  const int row0 = (blockIdx.x % blocks_per_head) * ROWS;
  const int bi = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool has_state = p.state != nullptr;

  if (p.flags & kFlagSelftestWaitTimeout) {
    // Self-test of the bounded-wait path: every thread waits on a barrier that nothing
    // arrives at, with a 1 ms limit.  No copy is issued, so nothing is in flight when the
    // waits give up; each records GDN_DEVERR_WAIT_TIMEOUT and the CTA returns without
    // touching out / new_state.
    if (threadIdx.x == 0) {
      mbar_init(&bars[0], 1);
      fence_barrier_init();
    }
    __syncthreads();
    mbar_wait(&bars[0], 0, kSelftestWaitLimitNs);  // gives up: the phase cannot complete
    return;
  }

  // the state block of sequence bi: its own, or slot indices[bi] of a pool
  int64_t slot = bi;
  if (p.indices) {
    slot = p.idx_is_int64 ? reinterpret_cast<const int64_t*>(p.indices)[bi]
                          : (int64_t) reinterpret_cast<const int32_t*>(p.indices)[bi];
    if (slot < 0 || slot >= p.P) {  // padded (or out-of-range) entry: zero outputs, no state touched
      if (slot >= p.P && threadIdx.x == 0) raise_device_error(kDevErrBadIndex);
      if (threadIdx.x < ROWS)
        p.out[(size_t)bi * p.o_sb + (size_t)h * p.o_sh + row0 + threadIdx.x] = __float2bfloat16_rn(0.f);
      return;
    }
  }
  const size_t in_off = (size_t)slot * p.s_sb + (size_t)h * p.s_sh + (size_t)row0 * kHeadDim;
  if (threadIdx.x == 0 && has_state) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mbar_init(&bars[w], 1);
    fence_barrier_init();
    constexpr uint32_t kBytes = kRowsPerWarp * kHeadDim * sizeof(float);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      mbar_arrive_expect_tx(&bars[w], kBytes);
      bulk_g2s_evict_first(tile + w * kRowsPerWarp * kHeadDim, p.state + in_off + w * kRowsPerWarp * kHeadDim,
                           kBytes, &bars[w]);
    }
  }

  // ---- per-head scalars and vectors (overlap the state copy) ----
  const int qh = h / p.ratio;
  float4 kv = load_bf16x4(p.k + (size_t)bi * p.k_sb + (size_t)qh * p.k_sh + lane * 4);
  float4 qv = load_bf16x4(p.q + (size_t)bi * p.q_sb + (size_t)qh * p.q_sh + lane * 4);
  if (L2NORM) {
    float kk = dot4(kv, kv), qq = dot4(qv, qv);
    warp_sum2(kk, qq);
    const float rk = rsqrtf(kk + 1e-6f), rq = rsqrtf(qq + 1e-6f);
    kv = make_float4(kv.x * rk, kv.y * rk, kv.z * rk, kv.w * rk);
    qv = make_float4(qv.x * rq, qv.y * rq, qv.z * rq, qv.w * rq);
  }
  float kq = dot4(kv, qv);
  kq = warp_sum(kq);
  float g, beta;
  gdn_gates(p.A_log[h], bf16_to_f32(p.a + (size_t)bi * p.a_sb + h), p.dt_bias[h],
            bf16_to_f32(p.b + (size_t)bi * p.b_sb + h), g, beta);
  const int wrow0 = row0 + warp * kRowsPerWarp;
  float v_mine = 0.0f;
  if (lane < kRowsPerWarp) v_mine = bf16_to_f32(p.v + (size_t)bi * p.v_sb + (size_t)h * p.v_sh + wrow0 + lane);
  const float scale = p.scale;

  __syncthreads();  // barrier initialisation visible to all warps
  const float* wtile = tile + warp * kRowsPerWarp * kHeadDim;
  if (has_state && !mbar_wait(&bars[warp], 0)) return;

  float* dst = p.new_state + (size_t)slot * p.n_sb + (size_t)h * p.n_sh + (size_t)wrow0 * kHeadDim + lane * 4;
  float o_mine = 0.0f;
#pragma unroll 4
  for (int r = 0; r < kRowsPerWarp; ++r) {
    float4 s = has_state ? *reinterpret_cast<const float4*>(wtile + r * kHeadDim + lane * 4)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    s.x *= g;
    s.y *= g;
    s.z *= g;
    s.w *= g;
    float pk = dot4(s, kv), pq = dot4(s, qv);
    warp_sum2(pk, pq);
    const float vr = __shfl_sync(0xffffffffu, v_mine, r);
    const float delta = beta * (vr - pk);
    s.x = fmaf(delta, kv.x, s.x);
    s.y = fmaf(delta, kv.y, s.y);
    s.z = fmaf(delta, kv.z, s.z);
    s.w = fmaf(delta, kv.w, s.w);
    st_cs_f4(dst + r * kHeadDim, s);
    if (lane == r) o_mine = scale * fmaf(delta, kq, pq);
  }
  if (lane < kRowsPerWarp)
    p.out[(size_t)bi * p.o_sb + (size_t)h * p.o_sh + wrow0 + lane] = __float2bfloat16_rn(o_mine);
}

template <int ROWS>
static cudaError_t launch_rows(const DecodeParams& p, cudaStream_t stream) {
  const dim3 grid(p.HV * (kHeadDim / ROWS), p.B);
  const size_t smem = ROWS * kHeadDim * sizeof(float) + 4 * sizeof(uint64_t);
  static_assert(ROWS * kHeadDim * sizeof(float) + 4 * sizeof(uint64_t) <= 48 * 1024, "default smem limit");
  if (p.flags & kFlagQkL2Norm)
    decode_kernel<ROWS, true><<<grid, 128, smem, stream>>>(p);
  else
    decode_kernel<ROWS, false><<<grid, 128, smem, stream>>>(p);
  return cudaGetLastError();
}

int decode_rows_for(int B, int HV) {
  // Enough CTAs for several waves on 148 SMs; larger tiles once the grid is big.
  const long units = (long)B * HV;  // 64 KB head states
  if (units >= 1024) return 32;
  return 16;
}

cudaError_t launch_decode(const DecodeParams& p, int rows, cudaStream_t stream) {
  switch (rows) {
    case 16: return launch_rows<16>(p, stream);
    case 32: return launch_rows<32>(p, stream);
    case 64: return launch_rows<64>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
