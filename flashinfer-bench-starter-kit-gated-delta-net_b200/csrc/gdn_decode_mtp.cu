// Multi-token GDN decode against a pool of states (sm_100a): the serving form
// with state slots, T >= 1 tokens per sequence.
//
// Semantics: flashinfer 0.6.11.post2 flashinfer/trace/templates/gdn.py
// _gdn_mtp_reference (third party): sequence b starts from pool[indices[b]] and
// runs T steps of the decode recurrence of solution/triton/kernel_decode.py:71-103
// (per state row v: S <- g S; u = S.k; delta = beta (v - u); S <- S + delta k;
// o = scale S.q), writing o[b, t] for every token, the state after token t to
// intermediate[slot, t] when that buffer is given, and the final state to
// new_pool[slot].  A negative index skips the sequence (its outputs are zeros);
// an index >= pool_size raises GDN_DEVERR_BAD_INDEX and is skipped.
//
// Design: as the single-token kernel (CTA = 4 warps owning ROWS state rows of one
// (sequence, v-head); rows arrive by 1-D bulk copies, one mbarrier per warp
// slice), but the rows stay in registers for all T tokens, so the state crosses
// HBM once per call.  Eight lanes share a row: lane c of the eight holds K
// elements 32 j + 4 c .. 32 j + 4 c + 3 (j = 0..3), so the eight lanes' 16-byte
// accesses cover 128 contiguous bytes.  A warp thus works on 4 rows at once and
// each dot product needs a 3-level shuffle reduction; the decay is folded in
// (S.k and S.q are taken on the undecayed row and scaled by g).  The row math
// runs on packed fp32x2 instructions (__ffma2_rn / __fmul2_rn / __fadd2_rn), two
// columns per instruction.  q, k, v and the gates of up to kTokGroup tokens are
// staged in shared memory (fp32) per group.
#include "gdn_common.cuh"
#include "gdn_kernels.h"

namespace gdn {

namespace {

constexpr int kTokGroup = 16;

__device__ __forceinline__ int64_t load_index(const DecodeMtpParams& p, int b) {
  return p.idx_is_int64 ? reinterpret_cast<const int64_t*>(p.indices)[b]
                        : (int64_t) reinterpret_cast<const int32_t*>(p.indices)[b];
}

template <int ROWS>
constexpr size_t mtp_smem_bytes() {
  return (size_t)ROWS * kHeadDim * 4                    // state rows
         + (size_t)kTokGroup * 2 * kHeadDim * 4         // q, k per token
         + (size_t)kTokGroup * ROWS * 4                 // v of this CTA's rows per token
         + (size_t)kTokGroup * 2 * 4                    // g, beta per token
         + 4 * sizeof(uint64_t);                        // mbarriers
}

template <int ROWS, bool L2NORM>
__global__ void __launch_bounds__(128) decode_mtp_kernel(DecodeMtpParams p) {
  constexpr int kWarps = 4;
  constexpr int R = ROWS / kWarps;  // rows per warp
  static_assert(R >= 1 && R <= 32, "rows per warp");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  float* tile = reinterpret_cast<float*>(smem_raw);         // [ROWS][128]
  float* sqk = tile + ROWS * kHeadDim;                      // [kTokGroup][2][128]
  float* sv = sqk + kTokGroup * 2 * kHeadDim;               // [kTokGroup][ROWS]
  float* sg = sv + kTokGroup * ROWS;                        // [kTokGroup][2] (g, beta)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sg + kTokGroup * 2);

  const int blocks_per_head = kHeadDim / ROWS;
  const int h = blockIdx.x / blocks_per_head;
  const int row0 = (blockIdx.x % blocks_per_head) * ROWS;
  const int bi = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wrow0 = row0 + warp * R;

  const int64_t slot = load_index(p, bi);
  if (slot < 0 || slot >= p.P) {
    if (slot >= p.P && tid == 0) raise_device_error(kDevErrBadIndex);
    // skipped sequence: zero outputs for this CTA's rows
    for (int e = tid; e < p.T * ROWS; e += blockDim.x) {
      const int t = e / ROWS, r = e % ROWS;
      p.out[(size_t)bi * p.o_sb + (size_t)t * p.o_st + (size_t)h * p.o_sh + row0 + r] = __float2bfloat16_rn(0.f);
    }
    return;
  }

  const size_t in_off = (size_t)slot * p.s_sn + (size_t)h * p.s_sh + (size_t)row0 * kHeadDim;
  if (tid == 0) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mbar_init(&bars[w], 1);
    fence_barrier_init();
    constexpr uint32_t kBytes = R * kHeadDim * sizeof(float);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      mbar_arrive_expect_tx(&bars[w], kBytes);
      bulk_g2s_evict_first(tile + w * R * kHeadDim, p.pool + in_off + w * R * kHeadDim, kBytes, &bars[w]);
    }
  }

  const int qh = h / p.ratio;
  const float A_log = p.A_log[h], dt_bias = p.dt_bias[h], scale = p.scale;
  constexpr int kPasses = R / 4;                      // rows per lane
  static_assert(R % 4 == 0, "four rows per warp pass");
  const int rg = lane >> 3, cs = lane & 7;             // row in the pass, column slice
  float2 s[kPasses][8];  // s[ps][2 j + e]: columns 32 j + 4 cs + 2 e, + 1 of row ps * 4 + rg
  bool have_rows = false, rows_ok = true;

  for (int tg = 0; tg < p.T; tg += kTokGroup) {
    const int nt = min(kTokGroup, p.T - tg);
    __syncthreads();  // previous group's staging consumed; barrier init visible (first group)
    // ---- stage q, k (fp32), v (this CTA's rows), gates for tokens tg .. tg + nt - 1 ----
    for (int e = tid; e < nt * 2 * (kHeadDim / 4); e += blockDim.x) {
      const int t = e / (2 * (kHeadDim / 4)), rem = e % (2 * (kHeadDim / 4));
      const int which = rem / (kHeadDim / 4), c4 = rem % (kHeadDim / 4);
      const __nv_bfloat16* src = which == 0
          ? p.q + (size_t)bi * p.q_sb + (size_t)(tg + t) * p.q_st + (size_t)qh * p.q_sh
          : p.k + (size_t)bi * p.k_sb + (size_t)(tg + t) * p.k_st + (size_t)qh * p.k_sh;
      *reinterpret_cast<float4*>(sqk + (t * 2 + which) * kHeadDim + c4 * 4) = load_bf16x4(src + c4 * 4);
    }
    for (int e = tid; e < nt * ROWS; e += blockDim.x) {
      const int t = e / ROWS, r = e % ROWS;
      sv[t * ROWS + r] = bf16_to_f32(p.v + (size_t)bi * p.v_sb + (size_t)(tg + t) * p.v_st + (size_t)h * p.v_sh + row0 + r);
    }
    if (tid < nt) {
      float g, beta;
      gdn_gates(A_log, bf16_to_f32(p.a + (size_t)bi * p.a_sb + (size_t)(tg + tid) * p.a_st + h), dt_bias,
                bf16_to_f32(p.b + (size_t)bi * p.b_sb + (size_t)(tg + tid) * p.b_st + h), g, beta);
      sg[tid * 2] = g;
      sg[tid * 2 + 1] = beta;
    }
    __syncthreads();
    if (!have_rows) {
      // a timed-out copy (recorded by mbar_wait) leaves this warp without rows: it
      // keeps taking part in the CTA barriers but computes and stores nothing
      rows_ok = mbar_wait(&bars[warp], 0);
#pragma unroll
      for (int ps = 0; ps < kPasses; ++ps) {
        const float* src = tile + (warp * R + ps * 4 + rg) * kHeadDim + cs * 4;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 x = rows_ok ? *reinterpret_cast<const float4*>(src + c4 * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
          s[ps][2 * c4] = make_float2(x.x, x.y);
          s[ps][2 * c4 + 1] = make_float2(x.z, x.w);
        }
      }
      have_rows = true;
    }
    if (!rows_ok) continue;
    // ---- nt sequential decode steps on the register-resident rows (packed fp32x2 math) ----
#pragma unroll 1
    for (int t = 0; t < nt; ++t) {
      float2 kv[8], qv[8];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        const float4 k4 = *reinterpret_cast<const float4*>(sqk + (t * 2 + 1) * kHeadDim + cs * 4 + c4 * 32);
        const float4 q4 = *reinterpret_cast<const float4*>(sqk + (t * 2) * kHeadDim + cs * 4 + c4 * 32);
        kv[2 * c4] = make_float2(k4.x, k4.y);
        kv[2 * c4 + 1] = make_float2(k4.z, k4.w);
        qv[2 * c4] = make_float2(q4.x, q4.y);
        qv[2 * c4 + 1] = make_float2(q4.z, q4.w);
      }
      // k.q (and |k|^2, |q|^2) over the row's 8 lanes (every 8-lane group holds all 128 elements)
      float2 akq = make_float2(0.f, 0.f), akk = akq, aqq = akq;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        akq = __ffma2_rn(kv[c], qv[c], akq);
        if (L2NORM) {
          akk = __ffma2_rn(kv[c], kv[c], akk);
          aqq = __ffma2_rn(qv[c], qv[c], aqq);
        }
      }
      float kq = akq.x + akq.y;
      float2 nrm = __fadd2_rn(make_float2(akk.x, aqq.x), make_float2(akk.y, aqq.y));
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        kq += __shfl_xor_sync(0xffffffffu, kq, o);
        if (L2NORM)
          nrm = __fadd2_rn(nrm, make_float2(__shfl_xor_sync(0xffffffffu, nrm.x, o),
                                            __shfl_xor_sync(0xffffffffu, nrm.y, o)));
      }
      if (L2NORM) {
        const float rk = rsqrtf(nrm.x + 1e-6f), rq = rsqrtf(nrm.y + 1e-6f);
        const float2 rk2 = make_float2(rk, rk), rq2 = make_float2(rq, rq);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          kv[c] = __fmul2_rn(kv[c], rk2);
          qv[c] = __fmul2_rn(qv[c], rq2);
        }
        kq *= rk * rq;
      }
      const float g = sg[t * 2], beta = sg[t * 2 + 1];
      const float2 g2 = make_float2(g, g);
#pragma unroll
      for (int ps = 0; ps < kPasses; ++ps) {
        const int r = ps * 4 + rg;  // row within the warp
        float2 ak = make_float2(0.f, 0.f), aq = ak;  // S.k, S.q on the undecayed row
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          ak = __ffma2_rn(s[ps][c], kv[c], ak);
          aq = __ffma2_rn(s[ps][c], qv[c], aq);
        }
        float2 pkq = __fadd2_rn(make_float2(ak.x, aq.x), make_float2(ak.y, aq.y));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
          pkq = __fadd2_rn(pkq, make_float2(__shfl_xor_sync(0xffffffffu, pkq.x, o),
                                            __shfl_xor_sync(0xffffffffu, pkq.y, o)));
        const float delta = beta * (sv[t * ROWS + warp * R + r] - g * pkq.x);
        const float2 d2 = make_float2(delta, delta);
#pragma unroll
        for (int c = 0; c < 8; ++c) s[ps][c] = __ffma2_rn(g2, s[ps][c], __fmul2_rn(d2, kv[c]));
        if (cs == 0)
          p.out[(size_t)bi * p.o_sb + (size_t)(tg + t) * p.o_st + (size_t)h * p.o_sh + wrow0 + r] =
              __float2bfloat16_rn(scale * fmaf(delta, kq, g * pkq.y));
        if (p.inter) {
          float* idst = p.inter + (size_t)slot * p.i_sn + (size_t)(tg + t) * p.i_st + (size_t)h * p.i_sh +
                        (size_t)(wrow0 + r) * kHeadDim + cs * 4;
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4)
            st_cs_f4(idst + c4 * 32, make_float4(s[ps][2 * c4].x, s[ps][2 * c4].y, s[ps][2 * c4 + 1].x,
                                                 s[ps][2 * c4 + 1].y));
        }
      }
    }
  }
  if (rows_ok) {
#pragma unroll
    for (int ps = 0; ps < kPasses; ++ps) {
      float* dst = p.new_pool + (size_t)slot * p.n_sn + (size_t)h * p.n_sh +
                   (size_t)(wrow0 + ps * 4 + rg) * kHeadDim + cs * 4;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4)
        st_cs_f4(dst + c4 * 32, make_float4(s[ps][2 * c4].x, s[ps][2 * c4].y, s[ps][2 * c4 + 1].x,
                                            s[ps][2 * c4 + 1].y));
    }
  }
}

template <int ROWS>
cudaError_t launch_mtp_rows(const DecodeMtpParams& p, cudaStream_t stream) {
  constexpr size_t smem = mtp_smem_bytes<ROWS>();
  static_assert(smem <= 48 * 1024, "default dynamic shared memory limit");
  const dim3 grid(p.HV * (kHeadDim / ROWS), p.B);
  if (p.flags & kFlagQkL2Norm)
    decode_mtp_kernel<ROWS, true><<<grid, 128, smem, stream>>>(p);
  else
    decode_mtp_kernel<ROWS, false><<<grid, 128, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_mtp(const DecodeMtpParams& p, cudaStream_t stream) {
  if (p.B == 0 || p.T == 0) return cudaSuccess;
  return decode_rows_for(p.B, p.HV) == 32 ? launch_mtp_rows<32>(p, stream) : launch_mtp_rows<16>(p, stream);
}

}  // namespace gdn
