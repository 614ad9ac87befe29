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
#include <algorithm>

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

// ---------------------------------------------------------------------------
// Warp-pipelined form for T <= kPipeMaxT and 16-byte aligned q/k/v rows (the
// serving case).  Every warp is an independent worker over items of
// kPipeRows = 8 state rows of one (sequence, v-head); items are strided over
// all warps of a persistent grid.  Each warp double-buffers two parts per item
// in its own shared memory:
//   rows   the item's 8 x 128 fp32 state rows (one 4 KB bulk copy from the
//          pool), released as soon as they are in registers, so the copy for
//          item j + 2 is in flight during items j and j + 1;
//   tokens q and k rows (bf16, 256 B per token each) and the item's 8 v values
//          per token (16 B), T * 3 bulk copies issued one per lane, released
//          after the item's T steps.
// Each step's q and k rows are widened to fp32 once (each lane converts 8
// elements) into a 1 KB per-warp buffer, the next step's during the current
// step's shuffle reductions (after every lane has read the current one).  All dot products of a step
// (S.k and S.q of the lane's two rows, k.q, and |k|^2, |q|^2 for the in-kernel
// L2 norm, which scales the dot products rather than the vectors) are formed
// together, so their 3-level reductions overlap.
// The gates (a, b, A_log, dt_bias) and the pool index are prefetched into
// registers one and two items ahead.  No CTA-wide barrier is used.
constexpr int kPipeRows = 8;
constexpr int kPipeMaxT = 8;
constexpr int kPipeWarps = 4;
constexpr uint32_t kPipeRowBytes = kPipeRows * kHeadDim * 4;  // 4096

__host__ __device__ constexpr uint32_t pipe_tok_bytes(int T) { return (uint32_t)T * (2 * kHeadDim * 2 + kPipeRows * 2); }
__host__ __device__ constexpr uint32_t pipe_warp_bytes(int T) {
  return 2 * kPipeRowBytes + 2 * pipe_tok_bytes(T) + 2 * kHeadDim * 4 + 4 * 8;
}

struct PipeItem {
  int bi, h, wrow0;
};

// item = (bi * HV + h) * 16 + row block; the division by HV is a multiply
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994: round-up multiplier for 32-bit operands)
__device__ __forceinline__ PipeItem pipe_item(int item, const DecodeMtpParams& p) {
  PipeItem it;
  it.wrow0 = (item & (kHeadDim / kPipeRows - 1)) * kPipeRows;
  const uint32_t bh = (uint32_t)item >> 4;
  it.bi = (int)((__umulhi(bh, p.hv_mul) + bh) >> p.hv_shr);
  it.h = (int)bh - it.bi * p.HV;
  return it;
}
static_assert(kHeadDim / kPipeRows == 16, "16 row blocks per head");

template <bool L2NORM>
__global__ void __launch_bounds__(kPipeWarps * 32, 4) decode_mtp_pipe_kernel(DecodeMtpParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = p.T;
  const uint32_t tok_bytes = pipe_tok_bytes(T);
  unsigned char* wbase = smem_raw + (size_t)warp * pipe_warp_bytes(T);
  float* rows_buf = reinterpret_cast<float*>(wbase);                              // [2][8][128] fp32
  unsigned char* tok_buf = wbase + 2 * kPipeRowBytes;                             // [2][tok_bytes]
  float* qk32 = reinterpret_cast<float*>(tok_buf + 2 * tok_bytes);                // [q 128 | k 128] fp32
  uint64_t* bars = reinterpret_cast<uint64_t*>(qk32 + 2 * kHeadDim);              // rows_full[2], tok_full[2]

  const int n_items = p.B * p.HV * (kHeadDim / kPipeRows);  // < 2^31 (checked by the launcher)
  const int first = blockIdx.x * kPipeWarps + warp, step = gridDim.x * kPipeWarps;
  if (first >= n_items) return;
  const int rg = lane >> 3, cs = lane & 7;

  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncwarp();

  auto slot_of = [&](int item) -> int64_t {
    return item < n_items ? load_index(p, pipe_item(item, p).bi) : -1;
  };
  auto issue_rows = [&](int item, int64_t slot, int st) {
    if (lane == 0) {
      const PipeItem it = pipe_item(item, p);
      if (slot >= 0 && slot < p.P) {
        mbar_arrive_expect_tx(&bars[st], kPipeRowBytes);
        bulk_g2s_evict_first(rows_buf + st * kPipeRows * kHeadDim,
                             p.pool + (size_t)slot * p.s_sn + (size_t)it.h * p.s_sh + (size_t)it.wrow0 * kHeadDim,
                             kPipeRowBytes, &bars[st]);
      } else {
        mbar_arrive(&bars[st]);  // nothing to load: complete the phase
      }
    }
  };
  auto issue_tok = [&](int item, int st) {
    const PipeItem it = pipe_item(item, p);
    if (lane == 0) mbar_arrive_expect_tx(&bars[2 + st], tok_bytes);
    __syncwarp();
    unsigned char* dst = tok_buf + st * tok_bytes;
    const int qh = it.h / p.ratio;
    if (lane < T) {
      bulk_g2s(dst + lane * 512, p.q + (size_t)it.bi * p.q_sb + (size_t)lane * p.q_st + (size_t)qh * p.q_sh, 256,
               &bars[2 + st]);
    } else if (lane < 2 * T) {
      const int t = lane - T;
      bulk_g2s(dst + t * 512 + 256, p.k + (size_t)it.bi * p.k_sb + (size_t)t * p.k_st + (size_t)qh * p.k_sh, 256,
               &bars[2 + st]);
    } else if (lane < 3 * T) {
      const int t = lane - 2 * T;
      bulk_g2s(dst + T * 512 + t * 16,
               p.v + (size_t)it.bi * p.v_sb + (size_t)t * p.v_st + (size_t)it.h * p.v_sh + it.wrow0, 16,
               &bars[2 + st]);
    }
  };
  // gate inputs of an item, lane t < T holding token t's a, b
  auto load_gate_inputs = [&](int item, float& ga, float& gb, float& alog, float& dtb) {
    ga = gb = alog = dtb = 0.f;
    if (item < n_items && lane < T) {
      const PipeItem it = pipe_item(item, p);
      ga = bf16_to_f32(p.a + (size_t)it.bi * p.a_sb + (size_t)lane * p.a_st + it.h);
      gb = bf16_to_f32(p.b + (size_t)it.bi * p.b_sb + (size_t)lane * p.b_st + it.h);
      alog = p.A_log[it.h];
      dtb = p.dt_bias[it.h];
    }
  };

  // prologue: items 0 and 1 of this warp in flight, indices up to item 2, gates of item 0
  int64_t slot0 = slot_of(first), slot1 = slot_of(first + step), slot2 = slot_of(first + 2 * step);
  issue_rows(first, slot0, 0);
  issue_tok(first, 0);
  if (first + step < n_items) {
    issue_rows(first + step, slot1, 1);
    issue_tok(first + step, 1);
  }
  float ga, gb, alog, dtb;
  load_gate_inputs(first, ga, gb, alog, dtb);

  int fail = 0;  // 1: a rows copy, 2: a tokens copy did not land in time
  int j = 0;
  for (int item = first; item < n_items; item += step, ++j) {
    const int st = (int)(j & 1);
    const uint32_t par = (uint32_t)((j >> 1) & 1);
    const PipeItem it = pipe_item(item, p);
    const int64_t slot = slot0;
    const bool valid = slot >= 0 && slot < p.P;
    // this item's gates (lane t: token t), then prefetch the next item's inputs
    float g_l = 0.f, beta_l = 0.f;
    if (lane < T) gdn_gates(alog, ga, dtb, gb, g_l, beta_l);
    load_gate_inputs(item + step, ga, gb, alog, dtb);
    const int64_t slot3 = slot_of(item + 3 * step);

    // ---- state rows -> registers; the rows buffer goes to item + 2 ----
    float2 s[2][8];
    if (!mbar_wait(&bars[st], par)) { fail = 1; break; }
    if (valid) {
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        const float* src = rows_buf + st * kPipeRows * kHeadDim + (ps * 4 + rg) * kHeadDim + cs * 4;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 x = *reinterpret_cast<const float4*>(src + c4 * 32);
          s[ps][2 * c4] = make_float2(x.x, x.y);
          s[ps][2 * c4 + 1] = make_float2(x.z, x.w);
        }
      }
    }
    __syncwarp();
    if (item + 2 * step < n_items) issue_rows(item + 2 * step, slot2, st);

    if (!mbar_wait(&bars[2 + st], par)) { fail = 2; break; }
    const unsigned char* tk = tok_buf + st * tok_bytes;
    __nv_bfloat16* out_item = p.out + (size_t)it.bi * p.o_sb + (size_t)it.h * p.o_sh + it.wrow0;
    if (valid) {
      const float scale = p.scale;
      // widen token t's q and k rows to fp32 in qk32 (lane: elements 4 lane .. 4 lane + 3)
      auto widen = [&](int t) {
        const uint2 qr = *reinterpret_cast<const uint2*>(tk + t * 512 + lane * 8);
        const uint2 kr = *reinterpret_cast<const uint2*>(tk + t * 512 + 256 + lane * 8);
        const float2 q0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qr.x));
        const float2 q1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qr.y));
        const float2 k0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kr.x));
        const float2 k1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&kr.y));
        float* dst = qk32;
        *reinterpret_cast<float4*>(dst + lane * 4) = make_float4(q0.x, q0.y, q1.x, q1.y);
        *reinterpret_cast<float4*>(dst + kHeadDim + lane * 4) = make_float4(k0.x, k0.y, k1.x, k1.y);
      };
      widen(0);
      __syncwarp();
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        float2 kv[8], qv[8];
        const float* src = qk32;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 q4 = *reinterpret_cast<const float4*>(src + c4 * 32 + cs * 4);
          const float4 k4 = *reinterpret_cast<const float4*>(src + kHeadDim + c4 * 32 + cs * 4);
          qv[2 * c4] = make_float2(q4.x, q4.y);
          qv[2 * c4 + 1] = make_float2(q4.z, q4.w);
          kv[2 * c4] = make_float2(k4.x, k4.y);
          kv[2 * c4 + 1] = make_float2(k4.z, k4.w);
        }
        // all dot products of the step at once (S.k, S.q of both rows on the
        // undecayed, un-normalised vectors; k.q; |k|^2, |q|^2)
        float2 akq = make_float2(0.f, 0.f), akk = akq, aqq = akq, ak0 = akq, aq0 = akq, ak1 = akq, aq1 = akq;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          ak0 = __ffma2_rn(s[0][c], kv[c], ak0);
          aq0 = __ffma2_rn(s[0][c], qv[c], aq0);
          ak1 = __ffma2_rn(s[1][c], kv[c], ak1);
          aq1 = __ffma2_rn(s[1][c], qv[c], aq1);
          akq = __ffma2_rn(kv[c], qv[c], akq);
          if (L2NORM) {
            akk = __ffma2_rn(kv[c], kv[c], akk);
            aqq = __ffma2_rn(qv[c], qv[c], aqq);
          }
        }
        __syncwarp();                  // every lane has read this step's q and k
        if (t + 1 < T) widen(t + 1);  // overlaps the reductions below
        float2 r0 = __fadd2_rn(make_float2(ak0.x, aq0.x), make_float2(ak0.y, aq0.y));
        float2 r1 = __fadd2_rn(make_float2(ak1.x, aq1.x), make_float2(ak1.y, aq1.y));
        float2 rn = __fadd2_rn(make_float2(akk.x, aqq.x), make_float2(akk.y, aqq.y));
        float kq = akq.x + akq.y;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
          const float x0 = __shfl_xor_sync(0xffffffffu, r0.x, o), y0 = __shfl_xor_sync(0xffffffffu, r0.y, o);
          const float x1 = __shfl_xor_sync(0xffffffffu, r1.x, o), y1 = __shfl_xor_sync(0xffffffffu, r1.y, o);
          const float xq = __shfl_xor_sync(0xffffffffu, kq, o);
          float xn = 0.f, yn = 0.f;
          if (L2NORM) {
            xn = __shfl_xor_sync(0xffffffffu, rn.x, o);
            yn = __shfl_xor_sync(0xffffffffu, rn.y, o);
          }
          r0 = __fadd2_rn(r0, make_float2(x0, y0));
          r1 = __fadd2_rn(r1, make_float2(x1, y1));
          kq += xq;
          if (L2NORM) rn = __fadd2_rn(rn, make_float2(xn, yn));
        }
        float rk = 1.f;
        if (L2NORM) {
          // k <- k / sqrt(|k|^2 + eps), q likewise: scale the dot products instead of the vectors
          const float rq = rsqrtf(rn.y + 1e-6f);
          rk = rsqrtf(rn.x + 1e-6f);
          const float2 s2 = make_float2(rk, rq);
          r0 = __fmul2_rn(r0, s2);
          r1 = __fmul2_rn(r1, s2);
          kq *= rk * rq;
        }
        const float g = __shfl_sync(0xffffffffu, g_l, t), beta = __shfl_sync(0xffffffffu, beta_l, t);
        const __nv_bfloat16* vt = reinterpret_cast<const __nv_bfloat16*>(tk + T * 512 + t * 16);
        const float delta0 = beta * (__bfloat162float(vt[rg]) - g * r0.x);
        const float delta1 = beta * (__bfloat162float(vt[4 + rg]) - g * r1.x);
        if (cs == 0) {
          __nv_bfloat16* out_t = out_item + (size_t)t * p.o_st;
          out_t[rg] = __float2bfloat16_rn(scale * fmaf(delta0, kq, g * r0.y));
          out_t[4 + rg] = __float2bfloat16_rn(scale * fmaf(delta1, kq, g * r1.y));
        }
        // S <- g S + delta k (k normalised: delta * rk times the raw k)
        const float2 g2 = make_float2(g, g), d0 = make_float2(delta0 * rk, delta0 * rk),
                     d1 = make_float2(delta1 * rk, delta1 * rk);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          s[0][c] = __ffma2_rn(g2, s[0][c], __fmul2_rn(d0, kv[c]));
          s[1][c] = __ffma2_rn(g2, s[1][c], __fmul2_rn(d1, kv[c]));
        }
        if (p.inter) {
#pragma unroll
          for (int ps = 0; ps < 2; ++ps) {
            float* idst = p.inter + (size_t)slot * p.i_sn + (size_t)t * p.i_st + (size_t)it.h * p.i_sh +
                          (size_t)(it.wrow0 + ps * 4 + rg) * kHeadDim + cs * 4;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              st_cs_f4(idst + c4 * 32, make_float4(s[ps][2 * c4].x, s[ps][2 * c4].y, s[ps][2 * c4 + 1].x,
                                                   s[ps][2 * c4 + 1].y));
          }
        }
        __syncwarp();  // token t + 1 widened
      }
    } else {
      if (slot >= p.P && lane == 0) raise_device_error(kDevErrBadIndex);
      for (int e = lane; e < T * kPipeRows; e += 32)
        p.out[(size_t)it.bi * p.o_sb + (size_t)(e / kPipeRows) * p.o_st + (size_t)it.h * p.o_sh + it.wrow0 +
              e % kPipeRows] = __float2bfloat16_rn(0.f);
    }
    __syncwarp();
    if (item + 2 * step < n_items) issue_tok(item + 2 * step, st);
    if (valid) {
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        float* dst = p.new_pool + (size_t)slot * p.n_sn + (size_t)it.h * p.n_sh +
                     (size_t)(it.wrow0 + ps * 4 + rg) * kHeadDim + cs * 4;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4)
          st_cs_f4(dst + c4 * 32, make_float4(s[ps][2 * c4].x, s[ps][2 * c4].y, s[ps][2 * c4 + 1].x,
                                              s[ps][2 * c4 + 1].y));
      }
    }
    slot0 = slot1;
    slot1 = slot2;
    slot2 = slot3;
  }
  if (fail) {
    // a copy did not land in time (recorded): wait, bounded, for this warp's
    // copies still in flight before its shared memory is released.  Item i of
    // this warp uses stage i & 1, phase i >> 1; rows are issued two items
    // ahead (item j + 2 only once item j's rows were waited for), tokens after
    // the previous item's steps.
    const int n_local = (n_items - first + step - 1) / step;
    const int rows_last = std::min(n_local - 1, fail == 2 ? j + 2 : j + 1);
    const int tok_last = std::min(n_local - 1, j + 1);
    for (int i = (fail == 2 ? j + 1 : j); i <= rows_last; ++i)
      if (!mbar_wait(&bars[i & 1], (uint32_t)((i >> 1) & 1))) return;
    for (int i = j; i <= tok_last; ++i)
      if (!mbar_wait(&bars[2 + (i & 1)], (uint32_t)((i >> 1) & 1))) return;
  }
}

bool pipe_supported(const DecodeMtpParams& p) {
  if ((long long)p.B * p.HV * (kHeadDim / kPipeRows) >= (1ll << 31)) return false;
  auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  auto m8 = [](int64_t s) { return (s & 7) == 0; };
  return p.T >= 1 && p.T <= kPipeMaxT && al16(p.q) && al16(p.k) && al16(p.v) && m8(p.q_sb) && m8(p.q_st) &&
         m8(p.q_sh) && m8(p.k_sb) && m8(p.k_st) && m8(p.k_sh) && m8(p.v_sb) && m8(p.v_st) && m8(p.v_sh);
}

template <bool L2NORM>
cudaError_t launch_pipe(const DecodeMtpParams& p, cudaStream_t stream) {
  const int dev_max_smem = (int)(kPipeWarps * pipe_warp_bytes(kPipeMaxT));
  // per-device opt-in and occupancy (per T), looked up once
  static bool attr_set[64] = {};
  static int occ[64][kPipeMaxT + 1] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(decode_mtp_pipe_kernel<L2NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, dev_max_smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const size_t smem = (size_t)kPipeWarps * pipe_warp_bytes(p.T);
  if (occ[dev][p.T] == 0) {
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mtp_pipe_kernel<L2NORM>, kPipeWarps * 32, smem);
    if (e != cudaSuccess) return e;
    occ[dev][p.T] = n > 0 ? n : 1;
  }
  DecodeMtpParams q = p;
  int l = 0;
  while ((1ll << l) < p.HV) ++l;
  q.hv_shr = l;
  q.hv_mul = (uint32_t)((((1ull << 32) * ((1ull << l) - (unsigned long long)p.HV)) / (unsigned long long)p.HV) + 1);
  const long n_items = (long)p.B * p.HV * (kHeadDim / kPipeRows);
  const long need = (n_items + kPipeWarps - 1) / kPipeWarps;
  const long grid = std::min<long>(need, (long)sms[dev] * occ[dev][p.T]);
  decode_mtp_pipe_kernel<L2NORM><<<(unsigned)grid, kPipeWarps * 32, smem, stream>>>(q);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_mtp(const DecodeMtpParams& p, cudaStream_t stream) {
  if (p.B == 0 || p.T == 0) return cudaSuccess;
  if (pipe_supported(p))
    return (p.flags & kFlagQkL2Norm) ? launch_pipe<true>(p, stream) : launch_pipe<false>(p, stream);
  return decode_rows_for(p.B, p.HV) == 32 ? launch_mtp_rows<32>(p, stream) : launch_mtp_rows<16>(p, stream);
}

}  // namespace gdn
