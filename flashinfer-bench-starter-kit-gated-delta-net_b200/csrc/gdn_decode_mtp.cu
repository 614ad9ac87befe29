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

// ---------------------------------------------------------------------------
// Chunked multi-token kernel (2 <= T <= kChunkMaxT tokens, no intermediate states,
// q/k/v rows 16-byte aligned): every token's dot products with the state come
// from the unit's initial rows at once instead of one token after another.
//
// For one state row s and tokens t = 0 .. T-1 the decode recurrence is
//   s_t = g_t s_{t-1} + d_t k_t,   d_t = beta_t (v_t - g_t s_{t-1}.k_t),
//   o_t = scale (g_t s_{t-1}.q_t + d_t k_t.q_t).
// Every dot product of a later state with a token vector w follows from the
// products with the initial row and the Gram scalars of the token vectors:
//   z_t(w) = s_t.w = g_t z_{t-1}(w) + d_t (k_t.w),   z_{-1}(w) = s.w,
// and the final row is s_{T-1} = (prod_t g_t) s + sum_j c_j k_j with
// c_j = d_j prod_{i>j} g_i.  Per work unit of 16 rows of one (sequence, v-head):
//   G  the T^2 Gram scalars k_j.k_t (j < t) and k_j.q_t (j <= t) (+ |k_t|^2 and
//      |q_t|^2 for the in-kernel L2 norm), each lane over 4 of the 128
//      features, reduce-scattered over the warp into shared memory;
//   A  S [16 x 128] times W [128 x 8] (the token vectors k_0.., q_0.., zero
//      padded to 8) on the warp's tensor cores (mma.sync m16n8k8, tf32 inputs,
//      fp32 accumulation; S split as tf32 hi + lo, so the products keep ~20
//      bits; k and q are bf16 values, exact in tf32);
//   B  the recurrence on scalars for the lane's two rows (z, d_t, o_t, c_j);
//   C  S <- (prod g) S + C K, the rank-T update as a second mma with the state
//      as the accumulator (c split as tf32 hi + lo), stored from the fragments.
// The k dimension of A is permuted within each 8-column step (logical columns
// t and t + 4 are physical columns 2t and 2t + 1), which makes the A fragment of
// step n the accumulator fragment of columns 8n .. 8n + 7: each lane holds its 64
// state values once, in that layout, for both products.  Against the
// token-serial form there is no shuffle reduction per token, one multiply-add per
// token and element in the state update, and no token waits for the previous
// one.  The state crosses HBM once per call; each unit's rows (into padded
// shared rows, so the fragment loads are free of bank conflicts) and token rows
// are bulk-copied one unit ahead.
constexpr int kChunkMaxT = 8;
constexpr int kChunkWarps = 4;

// Enumeration of the Gram scalars of T tokens (vectors w < T are k_w, w >= T are
// q_{w - T}): token t owns kk(j, t) = k_j.k_t for j < t, then kq(j, t) = k_j.q_t
// for j <= t (2 t + 1 scalars from index t^2); then |k_t|^2, |q_t|^2.
template <int T, bool L2NORM>
struct ChunkGram {
  static constexpr int kDots = T * T + (L2NORM ? 2 * T : 0);
  // up to 32: one power-of-two reduce-scatter; beyond: batches of 32
  static constexpr int kPad = kDots <= 1 ? 1 : kDots <= 2 ? 2 : kDots <= 4 ? 4 : kDots <= 8 ? 8 : kDots <= 16 ? 16
                            : (kDots + 31) / 32 * 32;
  static constexpr int kk(int j, int t) { return t * t + j; }
  static constexpr int kq(int j, int t) { return t * t + t + j; }
  static constexpr int nk(int t) { return T * T + t; }
  static constexpr int nq(int t) { return T * T + T + t; }
  static constexpr int va(int d) {  // first vector of scalar d
    for (int t = 0; t < T; ++t) {
      if (d < t * t + t) return d - t * t;
      if (d < t * t + 2 * t + 1) return d - t * t - t;
    }
    return d < T * T + T ? d - T * T : T + (d - T * T - T);
  }
  static constexpr int vb(int d) {  // second vector of scalar d
    for (int t = 0; t < T; ++t) {
      if (d < t * t + t) return t;
      if (d < t * t + 2 * t + 1) return T + t;
    }
    return d < T * T + T ? d - T * T : T + (d - T * T - T);
  }
  static constexpr uint32_t kBytes = (uint32_t)((kPad * 4 + 15) / 16 * 16);
};

// Reduce-scatter of N (a power of two) per-lane partial sums over the warp: after
// it, for N >= 32 lane l holds the full sums of scalars l N/32 .. l N/32 + N/32 - 1
// in v[0 ..]; for N < 32 it holds scalar l >> (5 - log2 N) in v[0].
template <int N, int M>
struct WarpReduceScatter {
  __device__ __forceinline__ static void run(float* v, int lane) {
    if constexpr (M > 0) {
      if constexpr (N > 1) {
        constexpr int H = N / 2;
        const bool up = (lane & M) != 0;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float send = up ? v[i] : v[i + H];
          const float keep = up ? v[i + H] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, M);
        }
        WarpReduceScatter<H, M / 2>::run(v, lane);
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], M);
        WarpReduceScatter<1, M / 2>::run(v, lane);
      }
    }
  }
};

constexpr int ilog2(int n) { return n <= 1 ? 0 : 1 + ilog2(n / 2); }

// Work unit of the chunked kernel: 16 consecutive state rows of one (sequence, v-head),
// processed as two 8-row halves; the token rows, the gates and the Gram scalars are
// prepared once per unit and serve both halves.
constexpr int kChunkRows = 16;
constexpr uint32_t kChunkRowBytes = kChunkRows * kHeadDim * 4;  // 8192
constexpr int kPadRow = kHeadDim + 8;                           // padded shared row (floats): 544 B
// token vectors (k_0 .., q_0 ..) in tiles of 8 (the N of one mma): one tile up to 4 tokens, two up to 8
__host__ __device__ constexpr int chunk_vec_tiles(int T) { return (2 * T + 7) / 8; }
// token rows of a unit: q and k (256 B each) per token, then v of the unit's 16 rows (32 B) per token
__host__ __device__ constexpr uint32_t chunk_tok_bytes(int T) { return (uint32_t)T * (2 * kHeadDim * 2 + kChunkRows * 2); }
// per token in shared memory: v of the 16 rows, g, beta (fp32)
constexpr int kChunkScal = kChunkRows + 2;

template <int T, bool L2NORM>
__host__ __device__ constexpr uint32_t chunk_warp_bytes() {
  // rows [16][kPadRow] fp32 | token rows | q, k widened [8 x vector tiles][kPadRow] fp32 (rows >= 2T
  // zero) | Gram scalars | per-token scalars | 2 mbarriers
  return (uint32_t)(kChunkRows * kPadRow * 4) + chunk_tok_bytes(T) + (uint32_t)(8 * chunk_vec_tiles(T) * kPadRow * 4) +
         ChunkGram<T, L2NORM>::kBytes + (uint32_t)((T * kChunkScal * 4 + 15) / 16 * 16) + 16;
}

// unit u = (b * HV + h) * 8 + row block of 16 (the division by HV as in pipe_item)
__device__ __forceinline__ PipeItem chunk_unit(int u, const DecodeMtpParams& p) {
  PipeItem it;
  it.wrow0 = (u & (kHeadDim / kChunkRows - 1)) * kChunkRows;
  const uint32_t bh = (uint32_t)u >> 3;
  it.bi = (int)((__umulhi(bh, p.hv_mul) + bh) >> p.hv_shr);
  it.h = (int)bh - it.bi * p.HV;
  return it;
}
static_assert(kHeadDim / kChunkRows == 8, "8 row blocks per head");

// x = hi + lo: hi = x with the 13 mantissa bits below tf32 cleared (exactly a tf32 value), lo =
// x - hi (exact in fp32); the tensor core reads lo as tf32, dropping its low 13 bits, so the pair
// keeps about 20 significant bits of x (two integer/float instructions, no rounding mode emulation)
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}
// d += a b, m16n8k8, tf32 inputs, fp32 accumulation (fragments as in the PTX ISA:
// lane = 4 g + t; a: (g, t), (g + 8, t), (g, t + 4), (g + 8, t + 4); b: (t, g), (t + 4, g);
// d: (g, 2t), (g, 2t + 1), (g + 8, 2t), (g + 8, 2t + 1))
__device__ __forceinline__ void mma_16x8x8_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int T, bool L2NORM>
__global__ void __launch_bounds__(kChunkWarps * 32, T > 4 ? 2 : 3) decode_mtp_chunk_kernel(DecodeMtpParams p) {
  using G = ChunkGram<T, L2NORM>;
  constexpr int NV = chunk_vec_tiles(T);  // 8-vector tiles of W
  constexpr uint32_t kTok = chunk_tok_bytes(T);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* wbase = smem_raw + (size_t)warp * chunk_warp_bytes<T, L2NORM>();
  float* rows_buf = reinterpret_cast<float*>(wbase);  // [16][kPadRow]
  unsigned char* tok_buf = wbase + kChunkRows * kPadRow * 4;
  float* qk32 = reinterpret_cast<float*>(tok_buf + kTok);  // [8 NV][kPadRow]: k_0 .. k_{T-1}, q_0 .. q_{T-1}, 0 ..
  float* gram = qk32 + 8 * NV * kPadRow;
  float* scal = gram + G::kBytes / 4;  // [T][kChunkScal]: v of rows 0-15, g, beta
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      reinterpret_cast<unsigned char*>(scal) + (T * kChunkScal * 4 + 15) / 16 * 16);  // rows, tokens

  const int n_units = p.B * p.HV * (kHeadDim / kChunkRows);  // < 2^31 (checked by the launcher)
  const int first = blockIdx.x * kChunkWarps + warp, step = gridDim.x * kChunkWarps;
  if (first >= n_units) return;
  const int g8 = lane >> 2, t4 = lane & 3;  // mma fragment coordinates

  if (lane == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_barrier_init();
  }
  // the zero padding vectors (w >= 2T) of W, written once
  for (int e = lane; e < (8 * NV - 2 * T) * kPadRow; e += 32) qk32[2 * T * kPadRow + e] = 0.f;
  __syncwarp();

  auto issue_rows = [&](const PipeItem& it, int64_t slot) {
    const bool have = slot >= 0 && slot < p.P;
    if (lane == 0) {
      if (have) mbar_arrive_expect_tx(&bars[0], kChunkRowBytes);
      else mbar_arrive(&bars[0]);  // nothing to load: complete the phase
    }
    __syncwarp();
    if (have && lane < kChunkRows)  // one 512-byte row per lane, into its padded shared row
      bulk_g2s_evict_first(rows_buf + lane * kPadRow,
                           p.pool + (size_t)slot * p.s_sn + (size_t)it.h * p.s_sh + (size_t)(it.wrow0 + lane) * kHeadDim,
                           kHeadDim * 4, &bars[0]);
  };
  auto issue_tok = [&](const PipeItem& it) {
    if (lane == 0) mbar_arrive_expect_tx(&bars[1], kTok);
    __syncwarp();
    const int qh = it.h / p.ratio;
    if (lane < T) {
      bulk_g2s(tok_buf + lane * 512, p.q + (size_t)it.bi * p.q_sb + (size_t)lane * p.q_st + (size_t)qh * p.q_sh, 256,
               &bars[1]);
    } else if (lane < 2 * T) {
      const int t = lane - T;
      bulk_g2s(tok_buf + t * 512 + 256, p.k + (size_t)it.bi * p.k_sb + (size_t)t * p.k_st + (size_t)qh * p.k_sh, 256,
               &bars[1]);
    } else if (lane < 3 * T) {
      const int t = lane - 2 * T;
      bulk_g2s(tok_buf + T * 512 + t * 32,
               p.v + (size_t)it.bi * p.v_sb + (size_t)t * p.v_st + (size_t)it.h * p.v_sh + it.wrow0, 32, &bars[1]);
    }
  };
  auto load_gate_inputs = [&](const PipeItem& it, bool have, float& ga, float& gb, float& alog, float& dtb) {
    ga = gb = alog = dtb = 0.f;
    if (have && lane < T) {
      ga = bf16_to_f32(p.a + (size_t)it.bi * p.a_sb + (size_t)lane * p.a_st + it.h);
      gb = bf16_to_f32(p.b + (size_t)it.bi * p.b_sb + (size_t)lane * p.b_st + it.h);
      alog = p.A_log[it.h];
      dtb = p.dt_bias[it.h];
    }
  };

  // prologue: the first unit's rows and tokens in flight, the next unit's pool index
  PipeItem cur = chunk_unit(first, p), nx = chunk_unit(first + step < n_units ? first + step : first, p);
  int64_t slot_cur = load_index(p, cur.bi);
  int64_t slot_next = first + step < n_units ? load_index(p, nx.bi) : -1;
  issue_rows(cur, slot_cur);
  issue_tok(cur);
  uint32_t rows_issued = 1, rows_done = 0, tok_issued = 1, tok_done = 0;  // per barrier: phases armed / waited
  float ga, gb, alog, dtb;
  load_gate_inputs(cur, true, ga, gb, alog, dtb);

  bool fail = false;
  for (int u = first; u < n_units; u += step) {
    const PipeItem it = cur;
    const int64_t slot = slot_cur;
    const bool valid = slot >= 0 && slot < p.P;
    const bool more = u + step < n_units;
    // this unit's gates (lane t: token t), then the next unit's inputs and the pool index after it
    float g_l = 0.f, beta_l = 0.f;
    if (lane < T) gdn_gates_fast(alog, ga, dtb, gb, g_l, beta_l);
    load_gate_inputs(nx, more, ga, gb, alog, dtb);
    const bool more2 = u + 2 * step < n_units;
    const PipeItem nn = chunk_unit(more2 ? u + 2 * step : u, p);
    const int64_t slot_nn = more2 ? load_index(p, nn.bi) : -1;

    // ---- tokens: q and k widened to fp32 (lane: features 4 lane .. 4 lane + 3 of every
    //      vector), the Gram partials from the same registers, v and gates as fp32 ----
    if (!mbar_wait(&bars[1], tok_done & 1)) { fail = true; break; }
    ++tok_done;
    float4 wv[2 * T];
#pragma unroll
    for (int w = 0; w < 2 * T; ++w) {
      const int t = w < T ? w : w - T;
      const uint2 r = *reinterpret_cast<const uint2*>(tok_buf + t * 512 + (w < T ? 256 : 0) + lane * 8);
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      wv[w] = make_float4(lo.x, lo.y, hi.x, hi.y);
      *reinterpret_cast<float4*>(qk32 + w * kPadRow + lane * 4) = wv[w];
    }
    {
      const __nv_bfloat16* vt = reinterpret_cast<const __nv_bfloat16*>(tok_buf + T * 512);
#pragma unroll
      for (int e = lane; e < kChunkRows * T; e += 32)  // token e / 16, row e % 16
        scal[(e >> 4) * kChunkScal + (e & 15)] = __bfloat162float(vt[e]);
    }
    if (lane < T) {
      scal[lane * kChunkScal + kChunkRows] = g_l;
      scal[lane * kChunkScal + kChunkRows + 1] = beta_l;
    }
    __syncwarp();  // the token buffer is read; every lane's q, k features are in qk32
    if (more) {
      issue_tok(nx);
      ++tok_issued;
    }
    if constexpr (G::kPad <= 32) {
      float gp[G::kPad];
#pragma unroll
      for (int d = 0; d < G::kPad; ++d) {
        if (d < G::kDots) {
          const float4 x = wv[G::va(d)], y = wv[G::vb(d)];
          gp[d] = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, x.w * y.w)));
        } else {
          gp[d] = 0.f;
        }
      }
      WarpReduceScatter<G::kPad, 16>::run(gp, lane);
      if constexpr (G::kPad == 32) {
        gram[lane] = gp[0];
      } else {
        constexpr int sh = 5 - ilog2(G::kPad);
        if ((lane & ((1 << sh) - 1)) == 0) gram[lane >> sh] = gp[0];
      }
    } else {
#pragma unroll
      for (int b0 = 0; b0 < G::kPad; b0 += 32) {  // 32 scalars per batch, lane l keeps scalar b0 + l
        float gp[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int d = b0 + i;
          if (d < G::kDots) {
            const float4 x = wv[G::va(d)], y = wv[G::vb(d)];
            gp[i] = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, x.w * y.w)));
          } else {
            gp[i] = 0.f;
          }
        }
        WarpReduceScatter<32, 16>::run(gp, lane);
        gram[b0 + lane] = gp[0];
      }
    }

    // ---- the unit's 16 rows -> registers in the mma accumulator layout: c[n] = rows g8 and
    //      g8 + 8, columns 8 n + 2 t4 and 8 n + 2 t4 + 1; then the rows buffer goes to the next unit ----
    if (!mbar_wait(&bars[0], rows_done & 1)) { fail = true; break; }
    ++rows_done;
    float c[16][4];
    if (valid) {
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const float2 x0 = *reinterpret_cast<const float2*>(rows_buf + g8 * kPadRow + 8 * n + 2 * t4);
        const float2 x1 = *reinterpret_cast<const float2*>(rows_buf + (g8 + 8) * kPadRow + 8 * n + 2 * t4);
        c[n][0] = x0.x;
        c[n][1] = x0.y;
        c[n][2] = x1.x;
        c[n][3] = x1.y;
      }
    }
    __syncwarp();  // rows read; Gram scalars written
    if (more) {
      issue_rows(nx, slot_next);
      ++rows_issued;
    }
    __nv_bfloat16* out_unit = p.out + (size_t)it.bi * p.o_sb + (size_t)it.h * p.o_sh + it.wrow0;
    if (!valid) {
      if (slot >= p.P && lane == 0) raise_device_error(kDevErrBadIndex);
      for (int e = lane; e < T * kChunkRows; e += 32)
        out_unit[(size_t)(e >> 4) * p.o_st + (e & 15)] = __float2bfloat16_rn(0.f);
    } else {
      // ---- A: D = S W (rows g8, g8 + 8 of the unit; token vectors 2 t4, 2 t4 + 1) ----
      // per vector tile, four independent accumulators (hi / lo x even / odd steps) keep the
      // mma chains short
      float da[NV][4][4] = {};
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        uint32_t ah[4], al[4];
        tf32_split(c[n][0], ah[0], al[0]);  // (g8, logical t4)
        tf32_split(c[n][2], ah[1], al[1]);  // (g8 + 8, t4)
        tf32_split(c[n][1], ah[2], al[2]);  // (g8, t4 + 4)
        tf32_split(c[n][3], ah[3], al[3]);  // (g8 + 8, t4 + 4)
#pragma unroll
        for (int vt = 0; vt < NV; ++vt) {  // vector 8 vt + g8
          const float2 bw = *reinterpret_cast<const float2*>(qk32 + (8 * vt + g8) * kPadRow + 8 * n + 2 * t4);
          const uint32_t b0 = __float_as_uint(bw.x), b1 = __float_as_uint(bw.y);
          mma_16x8x8_tf32(da[vt][2 * (n & 1)], ah[0], ah[1], ah[2], ah[3], b0, b1);
          mma_16x8x8_tf32(da[vt][2 * (n & 1) + 1], al[0], al[1], al[2], al[3], b0, b1);
        }
      }
      // every lane of the quad gathers all 2T products of rows g8 and g8 + 8
      float x[2][8 * NV];
#pragma unroll
      for (int vt = 0; vt < NV; ++vt) {
        float dacc[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) dacc[i] = (da[vt][0][i] + da[vt][2][i]) + (da[vt][1][i] + da[vt][3][i]);
#pragma unroll
        for (int tq = 0; tq < 4; ++tq) {
          const int src = (lane & ~3) | tq;
          x[0][8 * vt + 2 * tq] = __shfl_sync(0xffffffffu, dacc[0], src);
          x[0][8 * vt + 2 * tq + 1] = __shfl_sync(0xffffffffu, dacc[1], src);
          x[1][8 * vt + 2 * tq] = __shfl_sync(0xffffffffu, dacc[2], src);
          x[1][8 * vt + 2 * tq + 1] = __shfl_sync(0xffffffffu, dacc[3], src);
        }
      }
      // ---- B: the token recurrence on scalars for rows g8 (ps 0) and g8 + 8 (ps 1) ----
      float nkv[T], nqv[T];  // 1 / |k_t|, 1 / |q_t| with the L2 norm, else 1
#pragma unroll
      for (int t = 0; t < T; ++t) {
        nkv[t] = L2NORM ? rsqrtf(gram[G::nk(t)] + 1e-6f) : 1.f;
        nqv[t] = L2NORM ? rsqrtf(gram[G::nq(t)] + 1e-6f) : 1.f;
      }
      const float scale = p.scale;
      float cm[2][2], pg = 1.f;  // cm[ps][h]: c of token t4 + 4 h for the lane's two rows; pg = prod g
#pragma unroll
      for (int t = 0; t < T; ++t) pg *= scal[t * kChunkScal + kChunkRows];
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        float z[2 * T];
#pragma unroll
        for (int t = 0; t < T; ++t) {
          z[t] = x[ps][t] * nkv[t];
          z[T + t] = x[ps][T + t] * nqv[t];
        }
        const int vr = g8 + 8 * ps;
        float dl[T], om[2] = {0.f, 0.f};  // om[h]: the output of token t4 + 4 h (this lane's stores)
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float g = scal[t * kChunkScal + kChunkRows];
          const float d = scal[t * kChunkScal + kChunkRows + 1] * (scal[t * kChunkScal + vr] - g * z[t]);
          const float o = scale * fmaf(d, gram[G::kq(t, t)] * (nkv[t] * nqv[t]), g * z[T + t]);
          if ((t & 3) == t4) om[t >> 2] = o;
          dl[t] = d;
#pragma unroll
          for (int t2 = t + 1; t2 < T; ++t2) {
            z[t2] = fmaf(d, gram[G::kk(t, t2)] * (nkv[t] * nkv[t2]), g * z[t2]);
            z[T + t2] = fmaf(d, gram[G::kq(t, t2)] * (nkv[t] * nqv[t2]), g * z[T + t2]);
          }
        }
        float tail = 1.f;  // prod_{i > j} g_i
        cm[ps][0] = cm[ps][1] = 0.f;
#pragma unroll
        for (int t = T - 1; t >= 0; --t) {
          const float cj = dl[t] * tail * nkv[t];
          if ((t & 3) == t4) cm[ps][t >> 2] = cj;
          tail *= scal[t * kChunkScal + kChunkRows];
        }
        if (t4 < T) out_unit[(size_t)t4 * p.o_st + vr] = __float2bfloat16_rn(om[0]);  // token t4's output
        if (t4 + 4 < T) out_unit[(size_t)(t4 + 4) * p.o_st + vr] = __float2bfloat16_rn(om[1]);  // token t4 + 4
      }
      // ---- C: S <- (prod g) S + C K: A = c (rows g8, g8 + 8; tokens t4 and t4 + 4, 0 beyond T),
      //      B = k_t4, k_{t4 + 4} (0 beyond T) ----
      uint32_t ch[4], cl[4];
      tf32_split(cm[0][0], ch[0], cl[0]);  // (g8, t4)
      tf32_split(cm[1][0], ch[1], cl[1]);  // (g8 + 8, t4)
      tf32_split(cm[0][1], ch[2], cl[2]);  // (g8, t4 + 4)
      tf32_split(cm[1][1], ch[3], cl[3]);  // (g8 + 8, t4 + 4)
      const float* krow0 = qk32 + (t4 < T ? t4 : 0) * kPadRow;
      const float* krow1 = qk32 + (t4 + 4 < T ? t4 + 4 : 0) * kPadRow;
      float* dst0 = p.new_pool + (size_t)slot * p.n_sn + (size_t)it.h * p.n_sh + (size_t)(it.wrow0 + g8) * kHeadDim +
                    2 * t4;
      float* dst1 = dst0 + 8 * kHeadDim;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const float2 s01 = __fmul2_rn(make_float2(c[n][0], c[n][1]), make_float2(pg, pg));
        const float2 s23 = __fmul2_rn(make_float2(c[n][2], c[n][3]), make_float2(pg, pg));
        float acc[4] = {s01.x, s01.y, s23.x, s23.y};
        const uint32_t b0 = t4 < T ? __float_as_uint(krow0[8 * n + g8]) : 0u;
        const uint32_t b1 = t4 + 4 < T ? __float_as_uint(krow1[8 * n + g8]) : 0u;
        mma_16x8x8_tf32(acc, ch[0], ch[1], ch[2], ch[3], b0, b1);
        mma_16x8x8_tf32(acc, cl[0], cl[1], cl[2], cl[3], b0, b1);
        __stcs(reinterpret_cast<float2*>(dst0 + 8 * n), make_float2(acc[0], acc[1]));
        __stcs(reinterpret_cast<float2*>(dst1 + 8 * n), make_float2(acc[2], acc[3]));
      }
    }
    __syncwarp();  // qk32, the Gram and per-token scalars are read before the next unit overwrites them
    cur = nx;
    nx = nn;
    slot_cur = slot_next;
    slot_next = slot_nn;
  }
  if (fail) {
    // a copy did not land in time (recorded): wait, bounded, for this warp's copies still
    // in flight before its shared memory is released
    if (rows_issued > rows_done && !mbar_wait(&bars[0], rows_done & 1)) return;
    if (tok_issued > tok_done) mbar_wait(&bars[1], tok_done & 1);
  }
}

bool pipe_supported(const DecodeMtpParams& p) {
  if ((long long)p.B * p.HV * (kHeadDim / kPipeRows) >= (1ll << 31)) return false;
  auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  auto m8 = [](int64_t s) { return (s & 7) == 0; };
  return p.T >= 1 && p.T <= kPipeMaxT && al16(p.q) && al16(p.k) && al16(p.v) && m8(p.q_sb) && m8(p.q_st) &&
         m8(p.q_sh) && m8(p.k_sb) && m8(p.k_st) && m8(p.k_sh) && m8(p.v_sb) && m8(p.v_st) && m8(p.v_sh);
}

// The item -> (sequence, v-head) divisor of pipe_item for this call's HV.
DecodeMtpParams with_hv_divisor(const DecodeMtpParams& p) {
  DecodeMtpParams q = p;
  int l = 0;
  while ((1ll << l) < p.HV) ++l;
  q.hv_shr = l;
  q.hv_mul = (uint32_t)((((1ull << 32) * ((1ull << l) - (unsigned long long)p.HV)) / (unsigned long long)p.HV) + 1);
  return q;
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
  DecodeMtpParams q = with_hv_divisor(p);
  const long n_items = (long)p.B * p.HV * (kHeadDim / kPipeRows);
  const long need = (n_items + kPipeWarps - 1) / kPipeWarps;
  const long grid = std::min<long>(need, (long)sms[dev] * occ[dev][p.T]);
  decode_mtp_pipe_kernel<L2NORM><<<(unsigned)grid, kPipeWarps * 32, smem, stream>>>(q);
  return cudaGetLastError();
}

template <int T, bool L2NORM>
cudaError_t launch_chunk(const DecodeMtpParams& p, cudaStream_t stream) {
  constexpr size_t smem = (size_t)kChunkWarps * chunk_warp_bytes<T, L2NORM>();
  // per-device opt-in, SM count and occupancy, looked up once
  static bool attr_set[64] = {};
  static int occ[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(decode_mtp_chunk_kernel<T, L2NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    int n = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mtp_chunk_kernel<T, L2NORM>, kChunkWarps * 32,
                                                      smem);
    if (e != cudaSuccess) return e;
    occ[dev] = n > 0 ? n : 1;
    attr_set[dev] = true;
  }
  const DecodeMtpParams q = with_hv_divisor(p);
  const long n_units = (long)p.B * p.HV * (kHeadDim / kChunkRows);
  const long need = (n_units + kChunkWarps - 1) / kChunkWarps;
  const long grid = std::min<long>(need, (long)sms[dev] * occ[dev]);
  decode_mtp_chunk_kernel<T, L2NORM><<<(unsigned)grid, kChunkWarps * 32, smem, stream>>>(q);
  return cudaGetLastError();
}

template <bool L2NORM>
cudaError_t launch_chunk_any(const DecodeMtpParams& p, cudaStream_t stream) {
  static_assert(kChunkMaxT == 8, "one instantiation per token count");
  switch (p.T) {
    case 2: return launch_chunk<2, L2NORM>(p, stream);
    case 3: return launch_chunk<3, L2NORM>(p, stream);
    case 4: return launch_chunk<4, L2NORM>(p, stream);
    case 5: return launch_chunk<5, L2NORM>(p, stream);
    case 6: return launch_chunk<6, L2NORM>(p, stream);
    case 7: return launch_chunk<7, L2NORM>(p, stream);
    case 8: return launch_chunk<8, L2NORM>(p, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_decode_mtp(const DecodeMtpParams& p, cudaStream_t stream) {
  if (p.B == 0 || p.T == 0) return cudaSuccess;
  if (p.T == 1 && !p.inter) {
    // one token, no intermediate states: the single-token decode kernel on the indexed slots
    DecodeParams d;
    d.q = p.q;
    d.k = p.k;
    d.v = p.v;
    d.state = p.pool;
    d.A_log = p.A_log;
    d.a = p.a;
    d.dt_bias = p.dt_bias;
    d.b = p.b;
    d.out = p.out;
    d.new_state = p.new_pool;
    d.q_sb = p.q_sb;
    d.q_sh = p.q_sh;
    d.k_sb = p.k_sb;
    d.k_sh = p.k_sh;
    d.v_sb = p.v_sb;
    d.v_sh = p.v_sh;
    d.s_sb = p.s_sn;
    d.s_sh = p.s_sh;
    d.a_sb = p.a_sb;
    d.b_sb = p.b_sb;
    d.o_sb = p.o_sb;
    d.o_sh = p.o_sh;
    d.n_sb = p.n_sn;
    d.n_sh = p.n_sh;
    d.scale = p.scale;
    d.B = p.B;
    d.HQ = p.HQ;
    d.HV = p.HV;
    d.ratio = p.ratio;
    d.flags = p.flags;
    d.indices = p.indices;
    d.idx_is_int64 = p.idx_is_int64;
    d.P = p.P;
    return launch_decode(d, decode_rows_for(p.B, p.HV), stream);
  }
  if (pipe_supported(p)) {
    const bool l2 = (p.flags & kFlagQkL2Norm) != 0;
    // without intermediate states, 2 .. kChunkMaxT tokens: all tokens' products at once
    if (!p.inter && p.T >= 2 && p.T <= kChunkMaxT)
      return l2 ? launch_chunk_any<true>(p, stream) : launch_chunk_any<false>(p, stream);
    return l2 ? launch_pipe<true>(p, stream) : launch_pipe<false>(p, stream);
  }
  return decode_rows_for(p.B, p.HV) == 32 ? launch_mtp_rows<32>(p, stream) : launch_mtp_rows<16>(p, stream);
}

}  // namespace gdn
