// Chunk preparation for the chunked prefill (sm_100a): every state-independent
// quantity of every chunk of every (sequence, v-head), all at once.
//
// Reference semantics: solution/triton/kernel_prefill.py:42-142 (the per-token
// gates at :108-113).  For a chunk of C = 64 tokens with gates beta_t and
// log-decay prefix g_t (natural log, inclusive):
//   A[t][j] = beta_t exp(g_t - g_j) k_t.k_j   (j < t),   T = (I + A)^-1
// T is what turns the chunk's delta-rule recurrence into one product
// (D^T = R^T T^T in the chain kernel).  This kernel writes, per (chunk slot,
// v-head), the record described in gdn_prefill_chunk.cuh: the lower triangle of T
// as bf16 hi + lo core matrices (bulk-copied row block by row block into the chain
// kernel's MMA operand buffers) and the chunk's gate arrays.
//
// CTA = two consecutive chunk slots of one v-head, 8 warps in two groups of 4
// (group c = slot 2 * blockIdx.x + c):
//   threads 0 / 128 find their slot's chunk (binary search over cu_seqlens); thread 64
//              loads both chunks' K rows by TMA into one 128-row tile [K_slot0; K_slot1],
//              issues K_tile K_slot0^T and K_tile K_slot1^T on tcgen05 (fp32 in
//              TMEM; rows 0-63 of the first, 64-127 of the second are the
//              chunks' K K^T)
//   each group gates (64 threads, overlapping the TMA and MMA), A rows from
//              TMEM, then the inverse in place in one fp32 [64 x 68] array:
//              16x16 diagonal blocks by substitution, then block merges
//              16 -> 32 -> 64 (T_10 = -T_11 (A_10 T_00), the last one register-
//              blocked), and the record writes.
#include <cuda.h>

#include "gdn_prefill_chunk.cuh"

namespace gdn {
namespace {

using namespace chunk;

constexpr int kThreads = 256;
constexpr int kLd = 68;  // padded row stride (floats) of the in-place A / T array

constexpr uint32_t kSmK = 0;            // 2 tiles (feature cols 0-63 | 64-127) x [128 rows x 128 B]
constexpr uint32_t kKTile = 16384;
// per group: A, then T, in place [64][kLd] fp32.  It overlays the K tiles: A is written
// only after the K K^T products have completed (their commit barrier), when no
// tcgen05 read of the tiles is left.
constexpr uint32_t kSmAT = 0;
constexpr uint32_t kATBytes = 64 * kLd * 4;
constexpr uint32_t kSmGate = kSmAT + 2 * kATBytes;  // per group: GA_N x 64 fp32 + scan scratch
// per group, 64 fp32 each: g2_t, beta_t, G_t, g2_C (log2 e g_C), log2 m_t, m_t (q
// normalisation), scan scratch, then (after the K K^T diagonal) n_t and log2 n_t (k
// normalisation), the column term g2_t - log2 n_t and the row factor beta_t n_t of A
enum : int { PG_G2 = 0, PG_BETA, PG_G, PG_GC2, PG_LM, PG_M, PG_SCAN, PG_N, PG_LN, PG_G2C, PG_BN, PG_COUNT };
constexpr uint32_t kGateBytes = PG_COUNT * 64 * 4;
constexpr uint32_t kSmBar = kSmGate + 2 * kGateBytes;
constexpr uint32_t kSmMisc = kSmBar + 16;  // tmem base slot, per-group chunk info
constexpr uint32_t kSmBytes = kSmMisc + 80;
// Four CTAs per SM (64 registers, 128 TMEM columns each).  The allocation is padded
// so that a fifth cannot become resident and wait on TMEM (5 x 47 KB > 228 KB).
constexpr uint32_t kSmAlloc = (kSmBytes + 1024) > 46 * 1024 ? (kSmBytes + 1024) : 46 * 1024;
static_assert(kSmK + 2 * kKTile <= kSmGate && kSmAT + 2 * kATBytes <= kSmGate, "smem map");
static_assert((kSmAlloc + 1024) * 4 <= 228 * 1024 && (kSmAlloc + 1024) * 5 > 228 * 1024, "four CTAs per SM");

struct SlotInfo {
  int64_t slot;
  int64_t z;  // first token
  int nvalid;  // tokens of the chunk inside its sequence (0: no chunk in this slot)
  int pad;
};

// Chunk of slot `slot` (see gdn_prefill_chunk.cuh), or nvalid = 0 for a gap slot.
__device__ SlotInfo find_chunk(const PrefillParams& p, int64_t slot) {
  SlotInfo r{slot, 0, 0, 0};
  if (p.N <= 0 || slot_start(load_cu(p, 0), 0) > slot) return r;
  int lo = 0, hi = p.N - 1;  // largest n with slot_start(n) <= slot
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (slot_start(load_cu(p, mid), mid) <= slot) lo = mid;
    else hi = mid - 1;
  }
  const int64_t t0 = load_cu(p, lo), t1 = load_cu(p, lo + 1);
  if (t1 < t0 || t0 < 0 || t1 > p.T) return r;  // malformed: the chain kernel reports it
  const int64_t i = slot - slot_start(t0, lo);
  if (i * kC >= t1 - t0) return r;
  r.z = t0 + i * kC;
  const int64_t rem = t1 - r.z;
  r.nvalid = rem < kC ? (int)rem : kC;
  return r;
}

// 16x16 diagonal blocks of T, one column per thread (64 threads):
// x_r = delta_rc - sum_{q<r} A_rq x_q.  In place: all reads of a block finish
// (named barrier `bar`) before its T columns are written.
__device__ __forceinline__ void solve_diag16(float* AT, int p, int bar) {
  const int o = (p >> 4) * 16, c = p & 15;
  float x[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    const float* arow = AT + (o + r) * kLd + o;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int q4 = 0; q4 < r; q4 += 4) {
      const float4 a = *reinterpret_cast<const float4*>(arow + q4);
      s0 = fmaf(a.x, x[q4], s0);
      if (q4 + 1 < r) s1 = fmaf(a.y, x[q4 + 1], s1);
      if (q4 + 2 < r) s0 = fmaf(a.z, x[q4 + 2], s0);
      if (q4 + 3 < r) s1 = fmaf(a.w, x[q4 + 3], s1);
    }
    x[r] = (r == c ? 1.f : 0.f) - (s0 + s1);
  }
  named_sync(bar, 64);
#pragma unroll
  for (int r = 0; r < 16; ++r) AT[(o + r) * kLd + o + c] = x[r];
}

// ---- block merges on the warp-level tensor-core path (mma.sync, tf32 inputs,
// fp32 accumulation).  Each fp32 operand x is split as hi + lo (split_tf32) and a
// product accumulated as lo*hi + hi*lo + hi*hi, which keeps about 20 significant
// bits (fp32-level for these O(1) entries; T is stored as bf16 hi + lo, ~16 bits).  Fragments
// are read per lane from the fp32 array (m16n8k8 layouts: g = lane / 4,
// t = lane % 4), so no operand is broadcast through shared memory.
// hi = x with the 13 mantissa bits below tf32 cleared (exactly a tf32 value), lo = x - hi (exact in
// fp32; the tensor core reads it as tf32, dropping its low 13 bits)
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
struct FragA {
  uint32_t h[4], l[4];
};
struct FragB {
  uint32_t h[2], l[2];
};
// A fragment of the 16 x 8 block of AT at rows mr.., cols mc..
__device__ __forceinline__ FragA load_a(const float* AT, int mr, int mc, int lane) {
  const int g = lane >> 2, t = lane & 3;
  FragA f;
  split_tf32(AT[(mr + g) * kLd + mc + t], f.h[0], f.l[0]);
  split_tf32(AT[(mr + g + 8) * kLd + mc + t], f.h[1], f.l[1]);
  split_tf32(AT[(mr + g) * kLd + mc + t + 4], f.h[2], f.l[2]);
  split_tf32(AT[(mr + g + 8) * kLd + mc + t + 4], f.h[3], f.l[3]);
  return f;
}
// B fragment of the 8 x 8 block of AT at rows nr.. (K), cols nc.. (N)
__device__ __forceinline__ FragB load_b(const float* AT, int nr, int nc, int lane) {
  const int g = lane >> 2, t = lane & 3;
  FragB f;
  split_tf32(AT[(nr + t) * kLd + nc + g], f.h[0], f.l[0]);
  split_tf32(AT[(nr + t + 4) * kLd + nc + g], f.h[1], f.l[1]);
  return f;
}
// d += A B with the 3-term split
__device__ __forceinline__ void mma3(float (&d)[4], const FragA& a, const FragB& b) {
  mma_tf32(d, a.l[0], a.l[1], a.l[2], a.l[3], b.h[0], b.h[1]);
  mma_tf32(d, a.h[0], a.h[1], a.h[2], a.h[3], b.l[0], b.l[1]);
  mma_tf32(d, a.h[0], a.h[1], a.h[2], a.h[3], b.h[0], b.h[1]);
}
// d += M[mr.., mc..] (16 x 8) x N[nr.., nc..] (8 x 8), blocks of AT
__device__ __forceinline__ void mma_step(float (&d)[4], const float* AT, int mr, int mc, int nr, int nc, int lane) {
  mma3(d, load_a(AT, mr, mc, lane), load_b(AT, nr, nc, lane));
}
// store a 16 x 8 accumulator tile (times `sign`) at AT rows r0.., cols c0..
__device__ __forceinline__ void st_tile_f32(float* AT, int r0, int c0, const float (&d)[4], float sign, int lane) {
  const int g = lane >> 2, t = lane & 3;
  *reinterpret_cast<float2*>(AT + (r0 + g) * kLd + c0 + 2 * t) = make_float2(sign * d[0], sign * d[1]);
  *reinterpret_cast<float2*>(AT + (r0 + g + 8) * kLd + c0 + 2 * t) = make_float2(sign * d[2], sign * d[3]);
}

// Merge of the two 16-block pairs: for the pair rows/cols [jo, jo+16) (block 0)
// and [io = jo+16, io+16) (block 1), X = A_10 T_00 is stored above the diagonal
// at rows jo.., cols io.., then T_10 = -T_11 X is written over A_10.
// Warp w: pair w / 2, 8 output columns (w % 2) * 8.. ; T_00[k][c] = 0 for k < c.
__device__ __forceinline__ void solve_merge16(float* AT, int p, int bar) {
  const int w = p >> 5, lane = p & 31;
  const int jo = 32 * (w >> 1), io = jo + 16, n0 = 8 * (w & 1);
  {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int ks = w & 1; ks < 2; ++ks) mma_step(d, AT, io, jo + 8 * ks, jo + 8 * ks, jo + n0, lane);
    st_tile_f32(AT, jo, io + n0, d, 1.f, lane);
  }
  named_sync(bar, 128);
  {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) mma_step(d, AT, io, io + 8 * ks, jo + 8 * ks, io + n0, lane);
    st_tile_f32(AT, io, jo + n0, d, -1.f, lane);
  }
  named_sync(bar, 128);
}

// Merge of the two 32-blocks: X = A_10 T_00 (stored at rows 0-31, cols 32-63,
// above the diagonal), then T_10 = -T_11 X over A_10.  Warp w owns output
// columns [8w, 8w + 8) of both 16-row halves.  T_00[k][c] = 0 for k < c skips
// the first w k-steps; T_11 rows 0-15 stop at column 16 (rows 32-47 x cols
// 48-63 hold the 16-merge's scratch, not zeros).
__device__ __forceinline__ void solve_merge32(float* AT, int p, int bar) {
  const int w = p >> 5, lane = p & 31, n0 = 8 * w;
  {
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int ks = w; ks < 4; ++ks) {
      const FragB b = load_b(AT, 8 * ks, n0, lane);
      mma3(d0, load_a(AT, 32, 8 * ks, lane), b);
      mma3(d1, load_a(AT, 48, 8 * ks, lane), b);
    }
    st_tile_f32(AT, 0, 32 + n0, d0, 1.f, lane);
    st_tile_f32(AT, 16, 32 + n0, d1, 1.f, lane);
  }
  named_sync(bar, 128);
  {
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const FragB b = load_b(AT, 8 * ks, 32 + n0, lane);
      if (ks < 2) mma3(d0, load_a(AT, 32, 32 + 8 * ks, lane), b);
      mma3(d1, load_a(AT, 48, 32 + 8 * ks, lane), b);
    }
    st_tile_f32(AT, 32, n0, d0, -1.f, lane);
    st_tile_f32(AT, 48, n0, d1, -1.f, lane);
  }
  named_sync(bar, 128);
}

__global__ void __launch_bounds__(kThreads, 4)
    prefill_prep_kernel(const __grid_constant__ CUtensorMap mapK, PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = warp >> 2, gth = tid & 127;
  const int h = blockIdx.y, qh = h / p.ratio;
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(base + kSmBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + kSmMisc);
  SlotInfo* info = reinterpret_cast<SlotInfo*>(base + kSmMisc + 16);
  // named barriers: group g uses 1 + 2g (its 64 gate / diagonal threads) and 2 + 2g (all 128)
  const int bar64 = 1 + 2 * grp, bar128 = 2 + 2 * grp;

  if (gth == 0) info[grp] = find_chunk(p, 2 * (int64_t)blockIdx.x + grp);
  if (tid == 0) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, 128);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const SlotInfo mine = info[grp];
  const int n0 = info[0].nvalid, n1 = info[1].nvalid;

  // ---- K rows by TMA, then the two K K^T products (one thread) ----
  if (tid == 64 && (n0 | n1)) {  // a thread outside group 0's gate and A-row warps
    tc::prefetch_tensormap(&mapK);
    mbar_arrive_expect_tx(bar_tma, (n0 ? 16384u : 0u) + (n1 ? 16384u : 0u));
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      if (!info[c].nvalid) continue;
      const int z = (int)info[c].z;
      tc::tma_load_3d(base + kSmK + c * 8192, &mapK, 0, qh, z, bar_tma);
      tc::tma_load_3d(base + kSmK + kKTile + c * 8192, &mapK, 64, qh, z, bar_tma);
    }
    if (mbar_wait_sleep(bar_tma, 0)) {
      tc::fence_after_sync();
      const uint32_t id_n64 = tc::idesc_bf16(128, 64, false, false);
      const uint64_t dA = tc::kmajor_desc(smem_u32(base + kSmK), 0, 0);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint64_t dB = dA + ((uint64_t)(c * 8192) >> 4);  // rows 64c.. of the same tile
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + c * 64, dA + tc::kmajor_step(kKTile, ks), dB + tc::kmajor_step(kKTile, ks), id_n64,
                       ks > 0);
      }
      tc::mma_commit(bar_mma);
    }
  }

  float* AT = reinterpret_cast<float*>(base + kSmAT + grp * kATBytes);
  float* gates = reinterpret_cast<float*>(base + kSmGate + grp * kGateBytes);
  unsigned char* rec = mine.nvalid ? record(p, mine.slot, h) : nullptr;
  const bool l2norm = (p.flags & kFlagQkL2Norm) != 0;
  // ---- gates (threads 0-63 of the group, token t = gth); with the q/k L2 norm also the
  //      token's q norm (computed once per token and q/k head by qk_norm_kernel) ----
  if (mine.nvalid && gth < 64) {
    const float eA = tc::ex2_approx(p.A_log[h] * kLog2e), dt_bias = p.dt_bias[h];
    float lg = 0.f, bt = 0.f, lm = 0.f, m = 1.f;
    if (gth < mine.nvalid) {
      const int64_t tok = mine.z + gth;
      const float a = __bfloat162float(p.a[tok * p.a_st + h]);
      const float b = __bfloat162float(p.b[tok * p.b_st + h]);
      if (l2norm) {  // m_t = 1 / |q_t| and its log2
        const float2 mq = p.qnorm[tok * p.HQ + h / p.ratio];
        m = mq.x;
        lm = mq.y;
      }
      token_gates(eA, dt_bias, a, b, lg, bt);
    }
    float x = lg;  // inclusive scan over the 64 tokens: warp scans + carry
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    float* tmp = gates + PG_SCAN * 64;
    if (gth == 31) tmp[0] = x;
    named_sync(bar64, 64);
    if (gth >= 32) x += tmp[0];
    if (gth == 63) tmp[1] = x;
    named_sync(bar64, 64);
    const float x2 = x * kLog2e, gC2 = tmp[1] * kLog2e;
    gates[PG_G2 * 64 + gth] = x2;
    gates[PG_BETA * 64 + gth] = bt;
    gates[PG_G * 64 + gth] = tc::ex2_approx(x2);
    gates[PG_GC2 * 64 + gth] = gC2;
    gates[PG_LM * 64 + gth] = lm;
    gates[PG_M * 64 + gth] = m;
  }
  if (mine.nvalid) {
    named_sync(bar128, 128);
    // ---- A rows from TMEM (the two warps whose lane quarter holds this slot's rows) ----
    int ok = 1;
    if (gth == 0) ok = mbar_wait_sleep(bar_mma, 0) ? 1 : 0;
    {
      int all;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
          : "=r"(all)
          : "r"(ok), "r"(bar128)
          : "memory");
      ok = all;
    }
    if (ok) {
      const bool arow = ((warp & 3) >> 1) == grp;  // this warp's lane quarter holds slot rows
      const int t_row = ((warp & 1) << 5) | lane;
      const uint32_t d0 = tc::tmem_addr(tmem, (uint32_t)((warp & 3) * 32), (uint32_t)(grp * 64));
      tc::fence_after_sync();
      // k normalisation: n_t = 1 / |k_t| from the diagonal of K K^T (row t, column t)
      if (l2norm && arow) {
        float diag = 0.f;
        const int c0 = (warp & 1) * 4;  // the warp's rows are columns 8 c0 .. 8 c0 + 31
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          float v[8];
          tc::tmem_ld8(d0 + (c0 + g4) * 8, v);
          tc::tmem_wait_ld();
          if ((t_row >> 3) == c0 + g4) {
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if ((t_row & 7) == u) diag = v[u];
          }
        }
        gates[PG_N * 64 + t_row] = t_row < mine.nvalid ? l2_factor(diag) : 1.f;
        gates[PG_LN * 64 + t_row] = t_row < mine.nvalid ? -0.5f * tc::lg2_approx(diag + 1e-6f) : 0.f;
      }
      named_sync(bar128, 128);
      // ---- the chunk's gate arrays (record) and A's column term and row factor ----
      if (gth < 64) {
        const float n = l2norm ? gates[PG_N * 64 + gth] : 1.f;
        const float ln = l2norm ? gates[PG_LN * 64 + gth] : 0.f;  // log2 n_t
        const float x2 = gates[PG_G2 * 64 + gth], bt = gates[PG_BETA * 64 + gth], G = gates[PG_G * 64 + gth];
        const float gC2 = gates[PG_GC2 * 64 + gth], m = gates[PG_M * 64 + gth], lm = gates[PG_LM * 64 + gth];
        const float r = tc::ex2_approx(gC2 - x2);  // exp(g_C - g_t)
        const float vals[GA_N] = {x2 + lm, bt, G * m, bt * G * n, r * n, x2 - ln, tc::ex2_approx(gC2)};
        float* rg = reinterpret_cast<float*>(rec + kRecT);
#pragma unroll
        for (int a = 0; a < GA_N; ++a) rg[a * 64 + gth] = vals[a];
        gates[PG_G2C * 64 + gth] = x2 - ln;
        gates[PG_BN * 64 + gth] = bt * n;
      }
      named_sync(bar128, 128);
      if (arow) {
        const int t = t_row;
        // A[t][j] = beta_t n_t exp2(g2_t - (g2_j - log2 n_j)) (k_t.k_j) = beta_t exp(g_t - g_j) k^_t.k^_j
        const float* g2 = gates + PG_G2C * 64;
        const float gt = gates[PG_G2 * 64 + t], bt = gates[PG_BN * 64 + t];
#pragma unroll 2
        for (int j8 = 0; j8 < 8; ++j8) {
          float v[8];
          tc::tmem_ld8(d0 + j8 * 8, v);  // warp-wide: every lane takes part in the load
          const float4 g0 = *reinterpret_cast<const float4*>(g2 + j8 * 8);
          const float4 g1 = *reinterpret_cast<const float4*>(g2 + j8 * 8 + 4);
          tc::tmem_wait_ld();
          const float gj[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          float w[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (j8 * 8 < t) {  // columns j < t only
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = j8 * 8 + u < t ? bt * tc::ex2_approx(gt - gj[u]) * v[u] : 0.f;
          }
          *reinterpret_cast<float4*>(AT + t * kLd + j8 * 8) = make_float4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<float4*>(AT + t * kLd + j8 * 8 + 4) = make_float4(w[4], w[5], w[6], w[7]);
        }
      }
      tc::fence_before_sync();
      named_sync(bar128, 128);
      // ---- T = (I + A)^-1 in place ----
      if (gth < 64) solve_diag16(AT, gth, bar64);
      named_sync(bar128, 128);
      solve_merge16(AT, gth, bar128);
      solve_merge32(AT, gth, bar128);
      // ---- T hi / lo, compacted lower triangle (see gdn_prefill_chunk.cuh): 16-byte core-matrix
      //      rows in address order (coalesced) ----
#pragma unroll 1
      for (int q = gth; q < (int)kTriCM * 8; q += 128) {
        const int cm = q >> 3, i = q & 7;  // core matrix (row block rb, column block kc), row i
        int rb = 0;
#pragma unroll
        for (int b = 1; b < 8; ++b) rb += (int)tri_prefix(b) <= cm ? 1 : 0;
        const int kc = cm - (int)tri_prefix(rb), r = rb * 8 + i;
        const float4 x0 = *reinterpret_cast<const float4*>(AT + r * kLd + kc * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(AT + r * kLd + kc * 8 + 4);
        float t8[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        if (kc == rb) {  // the diagonal block: zero what lies above the diagonal
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e > i) t8[e] = 0.f;
        }
        uint4 hi, lo;
        split2(t8[0], t8[1], hi.x, lo.x);
        split2(t8[2], t8[3], hi.y, lo.y);
        split2(t8[4], t8[5], hi.z, lo.z);
        split2(t8[6], t8[7], hi.w, lo.w);
        *reinterpret_cast<uint4*>(rec + q * 16) = hi;
        *reinterpret_cast<uint4*>(rec + kRecTile + q * 16) = lo;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 128);
  }
}

// 1 / |q| and its log2 for every (token, q/k head): a streaming pass over q, 16 lanes per
// 256-byte row (coalesced 16-byte loads), 8 rows per warp per iteration.
__global__ void __launch_bounds__(256) qk_norm_kernel(PrefillParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = p.T * (int64_t)p.HQ;
  const int64_t nwarps = (int64_t)gridDim.x * 8;
  for (int64_t r0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * 8; r0 < rows; r0 += nwarps * 8) {
    float ss[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t row = r0 + 2 * i + (lane >> 4);
      ss[i] = 0.f;
      if (row < rows) {
        const int64_t tok = row / p.HQ;
        const int hq = (int)(row - tok * p.HQ);
        const uint4 w = *reinterpret_cast<const uint4*>(p.q + tok * p.q_st + (int64_t)hq * p.q_sh + (lane & 15) * 8);
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = __uint_as_float(u[e] << 16), hi = __uint_as_float(u[e] & 0xffff0000u);
          ss[i] = fmaf(lo, lo, fmaf(hi, hi, ss[i]));
        }
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < 4; ++i) ss[i] += __shfl_xor_sync(0xffffffffu, ss[i], o);
    if ((lane & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t row = r0 + 2 * i + (lane >> 4);
        if (row < rows) p.qnorm[row] = make_float2(l2_factor(ss[i]), -0.5f * tc::lg2_approx(ss[i] + 1e-6f));
      }
    }
  }
}

}  // namespace

cudaError_t launch_qk_norm(const PrefillParams& p, cudaStream_t stream) {
  const int64_t rows = p.T * (int64_t)p.HQ;
  if (rows <= 0) return cudaSuccess;
  const int64_t blocks = (rows + 63) / 64;
  qk_norm_kernel<<<(unsigned)(blocks < 148 * 8 ? blocks : 148 * 8), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill_prep(const PrefillParams& p, const CUtensorMap& mapK, cudaStream_t stream) {
  const int64_t slots = num_slots(p.T, p.N);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmAlloc);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const dim3 grid((unsigned)((slots + 1) / 2), (unsigned)p.HV);
  prefill_prep_kernel<<<grid, kThreads, kSmAlloc, stream>>>(mapK, p);
  return cudaGetLastError();
}

}  // namespace gdn
