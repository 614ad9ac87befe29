// Chunked (C = 64) varlen GDN prefill on tcgen05 tensor cores (sm_100a).
//
// Reference semantics: solution/triton/kernel_prefill.py:42-142 (token-serial
// decode recurrence per (sequence, v-head); an empty sequence passes its
// initial state through).  This kernel computes the same recurrence in the
// chunked WY/UT form.  For a chunk of C tokens with initial k-last state S0
// [V x K] (row v = one value index), in-chunk log-decay prefix
// g_t = sum_{i<=t} log g_i, G_t = exp(g_t), gates beta_t:
//   A[t][j] = beta_t exp(g_t - g_j) k_t.k_j  (j < t),   T = (I + A)^-1
//   R^T[v][t] = beta_t V[t][v] - beta_t G_t (S0 K^T)[v][t]
//   D^T = R^T T^T                                   (per-token deltas, [V x C])
//   O^T = scale (S0 Qg^T + D^T P^T),  Qg[t] = G_t q_t,  P[t][j] = exp(g_t - g_j) q_t.k_j (j <= t)
//   S_next = G_C S0 + Dt^T K,   Dt[j] = exp(g_C - g_j) D[j]
// Every product runs on tcgen05 with M = 128 = the state's V dimension on the
// TMEM lanes, bf16 operands and fp32 accumulation.  The operands whose rounding
// reaches the state at the scale of the deltas are split into bf16 hi + lo
// parts: S0 in S0 K^T (V - G S0 K^T cancels once the state has learned the
// values), R and T in D^T (3 products) and Dt in the state update (2 products).
// The state stays fp32 in TMEM for the whole sequence.
//
// CTA = one (sequence, v-head) chain, 14 warps:
//   warps 0-7   chain: thread (warp & 3, lane) owns state row v, warp >> 2
//               selects a column half; S0 hi/lo tiles and G_C scaling, R,
//               deltas, outputs, initial/final state I/O
//   warps 8-11  prep (one chunk ahead): gates, A and P from K K^T / Q K^T,
//               Q scaled by G in place, blocked fp32 inverse T, T hi/lo and P tiles
//   warp 12     TMA producer (K, Q: 128B-swizzled tiles, double-buffered; V plain)
//   warp 13     TMEM allocator and MMA issuer
// Hand-offs are mbarriers; every wait is bounded (kWaitLimitNs): a timeout
// raises GDN_DEVERR_WAIT_TIMEOUT and an in-CTA abort flag so every role leaves
// its loop, then in-flight copies and MMAs are drained before TMEM is freed.
#include <cuda.h>

#include "gdn_common.cuh"
#include "gdn_kernels.h"
#include "gdn_tc.cuh"

namespace gdn {
namespace {

constexpr int kC = 64;          // chunk length (tokens)
constexpr int kThreads = 448;   // 14 warps
constexpr int kChainThreads = 256;
constexpr int kWarpTma = 12, kWarpMma = 13;
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

// TMEM column map (fp32 accumulators; lanes = state row v unless noted)
constexpr uint32_t kTmS = 0;     // [0,128)    state S[v][k]
constexpr uint32_t kTmD1 = 128;  // [128,192)  S0 K^T
constexpr uint32_t kTmD0 = 192;  // [192,256), [256,320): K K^T / Q K^T (lanes = token), stage s
constexpr uint32_t kTmD2 = 320;  // [320,384)  D^T
constexpr uint32_t kTmD3 = 384;  // [384,448)  O^T (unscaled)

// Shared-memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kSmKQ = 0;          // 2 stages x 32 KB: [tile d0-63 | tile d64-127], rows 0-63 K, 64-127 Q
constexpr uint32_t kKQStage = 32768;
constexpr uint32_t kKQTile = 16384;    // one 64-column SW128 tile of 128 rows
constexpr uint32_t kSmV = 65536;       // V, plain row-major [64][128] bf16 (16 KB)
constexpr uint32_t kSmS0 = 81920;      // S0 hi: 2 tiles [128 x 64]
constexpr uint32_t kSmRD = 114688;     // S0 lo (2 tiles), then R^T hi|lo, then Dt^T hi|lo
constexpr uint32_t kSmDt = 147456;     // D^T bf16 tile [128 x 64]
constexpr uint32_t kSmT = 163840;      // T hi | lo: 2 tiles [64 x 64]
constexpr uint32_t kSmP = 180224;      // P tile [64 x 64]
constexpr int kLd = 68;                // padded row stride (floats) of the solve matrices
constexpr uint32_t kSmAs = 188416;     // A row-major [64][68] fp32
constexpr uint32_t kSmTs = 205824;     // T row-major [64][68] fp32
constexpr uint32_t kSmGate = 223232;   // 2 stages x 6 arrays x 64 fp32
constexpr uint32_t kSmBar = 226304;    // mbarriers (32 x 8 B)
constexpr uint32_t kSmMisc = 226560;   // tmem base slot, abort flag
constexpr uint32_t kSmX = 226624;      // solve block products [3][16][16] fp32
constexpr uint32_t kSmBytes = 229696;
constexpr uint32_t kSmAlloc = kSmBytes + 1024;  // + alignment slack
static_assert(kSmAs + 64 * kLd * 4 <= kSmTs && kSmTs + 64 * kLd * 4 <= kSmGate, "smem map");
static_assert(kSmX + 3 * 256 * 4 <= kSmBytes, "smem map");
static_assert(kSmAlloc <= 232448, "smem budget");

// gate arrays (per stage): log2-scaled prefix, beta, G, beta*G, exp(g_C - g), scratch
enum : int { GA_G2 = 0, GA_BETA = 1, GA_G = 2, GA_BG = 3, GA_R = 4, GA_TMP = 5, GA_N = 6 };

enum : int {
  B_KQ_FULL = 0,   // [2]
  B_KQ_EMPTY = 2,  // [2]
  B_KKQK = 4,      // [2]
  B_GATES = 6,     // [2]
  B_V_FULL = 8,
  B_V_EMPTY,
  B_S0_READY,
  B_MMA1,
  B_R_READY,
  B_MMA2,
  B_D_READY,
  B_MMA3,
  B_MMA4,
  B_OUT_DONE,
  B_PREP_DONE,
  B_DRAIN,
  B_COUNT
};
static_assert(B_COUNT <= 32, "barrier block");

struct Smem {
  unsigned char* base;
  __device__ uint64_t* bar(int i) const { return reinterpret_cast<uint64_t*>(base + kSmBar) + i; }
  __device__ float* gate(int s, int a) const { return reinterpret_cast<float*>(base + kSmGate) + (s * GA_N + a) * 64; }
  __device__ volatile int* abort_flag() const { return reinterpret_cast<volatile int*>(base + kSmMisc + 16); }
  __device__ uint32_t* tmem_slot() const { return reinterpret_cast<uint32_t*>(base + kSmMisc); }
  __device__ float* As() const { return reinterpret_cast<float*>(base + kSmAs); }
  __device__ float* Ts() const { return reinterpret_cast<float*>(base + kSmTs); }
  __device__ float* Xs() const { return reinterpret_cast<float*>(base + kSmX); }
  __device__ uint32_t addr(uint32_t off) const { return smem_u32(base + off); }
};

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

// Bounded wait that also gives up as soon as another role has aborted.
__device__ __forceinline__ bool wait_bar(const Smem& sm, uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
#pragma unroll 1
  for (int i = 0; i < 1024; ++i)
    if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (*sm.abort_flag()) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(kDevErrWaitTimeout);
      *sm.abort_flag() = 1;
      return false;
    }
  }
}

// Wait of a group of `n` threads: the leader polls the mbarrier, then the group
// meets at named barrier `bar_id` and AND-reduces the outcome, so all threads
// either proceed or leave together.
__device__ __forceinline__ bool group_wait(const Smem& sm, int bar_idx, uint32_t parity, int bar_id, int n,
                                           bool leader) {
  int ok = 1;
  if (leader) ok = wait_bar(sm, sm.bar(bar_idx), parity) ? 1 : 0;
  int all;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(all)
      : "r"(ok), "r"(bar_id), "r"(n)
      : "memory");
  return all != 0;
}

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int i) {
  return p.cu_is_int64 ? reinterpret_cast<const int64_t*>(p.cu_seqlens)[i]
                       : (int64_t) reinterpret_cast<const int32_t*>(p.cu_seqlens)[i];
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// (a, b) -> bf16x2 hi and bf16x2 lo with a = hi + lo to ~16 mantissa bits.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  lo = pack_bf16x2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xffff0000u));
}

// 16-byte store of 8 bf16 (columns 8*c8 .. 8*c8+7 of `row`) into a SW128 tile.
__device__ __forceinline__ void st_tile(unsigned char* tile, int row, int c8, uint4 w) {
  *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, c8 * 8)) = w;
}

__device__ __forceinline__ void fma4(float4& acc, float a, const float4& t) {
  acc.x = fmaf(a, t.x, acc.x);
  acc.y = fmaf(a, t.y, acc.y);
  acc.z = fmaf(a, t.z, acc.z);
  acc.w = fmaf(a, t.w, acc.w);
}

// ---------------------------------------------------------------------------
// Inverse of the unit lower-triangular 64x64 matrix I + A in fp32 by the prep
// warpgroup (128 threads).  As = A row-major (stride kLd, zero on and above the
// diagonal); the inverse is written to Ts (row-major, stride kLd; entries above
// the diagonal blocks are left unwritten).
//   1. diagonal 16x16 blocks, one column per thread (x_r = d_rc - sum_{q<r} A_rq x_q)
//   2. T_ij = -T_ii X_ij, X_ij = sum_{k=j}^{i-1} A_ik T_kj, by block distance 1, 2, 3;
//      each thread computes 1 x 4 output strips from float4 shared-memory loads.
__device__ void solve_unit_lower(const float* As, float* Ts, float* Xs, int p) {
  if (p < 64) {
    const int o = (p >> 4) * 16, c = p & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float* arow = As + (o + r) * kLd + o;
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
#pragma unroll
    for (int r = 0; r < 16; ++r) Ts[(o + r) * kLd + o + c] = x[r];
  }
  named_sync(2, 128);
#pragma unroll 1
  for (int d = 1; d <= 3; ++d) {
    const int items = (4 - d) * 64;  // (block, row r, column quad cq)
#pragma unroll 1
    for (int it = p; it < items; it += 128) {
      const int blk = it >> 6, r = (it >> 2) & 15, cq = it & 3;
      const int j = blk, i = blk + d;
      const float* arow = As + (16 * i + r) * kLd;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int kk = 16 * j; kk < 16 * i; kk += 4) {
        const float4 a = *reinterpret_cast<const float4*>(arow + kk);
        fma4(acc, a.x, *reinterpret_cast<const float4*>(Ts + (kk + 0) * kLd + 16 * j + 4 * cq));
        fma4(acc, a.y, *reinterpret_cast<const float4*>(Ts + (kk + 1) * kLd + 16 * j + 4 * cq));
        fma4(acc, a.z, *reinterpret_cast<const float4*>(Ts + (kk + 2) * kLd + 16 * j + 4 * cq));
        fma4(acc, a.w, *reinterpret_cast<const float4*>(Ts + (kk + 3) * kLd + 16 * j + 4 * cq));
      }
      *reinterpret_cast<float4*>(Xs + blk * 256 + r * 16 + 4 * cq) = acc;
    }
    named_sync(2, 128);
#pragma unroll 1
    for (int it = p; it < items; it += 128) {
      const int blk = it >> 6, r = (it >> 2) & 15, cq = it & 3;
      const int j = blk, i = blk + d;
      const float* trow = Ts + (16 * i + r) * kLd + 16 * i;
      const float* xb = Xs + blk * 256 + 4 * cq;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int q4 = 0; q4 < 16; q4 += 4) {
        const float4 a = *reinterpret_cast<const float4*>(trow + q4);
        fma4(acc, a.x, *reinterpret_cast<const float4*>(xb + (q4 + 0) * 16));
        fma4(acc, a.y, *reinterpret_cast<const float4*>(xb + (q4 + 1) * 16));
        fma4(acc, a.z, *reinterpret_cast<const float4*>(xb + (q4 + 2) * 16));
        fma4(acc, a.w, *reinterpret_cast<const float4*>(xb + (q4 + 3) * 16));
      }
      *reinterpret_cast<float4*>(Ts + (16 * i + r) * kLd + 16 * j + 4 * cq) =
          make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
    }
    named_sync(2, 128);
  }
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    prefill_chunk_kernel(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapQ,
                         const __grid_constant__ CUtensorMap mapV, PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem sm;
  sm.base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int h = blockIdx.x, n = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qh = h / p.ratio;

  const int64_t t0 = load_cu(p, n), t1 = load_cu(p, n + 1);
  const bool bad = t1 < t0 || t0 < 0 || t1 > p.T;
  const int64_t len = bad ? 0 : t1 - t0;
  const int nchunks = (int)((len + kC - 1) / kC);
  if (bad && tid == 0) raise_device_error(kDevErrBadSeqlens);

  if (tid == 0) {
    for (int i = 0; i < B_COUNT; ++i) mbar_init(sm.bar(i), 1);
    *sm.abort_flag() = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tc::tmem_alloc(sm.tmem_slot(), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *sm.tmem_slot();

  // ======================================================================= TMA producer
  if (warp == kWarpTma) {
    if (lane == 0 && nchunks > 0) {
      tc::prefetch_tensormap(&mapK);
      tc::prefetch_tensormap(&mapQ);
      tc::prefetch_tensormap(&mapV);
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i & 1;
        const int z = (int)(t0 + (int64_t)i * kC);
        if (i >= 2 && !wait_bar(sm, sm.bar(B_KQ_EMPTY + s), ((i - 2) >> 1) & 1)) break;
        uint64_t* full = sm.bar(B_KQ_FULL + s);
        mbar_arrive_expect_tx(full, 4 * 8192);
        unsigned char* kq = sm.base + kSmKQ + s * kKQStage;
        tc::tma_load_3d(kq, &mapK, 0, qh, z, full);
        tc::tma_load_3d(kq + kKQTile, &mapK, 64, qh, z, full);
        tc::tma_load_3d(kq + 8192, &mapQ, 0, qh, z, full);
        tc::tma_load_3d(kq + kKQTile + 8192, &mapQ, 64, qh, z, full);
        if (i >= 1 && !wait_bar(sm, sm.bar(B_V_EMPTY), (i - 1) & 1)) break;
        mbar_arrive_expect_tx(sm.bar(B_V_FULL), 16384);
        tc::tma_load_3d(sm.base + kSmV, &mapV, 0, h, z, sm.bar(B_V_FULL));
        issued = i + 1;
      }
      // drain: the last loads have landed before the CTA can exit (bounded)
      if (issued > 0) {
        const int i = issued - 1;
        wait_bar(sm, sm.bar(B_KQ_FULL + (i & 1)), (i >> 1) & 1);
        wait_bar(sm, sm.bar(B_V_FULL), i & 1);
      }
    }
  }
  // ======================================================================= MMA issuer
  else if (warp == kWarpMma) {
    if (lane == 0 && nchunks > 0) {
      const uint32_t id_n64 = tc::idesc_bf16(128, 64, false, false);
      const uint32_t id_st = tc::idesc_bf16(128, 128, false, true);  // Dt^T x K (K MN-major)
      const uint32_t aS0 = sm.addr(kSmS0), aRD = sm.addr(kSmRD), aDt = sm.addr(kSmDt);
      const uint32_t aT = sm.addr(kSmT), aP = sm.addr(kSmP);
      auto issue_kkqk = [&](int i) -> bool {
        const int s = i & 1;
        if (!wait_bar(sm, sm.bar(B_KQ_FULL + s), (i >> 1) & 1)) return false;
        tc::fence_after_sync();
        const uint32_t kq = sm.addr(kSmKQ + s * kKQStage);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD0 + s * 64, tc::kmajor_desc(kq, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks),
                       id_n64, ks > 0);
        tc::mma_commit(sm.bar(B_KKQK + s));
        return true;
      };
      bool ok = issue_kkqk(0);
      for (int i = 0; ok && i < nchunks; ++i) {
        const int s = i & 1;
        const uint32_t kq = sm.addr(kSmKQ + s * kKQStage);
        // MMA1: D1 = S0_hi K^T + S0_lo K^T
        if (!wait_bar(sm, sm.bar(B_S0_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD1, tc::kmajor_desc(aS0, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks), id_n64,
                       ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD1, tc::kmajor_desc(aRD, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks), id_n64,
                       true);
        tc::mma_commit(sm.bar(B_MMA1));
        // next chunk's K K^T / Q K^T
        if (i + 1 < nchunks && !issue_kkqk(i + 1)) break;
        // MMA2: D^T = R^T T^T (R and T split hi/lo: 3 products)
        if (!wait_bar(sm, sm.bar(B_R_READY), i & 1)) break;
        if (!wait_bar(sm, sm.bar(B_PREP_DONE), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD, 0, ks), tc::kmajor_desc(aT, 0, ks), id_n64, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD + 16384, 0, ks), tc::kmajor_desc(aT, 0, ks), id_n64, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD, 0, ks), tc::kmajor_desc(aT + 8192, 0, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA2));
        // O^T = S0_hi Qg^T + D^T P^T;   S += Dt^T K (hi/lo)
        if (!wait_bar(sm, sm.bar(B_D_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD3, tc::kmajor_desc(aS0, kKQTile, ks), tc::kmajor_desc(kq + 8192, kKQTile, ks),
                       id_n64, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD3, tc::kmajor_desc(aDt, 0, ks), tc::kmajor_desc(aP, 0, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA3));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmS, tc::kmajor_desc(aRD, 0, ks), tc::mnmajor_desc(kq, kKQTile, ks), id_st, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmS, tc::kmajor_desc(aRD + 16384, 0, ks), tc::mnmajor_desc(kq, kKQTile, ks), id_st,
                       true);
        tc::mma_commit(sm.bar(B_MMA4));
        tc::mma_commit(sm.bar(B_KQ_EMPTY + s));
      }
      // drain: every MMA issued above has completed before TMEM is released
      tc::mma_commit(sm.bar(B_DRAIN));
      wait_bar(sm, sm.bar(B_DRAIN), 0);
    }
  }
  // ======================================================================= prep warpgroup
  else if (warp >= 8) {
    const int pth = tid - 256;  // 0..127; TMEM lane quarter = warp & 3
    const int row = pth & 63;
    float* As = sm.As();
    float* Ts = sm.Ts();
    const float A_log = p.A_log[h], dt_bias = p.dt_bias[h];
    // gate inputs, loaded one chunk ahead
    float a_nx = 0.f, b_nx = 0.f;
    auto load_ab = [&](int i) {
      if (pth < 64 && (int64_t)i * kC + pth < len) {
        const int64_t tok = t0 + (int64_t)i * kC + pth;
        a_nx = bf16_to_f32(p.a + tok * p.a_st + h);
        b_nx = bf16_to_f32(p.b + tok * p.b_st + h);
      }
    };
    if (nchunks > 0) load_ab(0);
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      // ---- gates of chunk i into stage s (free once the chain finished chunk i-2) ----
      const float a_cur = a_nx, b_cur = b_nx;
      if (i + 1 < nchunks) load_ab(i + 1);
      if (i >= 2 && !group_wait(sm, B_OUT_DONE, (i - 2) & 1, 2, 128, pth == 0)) break;
      if (pth < 64) {
        const bool valid = (int64_t)i * kC + pth < len;
        float lg = 0.f, bt = 0.f;
        if (valid) {
          lg = gdn_log_decay(A_log, a_cur, dt_bias);
          bt = 1.0f / (1.0f + expf(-b_cur));
        }
        float x = lg;  // inclusive scan over the 64 tokens: warp scans + carry
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += y;
        }
        float* tmp = sm.gate(s, GA_TMP);
        if (pth == 31) tmp[0] = x;
        named_sync(3, 64);
        if (pth >= 32) x += tmp[0];
        if (pth == 63) tmp[1] = x;
        named_sync(3, 64);
        const float gC = tmp[1];
        const float G = expf(x);
        sm.gate(s, GA_G2)[pth] = x * kLog2e;
        sm.gate(s, GA_BETA)[pth] = bt;
        sm.gate(s, GA_G)[pth] = G;
        sm.gate(s, GA_BG)[pth] = bt * G;
        sm.gate(s, GA_R)[pth] = expf(gC - x);
      }
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_GATES + s));
      // ---- A (row-major fp32) and P (registers) from K K^T / Q K^T ----
      if (!group_wait(sm, B_KKQK + s, (i >> 1) & 1, 2, 128, pth == 0)) break;
      tc::fence_after_sync();
      const float* g2 = sm.gate(s, GA_G2);
      uint32_t prow[32];
      {
        float v[32];
        const float gt = g2[row];
        const float bt = sm.gate(s, GA_BETA)[row];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tc::tmem_ld32(tc::tmem_addr(tmem, (uint32_t)((warp & 3) * 32), kTmD0 + s * 64 + half * 32), v);
          tc::tmem_wait_ld();
          if (pth < 64) {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              const int j = half * 32 + q;
              const float4 gj = *reinterpret_cast<const float4*>(g2 + j);
              float4 w;
              w.x = j < row ? bt * tc::ex2_approx(gt - gj.x) * v[q] : 0.f;
              w.y = j + 1 < row ? bt * tc::ex2_approx(gt - gj.y) * v[q + 1] : 0.f;
              w.z = j + 2 < row ? bt * tc::ex2_approx(gt - gj.z) * v[q + 2] : 0.f;
              w.w = j + 3 < row ? bt * tc::ex2_approx(gt - gj.w) * v[q + 3] : 0.f;
              *reinterpret_cast<float4*>(As + row * kLd + j) = w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 32; q += 4) {
              const int j = half * 32 + q;
              const float4 gj = *reinterpret_cast<const float4*>(g2 + j);
              const float p0 = j <= row ? tc::ex2_approx(gt - gj.x) * v[q] : 0.f;
              const float p1 = j + 1 <= row ? tc::ex2_approx(gt - gj.y) * v[q + 1] : 0.f;
              const float p2 = j + 2 <= row ? tc::ex2_approx(gt - gj.z) * v[q + 2] : 0.f;
              const float p3 = j + 3 <= row ? tc::ex2_approx(gt - gj.w) * v[q + 3] : 0.f;
              prow[(half * 32 + q) >> 1] = pack_bf16x2(p0, p1);
              prow[((half * 32 + q) >> 1) + 1] = pack_bf16x2(p2, p3);
            }
          }
        }
      }
      tc::fence_before_sync();
      // ---- Q rows of the K/Q stage scaled by G in place (Qg for the output MMA) ----
      {
        const float Gt = sm.gate(s, GA_G)[row];
        unsigned char* qtile = sm.base + kSmKQ + s * kKQStage + (pth >> 6) * kKQTile;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const uint32_t off = tc::sw128_offset(64 + row, c8 * 8);
          uint4 w = *reinterpret_cast<const uint4*>(qtile + off);
          w.x = pack_bf16x2(__uint_as_float(w.x << 16) * Gt, __uint_as_float(w.x & 0xffff0000u) * Gt);
          w.y = pack_bf16x2(__uint_as_float(w.y << 16) * Gt, __uint_as_float(w.y & 0xffff0000u) * Gt);
          w.z = pack_bf16x2(__uint_as_float(w.z << 16) * Gt, __uint_as_float(w.z & 0xffff0000u) * Gt);
          w.w = pack_bf16x2(__uint_as_float(w.w << 16) * Gt, __uint_as_float(w.w & 0xffff0000u) * Gt);
          *reinterpret_cast<uint4*>(qtile + off) = w;
        }
      }
      named_sync(2, 128);
      // ---- T = (I + A)^-1 ----
      solve_unit_lower(As, Ts, sm.Xs(), pth);
      // ---- T hi/lo tiles (after MMA2 of chunk i-1), P tile (after MMA3 of chunk i-1) ----
      if (i >= 1 && !group_wait(sm, B_MMA2, (i - 1) & 1, 2, 128, pth == 0)) break;
      if (pth < 64) {
        unsigned char* thi = sm.base + kSmT;
        unsigned char* tlo = sm.base + kSmT + 8192;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const float4 x0 = *reinterpret_cast<const float4*>(Ts + pth * kLd + c8 * 8);
          const float4 x1 = *reinterpret_cast<const float4*>(Ts + pth * kLd + c8 * 8 + 4);
          float t8[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (c8 * 8 + e > pth) t8[e] = 0.f;  // above the diagonal (not written by the solve)
          uint4 hi, lo;
          split2(t8[0], t8[1], hi.x, lo.x);
          split2(t8[2], t8[3], hi.y, lo.y);
          split2(t8[4], t8[5], hi.z, lo.z);
          split2(t8[6], t8[7], hi.w, lo.w);
          st_tile(thi, pth, c8, hi);
          st_tile(tlo, pth, c8, lo);
        }
      }
      if (i >= 1 && !group_wait(sm, B_MMA3, (i - 1) & 1, 2, 128, pth == 0)) break;
      if (pth >= 64) {
        unsigned char* pt = sm.base + kSmP;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8)
          st_tile(pt, row, c8, make_uint4(prow[c8 * 4], prow[c8 * 4 + 1], prow[c8 * 4 + 2], prow[c8 * 4 + 3]));
      }
      tc::fence_proxy_async_smem();
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_PREP_DONE));
    }
  }
  // ======================================================================= chain warps
  else {
    const int quarter = warp & 3, hsel = warp >> 2;
    const int v = quarter * 32 + lane;  // state row / TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32);
    const bool leader = tid == 0;
    // initial state (this thread's 64-column half) -> TMEM S
    {
      const float* src =
          p.state ? p.state + (size_t)n * p.s_sn + (size_t)h * p.s_sh + (size_t)v * kHeadDim + hsel * 64 : nullptr;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) {
        float x[16];
#pragma unroll
        for (int q = 0; q < 16; q += 4) {
          const float4 f = src ? ld_nc_f4(src + c0 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[q] = f.x;
          x[q + 1] = f.y;
          x[q + 2] = f.z;
          x[q + 3] = f.w;
        }
        tc::tmem_st16(tc::tmem_addr(tmem, lane_base, kTmS + hsel * 64 + c0), x);
      }
      tc::tmem_wait_st();
    }
    const float scale = p.scale;
    unsigned char* s0t = sm.base + kSmS0 + hsel * kKQTile;  // this half's S0 hi tile
    unsigned char* s0l = sm.base + kSmRD + hsel * kKQTile;  // this half's S0 lo tile
    unsigned char* rd = sm.base + kSmRD;
    unsigned char* dtt = sm.base + kSmDt;
    const __nv_bfloat16* vt = reinterpret_cast<const __nv_bfloat16*>(sm.base + kSmV);
    const int tb = hsel * 32;  // this thread's token columns [tb, tb + 32)
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      const int64_t rem = len - (int64_t)i * kC;
      const int nvalid = rem < kC ? (int)rem : kC;
      if (!group_wait(sm, B_GATES + s, (i >> 1) & 1, 1, kChainThreads, leader)) break;
      const float GC = sm.gate(s, GA_G)[63];
      // ---- S0 hi/lo tiles and S <- G_C * S (64 columns per thread) ----
      if (i > 0 && !group_wait(sm, B_MMA4, (i - 1) & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32) {
        float x[32];
        const uint32_t ta = tc::tmem_addr(tmem, lane_base, kTmS + hsel * 64 + c32 * 32);
        tc::tmem_ld32(ta, x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          uint4 hi, lo;
          split2(x[c8 * 8 + 0], x[c8 * 8 + 1], hi.x, lo.x);
          split2(x[c8 * 8 + 2], x[c8 * 8 + 3], hi.y, lo.y);
          split2(x[c8 * 8 + 4], x[c8 * 8 + 5], hi.z, lo.z);
          split2(x[c8 * 8 + 6], x[c8 * 8 + 7], hi.w, lo.w);
          st_tile(s0t, v, c32 * 4 + c8, hi);
          st_tile(s0l, v, c32 * 4 + c8, lo);
        }
        float x0[16], x1[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          x0[q] = x[q] * GC;
          x1[q] = x[16 + q] * GC;
        }
        tc::tmem_st16(ta, x0);
        tc::tmem_st16(ta + 16, x1);
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_S0_READY));
      // ---- R^T = beta V^T - beta G (S0 K^T), split hi/lo (32 token columns per thread) ----
      if (!group_wait(sm, B_MMA1, i & 1, 1, kChainThreads, leader)) break;
      if (!group_wait(sm, B_V_FULL, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        float x[32];
        tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, kTmD1 + tb), x);
        tc::tmem_wait_ld();
        const float* bet = sm.gate(s, GA_BETA) + tb;
        const float* bg = sm.gate(s, GA_BG) + tb;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float r8[8];
#pragma unroll
          for (int q4 = 0; q4 < 8; q4 += 4) {
            const float4 b4 = *reinterpret_cast<const float4*>(bet + c8 * 8 + q4);
            const float4 g4 = *reinterpret_cast<const float4*>(bg + c8 * 8 + q4);
            const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int q = c8 * 8 + q4 + u;
              const float vv = __bfloat162float(vt[(tb + q) * kHeadDim + v]);
              r8[q4 + u] = fmaf(bb[u], vv, -gg[u] * x[q]);
            }
          }
          uint4 hi, lo;
          split2(r8[0], r8[1], hi.x, lo.x);
          split2(r8[2], r8[3], hi.y, lo.y);
          split2(r8[4], r8[5], hi.z, lo.z);
          split2(r8[6], r8[7], hi.w, lo.w);
          st_tile(rd, v, (tb >> 3) + c8, hi);
          st_tile(rd + 16384, v, (tb >> 3) + c8, lo);
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) {
        mbar_arrive(sm.bar(B_R_READY));
        mbar_arrive(sm.bar(B_V_EMPTY));
      }
      // ---- deltas: D^T (bf16, output MMA) and Dt^T = D^T exp(gC - g) (hi/lo, state MMA) ----
      if (!group_wait(sm, B_MMA2, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        float x[32];
        tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, kTmD2 + tb), x);
        tc::tmem_wait_ld();
        const float* rr = sm.gate(s, GA_R) + tb;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const float4 r0 = *reinterpret_cast<const float4*>(rr + c8 * 8);
          const float4 r1 = *reinterpret_cast<const float4*>(rr + c8 * 8 + 4);
          const float* d = x + c8 * 8;
          uint4 dd, hi, lo;
          dd.x = pack_bf16x2(d[0], d[1]);
          dd.y = pack_bf16x2(d[2], d[3]);
          dd.z = pack_bf16x2(d[4], d[5]);
          dd.w = pack_bf16x2(d[6], d[7]);
          split2(d[0] * r0.x, d[1] * r0.y, hi.x, lo.x);
          split2(d[2] * r0.z, d[3] * r0.w, hi.y, lo.y);
          split2(d[4] * r1.x, d[5] * r1.y, hi.z, lo.z);
          split2(d[6] * r1.z, d[7] * r1.w, hi.w, lo.w);
          st_tile(dtt, v, (tb >> 3) + c8, dd);
          st_tile(rd, v, (tb >> 3) + c8, hi);
          st_tile(rd + 16384, v, (tb >> 3) + c8, lo);
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_D_READY));
      // ---- outputs: o[t][v] = scale * O^T[v][t]; lane pairs exchange so each stores bf16x2 ----
      if (!group_wait(sm, B_MMA3, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        float x[32];
        tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, kTmD3 + tb), x);
        tc::tmem_wait_ld();
        const bool odd = lane & 1;
        const int vcol = v & ~1;
        __nv_bfloat16* out = p.out + (t0 + (int64_t)i * kC) * p.o_st + (int64_t)h * p.o_sh + vcol;
#pragma unroll
        for (int q = 0; q < 32; q += 2) {
          // even lane keeps token q (needs the odd neighbour's column), odd lane keeps token q + 1
          const float send = odd ? x[q] : x[q + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
          const float c0v = odd ? recv : x[q];      // column vcol
          const float c1v = odd ? x[q + 1] : recv;  // column vcol + 1
          const int t = tb + q + (odd ? 1 : 0);
          if (t < nvalid)
            *reinterpret_cast<uint32_t*>(out + (int64_t)t * p.o_st) = pack_bf16x2(scale * c0v, scale * c1v);
        }
      }
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_OUT_DONE));
    }
    // ---- final state ----
    bool ok = true;
    if (nchunks > 0) ok = group_wait(sm, B_MMA4, (nchunks - 1) & 1, 1, kChainThreads, leader) && !*sm.abort_flag();
    if (ok) {
      tc::fence_after_sync();
      float* dst = p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh + (size_t)v * kHeadDim + hsel * 64;
#pragma unroll
      for (int c32 = 0; c32 < 2; ++c32) {
        float x[32];
        tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, kTmS + hsel * 64 + c32 * 32), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<float4*>(dst + c32 * 32 + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
      }
    }
  }

  // ---- teardown: every role is out of its loop; MMAs and copies were drained ----
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kWarpMma) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D view [tokens][heads][128] of a bf16 activation with element strides
// (token, head); box = 64 tokens x 1 head x `box_x` features.
bool make_map(CUtensorMap* m, const void* base, int64_t tokens, int heads, int64_t st, int64_t sh, int box_x,
              bool swizzle) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)heads, (cuuint64_t)(tokens > 0 ? tokens : 1)};
  const cuuint64_t strides[2] = {(cuuint64_t)(sh * 2), (cuuint64_t)(st * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)box_x, 1u, (cuuint32_t)kC};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool prefill_chunk_supported(const PrefillParams& p) {
  auto ok16 = [](const void* ptr, int64_t a, int64_t b) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ((a * 2) & 15) == 0 && ((b * 2) & 15) == 0;
  };
  if (p.flags & kFlagQkL2Norm) return false;
  if (p.T <= 0) return false;
  // output rows are written as bf16 pairs
  if ((reinterpret_cast<uintptr_t>(p.out) & 3) || (p.o_st & 1) || (p.o_sh & 1)) return false;
  return ok16(p.q, p.q_st, p.q_sh) && ok16(p.k, p.k_st, p.k_sh) && ok16(p.v, p.v_st, p.v_sh);
}

cudaError_t launch_prefill_chunk(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  CUtensorMap mk, mq, mv;
  if (!make_map(&mk, p.k, p.T, p.HQ, p.k_st, p.k_sh, 64, true) ||
      !make_map(&mq, p.q, p.T, p.HQ, p.q_st, p.q_sh, 64, true) ||
      !make_map(&mv, p.v, p.T, p.HV, p.v_st, p.v_sh, 128, false))
    return cudaErrorInvalidValue;
  // The dynamic shared-memory opt-in is a per-device function attribute.
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmAlloc);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  prefill_chunk_kernel<<<dim3(p.HV, p.N), kThreads, kSmAlloc, stream>>>(mk, mq, mv, p);
  return cudaGetLastError();
}

}  // namespace gdn
