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
// Per chunk the state chain is S0 tiles -> [S0 [K;Qg]^T] -> R -> [R^T T^T] ->
// deltas -> [S += Dt^T K] -> next chunk; the output MMA (D^T P^T), the output
// stores and all prep work overlap it.  Hand-offs are mbarriers; every wait is
// bounded (kWaitLimitNs): a timeout raises GDN_DEVERR_WAIT_TIMEOUT and an
// in-CTA abort flag so every role leaves its loop, then in-flight copies and
// MMAs are drained before TMEM is freed.
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
constexpr float kLn2 = 0.6931471805599453f;

// TMEM column map (fp32 accumulators; lanes = state row v unless noted)
constexpr uint32_t kTmS = 0;     // [0,128)    state S[v][k]
constexpr uint32_t kTmD1 = 128;  // 2 buffers [128,256), [256,384): cols 0-63 S0 K^T, 64-127 O^T (unscaled)
constexpr uint32_t kTmD0 = 384;  // [384,448)  K K^T / Q K^T (lanes = token)
constexpr uint32_t kTmD2 = 448;  // [448,512)  D^T

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
constexpr uint32_t kSmX = 226624;      // solve: 32x32 block product X fp32 (4 KB)
constexpr uint32_t kSmBytes = 230720;
constexpr uint32_t kSmAlloc = kSmBytes + 1024;  // + alignment slack
static_assert(kSmAs + 64 * kLd * 4 <= kSmTs && kSmTs + 64 * kLd * 4 <= kSmGate, "smem map");
static_assert(kSmX + 32 * 32 * 4 <= kSmBytes, "smem map");
static_assert(kSmAlloc <= 232448, "smem budget");

// gate arrays (per stage): log2-scaled prefix, beta, G, beta*G, exp(g_C - g), scratch
enum : int { GA_G2 = 0, GA_BETA = 1, GA_G = 2, GA_BG = 3, GA_R = 4, GA_TMP = 5, GA_N = 6 };

enum : int {
  B_KQ_FULL = 0,   // [2]
  B_KQ_EMPTY = 2,  // [2]
  B_GATES = 4,     // [2]
  B_GFREE = 6,     // [2] the chain is done with a gate stage (per stage, so a wait can never alias)
  B_KKQK = 8,
  B_D0_FREE,
  B_QG_READY,
  B_V_FULL,
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
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    // suspended until the phase completes (or 0.1 ms), so waiting threads do not
    // take issue slots from the warps doing the work
    if (mbar_try_wait_sleep(addr, parity, 100000u)) return true;
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
// Inverse T of the unit lower-triangular 64x64 matrix I + A in fp32 (prep
// warpgroup).  As = A row-major (stride kLd, zero on and above the diagonal);
// T is written row-major to Ts (stride kLd; blocks above the diagonal blocks
// are left unwritten).
//   solve_diag16:  the four 16x16 diagonal blocks, one column per thread (64
//                  threads): x_r = d_rc - sum_{q<r} A_rq x_q
//   solve_merge:   for block pairs of size B (16, then 32): T_10 = -T_11 (A_10 T_00),
//                  two products over the 128 threads in 1x4 strips, skipping the
//                  zero triangles of T_00 and T_11; Xs holds A_10 T_00.
__device__ __forceinline__ void solve_diag16(const float* As, float* Ts, int p) {
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

// lgB = log2(B); pairs are (rows/cols) [2mB, 2mB+B) (block 0) and [2mB+B, 2mB+2B) (block 1).
__device__ __noinline__ void solve_merge(const float* As, float* Ts, float* Xs, int p, int lgB) {
  const int B = 1 << lgB, lgQ = lgB - 2, items = 8 * B;  // (64 / 2B pairs) x B rows x B/4 quads
  // X = A_10 T_00   (T_00[k][c] = 0 for k < c)
#pragma unroll 1
  for (int it = p; it < items; it += 128) {
    const int m = it >> (lgB + lgQ), r = (it >> lgQ) & (B - 1), cq = it & ((B >> 2) - 1);
    const int jo = 2 * m * B, io = jo + B;
    const float* arow = As + (io + r) * kLd + jo;
    const float* tcol = Ts + jo * kLd + jo + 4 * cq;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int kk = 4 * cq; kk < B; kk += 4) {
      const float4 a = *reinterpret_cast<const float4*>(arow + kk);
      fma4(acc, a.x, *reinterpret_cast<const float4*>(tcol + (kk + 0) * kLd));
      fma4(acc, a.y, *reinterpret_cast<const float4*>(tcol + (kk + 1) * kLd));
      fma4(acc, a.z, *reinterpret_cast<const float4*>(tcol + (kk + 2) * kLd));
      fma4(acc, a.w, *reinterpret_cast<const float4*>(tcol + (kk + 3) * kLd));
    }
    *reinterpret_cast<float4*>(Xs + ((m * B + r) << lgB) + 4 * cq) = acc;
  }
  named_sync(2, 128);
  // T_10 = -T_11 X   (T_11[r][q] = 0 for q > r)
#pragma unroll 1
  for (int it = p; it < items; it += 128) {
    const int m = it >> (lgB + lgQ), r = (it >> lgQ) & (B - 1), cq = it & ((B >> 2) - 1);
    const int jo = 2 * m * B, io = jo + B;
    const float* trow = Ts + (io + r) * kLd + io;
    const float* xb = Xs + ((m * B) << lgB) + 4 * cq;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int q4 = 0; q4 <= r; q4 += 4) {
      const float4 a = *reinterpret_cast<const float4*>(trow + q4);
      fma4(acc, a.x, *reinterpret_cast<const float4*>(xb + ((q4 + 0) << lgB)));
      fma4(acc, a.y, *reinterpret_cast<const float4*>(xb + ((q4 + 1) << lgB)));
      fma4(acc, a.z, *reinterpret_cast<const float4*>(xb + ((q4 + 2) << lgB)));
      fma4(acc, a.w, *reinterpret_cast<const float4*>(xb + ((q4 + 3) << lgB)));
    }
    *reinterpret_cast<float4*>(Ts + (io + r) * kLd + jo + 4 * cq) = make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
  }
  named_sync(2, 128);
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
      using tc::kmajor_step;
      using tc::mnmajor_step;
      const uint32_t id_n64 = tc::idesc_bf16(128, 64, false, false);
      const uint32_t id_n128 = tc::idesc_bf16(128, 128, false, false);
      const uint32_t id_st = tc::idesc_bf16(128, 128, false, true);  // Dt^T x K (K MN-major)
      // descriptor bases (start address of each operand buffer); per MMA step only a
      // constant is added (tc::kmajor_step / tc::mnmajor_step)
      const uint64_t dS0 = tc::kmajor_desc(sm.addr(kSmS0), 0, 0);
      const uint64_t dRD = tc::kmajor_desc(sm.addr(kSmRD), 0, 0);
      const uint64_t dRDlo = tc::kmajor_desc(sm.addr(kSmRD + 16384), 0, 0);
      const uint64_t dDt = tc::kmajor_desc(sm.addr(kSmDt), 0, 0);
      const uint64_t dT = tc::kmajor_desc(sm.addr(kSmT), 0, 0);
      const uint64_t dTlo = tc::kmajor_desc(sm.addr(kSmT + 8192), 0, 0);
      const uint64_t dP = tc::kmajor_desc(sm.addr(kSmP), 0, 0);
      const uint64_t dKQ0 = tc::kmajor_desc(sm.addr(kSmKQ), 0, 0);
      const uint64_t dKQ1 = tc::kmajor_desc(sm.addr(kSmKQ + kKQStage), 0, 0);
      const uint64_t dKmn0 = tc::mnmajor_desc(sm.addr(kSmKQ), kKQTile, 0);
      const uint64_t dKmn1 = tc::mnmajor_desc(sm.addr(kSmKQ + kKQStage), kKQTile, 0);
      auto issue_kkqk = [&](int i) -> bool {
        const int s = i & 1;
        if (!wait_bar(sm, sm.bar(B_KQ_FULL + s), (i >> 1) & 1)) return false;
        if (i >= 1 && !wait_bar(sm, sm.bar(B_D0_FREE), (i - 1) & 1)) return false;
        tc::fence_after_sync();
        const uint64_t d = s ? dKQ1 : dKQ0;
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD0, d + kmajor_step(kKQTile, ks), d + kmajor_step(kKQTile, ks), id_n64, ks > 0);
        tc::mma_commit(sm.bar(B_KKQK));
        return true;
      };
      bool ok = issue_kkqk(0);
      for (int i = 0; ok && i < nchunks; ++i) {
        const int s = i & 1;
        const uint64_t dK = s ? dKQ1 : dKQ0;
        const uint64_t dKmn = s ? dKmn1 : dKmn0;
        const uint32_t d1 = tmem + kTmD1 + (uint32_t)s * 128;
        // MMA1: D1 = S0_hi [K; Qg]^T (N = 128), then D1[:, K part] += S0_lo K^T
        if (!wait_bar(sm, sm.bar(B_S0_READY), i & 1)) break;
        if (!wait_bar(sm, sm.bar(B_QG_READY), i & 1)) break;
        if (i >= 2 && !wait_bar(sm, sm.bar(B_OUT_DONE), i & 1)) break;  // outputs of chunk i-2 read D1[s]
        tc::fence_after_sync();
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(d1, dS0 + kmajor_step(kKQTile, ks), dK + kmajor_step(kKQTile, ks), id_n128, ks > 0);
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(d1, dRD + kmajor_step(kKQTile, ks), dK + kmajor_step(kKQTile, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA1));
        // next chunk's K K^T / Q K^T
        if (i + 1 < nchunks && !issue_kkqk(i + 1)) break;
        // MMA2: D^T = R^T T^T (R and T split hi/lo: 3 products)
        if (!wait_bar(sm, sm.bar(B_R_READY), i & 1)) break;
        if (!wait_bar(sm, sm.bar(B_PREP_DONE), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, dRD + kmajor_step(0, ks), dT + kmajor_step(0, ks), id_n64, ks > 0);
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, dRDlo + kmajor_step(0, ks), dT + kmajor_step(0, ks), id_n64, true);
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, dRD + kmajor_step(0, ks), dTlo + kmajor_step(0, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA2));
        // state first: S += Dt^T K (hi/lo); then the output: D1[:, O part] += D^T P^T
        if (!wait_bar(sm, sm.bar(B_D_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmS, dRD + kmajor_step(0, ks), dKmn + mnmajor_step(ks), id_st, true);
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmS, dRDlo + kmajor_step(0, ks), dKmn + mnmajor_step(ks), id_st, true);
        tc::mma_commit(sm.bar(B_MMA4));
        tc::mma_commit(sm.bar(B_KQ_EMPTY + s));
#pragma unroll 1
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(d1 + 64, dDt + kmajor_step(0, ks), dP + kmajor_step(0, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA3));
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
    const float eA = tc::ex2_approx(A_log * kLog2e);
    // gate inputs (raw bf16 bits), loaded one chunk ahead and converted at use so
    // the load latency is not paid where they are issued
    unsigned short a_nx = 0, b_nx = 0;
    auto load_ab = [&](int i) {
      if (pth < 64 && (int64_t)i * kC + pth < len) {
        const int64_t tok = t0 + (int64_t)i * kC + pth;
        a_nx = reinterpret_cast<const unsigned short*>(p.a)[tok * p.a_st + h];
        b_nx = reinterpret_cast<const unsigned short*>(p.b)[tok * p.b_st + h];
      }
    };
    if (nchunks > 0) load_ab(0);
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      // ---- gates of chunk i into stage s (free once the chain's deltas of chunk i-2 are done) ----
      const float a_cur = __uint_as_float((uint32_t)a_nx << 16), b_cur = __uint_as_float((uint32_t)b_nx << 16);
      if (i + 1 < nchunks) load_ab(i + 1);
      if (i >= 2 && !group_wait(sm, B_GFREE + s, ((i - 2) >> 1) & 1, 2, 128, pth == 0)) break;
      if (pth < 64) {
        // g = exp(-exp(A_log) softplus(a + dt_bias)), softplus(x) = x for x > 20 else log(1 + e^x);
        // beta = sigmoid(b)  (kernel_prefill.py:108-113), with the hardware exp2/log2
        const bool valid = (int64_t)i * kC + pth < len;
        float lg = 0.f, bt = 0.f;
        if (valid) {
          const float x = a_cur + dt_bias;
          const float sp = x > 20.f ? x : kLn2 * tc::lg2_approx(1.f + tc::ex2_approx(x * kLog2e));
          lg = -eA * sp;
          bt = 1.f / (1.f + tc::ex2_approx(-b_cur * kLog2e));
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
        const float x2 = x * kLog2e, gC2 = tmp[1] * kLog2e;
        const float G = tc::ex2_approx(x2);
        sm.gate(s, GA_G2)[pth] = x2;
        sm.gate(s, GA_BETA)[pth] = bt;
        sm.gate(s, GA_G)[pth] = G;
        sm.gate(s, GA_BG)[pth] = bt * G;
        sm.gate(s, GA_R)[pth] = tc::ex2_approx(gC2 - x2);
      }
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_GATES + s));
      // ---- A (row-major fp32) and P (registers) from K K^T / Q K^T ----
      if (!group_wait(sm, B_KKQK, i & 1, 2, 128, pth == 0)) break;
      tc::fence_after_sync();
      const float* g2 = sm.gate(s, GA_G2);
      uint32_t prow[32];
      {
        const float gt = g2[row];
        const uint32_t d0 = tc::tmem_addr(tmem, (uint32_t)((warp & 3) * 32), kTmD0);
        if (pth < 64) {  // A row (warps 8, 9): rolled loop
          const float bt = sm.gate(s, GA_BETA)[row];
#pragma unroll 1
          for (int j8 = 0; j8 < 8; ++j8) {
            float v[8];
            tc::tmem_ld8(d0 + j8 * 8, v);
            const float4 g0 = *reinterpret_cast<const float4*>(g2 + j8 * 8);
            const float4 g1 = *reinterpret_cast<const float4*>(g2 + j8 * 8 + 4);
            tc::tmem_wait_ld();
            const float gj[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            float w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = j8 * 8 + u < row ? bt * tc::ex2_approx(gt - gj[u]) * v[u] : 0.f;
            *reinterpret_cast<float4*>(As + row * kLd + j8 * 8) = make_float4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<float4*>(As + row * kLd + j8 * 8 + 4) = make_float4(w[4], w[5], w[6], w[7]);
          }
        } else {  // P row (warps 10, 11): kept in registers until the P tile is free
#pragma unroll
          for (int j8 = 0; j8 < 8; ++j8) {
            float v[8];
            tc::tmem_ld8(d0 + j8 * 8, v);
            const float4 g0 = *reinterpret_cast<const float4*>(g2 + j8 * 8);
            const float4 g1 = *reinterpret_cast<const float4*>(g2 + j8 * 8 + 4);
            tc::tmem_wait_ld();
            const float gj[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            float w[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) w[u] = j8 * 8 + u <= row ? tc::ex2_approx(gt - gj[u]) * v[u] : 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) prow[j8 * 4 + u] = pack_bf16x2(w[2 * u], w[2 * u + 1]);
          }
        }
      }
      tc::fence_before_sync();
      named_sync(2, 128);  // A complete, D0 read
      if (pth == 0) mbar_arrive(sm.bar(B_D0_FREE));
      // ---- diagonal 16x16 blocks of T on threads 0-63, while threads 64-127 scale the
      //      Q rows of the K/Q stage by G in place (Qg for the first MMA of chunk i) ----
      if (pth < 64) {
        solve_diag16(As, Ts, pth);
      } else {
        const float Gt = sm.gate(s, GA_G)[row];
        unsigned char* qstage = sm.base + kSmKQ + s * kKQStage;
#pragma unroll 2
        for (int c16 = 0; c16 < 16; ++c16) {
          const uint32_t off = (uint32_t)(c16 >> 3) * kKQTile + tc::sw128_offset(64 + row, (c16 & 7) * 8);
          uint4 w = *reinterpret_cast<const uint4*>(qstage + off);
          w.x = pack_bf16x2(__uint_as_float(w.x << 16) * Gt, __uint_as_float(w.x & 0xffff0000u) * Gt);
          w.y = pack_bf16x2(__uint_as_float(w.y << 16) * Gt, __uint_as_float(w.y & 0xffff0000u) * Gt);
          w.z = pack_bf16x2(__uint_as_float(w.z << 16) * Gt, __uint_as_float(w.z & 0xffff0000u) * Gt);
          w.w = pack_bf16x2(__uint_as_float(w.w << 16) * Gt, __uint_as_float(w.w & 0xffff0000u) * Gt);
          *reinterpret_cast<uint4*>(qstage + off) = w;
        }
        tc::fence_proxy_async_smem();
      }
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_QG_READY));
      // ---- T = (I + A)^-1: off-diagonal blocks, 16 -> 32 -> 64 ----
      solve_merge(As, Ts, sm.Xs(), pth, 4);
      solve_merge(As, Ts, sm.Xs(), pth, 5);
      // ---- T hi/lo tiles (after MMA2 of chunk i-1), P tile (after MMA3 of chunk i-1) ----
      if (i >= 1 && !group_wait(sm, B_MMA2, (i - 1) & 1, 2, 128, pth == 0)) break;
      if (pth < 64) {
        unsigned char* thi = sm.base + kSmT;
        unsigned char* tlo = sm.base + kSmT + 8192;
#pragma unroll 1
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
    // outputs of chunk ci: o[t][v] = scale * O^T[v][t] (D1 buffer ci & 1, columns 64-127);
    // lane pairs exchange so each stores bf16x2.  Requires MMA3(ci) complete.
    auto emit_out = [&](int ci) {
      const int64_t rem = len - (int64_t)ci * kC;
      const int nvalid = rem < kC ? (int)rem : kC;
      const bool odd = lane & 1;
      const int vcol = v & ~1;
      __nv_bfloat16* out = p.out + (t0 + (int64_t)ci * kC) * p.o_st + (int64_t)h * p.o_sh + vcol;
#pragma unroll 1
      for (int c8 = 0; c8 < 4; ++c8) {
        float x[8];
        tc::tmem_ld8(tc::tmem_addr(tmem, lane_base, kTmD1 + (uint32_t)(ci & 1) * 128 + 64 + tb + c8 * 8), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 8; q += 2) {
          // even lane keeps token q (needs the odd neighbour's column), odd lane keeps token q + 1
          const float send = odd ? x[q] : x[q + 1];
          const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
          const float c0v = odd ? recv : x[q];      // column vcol
          const float c1v = odd ? x[q + 1] : recv;  // column vcol + 1
          const int t = tb + c8 * 8 + q + (odd ? 1 : 0);
          if (t < nvalid)
            *reinterpret_cast<uint32_t*>(out + (int64_t)t * p.o_st) = pack_bf16x2(scale * c0v, scale * c1v);
        }
      }
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_OUT_DONE));
    };
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      if (!group_wait(sm, B_GATES + s, (i >> 1) & 1, 1, kChainThreads, leader)) break;
      const float GC = sm.gate(s, GA_G)[63];
      // ---- S0 hi/lo tiles and S <- G_C * S (64 columns per thread) ----
      if (i > 0 && !group_wait(sm, B_MMA4, (i - 1) & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
#pragma unroll 2
      for (int c8 = 0; c8 < 8; ++c8) {
        float x[8];
        const uint32_t ta = tc::tmem_addr(tmem, lane_base, kTmS + hsel * 64 + c8 * 8);
        tc::tmem_ld8(ta, x);
        tc::tmem_wait_ld();
        uint4 hi, lo;
        split2(x[0], x[1], hi.x, lo.x);
        split2(x[2], x[3], hi.y, lo.y);
        split2(x[4], x[5], hi.z, lo.z);
        split2(x[6], x[7], hi.w, lo.w);
        st_tile(s0t, v, c8, hi);
        st_tile(s0l, v, c8, lo);
#pragma unroll
        for (int q = 0; q < 8; ++q) x[q] *= GC;
        tc::tmem_st8(ta, x);
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_S0_READY));
      // ---- R^T = beta V^T - beta G (S0 K^T), split hi/lo (32 token columns per thread) ----
      if (!group_wait(sm, B_V_FULL, i & 1, 1, kChainThreads, leader)) break;
      if (!group_wait(sm, B_MMA1, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        const float* bet = sm.gate(s, GA_BETA) + tb;
        const float* bg = sm.gate(s, GA_BG) + tb;
#pragma unroll 2
        for (int c8 = 0; c8 < 4; ++c8) {
          float x[8], vv[8];
          tc::tmem_ld8(tc::tmem_addr(tmem, lane_base, kTmD1 + (uint32_t)s * 128 + tb + c8 * 8), x);
#pragma unroll
          for (int u = 0; u < 8; ++u) vv[u] = __bfloat162float(vt[(tb + c8 * 8 + u) * kHeadDim + v]);
          const float4 b0 = *reinterpret_cast<const float4*>(bet + c8 * 8);
          const float4 b1 = *reinterpret_cast<const float4*>(bet + c8 * 8 + 4);
          const float4 g0 = *reinterpret_cast<const float4*>(bg + c8 * 8);
          const float4 g1 = *reinterpret_cast<const float4*>(bg + c8 * 8 + 4);
          tc::tmem_wait_ld();
          const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
          float r8[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) r8[u] = fmaf(bb[u], vv[u], -gg[u] * x[u]);
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
      // ---- previous chunk's outputs, in the shadow of this chunk's second MMA ----
      if (i > 0) {
        if (!group_wait(sm, B_MMA3, (i - 1) & 1, 1, kChainThreads, leader)) break;
        tc::fence_after_sync();
        emit_out(i - 1);
      }
      // ---- deltas: D^T (bf16, output MMA) and Dt^T = D^T exp(gC - g) (hi/lo, state MMA) ----
      if (!group_wait(sm, B_MMA2, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        const float* rr = sm.gate(s, GA_R) + tb;
#pragma unroll 2
        for (int c8 = 0; c8 < 4; ++c8) {
          float d[8];
          tc::tmem_ld8(tc::tmem_addr(tmem, lane_base, kTmD2 + tb + c8 * 8), d);
          const float4 r0 = *reinterpret_cast<const float4*>(rr + c8 * 8);
          const float4 r1 = *reinterpret_cast<const float4*>(rr + c8 * 8 + 4);
          tc::tmem_wait_ld();
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
      if (leader) {
        mbar_arrive(sm.bar(B_D_READY));
        mbar_arrive(sm.bar(B_GFREE + s));
      }
    }
    // ---- last chunk's outputs and the final state ----
    bool ok = true;
    if (nchunks > 0) {
      ok = group_wait(sm, B_MMA4, (nchunks - 1) & 1, 1, kChainThreads, leader) &&
           group_wait(sm, B_MMA3, (nchunks - 1) & 1, 1, kChainThreads, leader) && !*sm.abort_flag();
      if (ok) {
        tc::fence_after_sync();
        emit_out(nchunks - 1);
      }
    }
    if (ok) {
      tc::fence_after_sync();
      float* dst = p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh + (size_t)v * kHeadDim + hsel * 64;
#pragma unroll 1
      for (int c8 = 0; c8 < 8; ++c8) {
        float x[8];
        tc::tmem_ld8(tc::tmem_addr(tmem, lane_base, kTmS + hsel * 64 + c8 * 8), x);
        tc::tmem_wait_ld();
        *reinterpret_cast<float4*>(dst + c8 * 8) = make_float4(x[0], x[1], x[2], x[3]);
        *reinterpret_cast<float4*>(dst + c8 * 8 + 4) = make_float4(x[4], x[5], x[6], x[7]);
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
