// Chunked (C = 64) varlen GDN prefill on tcgen05 tensor cores (sm_100a).
//
// Reference semantics: solution/triton/kernel_prefill.py:42-142 (token-serial
// decode recurrence per (sequence, v-head); empty sequence passes its initial
// state through).  This kernel computes the same recurrence in the chunked
// WY/UT form.  For a chunk of C tokens with initial k-last state S0 [V x K]
// (row v = one value index), log-decay prefix g_t = sum_{i<=t} log g_i,
// G_t = exp(g_t), gates beta_t:
//   A[t][j] = beta_t exp(g_t - g_j) k_t.k_j  (j < t),  T = (I + A)^-1
//   R^T[v][t] = beta_t (V[t][v] - G_t (S0 K^T)[v][t])
//   D^T = R^T T^T                      (D = per-token deltas, D^T is [V x C])
//   O^T[v][t] = scale (G_t (S0 Q^T)[v][t] + (D^T P^T)[v][t]),
//               P[t][j] = exp(g_t - g_j) q_t.k_j (j <= t)
//   S_next = G_C S0 + Dt^T K,  Dt[j] = exp(g_C - g_j) D[j]
// All products run on tcgen05 with M = 128 = the state's V dimension on the
// TMEM lanes, bf16 operands and fp32 accumulation.  The operands whose
// rounding reaches the state at the scale of the deltas are split into bf16
// hi + lo parts: S0 in S0 K^T (2 MMAs; V - G S0 K^T cancels once the state has
// learned the values), R and T in D^T (3 MMAs) and Dt in the state update
// (2 MMAs).  The state itself stays fp32 in TMEM for the whole sequence.
//
// CTA = one (sequence, v-head) chain, 10 warps:
//   warps 0-3  chain warpgroup: thread v owns state row v (TMEM lane v):
//              S0 -> bf16 tile, R, deltas, outputs, initial/final state I/O
//   warps 4-7  prep warpgroup: gates, A and P from K K^T / Q K^T, blocked fp32
//              triangular inverse T, T hi/lo and P tiles — for chunk i+1
//              while the chain works on chunk i
//   warp 8     TMA producer (K, Q: 128B-swizzled tiles; V: plain tile)
//   warp 9     TMEM allocator and MMA issuer
// Every wait is bounded (kWaitLimitNs); a timeout raises GDN_DEVERR_WAIT_TIMEOUT
// and makes every role leave its loop.
#include <cuda.h>

#include "gdn_common.cuh"
#include "gdn_kernels.h"
#include "gdn_tc.cuh"

namespace gdn {
namespace {

constexpr int kC = 64;             // chunk length (tokens)
constexpr int kThreads = 320;      // 10 warps
constexpr uint32_t kTmemCols = 512;

// TMEM column map (fp32 accumulators, lanes = state row v unless noted)
constexpr uint32_t kTmS = 0;      // [0,128)   state S[v][k]
constexpr uint32_t kTmD1 = 128;   // [128,192) S0 K^T,  [192,256) S0 Q^T
constexpr uint32_t kTmD0 = 256;   // [256,320) and [320,384): K K^T / Q K^T (lanes = token; stage s)
constexpr uint32_t kTmD2 = 384;   // [384,448) D^T
constexpr uint32_t kTmD3 = 448;   // [448,512) D^T P^T

// Shared-memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kSmKQ = 0;             // 2 stages x 32 KB: [tile d0-63 | tile d64-127], rows 0-63 K, 64-127 Q
constexpr uint32_t kKQStage = 32768;
constexpr uint32_t kKQTile = 16384;       // one 64-column tile of 128 rows
constexpr uint32_t kSmV = 65536;          // V tile, plain row-major [64][128] bf16 (16 KB)
constexpr uint32_t kSmS0 = 81920;         // S0 bf16: 2 tiles [128 x 64] (32 KB); D^T bf16 reuses tile 0
constexpr uint32_t kSmRD = 114688;        // S0 lo (2 tiles), then R^T hi | lo, then Dt^T hi | lo: 2 tiles [128 x 64]
constexpr uint32_t kSmT = 147456;         // T hi | lo: 2 tiles [64 x 64] (16 KB)
constexpr uint32_t kSmP = 163840;         // P: tile [64 x 64] (8 KB)
constexpr uint32_t kSmA = 172032;         // solve: A^T fp32 [64][64] (16 KB)
constexpr uint32_t kSmTf = 188416;        // solve: T fp32 [64][64] (16 KB)
constexpr uint32_t kSmX = 204800;         // solve: products scratch fp32 [3][16][16] (3 KB)
constexpr uint32_t kSmGate = 207872;      // 2 stages x {gamma[64], beta[64], exp(gamma)[64]} fp32 (1.5 KB)
constexpr uint32_t kSmBar = 209408;       // mbarriers (32 x 8 B)
constexpr uint32_t kSmMisc = 209664;      // tmem base slot, abort flag
constexpr uint32_t kSmBytes = 209728;
constexpr uint32_t kSmAlloc = kSmBytes + 1024;  // + alignment slack

// barrier indices
enum : int {
  B_KQ_FULL = 0,    // [2]
  B_KQ_EMPTY = 2,   // [2]
  B_KKQK = 4,       // [2]
  B_GATES = 6,      // [2]
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
  __device__ float* gamma(int s) const { return reinterpret_cast<float*>(base + kSmGate) + s * 192; }
  __device__ float* beta(int s) const { return reinterpret_cast<float*>(base + kSmGate) + s * 192 + 64; }
  __device__ float* gexp(int s) const { return reinterpret_cast<float*>(base + kSmGate) + s * 192 + 128; }
  __device__ volatile int* abort_flag() const { return reinterpret_cast<volatile int*>(base + kSmMisc + 16); }
  __device__ uint32_t* tmem_slot() const { return reinterpret_cast<uint32_t*>(base + kSmMisc); }
  __device__ float* A() const { return reinterpret_cast<float*>(base + kSmA); }
  __device__ float* Tf() const { return reinterpret_cast<float*>(base + kSmTf); }
  __device__ float* X() const { return reinterpret_cast<float*>(base + kSmX); }
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

// Wait of a 128-thread warpgroup: the leader polls the mbarrier, then the group
// meets at named barrier `bar_id` and AND-reduces the outcome, so all threads
// either proceed or leave together.
__device__ __forceinline__ bool group_wait(const Smem& sm, int bar_idx, uint32_t parity, int bar_id, bool leader) {
  int ok = 1;
  if (leader) ok = wait_bar(sm, sm.bar(bar_idx), parity) ? 1 : 0;
  int all;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(all)
      : "r"(ok), "r"(bar_id)
      : "memory");
  return all != 0;
}

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int i) {
  return p.cu_is_int64 ? reinterpret_cast<const int64_t*>(p.cu_seqlens)[i]
                       : (int64_t) reinterpret_cast<const int32_t*>(p.cu_seqlens)[i];
}

__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16& hi, __nv_bfloat16& lo) {
  hi = __float2bfloat16_rn(x);
  lo = __float2bfloat16_rn(x - __bfloat162float(hi));
}

// Write 8 consecutive bf16 (columns c8*8 .. c8*8+7 of `row`) into a SW128 tile.
__device__ __forceinline__ void st_tile8(unsigned char* tile, int row, int c8, const __nv_bfloat16 (&v)[8]) {
  uint4 w;
  w.x = *reinterpret_cast<const uint32_t*>(&v[0]);
  w.y = *reinterpret_cast<const uint32_t*>(&v[2]);
  w.z = *reinterpret_cast<const uint32_t*>(&v[4]);
  w.w = *reinterpret_cast<const uint32_t*>(&v[6]);
  *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, c8 * 8)) = w;
}

// ---------------------------------------------------------------------------
// Blocked inverse of the unit lower-triangular 64x64 matrix I + A (prep warpgroup,
// 128 threads, fp32).  A is given transposed (At[j][t] = A[t][j], zero on and
// above the diagonal); the inverse T is written row-major to Tf[t][j].
//   diagonal 16x16 blocks by column forward substitution, then
//   T_ij = -T_ii * sum_{k=j}^{i-1} A_ik T_kj  by block distance 1, 2, 3.
__device__ void solve_unit_lower(const float* At, float* Tf, float* X, int p) {
  // zero the strictly upper part of Tf (rows: 2 per thread)
  for (int e = p; e < 64 * 64; e += 128) {
    const int t = e >> 6, j = e & 63;
    if (j > t) Tf[e] = 0.f;
  }
  if (p < 64) {
    const int b = p >> 4, c = p & 15, o = b * 16;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = 0.f;
    x[c] = 1.f;
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      if (r > c) {
        float s = 0.f;
#pragma unroll
        for (int q = 0; q < 15; ++q)
          if (q >= c && q < r) s = fmaf(At[(o + q) * 64 + o + r], x[q], s);
        x[r] = -s;
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r)
      if (r >= c) Tf[(o + r) * 64 + o + c] = x[r];
  }
  named_sync(2, 128);
  // block distance d = i - j
  for (int d = 1; d <= 3; ++d) {
    const int nblk = 4 - d;                 // blocks (i, j) with j = 0..nblk-1, i = j + d
    // X_ij = sum_{k=j}^{i-1} A_ik T_kj
    for (int e = p; e < nblk * 256; e += 128) {
      const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
      const int j = blk, i = blk + d;
      float s = 0.f;
      for (int k = j; k < i; ++k) {
#pragma unroll
        for (int q = 0; q < 16; ++q) s = fmaf(At[(16 * k + q) * 64 + 16 * i + r], Tf[(16 * k + q) * 64 + 16 * j + c], s);
      }
      X[blk * 256 + r * 16 + c] = s;
    }
    named_sync(2, 128);
    // T_ij = -T_ii X_ij
    for (int e = p; e < nblk * 256; e += 128) {
      const int blk = e >> 8, r = (e >> 4) & 15, c = e & 15;
      const int j = blk, i = blk + d;
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q) s = fmaf(Tf[(16 * i + r) * 64 + 16 * i + q], X[blk * 256 + q * 16 + c], s);
      Tf[(16 * i + r) * 64 + 16 * j + c] = -s;
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
  if (warp == 9) {
    tc::tmem_alloc(sm.tmem_slot(), kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *sm.tmem_slot();

  // ======================================================================= TMA producer
  if (warp == 8) {
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
  else if (warp == 9) {
    if (lane == 0 && nchunks > 0) {
      const uint32_t id_kq = tc::idesc_bf16(128, 64, false, false);    // [K;Q] x K^T
      const uint32_t id_s0 = tc::idesc_bf16(128, 128, false, false);   // S0 x [K;Q]^T
      const uint32_t id_64 = tc::idesc_bf16(128, 64, false, false);    // R^T x T^T, D^T x P^T
      const uint32_t id_st = tc::idesc_bf16(128, 128, false, true);    // Dt^T x K (K MN-major)
      const uint32_t aS0 = sm.addr(kSmS0), aRD = sm.addr(kSmRD), aT = sm.addr(kSmT), aP = sm.addr(kSmP);
      auto issue_kkqk = [&](int i) -> bool {
        const int s = i & 1;
        if (!wait_bar(sm, sm.bar(B_KQ_FULL + s), (i >> 1) & 1)) return false;
        tc::fence_after_sync();
        const uint32_t kq = sm.addr(kSmKQ + s * kKQStage);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD0 + s * 64, tc::kmajor_desc(kq, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks),
                       id_kq, ks > 0);
        tc::mma_commit(sm.bar(B_KKQK + s));
        return true;
      };
      bool ok = issue_kkqk(0);
      for (int i = 0; ok && i < nchunks; ++i) {
        const int s = i & 1;
        const uint32_t kq = sm.addr(kSmKQ + s * kKQStage);
        // MMA1: D1 = S0_hi [K;Q]^T, then D1[:, K part] += S0_lo K^T
        if (!wait_bar(sm, sm.bar(B_S0_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD1, tc::kmajor_desc(aS0, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks), id_s0,
                       ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16(tmem + kTmD1, tc::kmajor_desc(aRD, kKQTile, ks), tc::kmajor_desc(kq, kKQTile, ks), id_kq,
                       true);
        tc::mma_commit(sm.bar(B_MMA1));
        // next chunk's K K^T / Q K^T
        if (i + 1 < nchunks && !issue_kkqk(i + 1)) break;
        // MMA2: D^T = R^T T^T (hi/lo)
        if (!wait_bar(sm, sm.bar(B_R_READY), i & 1)) break;
        if (!wait_bar(sm, sm.bar(B_PREP_DONE), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD, 0, ks), tc::kmajor_desc(aT, 0, ks), id_64, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD + 16384, 0, ks), tc::kmajor_desc(aT, 0, ks), id_64, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD2, tc::kmajor_desc(aRD, 0, ks), tc::kmajor_desc(aT + 8192, 0, ks), id_64, true);
        tc::mma_commit(sm.bar(B_MMA2));
        // MMA3: D3 = D^T P^T;  MMA4: S += Dt^T K (hi/lo)
        if (!wait_bar(sm, sm.bar(B_D_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(tmem + kTmD3, tc::kmajor_desc(aS0, 0, ks), tc::kmajor_desc(aP, 0, ks), id_64, ks > 0);
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
  else if (warp >= 4) {
    const int pth = tid - 128;  // 0..127, TMEM lane pth
    float* At = sm.A();
    float* Tf = sm.Tf();
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      // ---- gates of chunk i (stage s free once the chain finished chunk i-2) ----
      if (i >= 2 && !group_wait(sm, B_OUT_DONE, (i - 2) & 1, 2, pth == 0)) break;
      if (pth < 64) {
        const int64_t tok = t0 + (int64_t)i * kC + pth;
        const bool valid = (int64_t)i * kC + pth < len;
        float lg = 0.f, bt = 0.f;
        if (valid) {
          const float a = bf16_to_f32(p.a + tok * p.a_st + h);
          const float b = bf16_to_f32(p.b + tok * p.b_st + h);
          lg = gdn_log_decay(p.A_log[h], a, p.dt_bias[h]);
          bt = 1.0f / (1.0f + expf(-b));
        }
        // inclusive scan of lg over the 64 tokens (two warps)
        float x = lg;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += y;
        }
        sm.gamma(s)[pth] = x;  // partial (per warp)
        sm.beta(s)[pth] = bt;
      }
      named_sync(2, 128);
      if (pth < 64) {
        float g = sm.gamma(s)[pth];
        if (pth >= 32) g += sm.gamma(s)[31];
        named_sync(3, 64);  // both warps read before the upper half is rewritten
        sm.gamma(s)[pth] = g;
        sm.gexp(s)[pth] = expf(g);
      }
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_GATES + s));
      // ---- A (transposed, fp32) and P (registers) from K K^T / Q K^T ----
      if (!group_wait(sm, B_KKQK + s, (i >> 1) & 1, 2, pth == 0)) break;
      tc::fence_after_sync();
      const float* gam = sm.gamma(s);
      const float* bet = sm.beta(s);
      uint32_t prow[32];  // P row (lanes 64..127) packed bf16x2
      {
        const int row = pth & 63;
        const float gt = gam[row];
        const float bt = bet[row];
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          float v[16];
          tc::tmem_ld16(tc::tmem_addr(tmem, (uint32_t)((warp & 3) * 32), kTmD0 + s * 64 + c0), v);
          tc::tmem_wait_ld();
          if (pth < 64) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int j = c0 + q;
              At[j * 64 + row] = j < row ? bt * expf(gt - gam[j]) * v[q] : 0.f;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 16; q += 2) {
              const int j = c0 + q;
              const float p0 = j <= row ? expf(gt - gam[j]) * v[q] : 0.f;
              const float p1 = j + 1 <= row ? expf(gt - gam[j + 1]) * v[q + 1] : 0.f;
              __nv_bfloat162 pr = __floats2bfloat162_rn(p0, p1);
              prow[(c0 + q) >> 1] = *reinterpret_cast<uint32_t*>(&pr);
            }
          }
        }
      }
      tc::fence_before_sync();
      named_sync(2, 128);
      // ---- T = (I + A)^-1 ----
      solve_unit_lower(At, Tf, sm.X(), pth);
      // ---- T hi/lo tile (after MMA2 of chunk i-1), P tile (after MMA3 of chunk i-1) ----
      if (i >= 1 && !group_wait(sm, B_MMA2, (i - 1) & 1, 2, pth == 0)) break;
      if (pth < 64) {
        unsigned char* thi = sm.base + kSmT;
        unsigned char* tlo = sm.base + kSmT + 8192;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          __nv_bfloat16 hi[8], lo[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) split_bf16(Tf[pth * 64 + c8 * 8 + q], hi[q], lo[q]);
          st_tile8(thi, pth, c8, hi);
          st_tile8(tlo, pth, c8, lo);
        }
      }
      if (i >= 1 && !group_wait(sm, B_MMA3, (i - 1) & 1, 2, pth == 0)) break;
      if (pth >= 64) {
        unsigned char* pt = sm.base + kSmP;
        const int row = pth - 64;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          uint4 w = make_uint4(prow[c8 * 4], prow[c8 * 4 + 1], prow[c8 * 4 + 2], prow[c8 * 4 + 3]);
          *reinterpret_cast<uint4*>(pt + tc::sw128_offset(row, c8 * 8)) = w;
        }
      }
      tc::fence_proxy_async_smem();
      named_sync(2, 128);
      if (pth == 0) mbar_arrive(sm.bar(B_PREP_DONE));
    }
  }
  // ======================================================================= chain warpgroup
  else {
    const int v = tid;  // state row / TMEM lane
    const uint32_t lane_base = (uint32_t)(warp * 32);
    // initial state -> TMEM S
    {
      const float* src = p.state ? p.state + (size_t)n * p.s_sn + (size_t)h * p.s_sh + (size_t)v * kHeadDim : nullptr;
#pragma unroll
      for (int c0 = 0; c0 < kHeadDim; c0 += 16) {
        float x[16];
#pragma unroll
        for (int q = 0; q < 16; q += 4) {
          const float4 f = src ? ld_nc_f4(src + c0 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
          x[q] = f.x;
          x[q + 1] = f.y;
          x[q + 2] = f.z;
          x[q + 3] = f.w;
        }
        tc::tmem_st16(tc::tmem_addr(tmem, lane_base, kTmS + c0), x);
      }
      tc::tmem_wait_st();
    }
    const float scale = p.scale;
    unsigned char* s0t = sm.base + kSmS0;
    unsigned char* rd = sm.base + kSmRD;
    const __nv_bfloat16* vt = reinterpret_cast<const __nv_bfloat16*>(sm.base + kSmV);
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      const int64_t rem = len - (int64_t)i * kC;
      const int nvalid = rem < kC ? (int)rem : kC;
      if (!group_wait(sm, B_GATES + s, (i >> 1) & 1, 1, v == 0)) break;
      const float* gam = sm.gamma(s);
      const float* bet = sm.beta(s);
      const float* gex = sm.gexp(s);
      const float gC = gam[63];
      const float GC = gex[63];
      // ---- S0 tiles (bf16 hi in kSmS0, lo in kSmRD) and S <- G_C * S ----
      if (i > 0 && !group_wait(sm, B_MMA4, (i - 1) & 1, 1, v == 0)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < kHeadDim; c0 += 16) {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmS + c0), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
          __nv_bfloat16 hi[8], lo[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) split_bf16(x[h8 * 8 + q], hi[q], lo[q]);
          st_tile8(s0t + (c0 >> 6) * kKQTile, v, ((c0 & 63) >> 3) + h8, hi);
          st_tile8(rd + (c0 >> 6) * kKQTile, v, ((c0 & 63) >> 3) + h8, lo);
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) x[q] *= GC;
        tc::tmem_st16(tc::tmem_addr(tmem, lane_base, kTmS + c0), x);
      }
      tc::tmem_wait_st();
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, 128);
      if (v == 0) mbar_arrive(sm.bar(B_S0_READY));
      // ---- R^T = beta (V^T - G * S0 K^T), split hi/lo ----
      if (!group_wait(sm, B_MMA1, i & 1, 1, v == 0)) break;
      if (!group_wait(sm, B_V_FULL, i & 1, 1, v == 0)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < kC; c0 += 16) {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmD1 + c0), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
          __nv_bfloat16 hi[8], lo[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int t = c0 + h8 * 8 + q;
            const float r = bet[t] * (__bfloat162float(vt[t * kHeadDim + v]) - gex[t] * x[h8 * 8 + q]);
            split_bf16(r, hi[q], lo[q]);
          }
          st_tile8(rd, v, (c0 >> 3) + h8, hi);
          st_tile8(rd + 16384, v, (c0 >> 3) + h8, lo);
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, 128);
      if (v == 0) {
        mbar_arrive(sm.bar(B_R_READY));
        mbar_arrive(sm.bar(B_V_EMPTY));
      }
      // ---- deltas: D^T (bf16, for the output) and Dt^T = D^T exp(gC - g) (hi/lo, for the state) ----
      if (!group_wait(sm, B_MMA2, i & 1, 1, v == 0)) break;
      tc::fence_after_sync();
#pragma unroll
      for (int c0 = 0; c0 < kC; c0 += 16) {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmD2 + c0), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
          __nv_bfloat16 d8[8], hi[8], lo[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int t = c0 + h8 * 8 + q;
            const float d = x[h8 * 8 + q];
            d8[q] = __float2bfloat16_rn(d);
            split_bf16(d * expf(gC - gam[t]), hi[q], lo[q]);
          }
          st_tile8(s0t, v, (c0 >> 3) + h8, d8);
          st_tile8(rd, v, (c0 >> 3) + h8, hi);
          st_tile8(rd + 16384, v, (c0 >> 3) + h8, lo);
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      named_sync(1, 128);
      if (v == 0) mbar_arrive(sm.bar(B_D_READY));
      // ---- outputs: o[t][v] = scale (G_t S0Q^T[v][t] + (D^T P^T)[v][t]) ----
      if (!group_wait(sm, B_MMA3, i & 1, 1, v == 0)) break;
      tc::fence_after_sync();
      __nv_bfloat16* out = p.out + (t0 + (int64_t)i * kC) * p.o_st + (int64_t)h * p.o_sh + v;
#pragma unroll
      for (int c0 = 0; c0 < kC; c0 += 16) {
        float xq[16], xd[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmD1 + 64 + c0), xq);
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmD3 + c0), xd);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int t = c0 + q;
          if (t < nvalid) out[(int64_t)t * p.o_st] = __float2bfloat16_rn(scale * fmaf(gex[t], xq[q], xd[q]));
        }
      }
      tc::fence_before_sync();
      named_sync(1, 128);
      if (v == 0) mbar_arrive(sm.bar(B_OUT_DONE));
    }
    // ---- final state ----
    bool ok = true;
    if (nchunks > 0) ok = group_wait(sm, B_MMA4, (nchunks - 1) & 1, 1, v == 0) && !*sm.abort_flag();
    if (ok) {
      tc::fence_after_sync();
      float* dst = p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh + (size_t)v * kHeadDim;
#pragma unroll
      for (int c0 = 0; c0 < kHeadDim; c0 += 16) {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmS + c0), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 16; q += 4)
          *reinterpret_cast<float4*>(dst + c0 + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
      }
    }
  }

  // ---- teardown: every role is out of its loop; drain in-flight MMAs before freeing TMEM ----
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 9) {
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
