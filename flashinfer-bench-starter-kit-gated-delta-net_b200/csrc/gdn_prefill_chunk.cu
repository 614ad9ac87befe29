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
// TMEM lanes, bf16 operands and fp32 accumulation.  The A operands the chain
// produces (S0, R, Dt) are written to TMEM and read from there by the MMA, so
// shared-memory bandwidth is left to the B operands (K, Qg, T) and the copies.  The operands whose rounding
// reaches the state at the scale of the deltas are split into bf16 hi + lo
// parts: S0 in S0 K^T (V - G S0 K^T cancels once the state has learned the
// values), R and T in D^T (3 products) and Dt in the state update (2 products).
// The state stays fp32 in TMEM for the whole sequence.
//
// The state-independent per-chunk work (gates, A, T and its hi/lo split) comes
// precomputed from the prep kernel (gdn_prefill_prep.cu) as one workspace record
// per (chunk slot, v-head), bulk-copied into shared memory one chunk ahead.
//
// CTA = one (sequence, v-head) chain (sequences started longest first), 4 kCW + 6 warps:
//   4 kCW chain warps: thread (warp & 3, lane) owns state row v, warp >> 2
//               selects 1/kCW of the columns; initial state (loaded before the
//               CTA setup), S0 hi/lo and G_C scaling, R, deltas, the D^T tile,
//               final state
//   4 P warps   P from Q K^T (Q rows on all 128 TMEM lanes), G-scaling of S0 Q^T
//               in TMEM, the outputs of the previous chunk (TMEM -> bf16 rows in
//               shared memory -> one TMA store)
//   1 TMA warp  record (T tiles + gates) by bulk copy, K, Q (128B-swizzled tiles),
//               V (plain); all double-buffered except V
//   1 MMA warp  TMEM allocator and MMA issuer
// Per chunk the state chain is S0 hi/lo -> [S0 [Q;K]^T] -> R -> [R^T T^T] ->
// deltas -> [S += Dt^T K] -> next chunk; the next chunk's Q K^T (in two halves, in
// the tensor pipe's idle windows), the output MMA (D^T P^T), the output stores and
// the P work overlap it.  Hand-offs are mbarriers, arranged so the MMA thread waits
// on one barrier per MMA group (a barrier probe costs it several hundred cycles even
// after the phase completed; a wait that blocks first wakes quickly): MMA1 waits on
// the chain's S0 split and the P warps' read of Q K^T together, MMA4 and the output
// MMA on the deltas and the P tile together, and one barrier completes when a chunk's
// record, gates and V have landed.  Every wait is bounded (kWaitLimitNs): a timeout
// raises GDN_DEVERR_WAIT_TIMEOUT and an in-CTA abort flag so every role leaves its
// loop, then in-flight copies and MMAs are drained before TMEM is freed.
#include <cuda.h>

#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <utility>
#include <vector>

#include "gdn_prefill_chunk.cuh"

namespace gdn {
namespace {

using namespace chunk;

// Chain warps per TMEM lane quarter (the warp's quarter is warp % 4, which is also
// its scheduler): each chain thread owns one state row and 1/kCW of the columns.
#ifndef GDN_CHAIN_WARPS_PER_QUARTER
#define GDN_CHAIN_WARPS_PER_QUARTER 4
#endif
constexpr int kCW = GDN_CHAIN_WARPS_PER_QUARTER;
constexpr int kChainWarps = 4 * kCW;
constexpr int kChainThreads = 32 * kChainWarps;
constexpr int kWarpP0 = kChainWarps;  // P warpgroup: 4 warps after the chain warps
constexpr int kWarpTma = kChainWarps + 4, kWarpMma = kChainWarps + 5;
constexpr int kThreads = 32 * (kChainWarps + 6);
constexpr int kStateCols = 128 / kCW, kTokCols = 64 / kCW;  // per chain thread
static_assert(kCW == 4, "chain split: a chain thread holds 32 state columns");
constexpr uint32_t kTmemCols = 512;

// TMEM column map (lanes = state row v unless noted)
constexpr uint32_t kTmS = 0;      // [0,128)  state S[v][k], fp32
constexpr uint32_t kTmD1 = 128;   // 2 buffers [128,256), [256,384), fp32: cols 0-63 S0 Q^T, scaled by G in
                                  //   place, + D^T P^T = O^T (unscaled); cols 64-127 [Q; Q] K^T scratch
                                  //   (lanes = token, twice), then S0 K^T, then D^T
                                  // [384,512) bf16 A operands, two per column, reused along the chain:
constexpr uint32_t kTmS0hi = 384; //   S0 hi [384,448), S0 lo [448,512)           (S0 split .. MMA1)
constexpr uint32_t kTmS0lo = 448;
constexpr uint32_t kTmRhi = 384;  //   R hi [384,416), R lo [416,448)             (R .. MMA2)
constexpr uint32_t kTmRlo = 416;
constexpr uint32_t kTmDthi = 448; //   Dt hi [448,480), Dt lo [480,512)           (deltas .. MMA4)
constexpr uint32_t kTmDtlo = 480;

// Shared-memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kSmKQ = 0;          // 2 stages x 48 KB: [tile d0-63 | tile d64-127]; in each 64-column
constexpr uint32_t kKQStage = 49152;   // SW128 tile rows 0-63 Q, 64-127 Q again, 128-191 K, so that
constexpr uint32_t kKQTile = 24576;    // [Q; Q] (A of Q K^T: the Q rows on all 128 TMEM lanes) and
constexpr uint32_t kRowsQ2 = 8192;     // [Q; K] (B of the first MMA) are both 128 contiguous rows
constexpr uint32_t kRowsK = 16384;
constexpr uint32_t kSmV = 98304;       // V, plain row-major [64][128] bf16 (16 KB)
constexpr uint32_t kSmD = 114688;      // D^T bf16 SW128 tile [128 x 64] (A of the output MMA)
constexpr uint32_t kSmT = 131072;      // 2 stages x (T hi | T lo: 2 tiles [64 x 64]) (record bytes 0-16383)
constexpr uint32_t kTStage = 2 * kTTileBytes;  // full T hi | T lo tiles (no swizzle, upper blocks zero)
constexpr uint32_t kSmP = 163840;      // P tile [64 x 64]
constexpr uint32_t kSmO = 172032;      // output rows of one chunk, [64 tokens][128] bf16 (TMA-store source)
constexpr uint32_t kSmGate = 188416;   // 2 stages x gate arrays (record bytes 16384-18175)
constexpr uint32_t kSmBar = 192000;    // mbarriers (32 x 8 B)
constexpr uint32_t kSmMisc = 192256;   // tmem base slot, abort flag
constexpr uint32_t kSmBytes = 192320;
constexpr uint32_t kSmAlloc = kSmBytes + 1024;  // + alignment slack
static_assert(kSmKQ + 2 * kKQStage <= kSmV && kSmT + 2 * kTStage <= kSmP && kSmO + 16384 <= kSmGate &&
                  kSmGate + 2 * kRecGates <= kSmBar,
              "smem map");
static_assert(kSmAlloc <= 232448, "smem budget");

enum : int {
  B_KQ_FULL = 0,    // [2]
  B_KQ_EMPTY = 2,   // [2]
  B_REC_FULL = 4,   // [2] chunk inputs landed: T (hi | lo), the gate arrays and V (one expect_tx,
                    //     three copies)
  B_GFREE = 6,      // [2] chain and P warpgroup are done with a gate stage (2 arrivals)
  B_T_EMPTY = 8,    // [2] the MMA reading a T stage has completed
  B_MMA4 = 10,      // [2] state update of a chunk done (per chunk parity)
  B_KKQK = 12,      // [Q; Q] K^T of a chunk is in its D1 buffer, columns 64-127
  B_V_EMPTY,
  B_S0_READY,       // MMA1 may go: S0 hi/lo written (chain) and the P warpgroup has read the Q K^T
                    // of the chunk's D1 buffer (having stored the outputs of chunk i - 2 from it)
  B_MMA1,
  B_R_READY,        // R written (also: S0 Q^T may be scaled by the P warpgroup from here on)
  B_MMA2,
  B_D_READY,        // MMA4 may go: Dt hi/lo written (chain), and the P warpgroup has written the
                    // P tile and scaled S0 Q^T (so the output MMA after MMA4 needs only the D^T tile)
  B_MMA3,
  B_DTILE,          // D^T bf16 tile written (A of the output MMA)
  B_DRAIN,
  B_COUNT
};
static_assert(B_COUNT <= 32, "barrier block");

struct Smem {
  unsigned char* base;
  __device__ uint64_t* bar(int i) const { return reinterpret_cast<uint64_t*>(base + kSmBar) + i; }
  __device__ float* gate(int s, int a) const { return reinterpret_cast<float*>(base + kSmGate + s * kRecGates) + a * 64; }
  __device__ volatile int* abort_flag() const { return reinterpret_cast<volatile int*>(base + kSmMisc + 16); }
  __device__ uint32_t* tmem_slot() const { return reinterpret_cast<uint32_t*>(base + kSmMisc); }
  __device__ uint32_t addr(uint32_t off) const { return smem_u32(base + off); }
};

// Bounded wait that also gives up as soon as another role has aborted: first
// blocking tests (the hardware suspends the thread until the phase completes or
// a short time limit passes, so a waiting thread takes no issue slots), then
// tests with a longer suspend hint between abort and time-limit checks.
__device__ __forceinline__ bool wait_bar_flag(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
#pragma unroll 1
  for (int k = 0; k < 64; ++k)
    if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll 1
  while (true) {
    // suspended until the phase completes (or 0.1 ms), so waiting threads do not
    // take issue slots from the warps doing the work
    if (mbar_try_wait_sleep(addr, parity, 100000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(kDevErrWaitTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ bool wait_bar(const Smem& sm, uint64_t* bar, uint32_t parity) {
  return wait_bar_flag(bar, parity, sm.abort_flag());
}

// Longest chains first.  CTAs start in blockIdx order, so blockIdx.y is mapped to
// the sequences by decreasing length (ties: lower index first): the long chains
// start in the first wave and the short ones fill the tail of the last.  `rank`
// < N; the ranks of a strict total order are a permutation, so exactly one
// thread finds it.  Up to kLptMaxSeqs sequences (each thread ranks one sequence
// against all others); above that the identity order is kept.
constexpr int kLptMaxSeqs = 128;
__device__ int lpt_sequence(const PrefillParams& p, int rank, unsigned char* scratch) {
  if (p.N <= 1 || p.N > kLptMaxSeqs) return rank;
  int64_t* len = reinterpret_cast<int64_t*>(scratch);
  int* pick = reinterpret_cast<int*>(scratch + kLptMaxSeqs * sizeof(int64_t));
  const int tid = threadIdx.x;
  if (tid < p.N) len[tid] = load_cu(p, tid + 1) - load_cu(p, tid);
  __syncthreads();
  if (tid < p.N) {
    const int64_t mine = len[tid];
    int r = 0;
#pragma unroll 4
    for (int m = 0; m < p.N; ++m) {
      const int64_t o = len[m];
      r += (o > mine || (o == mine && m < tid)) ? 1 : 0;
    }
    if (r == rank) *pick = tid;
  }
  __syncthreads();
  return *pick;
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

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    prefill_chunk_kernel(const __grid_constant__ CUtensorMap mapK, const __grid_constant__ CUtensorMap mapQ,
                         const __grid_constant__ CUtensorMap mapV, const __grid_constant__ CUtensorMap mapO,
                         const __grid_constant__ CUtensorMap mapPhi, PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem sm;
  sm.base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int h = blockIdx.x;
  const int n = lpt_sequence(p, blockIdx.y, sm.base + kSmO);  // the output stage is free until the first chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qh = h / p.ratio;

  const int64_t cu0 = load_cu(p, n), cu1 = load_cu(p, n + 1);
  const bool bad = cu1 < cu0 || cu0 < 0 || cu1 > p.T;
  if (bad && tid == 0 && blockIdx.z == 0) raise_device_error(kDevErrBadSeqlens);
  const int64_t seq_len = bad ? 0 : cu1 - cu0;

  // ---- this CTA's task: a chunk range of the sequence, where its state starts and ends ----
  // cp_pass 0: the whole sequence from p.state to p.new_state, with outputs.
  // cp_pass 1 (z): 0 = segment 0 from p.state, with outputs, its final state -> kCpIn[0];
  //   2 s - 1 = M of segment s (identity start, v taken as 0), its outputs (the homogeneous
  //   outputs Phi) -> p.cp_phi, final state -> kCpMap[s - 1];
  //   2 s = C of segment s (zero start), its outputs -> p.out (corrected later by
  //   S_in Phi), final state -> kCpOff[s - 1]   (s = 1 .. S - 1).
  // cp_pass 2 (z): the sequence's map, no outputs: z = 2 s -> M, 2 s + 1 -> C of segment s;
  //   one segment: straight to p.map_m / p.map_c, else to the map scratch (composed later).
  const int S = p.cp_segments, cz = blockIdx.z;
  const int seg = p.cp_pass == 1 ? (cz + 1) >> 1 : (p.cp_pass == 2 ? cz >> 1 : 0);
  const bool emit = p.cp_pass == 0 || p.cp_pass == 1;                                // outputs written
  const bool homog = (p.cp_pass == 1 && (cz & 1)) || (p.cp_pass == 2 && !(cz & 1));  // identity start, v = 0
  // where the range's state starts (nullptr: zero, or the identity when homog) and ends
  // (nullptr: not stored); evaluated where used, to keep them out of the loops' registers
  auto init_block = [&]() -> const float* {
    if ((p.cp_pass == 1 && cz != 0) || p.cp_pass == 2) return nullptr;
    return p.state ? p.state + (size_t)n * p.s_sn + (size_t)h * p.s_sh : nullptr;
  };
  auto final_block = [&]() -> float* {
    if (p.cp_pass == 1)
      return p.cp_scratch + (cz == 0 ? cp_offset(p.N, p.HV, S, kCpIn, n, 0, h)
                                     : cp_offset(p.N, p.HV, S, (cz & 1) ? kCpMap : kCpOff, n, seg - 1, h));
    if (p.cp_pass == 2) {
      if (S > 1) return p.cp_scratch + map_seg_offset(p.N, p.HV, S, cz & 1, n, seg, h);
      return !(cz & 1) ? p.map_m + (size_t)n * p.m_sn + (size_t)h * p.m_sh : p.map_c + (size_t)n * p.c_sn + (size_t)h * p.c_sh;
    }
    return p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh;
  };
  const int nch_seq = (int)((seq_len + kC - 1) / kC);
  int cb = 0, ce = nch_seq;
  if (p.cp_pass == 1) {
    segment_range(nch_seq, S, p.cp_w0, seg, cb, ce);
  } else if (p.cp_pass == 2) {
    cb = (int)((int64_t)seg * nch_seq / S);
    ce = (int)((int64_t)(seg + 1) * nch_seq / S);
  }
  const int64_t t0 = cu0 + (int64_t)cb * kC;  // first token of the range
  const int64_t len = ce > cb ? (seq_len < (int64_t)ce * kC ? seq_len : (int64_t)ce * kC) - (int64_t)cb * kC : 0;
  const int nchunks = ce - cb;
  const int64_t slot0 = slot_start(cu0, n) + cb;  // workspace record slot of the range's chunk 0

  // chain threads: their 32 columns of the initial state (row (warp % 4) * 32 + lane, columns
  // (warp / 4) * 32 ..), loaded before the setup below so the memory round trip overlaps it
  float st_init[kStateCols];
  if (warp < kChainWarps) {
    const float* init_blk = init_block();
    const float* src =
        init_blk ? init_blk + (size_t)((warp & 3) * 32 + lane) * kHeadDim + (warp >> 2) * kStateCols : nullptr;
#pragma unroll
    for (int q = 0; q < kStateCols; q += 4) {
      const float4 f = src ? ld_nc_f4(src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      st_init[q] = f.x;
      st_init[q + 1] = f.y;
      st_init[q + 2] = f.z;
      st_init[q + 3] = f.w;
    }
  }

  // the T buffers' core matrices above the diagonal are never copied: zero them once
  for (int e = tid; e < (int)(2 * kTStage / 16); e += kThreads)
    reinterpret_cast<uint4*>(sm.base + kSmT)[e] = make_uint4(0u, 0u, 0u, 0u);
  tc::fence_proxy_async_smem();  // visible to the tensor core (async proxy) after the barrier below
  if (tid == 0) {
    for (int i = 0; i < B_COUNT; ++i)
      mbar_init(sm.bar(i), (i == B_GFREE || i == B_GFREE + 1 || i == B_S0_READY || i == B_D_READY) ? 2 : 1);
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
  // Lane 0 waits and issues; the 16 row-block copies of a chunk's T tiles are spread over
  // lanes 0-15 (all lanes follow lane 0's outcome, so they leave the loop together).
  if (warp == kWarpTma) {
    if (nchunks > 0) {
      if (lane == 0) {
        tc::prefetch_tensormap(&mapK);
        tc::prefetch_tensormap(&mapQ);
        tc::prefetch_tensormap(&mapV);
        tc::prefetch_tensormap(&mapO);
        if (homog && emit) tc::prefetch_tensormap(&mapPhi);
      }
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int s = i & 1;
        const uint32_t ph = ((i - 2) >> 1) & 1;  // phase of this stage's previous use (chunk i - 2)
        const int z = (int)(t0 + (int64_t)i * kC);
        const unsigned char* rec = record(p, slot0 + i, h);
        // waits in the order their phases complete: MMA2(i-2), deltas(i-2), MMA4(i-2), R(i-1).
        // One barrier counts the record's two parts and V (its phase completes once all landed;
        // V, the last, is issued once R of chunk i - 1 has read the previous V).
        int ok = 1;
        if (lane == 0) {
          ok = (i < 2 || wait_bar(sm, sm.bar(B_T_EMPTY + s), ph)) ? 1 : 0;
          if (ok) mbar_arrive_expect_tx(sm.bar(B_REC_FULL + s), kRecBytes + 16384);
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        if (lane < 16) {  // T hi / lo: row block rb of a tile is the run of its rb + 1 nonzero core matrices
          const int tile = lane >> 3, rb = lane & 7;
          bulk_g2s(sm.base + kSmT + s * kTStage + tile * kTTileBytes + rb * 1024,
                   rec + tile * kRecTile + tri_prefix(rb) * 128, (uint32_t)(rb + 1) * 128, sm.bar(B_REC_FULL + s));
        }
        if (lane == 0) {
          ok = 0;
          if (i < 2 || wait_bar(sm, sm.bar(B_GFREE + s), ph)) {
            bulk_g2s(sm.base + kSmGate + s * kRecGates, rec + kRecT, kRecGates, sm.bar(B_REC_FULL + s));
            if (i < 2 || wait_bar(sm, sm.bar(B_KQ_EMPTY + s), ph)) {
              uint64_t* full = sm.bar(B_KQ_FULL + s);
              mbar_arrive_expect_tx(full, 6 * 8192);
              unsigned char* kq = sm.base + kSmKQ + s * kKQStage;
#pragma unroll
              for (int f = 0; f < 2; ++f) {  // the two 64-feature tiles: Q, Q, K
                tc::tma_load_3d(kq + f * kKQTile, &mapQ, 64 * f, qh, z, full);
                tc::tma_load_3d(kq + f * kKQTile + kRowsQ2, &mapQ, 64 * f, qh, z, full);
                tc::tma_load_3d(kq + f * kKQTile + kRowsK, &mapK, 64 * f, qh, z, full);
              }
              if (i < 1 || wait_bar(sm, sm.bar(B_V_EMPTY), (i - 1) & 1)) {
                tc::tma_load_3d(sm.base + kSmV, &mapV, 0, h, z, sm.bar(B_REC_FULL + s));
                ok = 1;
              }
            }
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        issued = i + 1;
      }
      // drain: the last loads have landed before the CTA can exit (bounded)
      if (lane == 0 && issued > 0) {
        const int i = issued - 1, s = i & 1;
        wait_bar(sm, sm.bar(B_REC_FULL + s), (i >> 1) & 1);
        wait_bar(sm, sm.bar(B_KQ_FULL + s), (i >> 1) & 1);
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
      const uint64_t dD = tc::kmajor_desc(sm.addr(kSmD), 0, 0);
      // T tiles without swizzle: core matrices 128 B apart along K, row blocks 1 KB apart; one
      // MMA step of 16 columns is two core matrices (+256 B)
      const uint64_t dT0 = tc::sdesc_noswizzle(sm.addr(kSmT), 128u, 1024u);
      const uint64_t dT1 = tc::sdesc_noswizzle(sm.addr(kSmT + kTStage), 128u, 1024u);
      constexpr uint64_t kTlo = kTTileBytes >> 4;  // T lo follows T hi in a stage
      auto tstep = [](int ks) { return (uint64_t)(ks * 16); };
      const uint64_t dP = tc::kmajor_desc(sm.addr(kSmP), 0, 0);
      const uint64_t dKQ0 = tc::kmajor_desc(sm.addr(kSmKQ), 0, 0);
      const uint64_t dKQ1 = tc::kmajor_desc(sm.addr(kSmKQ + kKQStage), 0, 0);
      const uint64_t dKmn0 = tc::mnmajor_desc(sm.addr(kSmKQ + kRowsK), kKQTile, 0);
      const uint64_t dKmn1 = tc::mnmajor_desc(sm.addr(kSmKQ + kKQStage + kRowsK), kKQTile, 0);
      constexpr uint64_t kOffQ2 = kRowsQ2 >> 4, kOffK = kRowsK >> 4;  // descriptor offsets of the [Q; K] and K rows
      // [Q; Q] K^T of chunk j goes into D1[j & 1] columns 64-127 (Q K^T on lanes 0-63 and again
      // on 64-127); that half of the buffer was last read by the deltas of chunk j - 2
      // [Q; Q] K^T steps k0 .. k1 - 1 of chunk j (K = 128 in 8 steps of 16)
      auto kk_steps = [&](int j, int k0, int k1) {
        const uint64_t d = (j & 1) ? dKQ1 : dKQ0;
        const uint32_t dst = tmem + kTmD1 + (uint32_t)(j & 1) * 128 + 64;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          if (ks >= k0 && ks < k1)
            tc::mma_bf16(dst, d + kmajor_step(kKQTile, ks), d + kOffK + kmajor_step(kKQTile, ks), id_n64, ks > 0);
      };
      bool ok = wait_bar(sm, sm.bar(B_KQ_FULL), 0);
      if (ok) {
        tc::fence_after_sync();
        kk_steps(0, 0, 8);
        tc::mma_commit(sm.bar(B_KKQK));
      }
      // Probes of a barrier cost this thread several hundred cycles even when its phase is
      // complete, and the thread issues every MMA of the chain, so the waits on its critical
      // path are kept to one per MMA group: the preconditions of MMA1 (S0 split, Q K^T read by
      // the P warpgroup) share a barrier, and so do those of MMA4 and the output MMA (deltas,
      // P tile); the T record is covered by the chain's wait on the record before its split.
      for (int i = 0; ok && i < nchunks; ++i) {
        const int s = i & 1;
        const uint64_t dK = s ? dKQ1 : dKQ0;
        const uint64_t dKmn = s ? dKmn1 : dKmn0;
        const uint32_t d1 = tmem + kTmD1 + (uint32_t)s * 128;
        // MMA1: D1 = S0_hi [Q; K]^T (N = 128), then D1[:, K part] += S0_lo K^T
        if (!wait_bar(sm, sm.bar(B_S0_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16_ta(d1, tmem + kTmS0hi + 8 * ks, dK + kOffQ2 + kmajor_step(kKQTile, ks), id_n128, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16_ta(d1 + 64, tmem + kTmS0lo + 8 * ks, dK + kOffK + kmajor_step(kKQTile, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA1));
        // the next chunk's Q K^T in two halves, in the tensor pipe's idle windows: while the
        // chain computes R and while it computes the deltas
        const bool more = i + 1 < nchunks;
        if (more) {
          if (!wait_bar(sm, sm.bar(B_KQ_FULL + ((i + 1) & 1)), ((i + 1) >> 1) & 1)) break;
          tc::fence_after_sync();
          kk_steps(i + 1, 0, 4);
        }
        // MMA2: D^T = R^T T^T into D1 columns 64-127 (R and T split hi/lo: 3 products)
        if (!wait_bar(sm, sm.bar(B_R_READY), i & 1)) break;
        tc::fence_after_sync();
        const uint64_t dT = s ? dT1 : dT0;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ta(d1 + 64, tmem + kTmRhi + 8 * ks, dT + tstep(ks), id_n64, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ta(d1 + 64, tmem + kTmRlo + 8 * ks, dT + tstep(ks), id_n64, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ta(d1 + 64, tmem + kTmRhi + 8 * ks, dT + kTlo + tstep(ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA2));
        tc::mma_commit(sm.bar(B_T_EMPTY + s));
        if (more) {
          kk_steps(i + 1, 4, 8);
          tc::mma_commit(sm.bar(B_KKQK));
        }
        // state first: S += Dt^T K (hi/lo); then the output: D1[:, O part] += D^T P^T
        if (!wait_bar(sm, sm.bar(B_D_READY), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ta(tmem + kTmS, tmem + kTmDthi + 8 * ks, dKmn + mnmajor_step(ks), id_st, true);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16_ta(tmem + kTmS, tmem + kTmDtlo + 8 * ks, dKmn + mnmajor_step(ks), id_st, true);
        tc::mma_commit(sm.bar(B_MMA4 + s));
        tc::mma_commit(sm.bar(B_KQ_EMPTY + s));
        if (!wait_bar(sm, sm.bar(B_DTILE), i & 1)) break;
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_bf16(d1, dD + kmajor_step(0, ks), dP + kmajor_step(0, ks), id_n64, true);
        tc::mma_commit(sm.bar(B_MMA3));
      }
      // drain: every MMA issued above has completed before TMEM is released
      tc::mma_commit(sm.bar(B_DRAIN));
      wait_bar(sm, sm.bar(B_DRAIN), 0);
    }
  }
  // ======================================================================= P warpgroup
  else if (warp >= kWarpP0) {
    const int pth = tid - 32 * kWarpP0;  // 0..127; TMEM lane quarter = warp & 3
    const bool pleader = pth == 0;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32);
    const int v = (warp & 3) * 32 + lane;  // state row (TMEM lane) in the O^T passes
    __nv_bfloat16* ostage = reinterpret_cast<__nv_bfloat16*>(sm.base + kSmO);
    const float scale = p.scale;
    // outputs of chunk ci: o[t][v] = scale * O^T[v][t] (D1 buffer ci & 1, columns 0-63),
    // staged as bf16 rows in shared memory, then stored by TMA
    auto emit_out = [&](int ci) {
      const int64_t rem = len - (int64_t)ci * kC;
      const int nvalid = rem < kC ? (int)rem : kC;
      if (warp == kWarpP0) tc::bulk_wait_read_all();  // the previous chunk's row stores have read the stage
      named_sync(2, 128);
#pragma unroll 1
      for (int q16 = 0; q16 < (emit ? 4 : 0); ++q16) {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, kTmD1 + (uint32_t)(ci & 1) * 128 + q16 * 16), x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 16; ++u) ostage[(q16 * 16 + u) * kHeadDim + v] = __float2bfloat16_rn(scale * x[u]);
      }
      tc::fence_before_sync();
      tc::fence_proxy_async_smem();
      named_sync(2, 128);
      if (warp == kWarpP0 && emit) {
        // a pass-1 homogeneous chain writes Phi ([T][HV][128], rows contiguous) instead of out
        const bool to_phi = homog;
        if (nvalid == kC) {  // whole chunk: one tiled store of the [64 x 128] box
          if (lane == 0) tc::tma_store_3d(to_phi ? &mapPhi : &mapO, 0, h, (int)(t0 + (int64_t)ci * kC), ostage);
        } else {  // a sequence's last, partial chunk: only its own rows
          const int64_t ost = to_phi ? (int64_t)p.HV * kHeadDim : p.o_st;
          __nv_bfloat16* out = (to_phi ? p.cp_phi : p.out) + (t0 + (int64_t)ci * kC) * ost +
                               (int64_t)h * (to_phi ? (int64_t)kHeadDim : p.o_sh);
          for (int t = lane; t < nvalid; t += 32)
            tc::bulk_s2g(out + (int64_t)t * ost, ostage + t * kHeadDim, 256);
        }
        tc::bulk_commit();
      }
    };
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      const uint32_t d1 = kTmD1 + (uint32_t)s * 128;
      // ---- P rows from Q K^T (warps 10, 11: TMEM lanes 64-127), kept in registers until the
      //      P tile is free: P[t][j] = exp(g_t - g_j) q_t.k_j for j <= t ----
      if (!group_wait(sm, B_REC_FULL + s, (i >> 1) & 1, 2, 128, pleader)) break;
      if (!group_wait(sm, B_KKQK, i & 1, 2, 128, pleader)) break;
      tc::fence_after_sync();
      // P rows from Q K^T (D1 columns 64-127; every lane quarter holds the 64 Q rows):
      // thread (row r, column half ch) keeps P[r][32 ch .. 32 ch + 31] in registers until
      // the P tile is free; P[t][j] = exp(g_t - g_j) q_t.k_j for j <= t
      const int ch = (warp & 3) >> 1, prow_r = ((warp & 1) << 5) | lane;
      uint32_t prow[16];
      {
        // P[t][j] = exp2((g2_t + log2 m_t) - (g2_j - log2 n_j)) (q_t.k_j) = exp(g_t - g_j) q^_t.k^_j
        // (row and column terms of the gate arrays; m = n = 1 without the q/k L2 norm)
        const float* g2 = sm.gate(s, GA_G2C) + 32 * ch;
        const float gt = sm.gate(s, GA_G2)[prow_r];
        const uint32_t d0 = tc::tmem_addr(tmem, lane_base, d1 + 64 + 32 * ch);
#pragma unroll
        for (int q16 = 0; q16 < 2; ++q16) {
          float w[16];
          tc::tmem_ld16(d0 + q16 * 16, w);
          tc::tmem_wait_ld();
          if (32 * ch + 16 * q16 <= prow_r) {  // some j <= r in this group of 16
#pragma unroll
            for (int u4 = 0; u4 < 4; ++u4) {
              const float4 gj = *reinterpret_cast<const float4*>(g2 + 16 * q16 + 4 * u4);
              const int j = 32 * ch + 16 * q16 + 4 * u4;
              w[4 * u4 + 0] = j + 0 <= prow_r ? tc::ex2_approx(gt - gj.x) * w[4 * u4 + 0] : 0.f;
              w[4 * u4 + 1] = j + 1 <= prow_r ? tc::ex2_approx(gt - gj.y) * w[4 * u4 + 1] : 0.f;
              w[4 * u4 + 2] = j + 2 <= prow_r ? tc::ex2_approx(gt - gj.z) * w[4 * u4 + 2] : 0.f;
              w[4 * u4 + 3] = j + 3 <= prow_r ? tc::ex2_approx(gt - gj.w) * w[4 * u4 + 3] : 0.f;
            }
          } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) w[u] = 0.f;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) prow[8 * q16 + u] = pack_bf16x2(w[2 * u], w[2 * u + 1]);
        }
      }
      tc::fence_before_sync();
      named_sync(2, 128);
      if (pleader) mbar_arrive(sm.bar(B_S0_READY));  // this chunk's Q K^T has been read
      // ---- P tile, once the output MMA of chunk i-1 has read the previous one ----
      if (i >= 1 && !group_wait(sm, B_MMA3, (i - 1) & 1, 2, 128, pleader)) break;
      {
        unsigned char* pt = sm.base + kSmP;
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8)
          st_tile(pt, prow_r, 4 * ch + c8,
                  make_uint4(prow[c8 * 4], prow[c8 * 4 + 1], prow[c8 * 4 + 2], prow[c8 * 4 + 3]));
      }
      tc::fence_proxy_async_smem();
      // ---- outputs of chunk i-1 (its output MMA completed above) ----
      if (i >= 1) {
        tc::fence_after_sync();
        emit_out(i - 1);
      }
      // ---- S0 Q^T of chunk i scaled by G (column t by G_t), once the chain has read R's
      //      inputs (the first MMA is done; its TMEM traffic is over) ----
      if (!group_wait(sm, B_R_READY, i & 1, 2, 128, pleader)) break;
      tc::fence_after_sync();
      {
        const float* G = sm.gate(s, GA_G);
#pragma unroll 1
        for (int q16 = 0; q16 < 4; ++q16) {
          float x[16];
          const uint32_t ta = tc::tmem_addr(tmem, lane_base, d1 + q16 * 16);
          tc::tmem_ld16(ta, x);
          tc::tmem_wait_ld();
#pragma unroll
          for (int u4 = 0; u4 < 4; ++u4) {
            const float4 g4 = *reinterpret_cast<const float4*>(G + q16 * 16 + 4 * u4);
            x[4 * u4 + 0] *= g4.x;
            x[4 * u4 + 1] *= g4.y;
            x[4 * u4 + 2] *= g4.z;
            x[4 * u4 + 3] *= g4.w;
          }
          tc::tmem_st16(ta, x);
        }
        tc::tmem_wait_st();
      }
      tc::fence_before_sync();
      named_sync(2, 128);
      if (pleader) {
        mbar_arrive(sm.bar(B_D_READY));  // P tile written, S0 Q^T scaled
        mbar_arrive(sm.bar(B_GFREE + s));
      }
    }
    // ---- last chunk's outputs ----
    if (nchunks > 0 && group_wait(sm, B_MMA3, (nchunks - 1) & 1, 2, 128, pleader) && !*sm.abort_flag()) {
      tc::fence_after_sync();
      emit_out(nchunks - 1);
    }
    if (warp == kWarpP0) tc::bulk_wait_all();
  }
  // ======================================================================= chain warps
  else {
    const int quarter = warp & 3, hsel = warp >> 2;  // hsel: column slice 0..kCW-1
    const int v = quarter * 32 + lane;               // state row / TMEM lane
    const uint32_t lane_base = (uint32_t)(quarter * 32);
    const bool leader = tid == 0;
    const int sc = hsel * kStateCols;  // this thread's state columns [sc, sc + kStateCols)
    const int tb = hsel * kTokCols;    // this thread's token columns [tb, tb + kTokCols)
    // initial state (this thread's columns, loaded above) -> TMEM S: loaded, zero or the identity
    {
      if (homog) {
#pragma unroll
        for (int q = 0; q < kStateCols; ++q) st_init[q] = (sc + q == v) ? 1.f : 0.f;
      }
      tc::tmem_st32(tc::tmem_addr(tmem, lane_base, kTmS + sc), st_init);
      tc::tmem_wait_st();
    }
    unsigned char* dtile = sm.base + kSmD;
    const __nv_bfloat16* vt = reinterpret_cast<const __nv_bfloat16*>(sm.base + kSmV);
    for (int i = 0; i < nchunks; ++i) {
      const int s = i & 1;
      const uint32_t d1 = kTmD1 + (uint32_t)s * 128;
      if (!group_wait(sm, B_REC_FULL + s, (i >> 1) & 1, 1, kChainThreads, leader)) break;
      // ---- S0 hi/lo into TMEM (A of the first MMA): the thread's 32 state columns in one
      //      load, kept in registers for the G_C scaling below ----
      if (i > 0 && !group_wait(sm, B_MMA4 + ((i - 1) & 1), ((i - 1) >> 1) & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      float xs[kStateCols];
      tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, kTmS + sc), xs);
      tc::tmem_wait_ld();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) split2(xs[16 * half + 2 * u], xs[16 * half + 2 * u + 1], hi[u], lo[u]);
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmS0hi + sc / 2 + half * 8), hi);
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmS0lo + sc / 2 + half * 8), lo);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_S0_READY));
      // ---- S <- G_C * S while the first MMA runs (it reads only the hi/lo copies; the
      //      state MMA of this chunk comes after the deltas) ----
      {
        const float GC = sm.gate(s, GA_GC)[0];
#pragma unroll
        for (int q = 0; q < kStateCols; q += 2) {
          const float2 y = __fmul2_rn(make_float2(xs[q], xs[q + 1]), make_float2(GC, GC));
          xs[q] = y.x;
          xs[q + 1] = y.y;
        }
        tc::tmem_st32(tc::tmem_addr(tmem, lane_base, kTmS + sc), xs);
        tc::tmem_wait_st();
      }
      // ---- while the first MMA runs: beta_t V[t][v] and beta_t G_t of this thread's 16 token
      //      columns into registers ----
      static_assert(kTokCols == 16, "one 16-token piece per chain thread");
      float bv[16], bgx[16];
      {
        const float* bet = sm.gate(s, GA_BETA) + tb;
        const float* bg = sm.gate(s, GA_BG) + tb;
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const float4 b4 = *reinterpret_cast<const float4*>(bet + 4 * u4);
          const float4 g4 = *reinterpret_cast<const float4*>(bg + 4 * u4);
          const float bb[4] = {b4.x, b4.y, b4.z, b4.w}, gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int u = 4 * u4 + e;
            // a state map's homogeneous part takes v as 0
            bv[u] = homog ? 0.f : bb[e] * __bfloat162float(vt[(tb + u) * kHeadDim + v]);
            bgx[u] = -gg[e];  // negated: R = beta V - beta G x as one FMA
          }
        }
      }
      // ---- R^T = beta V^T - beta G (S0 K^T), split hi/lo into TMEM ----
      if (!group_wait(sm, B_MMA1, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      {
        float x[16];
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, d1 + 64 + tb), x);
        tc::tmem_wait_ld();
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float2 r = __ffma2_rn(make_float2(bgx[2 * u], bgx[2 * u + 1]), make_float2(x[2 * u], x[2 * u + 1]),
                                      make_float2(bv[2 * u], bv[2 * u + 1]));
          split2(r.x, r.y, hi[u], lo[u]);
        }
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmRhi + tb / 2), hi);
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmRlo + tb / 2), lo);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) {
        mbar_arrive(sm.bar(B_R_READY));
        mbar_arrive(sm.bar(B_V_EMPTY));
      }
      // ---- deltas: Dt^T = D^T exp(gC - g) (hi/lo into TMEM, state MMA) first; then D^T as a
      //      bf16 tile for the output MMA, after the state MMA has been released.  The decays
      //      exp(g_C - g_t) are loaded while MMA2 runs. ----
      float rdec[16];
      {
        const float* rr = sm.gate(s, GA_R) + tb;
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const float4 r4 = *reinterpret_cast<const float4*>(rr + 4 * u4);
          rdec[4 * u4] = r4.x;
          rdec[4 * u4 + 1] = r4.y;
          rdec[4 * u4 + 2] = r4.z;
          rdec[4 * u4 + 3] = r4.w;
        }
      }
      if (!group_wait(sm, B_MMA2, i & 1, 1, kChainThreads, leader)) break;
      tc::fence_after_sync();
      float d[16];
      {
        tc::tmem_ld16(tc::tmem_addr(tmem, lane_base, d1 + 64 + tb), d);
        tc::tmem_wait_ld();
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float2 e = __fmul2_rn(make_float2(d[2 * u], d[2 * u + 1]), make_float2(rdec[2 * u], rdec[2 * u + 1]));
          split2(e.x, e.y, hi[u], lo[u]);
        }
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmDthi + tb / 2), hi);
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, kTmDtlo + tb / 2), lo);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      named_sync(1, kChainThreads);
      if (leader) {
        mbar_arrive(sm.bar(B_D_READY));
        mbar_arrive(sm.bar(B_GFREE + s));
      }
      // the output MMA of chunk i - 1 (which read the tile) completed before MMA2 of chunk i
#pragma unroll
      for (int c8 = 0; c8 < 2; ++c8) {
        uint4 dd;
        dd.x = pack_bf16x2(d[8 * c8 + 0], d[8 * c8 + 1]);
        dd.y = pack_bf16x2(d[8 * c8 + 2], d[8 * c8 + 3]);
        dd.z = pack_bf16x2(d[8 * c8 + 4], d[8 * c8 + 5]);
        dd.w = pack_bf16x2(d[8 * c8 + 6], d[8 * c8 + 7]);
        st_tile(dtile, v, (tb >> 3) + c8, dd);
      }
      tc::fence_proxy_async_smem();
      named_sync(1, kChainThreads);
      if (leader) mbar_arrive(sm.bar(B_DTILE));
    }
    // ---- final state ----
    bool ok = true;
    if (nchunks > 0)
      ok = group_wait(sm, B_MMA4 + ((nchunks - 1) & 1), ((nchunks - 1) >> 1) & 1, 1, kChainThreads, leader) &&
           !*sm.abort_flag();
    float* fin_blk = final_block();
    if (ok && fin_blk) {
      tc::fence_after_sync();
      float* dst = fin_blk + (size_t)v * kHeadDim + sc;
#pragma unroll 1
      for (int c8 = 0; c8 < kStateCols / 8; ++c8) {
        float x[8];
        tc::tmem_ld8(tc::tmem_addr(tmem, lane_base, kTmS + sc + c8 * 8), x);
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

// Composition of the segment state maps (context parallelism):
// S_in(s + 1) = S_in(s) M_s + C_s for s = 1 .. S - 1, fp32 on the CUDA cores; S_in(S) is
// the sequence's final state (new_state).  S_in(1) comes from kCpIn[0] (p.cp_combine 0: the
// state leaving segment 0) or from p.state (3: the state entering a rank's range, also kept
// in kCpIn[0]).  With p.cp_combine 1 / 2 the same fold from the identity without the C
// terms / from zero gives the whole range's map M / C (into map_m / map_c).  The state rows
// are independent under the maps, so a CTA carries its 32 rows of one (sequence, v-head)
// through every step without synchronising with other CTAs.
// rows <- rows M + C (C optional) for a CTA's 32 state rows r0 .. r0 + 31 (thread: column c
// of 16 rows rh ..), then stored to out when given; M [128][128] and C's rows in global memory.
__device__ __forceinline__ void fold_rows(float (*rows)[kHeadDim], const float* M, const float* C, float* out, int r0,
                                          int c, int rh) {
  float acc[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) acc[r] = C ? C[(int64_t)(r0 + rh + r) * kHeadDim + c] : 0.f;
#pragma unroll 2
  for (int k = 0; k < kHeadDim; k += 4) {
    const float m0 = M[(k + 0) * kHeadDim + c], m1 = M[(k + 1) * kHeadDim + c];
    const float m2 = M[(k + 2) * kHeadDim + c], m3 = M[(k + 3) * kHeadDim + c];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(&rows[rh + r][k]);
      acc[r] = fmaf(x.x, m0, acc[r]);
      acc[r] = fmaf(x.y, m1, acc[r]);
      acc[r] = fmaf(x.z, m2, acc[r]);
      acc[r] = fmaf(x.w, m3, acc[r]);
    }
  }
  __syncthreads();  // every thread has read the rows
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    rows[rh + r][c] = acc[r];
    if (out) out[(int64_t)(r0 + rh + r) * kHeadDim + c] = acc[r];
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) prefill_combine_kernel(PrefillParams p) {
  __shared__ __align__(16) float rows[32][kHeadDim];
  const int h = blockIdx.x, n = blockIdx.y, r0 = blockIdx.z * 32;
  const int tid = threadIdx.x, c = tid & 127, rh = (tid >> 7) * 16;  // column; first of 16 rows
  const int S = p.cp_segments, mode = p.cp_combine;
  float* in0 = p.cp_scratch + cp_offset(p.N, p.HV, S, kCpIn, n, 0, h);
  if (mode == 3 && p.cp_prev_count > 0) {
    // the state entering the range: S = 0, S <- S M_j + C_j over the preceding ranges' maps
    for (int e = tid; e < 32 * kHeadDim; e += 256) rows[e / kHeadDim][e % kHeadDim] = 0.f;
    __syncthreads();
    for (int j = 0; j < p.cp_prev_count; ++j) {
      const float* M = p.cp_prev + (((int64_t)(2 * j) * p.N + n) * p.HV + h) * kStateFloats;
      const float* C = p.cp_prev + (((int64_t)(2 * j + 1) * p.N + n) * p.HV + h) * kStateFloats;
      fold_rows(rows, M, C, j + 1 == p.cp_prev_count ? in0 : nullptr, r0, c, rh);  // S_in(1) kept
    }
  } else if (mode == 0 || mode == 3) {
    const float* src = mode == 0 ? in0 + (int64_t)r0 * kHeadDim
                       : p.state ? p.state + (size_t)n * p.s_sn + (size_t)h * p.s_sh + (int64_t)r0 * kHeadDim
                                 : nullptr;  // zero incoming state
    for (int e = tid; e < 32 * kHeadDim / 4; e += 256) {
      const float4 x = src ? reinterpret_cast<const float4*>(src)[e] : make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(&rows[0][0])[e] = x;
      if (mode == 3) reinterpret_cast<float4*>(in0 + (int64_t)r0 * kHeadDim)[e] = x;  // S_in(1), for the correction
    }
    __syncthreads();
  } else {
    for (int e = tid; e < 32 * kHeadDim; e += 256)
      rows[e / kHeadDim][e % kHeadDim] = (mode == 1 && r0 + e / kHeadDim == e % kHeadDim) ? 1.f : 0.f;
    __syncthreads();
  }
  for (int sg = 1; sg <= S - 1; ++sg) {
    const float* M = p.cp_scratch + cp_offset(p.N, p.HV, S, kCpMap, n, sg - 1, h);
    const float* C = mode == 1 ? nullptr : p.cp_scratch + cp_offset(p.N, p.HV, S, kCpOff, n, sg - 1, h);
    float* out = nullptr;
    if (sg < S - 1) {
      if (mode == 0 || mode == 3) out = p.cp_scratch + cp_offset(p.N, p.HV, S, kCpIn, n, sg, h);
    } else {
      out = mode == 1   ? p.map_m + (size_t)n * p.m_sn + (size_t)h * p.m_sh
            : mode == 2 ? p.map_c + (size_t)n * p.c_sn + (size_t)h * p.c_sh
                        : p.new_state + (size_t)n * p.n_sn + (size_t)h * p.n_sh;
    }
    fold_rows(rows, M, C, out, r0, c, rh);
  }
}

// Output correction of the context-parallel segments (after pass 1 and the map
// composition, cp_segments >= 2).  Every (sequence, v-head) state evolves affinely in its
// initial state, and so do the outputs: for a token t of segment s >= 1,
//   o_t = o_t(zero initial state) + S_in(s) Phi_t,
// with Phi_t the output of the segment's homogeneous chain (run from the identity, v = 0).
// Pass 1 wrote the first term to out and Phi to p.cp_phi; this kernel adds the second:
//   out[t][v] += sum_j S_in(s)[v][j] Phi[t][j].
// tcgen05: D [128 v x 64 tokens] = S_in [128 v x 128 j] Phi^T per chunk, S_in split into
// bf16 hi + lo (two products) and held in TMEM as the A operand, Phi from shared memory,
// fp32 accumulation in TMEM (two 64-column buffers).  256 TMEM columns and 97 KB of shared
// memory per CTA, so two CTAs share an SM.
// CTA = (v-head, sequence, segment - 1 and a part of its chunks: grid z = (S - 1) x
// p.cp_parts), looping over those chunks; 6 warps:
//   0-3  thread = state row v: S_in hi / lo into TMEM (while the first loads are in
//        flight), then per chunk D from TMEM added to the out tile in shared memory,
//        which is stored back (TMA)
//   4    TMA loads of the Phi tile and the out tile, kStages deep
//   5    TMEM allocation and the MMA issue
namespace corr {
constexpr int kThreads = 192;
constexpr int kStages = 3;            // shared-memory stages (Phi tile | out tile)
constexpr int kDBufs = 2;             // TMEM accumulators
constexpr uint32_t kSmStage = 0;      // kStages x (Phi chunk: 2 SW128 tiles [64 tokens x 64 j], 8 KB each |
constexpr uint32_t kStageBytes = 32768;  //            out tile [64 tokens][128 v] bf16, plain, 16 KB)
constexpr uint32_t kOOff = 16384;
constexpr uint32_t kSmBar = kSmStage + kStages * kStageBytes;
constexpr uint32_t kSmMisc = kSmBar + 128;
constexpr uint32_t kSmBytes = kSmMisc + 32;
constexpr uint32_t kSmAlloc = kSmBytes + 1024;
constexpr uint32_t kTmemCols = 256;   // A hi [0, 64), A lo [64, 128) (bf16 pairs), D buffers [128, 256)
constexpr uint32_t kTmAhi = 0, kTmAlo = 64, kTmD = 128;
enum : int {
  B_FULL = 0,                    // [kStages] Phi and out tiles landed
  B_EMPTY = kStages,             // [kStages] the stage's out tile has been read by its store
  B_MMA = 2 * kStages,           // [kDBufs] D of a chunk complete
  B_TFREE = 2 * kStages + kDBufs,  // [kDBufs] the epilogue has read a D buffer
  B_AREADY = 2 * kStages + 2 * kDBufs,
  B_DRAIN,
  B_COUNT
};
static_assert(B_COUNT * 8 <= 128 && kTmD + kDBufs * 64 <= kTmemCols && 2 * (kSmAlloc + 1024) <= 232448, "layout");
}  // namespace corr

__global__ void __launch_bounds__(corr::kThreads, 2)
    prefill_correct_kernel(const __grid_constant__ CUtensorMap mapPhi, const __grid_constant__ CUtensorMap mapO,
                           PrefillParams p) {
  using corr::kDBufs;
  using corr::kStages;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int parts = p.cp_parts;
  const int h = blockIdx.x, n = blockIdx.y, seg = (int)blockIdx.z / parts + 1, part = (int)blockIdx.z % parts;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.cp_segments;
  const int64_t cu0 = load_cu(p, n), cu1 = load_cu(p, n + 1);
  const bool bad = cu1 < cu0 || cu0 < 0 || cu1 > p.T;
  const int64_t seq_len = bad ? 0 : cu1 - cu0;
  int sb = 0, se = 0;
  segment_range((int)((seq_len + kC - 1) / kC), S, p.cp_w0, seg, sb, se);
  const int cb = sb + (se - sb) * part / parts, ce = sb + (se - sb) * (part + 1) / parts;
  const int nchunks = ce - cb;
  if (nchunks <= 0) return;  // the same for every thread of the CTA, before any barrier
  const int64_t t0 = cu0 + (int64_t)cb * kC;
  const int64_t len = (seq_len < (int64_t)ce * kC ? seq_len : (int64_t)ce * kC) - (int64_t)cb * kC;
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + corr::kSmBar);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(base + corr::kSmMisc + 16);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + corr::kSmMisc);

  if (tid == 0) {
    for (int i = 0; i < corr::B_COUNT; ++i) mbar_init(&bar[i], i == corr::B_AREADY ? 4 : 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(tmem_slot, corr::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---- TMA: Phi tile (two 64-column SW128 boxes) and the out tile of each chunk ----
    if (lane == 0) {
      tc::prefetch_tensormap(&mapPhi);
      tc::prefetch_tensormap(&mapO);
      int issued = 0;
      for (int i = 0; i < nchunks; ++i) {
        const int st = i % kStages;
        if (i >= kStages && !wait_bar_flag(&bar[corr::B_EMPTY + st], ((i - kStages) / kStages) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bar[corr::B_FULL + st], corr::kStageBytes);
        const int z = (int)(t0 + (int64_t)i * kC);
        unsigned char* b = base + corr::kSmStage + st * corr::kStageBytes;
        tc::tma_load_3d(b, &mapPhi, 0, h, z, &bar[corr::B_FULL + st]);
        tc::tma_load_3d(b + 8192, &mapPhi, 64, h, z, &bar[corr::B_FULL + st]);
        tc::tma_load_3d(b + corr::kOOff, &mapO, 0, h, z, &bar[corr::B_FULL + st]);
        issued = i + 1;
      }
      if (issued > 0) {
        const int i = issued - 1;
        wait_bar_flag(&bar[corr::B_FULL + i % kStages], (i / kStages) & 1, abort_flag);
      }
    }
  } else if (warp == 5) {
    // ---- MMA: D[buf] = S_in_hi Phi^T + S_in_lo Phi^T (K = 128 in 8 steps of 16 each) ----
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(128, 64, false, false);
      bool ok = wait_bar_flag(&bar[corr::B_AREADY], 0, abort_flag);
      for (int i = 0; ok && i < nchunks; ++i) {
        const int st = i % kStages, db = i % kDBufs;
        if (!wait_bar_flag(&bar[corr::B_FULL + st], (i / kStages) & 1, abort_flag)) break;
        // TMEM buffer db was last read by the epilogue of chunk i - kDBufs
        if (i >= kDBufs && !wait_bar_flag(&bar[corr::B_TFREE + db], ((i - kDBufs) / kDBufs) & 1, abort_flag)) break;
        tc::fence_after_sync();
        const uint64_t dB = tc::kmajor_desc(smem_u32(base + corr::kSmStage + st * corr::kStageBytes), 0, 0);
        const uint32_t d = tmem + corr::kTmD + (uint32_t)db * 64;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16_ta(d, tmem + corr::kTmAhi + 8 * ks, dB + tc::kmajor_step(8192, ks), idesc, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          tc::mma_bf16_ta(d, tmem + corr::kTmAlo + 8 * ks, dB + tc::kmajor_step(8192, ks), idesc, true);
        tc::mma_commit(&bar[corr::B_MMA + db]);
      }
      tc::mma_commit(&bar[corr::B_DRAIN]);
      wait_bar_flag(&bar[corr::B_DRAIN], 0, abort_flag);
    }
  } else {
    const uint32_t lane_base = (uint32_t)(warp * 32);
    // ---- S_in(seg) as bf16 hi / lo pairs in TMEM (A operand): thread v writes state row v ----
    {
      const float* src = p.cp_scratch + cp_offset(p.N, p.HV, S, kCpIn, n, seg - 1, h) + (size_t)tid * kHeadDim;
#pragma unroll 1
      for (int c16 = 0; c16 < 8; ++c16) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 x = ld_nc_f4(src + c16 * 16 + 4 * q);
          split2(x.x, x.y, hi[2 * q], lo[2 * q]);
          split2(x.z, x.w, hi[2 * q + 1], lo[2 * q + 1]);
        }
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, corr::kTmAhi + c16 * 8), hi);
        tc::tmem_st8u(tc::tmem_addr(tmem, lane_base, corr::kTmAlo + c16 * 8), lo);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[corr::B_AREADY]);  // one arrival per warp
    }
    // ---- epilogue: out tile += D^T, stored back (thread = state row v = tid) ----
    for (int i = 0; i < nchunks; ++i) {
      const int st = i % kStages, db = i % kDBufs;
      int ok = 1;
      if (tid == 0)
        ok = (wait_bar_flag(&bar[corr::B_FULL + st], (i / kStages) & 1, abort_flag) &&
              wait_bar_flag(&bar[corr::B_MMA + db], (i / kDBufs) & 1, abort_flag))
                 ? 1
                 : 0;
      int all;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
          : "=r"(all)
          : "r"(ok)
          : "memory");
      if (!all) break;
      tc::fence_after_sync();
      __nv_bfloat16* ot = reinterpret_cast<__nv_bfloat16*>(base + corr::kSmStage + st * corr::kStageBytes + corr::kOOff);
      float x[64];
      tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, corr::kTmD + (uint32_t)db * 64), *reinterpret_cast<float(*)[32]>(x));
      tc::tmem_ld32(tc::tmem_addr(tmem, lane_base, corr::kTmD + (uint32_t)db * 64 + 32),
                    *reinterpret_cast<float(*)[32]>(x + 32));
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      named_sync(1, 128);
      if (tid == 0) mbar_arrive(&bar[corr::B_TFREE + db]);  // D buffer read: the next MMA may overwrite it
#pragma unroll
      for (int u = 0; u < 64; ++u) {
        __nv_bfloat16* e = ot + u * kHeadDim + tid;
        *e = __float2bfloat16_rn(__bfloat162float(*e) + x[u]);
      }
      tc::fence_proxy_async_smem();  // the tile is read by the TMA store
      named_sync(1, 128);
      if (tid == 0) {
        const int64_t rem = len - (int64_t)i * kC;
        const int nvalid = rem < kC ? (int)rem : kC;
        const int64_t z = t0 + (int64_t)i * kC;
        if (nvalid == kC) {
          tc::tma_store_3d(&mapO, 0, h, (int)z, ot);
        } else {  // the sequence's last, partial chunk: only its own rows
          __nv_bfloat16* out = p.out + z * p.o_st + (int64_t)h * p.o_sh;
          for (int t = 0; t < nvalid; ++t) tc::bulk_s2g(out + (int64_t)t * p.o_st, ot + t * kHeadDim, 256);
        }
        tc::bulk_commit();
        // the previous chunk's store has read its tile (this one's may still be reading):
        // that stage may be refilled
        if (i >= 1) {
          asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          mbar_arrive(&bar[corr::B_EMPTY + (i - 1) % kStages]);
        }
      }
    }
    if (tid == 0) tc::bulk_wait_all();
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, corr::kTmemCols);
  }
}

int device_sm_count() {
  static int cached[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace

namespace {
// Composition of segment maps into the map of the whole range: M = M_0 M_1 .. M_{S-1},
// C = (..((C_0 M_1 + C_1) M_2 + C_2) ..).  z = row block (4) x {M, C}; fp32 CUDA cores.
__global__ void __launch_bounds__(256) map_combine_kernel(PrefillParams p) {
  __shared__ __align__(16) float rows[32][kHeadDim];
  const int h = blockIdx.x, n = blockIdx.y, r0 = (blockIdx.z & 3) * 32, which = blockIdx.z >> 2;
  const int tid = threadIdx.x, c = tid & 127, rh = (tid >> 7) * 16;
  const int S = p.cp_segments;
  const float* first = p.cp_scratch + map_seg_offset(p.N, p.HV, S, which, n, 0, h) + (int64_t)r0 * kHeadDim;
  for (int e = tid; e < 32 * kHeadDim / 4; e += 256)
    reinterpret_cast<float4*>(&rows[0][0])[e] = reinterpret_cast<const float4*>(first)[e];
  __syncthreads();
  float acc[16];
  for (int sg = 1; sg < S; ++sg) {
    const float* M = p.cp_scratch + map_seg_offset(p.N, p.HV, S, 0, n, sg, h);
    const float* C = p.cp_scratch + map_seg_offset(p.N, p.HV, S, 1, n, sg, h) + (int64_t)r0 * kHeadDim;
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = which ? C[(rh + r) * kHeadDim + c] : 0.f;
#pragma unroll 2
    for (int k = 0; k < kHeadDim; k += 4) {
      const float m0 = M[(k + 0) * kHeadDim + c], m1 = M[(k + 1) * kHeadDim + c];
      const float m2 = M[(k + 2) * kHeadDim + c], m3 = M[(k + 3) * kHeadDim + c];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const float4 x = *reinterpret_cast<const float4*>(&rows[rh + r][k]);
        acc[r] = fmaf(x.x, m0, acc[r]);
        acc[r] = fmaf(x.y, m1, acc[r]);
        acc[r] = fmaf(x.z, m2, acc[r]);
        acc[r] = fmaf(x.w, m3, acc[r]);
      }
    }
    __syncthreads();  // every thread has read the rows of the previous product
#pragma unroll
    for (int r = 0; r < 16; ++r) rows[rh + r][c] = acc[r];
    __syncthreads();
  }
  float* dst = which ? p.map_c + (size_t)n * p.c_sn + (size_t)h * p.c_sh : p.map_m + (size_t)n * p.m_sn + (size_t)h * p.m_sh;
#pragma unroll
  for (int r = 0; r < 16; ++r) dst[(int64_t)(r0 + rh + r) * kHeadDim + c] = rows[rh + r][c];
}
}  // namespace

cudaError_t launch_prefill_combine(const PrefillParams& p, cudaStream_t stream) {
  if (p.cp_segments < 2) return cudaSuccess;
  prefill_combine_kernel<<<dim3(p.HV, p.N, kHeadDim / 32), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

namespace {
// How the chunked prefill cuts sequences into context-parallel segments.
struct CpPlan {
  int S = 1;      // segments per sequence (1: none)
  int w0 = 1024;  // segment 0's share of a sequence's chunks, in 1/1024
};

// Makespan, in chain-lengths, of longest-first list scheduling of `na` jobs of length a and
// `nb` jobs of length b on m SMs (CTAs start in blockIdx order as SMs free up).
double lpt_makespan(int64_t na, double a, int64_t nb, double b, int64_t m) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> load;
  for (int64_t i = 0; i < m; ++i) load.push(0.0);
  auto place = [&](int64_t cnt, double len) {
    for (int64_t i = 0; i < cnt; ++i) {
      const double x = load.top();
      load.pop();
      load.push(x + len);
    }
  };
  if (a >= b) {
    place(na, a);
    place(nb, b);
  } else {
    place(nb, b);
    place(na, a);
  }
  double mk = 0.0;
  while (!load.empty()) {
    mk = load.top() > mk ? load.top() : mk;
    load.pop();
  }
  return mk;
}

// Automatic plan for c (sequence, v-head) chains of about 2^lg_chunks chunks on m SMs.
// Without segments the chains take waves(c) = ceil(c / m) chain-lengths.  With S segments,
// segment 0 (fraction a of the chunks) is one chain with outputs and every later segment
// two (its maps, with the homogeneous outputs), so pass 1 is c jobs of length a and
// 2 c (S - 1) jobs of length (1 - a) / (S - 1), each plus a fixed ~2 chunks (CTA start,
// pipeline fill), then the output correction (one memory-bound pass over the later
// segments' tokens, ~0.0035 c (1 - a) chain-lengths, measured) and the map composition
// (~0.01).
// Candidates: S in [2, 8], segment 0 1 .. 4 times as long as the others; used if it saves
// at least 10 %.
CpPlan cp_plan_auto(int64_t chains, int64_t sms, int lg_chunks) {
  static std::mutex mu;
  static std::map<std::pair<int64_t, int64_t>, CpPlan> cache;
  const std::pair<int64_t, int64_t> key(chains * 64 + lg_chunks, sms);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  CpPlan plan;
  const double one = (double)((chains + sms - 1) / sms);
  if (chains < 4 * sms) {
    double best = one;
    const double eps = 2.0 / (double)(1LL << lg_chunks);
    const double ks[] = {1.0, 1.5, 2.0, 2.5, 3.0, 4.0};
    for (int sg = 2; sg <= 8; ++sg) {
      for (double k : ks) {
        const double a = k / (k + sg - 1);
        const double cost =
            lpt_makespan(chains, a + eps, 2 * chains * (sg - 1), (1.0 - a) / (sg - 1) + eps, sms) +
            0.0035 * (double)chains * (1.0 - a) + 0.01;
        if (cost < best - 1e-9) {
          best = cost;
          plan.S = sg;
          plan.w0 = (int)(a * 1024.0 + 0.5);
        }
      }
    }
    if (best > 0.9 * one) plan = CpPlan();
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = plan;
  return plan;
}

CpPlan cp_plan(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  const int req = (int)((flags >> kPrefillSegmentsShift) & 15u);
  if (req >= 1) return CpPlan{req, req > 1 ? 1024 / req : 1024};  // forced: equal segments
  // automatic, for sequences of 16 chunks or more on average
  const int64_t chains = (int64_t)num_seqs * num_v_heads;
  if (chains <= 0 || total_tokens < (int64_t)num_seqs * 16 * kC) return CpPlan();
  int lg = 4;  // floor(log2(average chunks per sequence)), 16 .. 2^20
  while (lg < 20 && total_tokens >= (int64_t)num_seqs * kC * (2LL << lg)) ++lg;
  return cp_plan_auto(chains, device_sm_count(), lg);
}
}  // namespace

int prefill_cp_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  return cp_plan(num_seqs, total_tokens, num_v_heads, flags).S;
}

int prefill_map_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  const int req = (int)((flags >> kPrefillSegmentsShift) & 15u);
  if (req >= 1) return req;
  // automatic: a map takes two chains per (sequence, v-head) (M and C); S segments of
  // 1/S of the chunks each take waves(2 c S) segment-lengths against waves(2 c) for one.
  // The cheapest S in [2, 8] (the smallest on ties) if it saves at least 10 %, for
  // sequences of 16 chunks or more on average.
  const int64_t chains = (int64_t)num_seqs * num_v_heads;
  if (chains <= 0 || total_tokens < (int64_t)num_seqs * 16 * kC) return 1;
  const int64_t sms = device_sm_count();
  auto waves = [&](int64_t ctas) { return (double)((ctas + sms - 1) / sms); };
  const double one = waves(2 * chains);
  double best = one;
  int best_s = 1;
  for (int sg = 2; sg <= 8; ++sg) {
    const double cost = waves(2 * chains * sg) / sg;
    if (cost < best - 1e-9) {
      best = cost;
      best_s = sg;
    }
  }
  return best <= 0.9 * one ? best_s : 1;
}

size_t prefill_map_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  if (num_seqs <= 0 || total_tokens <= 0 || num_v_heads <= 0) return 0;
  const size_t records = (size_t)chunk::num_slots(total_tokens, num_seqs) * (size_t)num_v_heads * chunk::kRecBytes;
  const int S = prefill_map_segments(num_seqs, total_tokens, num_v_heads, flags);
  if (S <= 1) return records;
  return ((records + 255) & ~(size_t)255) + (size_t)2 * S * num_seqs * num_v_heads * kStateFloats * sizeof(float);
}

namespace {
// Workspace of the chunked prefill: [records][context-parallel states and maps][Phi (the
// segments' homogeneous outputs, [T][HV][128] bf16)][q norms (GDN_FLAG_QK_L2NORM: [T][HQ]
// float2, sized for HV >= HQ heads)], each part 256-byte aligned; no segment parts without
// segments.
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
size_t chunk_records_bytes(int num_seqs, int64_t total_tokens, int num_v_heads) {
  return (size_t)chunk::num_slots(total_tokens, num_seqs) * (size_t)num_v_heads * chunk::kRecBytes;
}
size_t cp_states_bytes(int num_seqs, int num_v_heads, int S) {
  return (size_t)cp_floats(num_seqs, num_v_heads, S) * sizeof(float);
}
size_t chunk_records_and_cp_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  const size_t records = chunk_records_bytes(num_seqs, total_tokens, num_v_heads);
  const int S = prefill_cp_segments(num_seqs, total_tokens, num_v_heads, flags);
  if (S <= 1) return records;
  return align256(records) + align256(cp_states_bytes(num_seqs, num_v_heads, S)) +
         (size_t)total_tokens * (size_t)num_v_heads * kHeadDim * sizeof(__nv_bfloat16);
}
}  // namespace

size_t prefill_chunk_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  if (num_seqs <= 0 || total_tokens <= 0 || num_v_heads <= 0) return 0;
  const size_t base = chunk_records_and_cp_bytes(num_seqs, total_tokens, num_v_heads, flags);
  if (!(flags & kFlagQkL2Norm)) return base;
  return ((base + 255) & ~(size_t)255) + (size_t)total_tokens * (size_t)num_v_heads * sizeof(float2);
}

bool prefill_chunk_supported(const PrefillParams& p) {
  auto ok16 = [](const void* ptr, int64_t a, int64_t b) {
    return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && ((a * 2) & 15) == 0 && ((b * 2) & 15) == 0;
  };
  if (p.T <= 0) return false;
  // the prep kernel's records
  if (!p.workspace || (reinterpret_cast<uintptr_t>(p.workspace) & 15) ||
      p.workspace_bytes < prefill_chunk_workspace_bytes(p.N, p.T, p.HV, p.flags))
    return false;
  // output rows leave through 256-byte bulk stores
  if ((reinterpret_cast<uintptr_t>(p.out) & 15) || (p.o_st & 7) || (p.o_sh & 7)) return false;
  return ok16(p.q, p.q_st, p.q_sh) && ok16(p.k, p.k_st, p.k_sh) && ok16(p.v, p.v_st, p.v_sh);
}

namespace {
// Tensor maps of one call, the prep launch and the chain kernel's shared-memory opt-in.
// A state-map call has no output tensor: its output map is built on q (never stored to).
cudaError_t prefill_setup(const PrefillParams& p, cudaStream_t stream, CUtensorMap* mk, CUtensorMap* mq,
                          CUtensorMap* mv, CUtensorMap* mo) {
  const bool map_only = p.cp_pass == 2;
  if (!make_map(mk, p.k, p.T, p.HQ, p.k_st, p.k_sh, 64, true) ||
      !make_map(mq, p.q, p.T, p.HQ, p.q_st, p.q_sh, 64, true) ||
      !make_map(mv, p.v, p.T, p.HV, p.v_st, p.v_sh, 128, false) ||
      !make_map(mo, map_only ? const_cast<__nv_bfloat16*>(p.q) : p.out, p.T, map_only ? p.HQ : p.HV,
                map_only ? p.q_st : p.o_st, map_only ? p.q_sh : p.o_sh, 128, false))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaSuccess;
  if (p.flags & kFlagQkL2Norm) {
    if (!p.qnorm) return cudaErrorInvalidValue;  // the q norms live in the caller's workspace
    e = launch_qk_norm(p, stream);
    if (e != cudaSuccess) return e;
  }
  e = launch_prefill_prep(p, *mk, stream);
  if (e != cudaSuccess) return e;
  // The dynamic shared-memory opt-in is a per-device function attribute.
  static bool attr_set[64] = {};
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmAlloc);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  return cudaSuccess;
}

__global__ void identity_maps_kernel(PrefillParams p) {
  const int h = blockIdx.x, n = blockIdx.y;
  float* m = p.map_m + (size_t)n * p.m_sn + (size_t)h * p.m_sh;
  float* c = p.map_c + (size_t)n * p.c_sn + (size_t)h * p.c_sh;
  for (int e = threadIdx.x; e < kHeadDim * kHeadDim; e += blockDim.x) {
    m[e] = (e / kHeadDim == e % kHeadDim) ? 1.f : 0.f;
    c[e] = 0.f;
  }
}
}  // namespace

cudaError_t launch_identity_maps(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  identity_maps_kernel<<<dim3(p.HV, p.N), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill_state_map(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  PrefillParams q = p;
  const int S = prefill_map_segments(p.N, p.T, p.HV, p.flags);
  q.cp_segments = S;
  q.cp_pass = 2;
  q.out = nullptr;
  q.new_state = nullptr;
  if (S > 1) {
    const size_t records = (size_t)chunk::num_slots(p.T, p.N) * (size_t)p.HV * chunk::kRecBytes;
    q.cp_scratch =
        reinterpret_cast<float*>(static_cast<unsigned char*>(p.workspace) + ((records + 255) & ~(size_t)255));
  }
  CUtensorMap mk, mq, mv, mo;
  cudaError_t e = prefill_setup(q, stream, &mk, &mq, &mv, &mo);
  if (e != cudaSuccess) return e;
  prefill_chunk_kernel<<<dim3(p.HV, p.N, 2 * S), kThreads, kSmAlloc, stream>>>(mk, mq, mv, mo, mo, q);
  e = cudaGetLastError();
  if (e != cudaSuccess || S == 1) return e;
  map_combine_kernel<<<dim3(p.HV, p.N, 8), 256, 0, stream>>>(q);
  return cudaGetLastError();
}

namespace {
// The output correction of segments 1 .. S - 1 (q.cp_w0: segment 0's share of the chunks);
// each CTA corrects ~16 chunks of one segment.
cudaError_t launch_correct(PrefillParams q, const CUtensorMap& mphi_ld, const CUtensorMap& mo, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    e = cudaFuncSetAttribute(prefill_correct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)corr::kSmAlloc);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int S = q.cp_segments;
  const int64_t seg_chunks = (q.T / q.N / kC) * (1024 - q.cp_w0) / 1024 / (S - 1);
  q.cp_parts = (int)(seg_chunks / 16 < 1 ? 1 : (seg_chunks / 16 > 64 ? 64 : seg_chunks / 16));
  prefill_correct_kernel<<<dim3(q.HV, q.N, (S - 1) * q.cp_parts), corr::kThreads, corr::kSmAlloc, stream>>>(
      mphi_ld, mo, q);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_prefill_chunk(const PrefillParams& p_in, cudaStream_t stream) {
  if (p_in.N == 0) return cudaSuccess;
  PrefillParams p = p_in;
  if (p.flags & kFlagQkL2Norm) {
    const size_t base = chunk_records_and_cp_bytes(p.N, p.T, p.HV, p.flags);
    p.qnorm = reinterpret_cast<float2*>(static_cast<unsigned char*>(p.workspace) + align256(base));
  }
  CUtensorMap mk, mq, mv, mo;
  cudaError_t e = prefill_setup(p, stream, &mk, &mq, &mv, &mo);
  if (e != cudaSuccess) return e;
  const CpPlan plan = cp_plan(p.N, p.T, p.HV, p.flags);
  if (plan.S <= 1) {
    PrefillParams q = p;
    q.cp_segments = 1;
    q.cp_pass = 0;
    prefill_chunk_kernel<<<dim3(p.HV, p.N), kThreads, kSmAlloc, stream>>>(mk, mq, mv, mo, mo, q);
    return cudaGetLastError();
  }
  // context parallelism: segment 0 and the later segments' maps with their homogeneous
  // outputs (one launch), the map composition (initial states, final state), the output
  // correction of the later segments
  const int S = plan.S;
  unsigned char* ws = static_cast<unsigned char*>(p.workspace);
  const size_t states_at = align256(chunk_records_bytes(p.N, p.T, p.HV));
  PrefillParams q = p;
  q.cp_segments = S;
  q.cp_w0 = plan.w0;
  q.cp_pass = 1;
  q.cp_scratch = reinterpret_cast<float*>(ws + states_at);
  q.cp_phi = reinterpret_cast<__nv_bfloat16*>(ws + states_at + align256(cp_states_bytes(p.N, p.HV, S)));
  CUtensorMap mphi_st, mphi_ld;
  const int64_t phi_st = (int64_t)p.HV * kHeadDim;
  if (!make_map(&mphi_st, q.cp_phi, p.T, p.HV, phi_st, kHeadDim, 128, false) ||
      !make_map(&mphi_ld, q.cp_phi, p.T, p.HV, phi_st, kHeadDim, 64, true))
    return cudaErrorInvalidValue;
  prefill_chunk_kernel<<<dim3(p.HV, p.N, 2 * S - 1), kThreads, kSmAlloc, stream>>>(mk, mq, mv, mo, mphi_st, q);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = launch_prefill_combine(q, stream);
  if (e != cudaSuccess) return e;
  return launch_correct(q, mphi_ld, mo, stream);
}

// ---- context parallelism across GPUs: a later token range of each sequence ----

int prefill_range_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  // S - 1 map-pair segments (segment 0 is empty): forced by the segment flag (n pairs), else
  // the count k in [1, 8] minimising waves(2 c k) / k (+ ~2 chunks per CTA), with at least
  // 4 chunks per segment on average
  const int req = (int)((flags >> kPrefillSegmentsShift) & 15u);
  if (req >= 1) return req + 1;
  const int64_t chains = (int64_t)num_seqs * num_v_heads;
  if (chains <= 0 || num_seqs <= 0) return 2;
  const double avg_chunks = (double)total_tokens / (double)num_seqs / kC;
  const int64_t sms = device_sm_count();
  double best = 1e30;
  int best_k = 1;
  for (int k = 1; k <= 8; ++k) {
    if (k > 1 && avg_chunks < 4.0 * k) break;
    const double waves = (double)((2 * chains * k + sms - 1) / sms);
    const double cost = waves * (1.0 / k + (avg_chunks > 0 ? 2.0 / avg_chunks : 0.0));
    if (cost < best - 1e-9) {
      best = cost;
      best_k = k;
    }
  }
  return best_k + 1;
}

size_t prefill_range_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags) {
  if (num_seqs <= 0 || num_v_heads <= 0) return 0;
  const int S = prefill_range_segments(num_seqs, total_tokens, num_v_heads, flags);
  return align256(chunk_records_bytes(num_seqs, total_tokens, num_v_heads)) +
         align256(cp_states_bytes(num_seqs, num_v_heads, S)) +
         (size_t)total_tokens * (size_t)num_v_heads * kHeadDim * sizeof(__nv_bfloat16);
}

namespace {
// The range's parameters: segment 0 empty (w0 = 0), S - 1 map-pair segments, the
// scratch and Phi in the workspace after the records.
PrefillParams range_params(const PrefillParams& p) {
  PrefillParams q = p;
  const int S = prefill_range_segments(p.N, p.T, p.HV, p.flags);
  unsigned char* ws = static_cast<unsigned char*>(p.workspace);
  const size_t states_at = align256(chunk_records_bytes(p.N, p.T, p.HV));
  q.cp_segments = S;
  q.cp_w0 = 0;
  q.cp_pass = 1;
  q.cp_scratch = reinterpret_cast<float*>(ws + states_at);
  q.cp_phi = reinterpret_cast<__nv_bfloat16*>(ws + states_at + align256(cp_states_bytes(p.N, p.HV, S)));
  return q;
}
}  // namespace

cudaError_t launch_prefill_range_affine(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  PrefillParams q = range_params(p);
  q.state = nullptr;  // segment 0 is empty; the map pairs start from the identity and from zero
  q.new_state = nullptr;
  CUtensorMap mk, mq, mv, mo, mphi_st;
  cudaError_t e = prefill_setup(q, stream, &mk, &mq, &mv, &mo);
  if (e != cudaSuccess) return e;
  if (!make_map(&mphi_st, q.cp_phi, p.T, p.HV, (int64_t)p.HV * kHeadDim, kHeadDim, 128, false))
    return cudaErrorInvalidValue;
  prefill_chunk_kernel<<<dim3(p.HV, p.N, 2 * q.cp_segments - 1), kThreads, kSmAlloc, stream>>>(mk, mq, mv, mo,
                                                                                              mphi_st, q);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  for (int mode = 1; mode <= 2; ++mode) {  // the range's M, then its C
    q.cp_combine = mode;
    e = launch_prefill_combine(q, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_prefill_range_finish(const PrefillParams& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  PrefillParams q = range_params(p);
  q.cp_combine = 3;  // from the incoming state p.state to new_state, keeping every segment's start
  cudaError_t e = launch_prefill_combine(q, stream);
  if (e != cudaSuccess) return e;
  if (p.T <= 0) return cudaSuccess;
  CUtensorMap mo, mphi_ld;
  if (!make_map(&mo, p.out, p.T, p.HV, p.o_st, p.o_sh, 128, false) ||
      !make_map(&mphi_ld, q.cp_phi, p.T, p.HV, (int64_t)p.HV * kHeadDim, kHeadDim, 64, true))
    return cudaErrorInvalidValue;
  return launch_correct(q, mphi_ld, mo, stream);
}

}  // namespace gdn
