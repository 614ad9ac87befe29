// Pieces shared by the two kernels of the chunked prefill (sm_100a):
//   prefill_prep_kernel   (gdn_prefill_prep.cu)   state-independent per-chunk
//                         work for every chunk of every (sequence, v-head) at
//                         once: gates, A, T = (I + A)^-1 and its bf16 split
//   prefill_chunk_kernel  (gdn_prefill_chunk.cu)  the sequential state chain
// They meet in the workspace: one record per (chunk slot, v-head).
//
// Chunk slots.  cu_seqlens lives on the device, so the host sizes the workspace
// from (num_seqs, total_tokens) alone: chunk i of sequence n (tokens
// [cu[n] + 64 i, min(cu[n] + 64 (i + 1), cu[n + 1]))) owns slot
//   slot(n, i) = floor(cu[n] / 64) + n + i.
// For monotone cu_seqlens the slots of different sequences never collide
// (floor(c0/64) + ceil((c1-c0)/64) <= floor(c1/64) + 1) and every slot is
// below total_tokens / 64 + num_seqs + 1.
//
// Record (kRecBytes, 16-byte aligned), written by the prep kernel and bulk-copied
// into shared memory by the chain kernel:
//   [0, 4608)      T hi: the lower triangle of T [64 rows t][64 cols j] bf16 as the 36
//                  nonzero 8x8 core matrices of a K-major tile without swizzle, row
//                  block by row block, core matrices 0 .. rb of row block rb contiguous
//                  (128 B each: 8 rows of 16 B)
//   [4608, 9216)   T lo: same, T - hi
//   [9216, 11008)  gates: 7 x 64 fp32 (GA_* order below)
// In shared memory a T tile is the full [8 row blocks][8 core matrices] array (1 KB per
// row block, LBO 128 B along K, SBO 1 KB along the rows); the chain kernel zeroes its
// T buffers once, so the core matrices above the diagonal, never copied, stay zero.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gdn_common.cuh"
#include "gdn_kernels.h"
#include "gdn_tc.cuh"

namespace gdn {
namespace chunk {

constexpr int kC = 64;  // chunk length (tokens)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr uint32_t kTriCM = 36;                   // nonzero core matrices of a 64 x 64 lower triangle
constexpr uint32_t kRecTile = kTriCM * 128;       // one compacted T tile: 4608 B
constexpr uint32_t kRecT = 2 * kRecTile;          // T hi | T lo
constexpr uint32_t kRecGates = 1792;              // 7 x 64 fp32
constexpr uint32_t kRecBytes = kRecT + kRecGates; // 11008
constexpr uint32_t kTTileBytes = 8192;            // a full T tile in shared memory
static_assert(kRecBytes % 16 == 0 && kRecTile % 16 == 0, "record alignment");
// core matrices of the compacted tile before row block rb
__host__ __device__ constexpr uint32_t tri_prefix(int rb) { return (uint32_t)(rb * (rb + 1) / 2); }

// gate arrays (per chunk, 64 tokens each), with n_t = 1 / |k_t| and m_t = 1 / |q_t| when q
// and k are L2-normalised in the kernels (GDN_FLAG_QK_L2NORM), n_t = m_t = 1 otherwise:
//   GA_G2   g2_t + log2 m_t, g2_t = log2 e * sum_{i<=t} log g_i the log2-scaled decay prefix
//           (row term of the decayed Q K^T product)
//   GA_BETA beta_t
//   GA_G    G_t m_t, G_t = exp(g_t) (scales column t of S0 Q^T)
//   GA_BG   beta_t G_t n_t
//   GA_R    exp(g_C - g_t) n_t (the decay to the chunk end)
//   GA_G2C  g2_t - log2 n_t (column term of the decayed K K^T and Q K^T products)
//   GA_GC   G_C = exp(g_C) in every entry
// The normalisation is folded into these per-token factors: q and k stay raw bf16 in
// every product, so the chain kernel is the same with and without it.  Tokens past the
// sequence end carry beta = 0, log g = 0 (the prefix stays flat) and n = m = 1, so they
// change nothing.
enum : int { GA_G2 = 0, GA_BETA = 1, GA_G = 2, GA_BG = 3, GA_R = 4, GA_G2C = 5, GA_GC = 6, GA_N = 7 };

// 1 / sqrt(sum of squares + eps): the L2 normalisation factor (eps 1e-6, as the decode and
// token-serial kernels use).
__device__ __forceinline__ float l2_factor(float sumsq) { return rsqrtf(sumsq + 1e-6f); }

__host__ __device__ inline int64_t num_slots(int64_t total_tokens, int num_seqs) {
  return total_tokens / kC + num_seqs + 1;
}

// Context-parallel scratch (a sequence's chunks cut into S >= 2 segments): three arrays of
// [N][S - 1][HV][128 x 128] fp32 states, idx = segment - 1:
//   kCpIn  the initial state of segment idx + 1
//   kCpMap M of segment idx + 1 (its state map is S_out = S_in M + C)
//   kCpOff C of segment idx + 1
// followed (256-byte aligned) by Phi [T][HV][128] bf16: the outputs of each segment's
// homogeneous chain (run from the identity with v = 0), for the output correction.
enum CpArray { kCpIn = 0, kCpMap = 1, kCpOff = 2 };
constexpr int64_t kStateFloats = 128 * 128;
__host__ __device__ inline int64_t cp_floats(int N, int HV, int S) {
  return S < 2 ? 0 : (int64_t)N * HV * kStateFloats * 3 * (S - 1);
}
__host__ __device__ inline int64_t cp_offset(int N, int HV, int S, int which, int n, int idx, int h) {
  const int64_t per_array = (int64_t)N * (S - 1) * HV * kStateFloats;
  return which * per_array + (((int64_t)n * (S - 1) + idx) * HV + h) * kStateFloats;
}
// Chunk range [cb, ce) of segment `seg` of a sequence of `nch` chunks cut into S segments:
// segment 0 (one chain, with outputs) takes w0 / 1024 of the chunks, the others (two chains
// each: the maps) share the rest evenly.
__host__ __device__ inline void segment_range(int nch, int S, int w0, int seg, int& cb, int& ce) {
  const int c0 = S <= 1 ? nch : (int)(((int64_t)nch * w0) >> 10);
  if (seg == 0) {
    cb = 0;
    ce = c0;
    return;
  }
  const int rest = nch - c0;
  cb = c0 + (int)((int64_t)(seg - 1) * rest / (S - 1));
  ce = c0 + (int)((int64_t)seg * rest / (S - 1));
}

// State-map scratch when the map of each sequence is computed in S segments:
// [2 (M, C)][N][S][HV][128 x 128] fp32.
__host__ __device__ inline int64_t map_seg_offset(int N, int HV, int S, int which, int n, int sg, int h) {
  return ((((int64_t)which * N + n) * S + sg) * HV + h) * kStateFloats;
}

__device__ __forceinline__ int64_t load_cu(const PrefillParams& p, int i) {
  return p.cu_is_int64 ? reinterpret_cast<const int64_t*>(p.cu_seqlens)[i]
                       : (int64_t) reinterpret_cast<const int32_t*>(p.cu_seqlens)[i];
}

__device__ __forceinline__ int64_t slot_start(int64_t cu_n, int n) { return (cu_n >> 6) + n; }

__device__ __forceinline__ unsigned char* record(const PrefillParams& p, int64_t slot, int h) {
  return static_cast<unsigned char*>(p.workspace) + ((size_t)slot * (size_t)p.HV + (size_t)h) * kRecBytes;
}

__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// (a, b) -> bf16x2 hi and bf16x2 lo with a = hi + lo to ~16 mantissa bits.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(a, b);
  // both residuals (a, b) - hi in one packed fp32x2 FMA (exact: hi is a's / b's leading bits)
  const float2 r = __ffma2_rn(make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u)),
                              make_float2(-1.f, -1.f), make_float2(a, b));
  lo = pack_bf16x2(r.x, r.y);
}

// 16-byte store of 8 bf16 (columns 8*c8 .. 8*c8+7 of `row`) into a SW128 tile.
__device__ __forceinline__ void st_tile(unsigned char* tile, int row, int c8, uint4 w) {
  *reinterpret_cast<uint4*>(tile + tc::sw128_offset(row, c8 * 8)) = w;
}

// Gates of one token (kernel_prefill.py:108-113): log g = -exp(A_log) softplus(a + dt_bias)
// with softplus(x) = x for x > 20, and beta = sigmoid(b); hardware exp2 / log2.
__device__ __forceinline__ void token_gates(float eA, float dt_bias, float a, float b, float& lg, float& beta) {
  const float x = a + dt_bias;
  const float sp = x > 20.f ? x : kLn2 * tc::lg2_approx(1.f + tc::ex2_approx(x * kLog2e));
  lg = -eA * sp;
  beta = 1.f / (1.f + tc::ex2_approx(-b * kLog2e));
}

}  // namespace chunk

// Launches the prep kernel over every chunk slot and v-head (mapK: the chain
// kernel's K tensor map, 64-token x 64-feature SW128 boxes).
cudaError_t launch_prefill_combine(const PrefillParams& p, cudaStream_t stream);
cudaError_t launch_prefill_prep(const PrefillParams& p, const CUtensorMap& mapK, cudaStream_t stream);
// 1 / |q| and log2 (1 / |q|) of every (token, q/k head) into p.qnorm (GDN_FLAG_QK_L2NORM).
cudaError_t launch_qk_norm(const PrefillParams& p, cudaStream_t stream);

}  // namespace gdn
