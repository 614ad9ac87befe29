// Internal launch interface between the C ABI (gdn_abi.cu) and the kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr uint32_t kFlagQkL2Norm = 1u;        // mirrors GDN_FLAG_QK_L2NORM
constexpr uint32_t kFlagPrefillSerial = 2u;   // mirrors GDN_FLAG_PREFILL_SERIAL
constexpr uint32_t kFlagSelftestWaitTimeout = 1u << 31;  // mirrors GDN_FLAG_SELFTEST_WAIT_TIMEOUT
// Wait limit of the self-test: long enough to leave the fast spin, short enough for a test.
constexpr unsigned long long kSelftestWaitLimitNs = 1000000ull;  // 1 ms

// Strides are in elements; the innermost (feature) stride is 1 for every tensor.
struct DecodeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* state;  // nullptr -> zero initial state
  const float* A_log;
  const __nv_bfloat16* a;
  const float* dt_bias;
  const __nv_bfloat16* b;
  __nv_bfloat16* out;
  float* new_state;
  int64_t q_sb, q_sh, k_sb, k_sh, v_sb, v_sh;
  int64_t s_sb, s_sh;  // state: [B, HV, 128, 128], rows contiguous
  int64_t a_sb, b_sb;  // a, b: [B, HV] (head stride 1)
  int64_t o_sb, o_sh;  // out: [B, HV, 128]
  int64_t n_sb, n_sh;  // new_state: [B, HV, 128, 128], rows contiguous
  float scale;
  int B, HQ, HV, ratio;
  uint32_t flags;
  // pooled form (one token against a state pool): sequence b reads slot indices[b] of `state`
  // (a pool of P slots, s_sb = slot stride) and writes the same slot of `new_state`; a negative
  // index is a padded entry (zero outputs), one >= P raises GDN_DEVERR_BAD_INDEX
  const void* indices = nullptr;
  int idx_is_int64 = 0;
  int64_t P = 0;
};

struct PrefillParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* state;  // nullptr -> zero initial state
  const float* A_log;
  const __nv_bfloat16* a;
  const float* dt_bias;
  const __nv_bfloat16* b;
  const void* cu_seqlens;  // [N + 1], int32 or int64 (device)
  int cu_is_int64;
  __nv_bfloat16* out;
  float* new_state;
  int64_t q_st, q_sh, k_st, k_sh, v_st, v_sh;
  int64_t s_sn, s_sh;
  int64_t a_st, b_st;
  int64_t o_st, o_sh;
  int64_t n_sn, n_sh;
  float scale;
  int N, HQ, HV, ratio;
  int64_t T;
  uint32_t flags;
  void* workspace;
  size_t workspace_bytes;
  // context parallelism inside the GPU (set by the chunked launcher): each sequence's
  // chunks split into cp_segments ranges (segment 0 takes cp_w0 / 1024 of them);
  // cp_pass 0 = one chain per sequence, 1 = segment 0 and the maps and homogeneous
  // outputs of the others; cp_scratch = segment states and maps, cp_phi = the
  // homogeneous outputs [T][HV][128]
  int cp_segments = 1;
  int cp_pass = 0;
  int cp_w0 = 0;
  int cp_parts = 1;  // output correction: CTAs per segment (each a contiguous part of its chunks)
  // map composition: 0 = segment initial states from kCpIn[0] (in-GPU prefill), 3 = from
  // state (a range's incoming state, also copied to kCpIn[0]), both ending in new_state;
  // 1 = the range's M (from the identity, no C) into map_m, 2 = its C (from zero) into map_c
  int cp_combine = 0;
  // cp_combine 3: when cp_prev_count > 0 the incoming state is the fold S = 0,
  // S <- S M_j + C_j over cp_prev [cp_prev_count][2 (M, C)][N][HV][128][128] (p.state unused)
  const float* cp_prev = nullptr;
  int cp_prev_count = 0;
  float* cp_scratch = nullptr;
  __nv_bfloat16* cp_phi = nullptr;
  // GDN_FLAG_QK_L2NORM: per (token, q/k head) (1 / |q|, log2 (1 / |q|)), [T][HQ] (workspace)
  float2* qnorm = nullptr;
  // cp_pass 2: each sequence's affine state map S_out = S_in M + C instead of a prefill
  float* map_m = nullptr;
  float* map_c = nullptr;
  int64_t m_sn = 0, m_sh = 0, c_sn = 0, c_sh = 0;
};

// Multi-token decode against a state pool (serving form).  Strides in elements;
// q, k [B, T, HQ, 128], v [B, T, HV, 128], a, b [B, T, HV], out [B, T, HV, 128],
// pool / new_pool [P, HV, 128, 128] (rows contiguous), intermediate [P, T, HV, 128, 128].
struct DecodeMtpParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const float* pool;
  float* new_pool;  // may equal pool
  const void* indices;  // [B] int32 or int64 (device)
  int idx_is_int64;
  const float* A_log;
  const __nv_bfloat16* a;
  const float* dt_bias;
  const __nv_bfloat16* b;
  __nv_bfloat16* out;
  float* inter;  // nullptr: not cached
  int64_t q_sb, q_st, q_sh, k_sb, k_st, k_sh, v_sb, v_st, v_sh;
  int64_t a_sb, a_st, b_sb, b_st;
  int64_t o_sb, o_st, o_sh;
  int64_t s_sn, s_sh;  // pool
  int64_t n_sn, n_sh;  // new_pool
  int64_t i_sn, i_st, i_sh;  // intermediate
  float scale;
  int B, T, P, HQ, HV, ratio;
  uint32_t flags;
  uint32_t hv_mul;  // n / HV = (umulhi(n, hv_mul) + n) >> hv_shr for n < 2^31 (set by the launcher)
  int hv_shr;
};

int decode_rows_for(int B, int HV);
cudaError_t launch_decode_mtp(const DecodeMtpParams& p, cudaStream_t stream);
cudaError_t launch_decode(const DecodeParams& p, int rows, cudaStream_t stream);

cudaError_t launch_prefill_serial(const PrefillParams& p, cudaStream_t stream);

// Chunked tensor-core prefill: usable when q/k/v rows and strides are 16-byte
// aligned (TMA), no in-kernel q/k normalisation is requested and the workspace
// holds prefill_chunk_workspace_bytes (one record per chunk slot and v-head).
size_t prefill_chunk_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
// Segments per sequence the chunked prefill uses for this problem (1 = none):
// flags bits kPrefillSegmentsShift .. + 3 request a count (0 = automatic).
constexpr int kPrefillSegmentsShift = 8;
int prefill_cp_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
// Context parallelism across GPUs, a rank holding a later token range of each sequence: the
// range as map-pair segments only, with outputs from a zero initial state and the
// homogeneous outputs (launch_prefill_range_affine: out, map_m, map_c), then, once the state
// entering the range is known (p.state), the output correction and the final state
// (launch_prefill_range_finish).  Both take the same workspace (prefill_range_workspace_bytes).
int prefill_range_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
size_t prefill_range_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
cudaError_t launch_prefill_range_affine(const PrefillParams& p, cudaStream_t stream);
cudaError_t launch_prefill_range_finish(const PrefillParams& p, cudaStream_t stream);
bool prefill_chunk_supported(const PrefillParams& p);
cudaError_t launch_prefill_chunk(const PrefillParams& p, cudaStream_t stream);
// Per sequence the affine map of its token range, M [HV][K][K] and C [HV][V][K]
// (S_out = S_in M + C): the chunked chain from the identity with v = 0 and from zero,
// in prefill_map_segments(...) segments whose maps are then composed.
cudaError_t launch_prefill_state_map(const PrefillParams& p, cudaStream_t stream);
int prefill_map_segments(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
size_t prefill_map_workspace_bytes(int num_seqs, int64_t total_tokens, int num_v_heads, uint32_t flags);
// The maps of empty token ranges: M = I, C = 0 for every sequence and v-head.
cudaError_t launch_identity_maps(const PrefillParams& p, cudaStream_t stream);

}  // namespace gdn
