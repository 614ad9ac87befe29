// C ABI of libgdn_b200.so (declared in include/gdn_b200.h).
//
// Host-side argument validation, workspace sizing and kernel dispatch.  No
// allocation, no synchronisation: every call only enqueues kernels on the
// caller's stream.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_kernels.h"

namespace gdn {
__device__ unsigned int g_gdn_device_error = 0;
}

namespace {

// Scratch of gdn_prefill_noalloc: a static device array in the library's module, so that
// entry point allocates nothing.  64 MiB holds 3,692 prepared chunk records (18,176 B each),
// e.g. total_tokens / 64 + num_seqs + 1 <= 115 chunk slots at 32 v-heads.  No part of it needs
// to start at zero: the prep kernel writes every record before the chain kernel reads it.
constexpr size_t kStaticScratchBytes = size_t(GDN_PREFILL_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
std::mutex g_scratch_mutex;
void* g_scratch_addr[64] = {};  // per device, looked up once with that device current

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return GDN_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned(const void* p, int64_t stride_elems, int64_t stride2_elems, size_t elem, size_t align) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  return a % align == 0 && ((uint64_t)(stride_elems * (int64_t)elem)) % align == 0 &&
         ((uint64_t)(stride2_elems * (int64_t)elem)) % align == 0;
}

// Byte extent [lo, hi) touched by a [n0, n1, 128, 128] fp32 tensor with strides (s0, s1).
void state_extent(const float* p, int64_t n0, int64_t n1, int64_t s0, int64_t s1, uintptr_t& lo, uintptr_t& hi) {
  const int64_t last = (n0 - 1) * s0 + (n1 - 1) * s1 + (int64_t)gdn::kHeadDim * gdn::kHeadDim;
  lo = reinterpret_cast<uintptr_t>(p);
  hi = lo + (uintptr_t)last * sizeof(float);
}

int check_common(int32_t HQ, int32_t HV, int32_t D) {
  if (D != gdn::kHeadDim) return fail(GDN_ERR_UNSUPPORTED, "head_dim must be 128 (got %d)", D);
  if (HQ <= 0 || HV <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "head counts must be positive (qk %d, v %d)", HQ, HV);
  if (HV % HQ != 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_v_heads (%d) must be a multiple of num_qk_heads (%d)", HV, HQ);
  return GDN_OK;
}

int check_state_pair(const float* state, int64_t s0, int64_t s1, const float* new_state, int64_t n0, int64_t n1,
                     int64_t count, int32_t HV) {
  if (!new_state) return fail(GDN_ERR_INVALID_ARGUMENT, "new_state must not be NULL");
  if (!aligned(new_state, n0, n1, sizeof(float), 16))
    return fail(GDN_ERR_UNSUPPORTED, "new_state rows must be 16-byte aligned (base and strides)");
  if (state && !aligned(state, s0, s1, sizeof(float), 16))
    return fail(GDN_ERR_UNSUPPORTED, "state rows must be 16-byte aligned (base and strides)");
  if (n1 < 0 || n0 < 0 || s0 < 0 || s1 < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "negative state stride");
  if (state && count > 0) {
    uintptr_t alo, ahi, blo, bhi;
    state_extent(state, count, HV, s0, s1, alo, ahi);
    state_extent(new_state, count, HV, n0, n1, blo, bhi);
    const bool overlap = alo < bhi && blo < ahi;
    const bool identical = state == new_state && s0 == n0 && s1 == n1;
    if (overlap && !identical)
      return fail(GDN_ERR_INVALID_ARGUMENT, "new_state partially overlaps state (only exact aliasing is allowed)");
  }
  return GDN_OK;
}

}  // namespace

extern "C" {

int gdn_version(void) { return 100; }

const char* gdn_last_error(void) { return g_last_error.c_str(); }

int gdn_device_error(uint32_t* bits_out, int clear) {
  unsigned int bits = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&bits, gdn::g_gdn_device_error, sizeof(bits));
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
  if (bits_out) *bits_out = bits;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(gdn::g_gdn_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device error word");
  }
  return ok();
}

int gdn_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k, int64_t k_stride_b,
               int64_t k_stride_h, const void* v, int64_t v_stride_b, int64_t v_stride_h, const float* state,
               int64_t state_stride_b, int64_t state_stride_h, const float* A_log, const void* a,
               int64_t a_stride_b, const float* dt_bias, const void* b, int64_t b_stride_b, float scale, void* out,
               int64_t out_stride_b, int64_t out_stride_h, float* new_state, int64_t new_state_stride_b,
               int64_t new_state_stride_h, int32_t batch, int32_t num_qk_heads, int32_t num_v_heads,
               int32_t head_dim, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (batch < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "batch must be >= 0 (got %d)", batch);
  if (batch > 65535) return fail(GDN_ERR_UNSUPPORTED, "batch > 65535 per call is not supported (got %d)", batch);
  if (flags & ~(GDN_FLAG_QK_L2NORM | GDN_FLAG_SELFTEST_WAIT_TIMEOUT))
    return fail(GDN_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags);
  if (batch == 0) return ok();
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !out)
    return fail(GDN_ERR_INVALID_ARGUMENT, "a required tensor pointer is NULL");
  if (!aligned(q, q_stride_b, q_stride_h, 2, 8) || !aligned(k, k_stride_b, k_stride_h, 2, 8) ||
      !aligned(v, v_stride_b, v_stride_h, 2, 8))
    return fail(GDN_ERR_UNSUPPORTED, "q/k/v rows must be 8-byte aligned (base and strides)");
  rc = check_state_pair(state, state_stride_b, state_stride_h, new_state, new_state_stride_b, new_state_stride_h,
                        batch, num_v_heads);
  if (rc) return rc;

  gdn::DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state = state;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.new_state = new_state;
  p.q_sb = q_stride_b;
  p.q_sh = q_stride_h;
  p.k_sb = k_stride_b;
  p.k_sh = k_stride_h;
  p.v_sb = v_stride_b;
  p.v_sh = v_stride_h;
  p.s_sb = state_stride_b;
  p.s_sh = state_stride_h;
  p.a_sb = a_stride_b;
  p.b_sb = b_stride_b;
  p.o_sb = out_stride_b;
  p.o_sh = out_stride_h;
  p.n_sb = new_state_stride_b;
  p.n_sh = new_state_stride_h;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  p.B = batch;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.flags = flags;
  const cudaError_t e =
      gdn::launch_decode(p, gdn::decode_rows_for(batch, num_v_heads), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_decode launch");
  return ok();
}

size_t gdn_prefill_workspace_size(int32_t num_seqs, int64_t total_tokens, int32_t num_qk_heads, int32_t num_v_heads,
                                  int32_t head_dim, uint32_t flags) {
  (void)num_qk_heads;
  (void)head_dim;
  // gdn_prefill_range_affine / _finish: records, segment states and maps, homogeneous outputs
  if (flags & GDN_FLAG_RANGE_AFFINE)
    return gdn::prefill_range_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
  // gdn_prefill_state_map: records + the per-segment maps
  if (flags & GDN_FLAG_STATE_MAP) return gdn::prefill_map_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
  // the token-serial kernel (forced) needs none; the chunked kernel keeps one prepared
  // record per chunk slot and v-head (with or without in-kernel q/k normalisation)
  if (flags & GDN_FLAG_PREFILL_SERIAL) return 0;
  return gdn::prefill_chunk_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
}

int gdn_decode_pooled(const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                      int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_b,
                      int64_t v_stride_t, int64_t v_stride_h, const float* pool, int64_t pool_stride_n,
                      int64_t pool_stride_h, const void* indices, int32_t indices_is_int64, const float* A_log,
                      const void* a, int64_t a_stride_b, int64_t a_stride_t, const float* dt_bias, const void* b,
                      int64_t b_stride_b, int64_t b_stride_t, float scale, void* out, int64_t out_stride_b,
                      int64_t out_stride_t, int64_t out_stride_h, float* new_pool, int64_t new_pool_stride_n,
                      int64_t new_pool_stride_h, float* intermediate, int64_t inter_stride_n, int64_t inter_stride_t,
                      int64_t inter_stride_h, int32_t batch, int32_t tokens, int32_t pool_size, int32_t num_qk_heads,
                      int32_t num_v_heads, int32_t head_dim, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (batch < 0 || tokens < 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "batch and tokens must be >= 0 (got %d, %d)", batch, tokens);
  if (batch > 65535) return fail(GDN_ERR_UNSUPPORTED, "batch > 65535 per call is not supported (got %d)", batch);
  if (flags & ~(GDN_FLAG_QK_L2NORM | GDN_FLAG_SELFTEST_WAIT_TIMEOUT))
    return fail(GDN_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags);
  if (batch == 0 || tokens == 0) return ok();
  if (pool_size <= 0) return fail(GDN_ERR_INVALID_ARGUMENT, "pool_size must be positive (got %d)", pool_size);
  if (!q || !k || !v || !pool || !indices || !A_log || !a || !dt_bias || !b || !out)
    return fail(GDN_ERR_INVALID_ARGUMENT, "a required tensor pointer is NULL");
  if (!aligned(q, q_stride_b, q_stride_h, 2, 8) || !aligned(k, k_stride_b, k_stride_h, 2, 8) ||
      !aligned(v, v_stride_b, v_stride_h, 2, 8) || (q_stride_t * 2) % 8 || (k_stride_t * 2) % 8)
    return fail(GDN_ERR_UNSUPPORTED, "q/k/v rows must be 8-byte aligned (base and strides)");
  rc = check_state_pair(pool, pool_stride_n, pool_stride_h, new_pool, new_pool_stride_n, new_pool_stride_h, pool_size,
                        num_v_heads);
  if (rc) return rc;
  if (intermediate) {
    if (!aligned(intermediate, inter_stride_n, inter_stride_h, sizeof(float), 16) || (inter_stride_t * 4) % 16)
      return fail(GDN_ERR_UNSUPPORTED, "intermediate rows must be 16-byte aligned (base and strides)");
    if (inter_stride_n < 0 || inter_stride_t < 0 || inter_stride_h < 0)
      return fail(GDN_ERR_INVALID_ARGUMENT, "negative intermediate stride");
  }

  gdn::DecodeMtpParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.pool = pool;
  p.new_pool = new_pool;
  p.indices = indices;
  p.idx_is_int64 = indices_is_int64 ? 1 : 0;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.inter = intermediate;
  p.q_sb = q_stride_b;
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.k_sb = k_stride_b;
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v_sb = v_stride_b;
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.a_sb = a_stride_b;
  p.a_st = a_stride_t;
  p.b_sb = b_stride_b;
  p.b_st = b_stride_t;
  p.o_sb = out_stride_b;
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.s_sn = pool_stride_n;
  p.s_sh = pool_stride_h;
  p.n_sn = new_pool_stride_n;
  p.n_sh = new_pool_stride_h;
  p.i_sn = inter_stride_n;
  p.i_st = inter_stride_t;
  p.i_sh = inter_stride_h;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  p.B = batch;
  p.T = tokens;
  p.P = pool_size;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.flags = flags;
  const cudaError_t e = gdn::launch_decode_mtp(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_decode_pooled launch");
  return ok();
}

int gdn_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h, const float* state,
                int64_t state_stride_n, int64_t state_stride_h, const float* A_log, const void* a, int64_t a_stride_t,
                const float* dt_bias, const void* b, int64_t b_stride_t, const void* cu_seqlens,
                int32_t cu_seqlens_is_int64, float scale, void* out, int64_t out_stride_t, int64_t out_stride_h,
                float* new_state, int64_t new_state_stride_n, int64_t new_state_stride_h, int32_t num_seqs,
                int64_t total_tokens, int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim, void* workspace,
                size_t workspace_bytes, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0 (got %d, %lld)", num_seqs,
                (long long)total_tokens);
  if (num_seqs > 65535) return fail(GDN_ERR_UNSUPPORTED, "num_seqs > 65535 per call is not supported");
  if (flags & ~(GDN_FLAG_QK_L2NORM | GDN_FLAG_PREFILL_SERIAL | GDN_PREFILL_SEGMENTS(15)))
    return fail(GDN_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags);
  if (num_seqs == 0) return ok();
  if (!cu_seqlens) return fail(GDN_ERR_INVALID_ARGUMENT, "cu_seqlens must not be NULL");
  if (!A_log || !dt_bias) return fail(GDN_ERR_INVALID_ARGUMENT, "A_log and dt_bias must not be NULL");
  if (total_tokens > 0) {
    if (!q || !k || !v || !a || !b || !out)
      return fail(GDN_ERR_INVALID_ARGUMENT, "a required tensor pointer is NULL");
    if (!aligned(q, q_stride_t, q_stride_h, 2, 8) || !aligned(k, k_stride_t, k_stride_h, 2, 8) ||
        !aligned(v, v_stride_t, v_stride_h, 2, 8))
      return fail(GDN_ERR_UNSUPPORTED, "q/k/v rows must be 8-byte aligned (base and strides)");
  }
  rc = check_state_pair(state, state_stride_n, state_stride_h, new_state, new_state_stride_n, new_state_stride_h,
                        num_seqs, num_v_heads);
  if (rc) return rc;
  const size_t need =
      gdn_prefill_workspace_size(num_seqs, total_tokens, num_qk_heads, num_v_heads, head_dim, flags);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, workspace_bytes);

  gdn::PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state = state;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.cu_seqlens = cu_seqlens;
  p.cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.new_state = new_state;
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.s_sn = state_stride_n;
  p.s_sh = state_stride_h;
  p.a_st = a_stride_t;
  p.b_st = b_stride_t;
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.n_sn = new_state_stride_n;
  p.n_sh = new_state_stride_h;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  p.N = num_seqs;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.T = total_tokens;
  p.flags = flags;
  p.workspace = workspace;
  p.workspace_bytes = workspace_bytes;
  const bool chunked = !(flags & GDN_FLAG_PREFILL_SERIAL) && gdn::prefill_chunk_supported(p);
  const cudaError_t e = chunked ? gdn::launch_prefill_chunk(p, static_cast<cudaStream_t>(stream))
                                : gdn::launch_prefill_serial(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, chunked ? "gdn_prefill (chunked) launch" : "gdn_prefill launch");
  return ok();
}

int gdn_prefill_state_map(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                          int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                          int64_t v_stride_h, const float* A_log, const void* a, int64_t a_stride_t,
                          const float* dt_bias, const void* b, int64_t b_stride_t, const void* cu_seqlens,
                          int32_t cu_seqlens_is_int64, float* map_m, int64_t map_m_stride_n, int64_t map_m_stride_h,
                          float* map_c, int64_t map_c_stride_n, int64_t map_c_stride_h, int32_t num_seqs,
                          int64_t total_tokens, int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                          void* workspace, size_t workspace_bytes, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0 (got %d, %lld)", num_seqs,
                (long long)total_tokens);
  if (num_seqs > 65535) return fail(GDN_ERR_UNSUPPORTED, "num_seqs > 65535 per call is not supported");
  if (flags & ~(GDN_FLAG_STATE_MAP | GDN_PREFILL_SEGMENTS(15)))
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_prefill_state_map: unknown flag bits 0x%x", flags);
  if (num_seqs == 0) return ok();
  if (!cu_seqlens || !A_log || !dt_bias || !map_m || !map_c)
    return fail(GDN_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!aligned(map_m, map_m_stride_n, map_m_stride_h, sizeof(float), 16) ||
      !aligned(map_c, map_c_stride_n, map_c_stride_h, sizeof(float), 16))
    return fail(GDN_ERR_UNSUPPORTED, "map rows must be 16-byte aligned (base and strides)");
  if (total_tokens > 0) {
    if (!q || !k || !v || !a || !b) return fail(GDN_ERR_INVALID_ARGUMENT, "a required tensor pointer is NULL");
    if (!aligned(q, q_stride_t, q_stride_h, 2, 16) || !aligned(k, k_stride_t, k_stride_h, 2, 16) ||
        !aligned(v, v_stride_t, v_stride_h, 2, 16))
      return fail(GDN_ERR_UNSUPPORTED, "gdn_prefill_state_map needs 16-byte aligned q/k/v rows (base and strides)");
  }
  const size_t need = gdn::prefill_map_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
  if (need > 0 && (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15)))
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required (got %zu)", need,
                workspace_bytes);
  gdn::PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state = nullptr;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.cu_seqlens = cu_seqlens;
  p.cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p.out = nullptr;
  p.new_state = nullptr;
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.s_sn = p.s_sh = 0;
  p.a_st = a_stride_t;
  p.b_st = b_stride_t;
  p.o_st = p.o_sh = 0;
  p.n_sn = p.n_sh = 0;
  p.scale = 1.0f;
  p.N = num_seqs;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.T = total_tokens;
  p.flags = flags;
  p.workspace = workspace;
  p.workspace_bytes = workspace_bytes;
  p.map_m = map_m;
  p.m_sn = map_m_stride_n;
  p.m_sh = map_m_stride_h;
  p.map_c = map_c;
  p.c_sn = map_c_stride_n;
  p.c_sh = map_c_stride_h;
  const cudaError_t e = total_tokens > 0 ? gdn::launch_prefill_state_map(p, static_cast<cudaStream_t>(stream))
                                         : gdn::launch_identity_maps(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill_state_map launch");
  return ok();
}

int gdn_prefill_range_affine(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                             int64_t k_stride_t, int64_t k_stride_h, const void* v, int64_t v_stride_t,
                             int64_t v_stride_h, const float* A_log, const void* a, int64_t a_stride_t,
                             const float* dt_bias, const void* b, int64_t b_stride_t, const void* cu_seqlens,
                             int32_t cu_seqlens_is_int64, float scale, void* out, int64_t out_stride_t,
                             int64_t out_stride_h, float* map_m, int64_t map_m_stride_n, int64_t map_m_stride_h,
                             float* map_c, int64_t map_c_stride_n, int64_t map_c_stride_h, int32_t num_seqs,
                             int64_t total_tokens, int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                             void* workspace, size_t workspace_bytes, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0 (got %d, %lld)", num_seqs,
                (long long)total_tokens);
  if (num_seqs > 65535) return fail(GDN_ERR_UNSUPPORTED, "num_seqs > 65535 per call is not supported");
  if (flags & ~(GDN_FLAG_RANGE_AFFINE | GDN_PREFILL_SEGMENTS(15)))
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_prefill_range_affine: unsupported flag bits 0x%x", flags);
  if (num_seqs == 0) return ok();
  if (!cu_seqlens || !A_log || !dt_bias || !map_m || !map_c)
    return fail(GDN_ERR_INVALID_ARGUMENT, "a required pointer is NULL");
  if (!aligned(map_m, map_m_stride_n, map_m_stride_h, sizeof(float), 16) ||
      !aligned(map_c, map_c_stride_n, map_c_stride_h, sizeof(float), 16))
    return fail(GDN_ERR_UNSUPPORTED, "map rows must be 16-byte aligned (base and strides)");
  if (total_tokens > 0) {
    if (!q || !k || !v || !a || !b || !out) return fail(GDN_ERR_INVALID_ARGUMENT, "a required tensor pointer is NULL");
    if (!aligned(q, q_stride_t, q_stride_h, 2, 16) || !aligned(k, k_stride_t, k_stride_h, 2, 16) ||
        !aligned(v, v_stride_t, v_stride_h, 2, 16))
      return fail(GDN_ERR_UNSUPPORTED, "gdn_prefill_range_affine needs 16-byte aligned q/k/v rows (base and strides)");
    if ((reinterpret_cast<uintptr_t>(out) & 15) || (out_stride_t & 7) || (out_stride_h & 7))
      return fail(GDN_ERR_UNSUPPORTED, "out rows must be 16-byte aligned (base and strides)");
  }
  const size_t need = gdn::prefill_range_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required (got %zu)", need,
                workspace_bytes);
  gdn::PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.state = nullptr;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.cu_seqlens = cu_seqlens;
  p.cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.new_state = nullptr;
  p.q_st = q_stride_t;
  p.q_sh = q_stride_h;
  p.k_st = k_stride_t;
  p.k_sh = k_stride_h;
  p.v_st = v_stride_t;
  p.v_sh = v_stride_h;
  p.s_sn = p.s_sh = 0;
  p.a_st = a_stride_t;
  p.b_st = b_stride_t;
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.n_sn = p.n_sh = 0;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)head_dim);
  p.N = num_seqs;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.T = total_tokens;
  p.flags = flags;
  p.workspace = workspace;
  p.workspace_bytes = workspace_bytes;
  p.map_m = map_m;
  p.m_sn = map_m_stride_n;
  p.m_sh = map_m_stride_h;
  p.map_c = map_c;
  p.c_sn = map_c_stride_n;
  p.c_sh = map_c_stride_h;
  const cudaError_t e = total_tokens > 0 ? gdn::launch_prefill_range_affine(p, static_cast<cudaStream_t>(stream))
                                         : gdn::launch_identity_maps(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill_range_affine launch");
  return ok();
}

int gdn_prefill_range_finish(const void* cu_seqlens, int32_t cu_seqlens_is_int64, const float* state,
                             int64_t state_stride_n, int64_t state_stride_h, const float* prev_maps,
                             int32_t num_prev_maps, void* out, int64_t out_stride_t,
                             int64_t out_stride_h, float* new_state, int64_t new_state_stride_n,
                             int64_t new_state_stride_h, int32_t num_seqs, int64_t total_tokens,
                             int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim, void* workspace,
                             size_t workspace_bytes, uint32_t flags, void* stream) {
  int rc = check_common(num_qk_heads, num_v_heads, head_dim);
  if (rc) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0 (got %d, %lld)", num_seqs,
                (long long)total_tokens);
  if (num_seqs > 65535) return fail(GDN_ERR_UNSUPPORTED, "num_seqs > 65535 per call is not supported");
  if (flags & ~(GDN_FLAG_RANGE_AFFINE | GDN_PREFILL_SEGMENTS(15)))
    return fail(GDN_ERR_INVALID_ARGUMENT, "gdn_prefill_range_finish: unsupported flag bits 0x%x", flags);
  if (num_seqs == 0) return ok();
  if (!cu_seqlens) return fail(GDN_ERR_INVALID_ARGUMENT, "cu_seqlens must not be NULL");
  if (total_tokens > 0) {
    if (!out) return fail(GDN_ERR_INVALID_ARGUMENT, "out must not be NULL");
    if ((reinterpret_cast<uintptr_t>(out) & 15) || (out_stride_t & 7) || (out_stride_h & 7))
      return fail(GDN_ERR_UNSUPPORTED, "out rows must be 16-byte aligned (base and strides)");
  }
  if (num_prev_maps < 0) return fail(GDN_ERR_INVALID_ARGUMENT, "num_prev_maps must be >= 0");
  if (num_prev_maps > 0) {
    if (state) return fail(GDN_ERR_INVALID_ARGUMENT, "give either state or prev_maps, not both");
    if (!prev_maps || (reinterpret_cast<uintptr_t>(prev_maps) & 15))
      return fail(GDN_ERR_INVALID_ARGUMENT, "prev_maps must be a 16-byte aligned device pointer");
  }
  rc = check_state_pair(state, state_stride_n, state_stride_h, new_state, new_state_stride_n, new_state_stride_h,
                        num_seqs, num_v_heads);
  if (rc) return rc;
  const size_t need = gdn::prefill_range_workspace_bytes(num_seqs, total_tokens, num_v_heads, flags);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(GDN_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) required (got %zu)", need,
                workspace_bytes);
  gdn::PrefillParams p;
  p.cp_prev = prev_maps;
  p.cp_prev_count = num_prev_maps;
  p.cu_seqlens = cu_seqlens;
  p.cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p.state = state;
  p.s_sn = state_stride_n;
  p.s_sh = state_stride_h;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_st = out_stride_t;
  p.o_sh = out_stride_h;
  p.new_state = new_state;
  p.n_sn = new_state_stride_n;
  p.n_sh = new_state_stride_h;
  p.N = num_seqs;
  p.HQ = num_qk_heads;
  p.HV = num_v_heads;
  p.ratio = num_v_heads / num_qk_heads;
  p.T = total_tokens;
  p.flags = flags;
  p.workspace = workspace;
  p.workspace_bytes = workspace_bytes;
  const cudaError_t e = gdn::launch_prefill_range_finish(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill_range_finish launch");
  return ok();
}

int gdn_prefill_noalloc(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k, int64_t k_stride_t,
                        int64_t k_stride_h, const void* v, int64_t v_stride_t, int64_t v_stride_h,
                        const float* state, int64_t state_stride_n, int64_t state_stride_h, const float* A_log,
                        const void* a, int64_t a_stride_t, const float* dt_bias, const void* b, int64_t b_stride_t,
                        const void* cu_seqlens, int32_t cu_seqlens_is_int64, float scale, void* out,
                        int64_t out_stride_t, int64_t out_stride_h, float* new_state, int64_t new_state_stride_n,
                        int64_t new_state_stride_h, int32_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                        int32_t num_v_heads, int32_t head_dim, uint32_t flags, void* stream) {
  const size_t need =
      gdn_prefill_workspace_size(num_seqs, total_tokens, num_qk_heads, num_v_heads, head_dim, flags);
  if (need > kStaticScratchBytes)
    return fail(GDN_ERR_WORKSPACE,
                "gdn_prefill_noalloc: the problem needs %zu bytes of scratch, the static scratch holds %zu "
                "(call gdn_prefill with a workspace instead)",
                need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(GDN_ERR_UNSUPPORTED, "gdn_prefill_noalloc: device index %d >= 64", dev);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_static_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "gdn_prefill_noalloc: cudaGetSymbolAddress");
      g_scratch_addr[dev] = addr;
    }
    scratch = g_scratch_addr[dev];
  }
  return gdn_prefill(q, q_stride_t, q_stride_h, k, k_stride_t, k_stride_h, v, v_stride_t, v_stride_h, state,
                     state_stride_n, state_stride_h, A_log, a, a_stride_t, dt_bias, b, b_stride_t, cu_seqlens,
                     cu_seqlens_is_int64, scale, out, out_stride_t, out_stride_h, new_state, new_state_stride_n,
                     new_state_stride_h, num_seqs, total_tokens, num_qk_heads, num_v_heads, head_dim, scratch,
                     scratch ? kStaticScratchBytes : 0, flags, stream);
}

}  // extern "C"
