/*
 * gdn_b200 — C ABI of the B200-native Gated DeltaNet (GDN) operators.
 *
 * Library: libgdn_b200.so (built for sm_100a).  Every entry point is
 * asynchronous on the given CUDA stream (a cudaStream_t passed as void*; NULL
 * means the legacy default stream), performs no host<->device
 * synchronisation, and returns GDN_OK or an error code; the message of the
 * last failure on the calling thread is available from gdn_last_error().
 *
 * Tensor conventions (all device pointers, innermost dimension contiguous,
 * strides given in ELEMENTS):
 *   bf16 tensors   q, k, v, a, b, out (passed as void*: raw bf16 storage)
 *   fp32 tensors   state, new_state, A_log, dt_bias
 *   state layout   "k-last" [.., HV, V = head_dim, K = head_dim]; each 128-float
 *                  row is contiguous and rows of one head are adjacent, so only
 *                  the sequence and head strides are passed.
 *   GVA mapping    v-head h reads q/k head h / (num_v_heads / num_qk_heads).
 *   scale          <= 0 selects 1 / sqrt(head_dim).
 *   state == NULL  zero initial state.
 *   new_state      may alias state exactly (in-place update); partial overlap
 *                  is rejected.
 * Alignment: q, k and v rows must start on 8-byte boundaries and state /
 * new_state rows on 16-byte boundaries (GDN_ERR_UNSUPPORTED otherwise).
 * head_dim must be 128 (the definitions' fixed head size).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GDN_API __attribute__((visibility("default")))
#else
#define GDN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_OK 0
#define GDN_ERR_INVALID_ARGUMENT 1 /* shapes, strides, null pointers, overlap */
#define GDN_ERR_UNSUPPORTED 2      /* valid but not implemented (head_dim != 128, alignment) */
#define GDN_ERR_CUDA 3             /* a CUDA runtime call or kernel launch failed */
#define GDN_ERR_WORKSPACE 4        /* workspace missing or too small */

#define GDN_FLAG_QK_L2NORM 0x1u      /* L2-normalise q and k inside the kernel (eps 1e-6); default off */
#define GDN_FLAG_PREFILL_SERIAL 0x2u /* prefill: use the token-serial kernel instead of the chunked
                                        tensor-core kernel (cross-checking; prefill only) */
/* Prefill: split each sequence's chunks into n segments (2..15) that run on separate SMs
 * (context parallelism: segment 0 from the initial state; every later segment's affine
 * state map and its outputs from a zero and from the identity state; the maps composed;
 * the later segments' outputs corrected by their initial states).  0 = automatic
 * (segments only when the (sequence, v-head) chains leave most SMs idle and sequences are
 * long), 1 = never.  Bits 8-11.  gdn_prefill_range_affine / _finish: n map-pair segments
 * (1..15) instead, 0 = automatic. */
#define GDN_PREFILL_SEGMENTS(n) ((((uint32_t)(n)) & 15u) << 8)
/* gdn_prefill_workspace_size: size the workspace of gdn_prefill_state_map instead. */
#define GDN_FLAG_STATE_MAP 0x4u
/* gdn_prefill_workspace_size: size the workspace of gdn_prefill_range_affine / _finish
 * instead; those two calls take it in their flags as well. */
#define GDN_FLAG_RANGE_AFFINE 0x8u
/* gdn_decode self-test of the device-side failure path: every thread of the launch waits
 * on a barrier that nothing completes, gives up after 1 ms, records
 * GDN_DEVERR_WAIT_TIMEOUT and returns; out and new_state are not written.  No copy or
 * tensor-core work is in flight when the waits give up, so the context stays usable. */
#define GDN_FLAG_SELFTEST_WAIT_TIMEOUT 0x80000000u

/* Device-side error bits reported by gdn_device_error(). */
#define GDN_DEVERR_WAIT_TIMEOUT 0x1u /* a bounded wait inside a kernel gave up */
#define GDN_DEVERR_BAD_SEQLENS 0x2u  /* cu_seqlens not monotone or beyond total_tokens */
#define GDN_DEVERR_BAD_INDEX 0x4u    /* a state-pool index >= pool_size (gdn_decode_pooled) */

/* Version of this ABI (major * 10000 + minor * 100 + patch). */
GDN_API int gdn_version(void);

/* Message describing the last failure on the calling thread ("" if none). */
GDN_API const char* gdn_last_error(void);

/*
 * Reads (and optionally clears) the device-side error word of the current
 * device.  Synchronous: waits for prior work on the device.  For tests and
 * debugging only; the operator entry points never call it.
 */
GDN_API int gdn_device_error(uint32_t* bits_out, int clear);

/*
 * Single-token decode step.
 * Replaces solution/triton/kernel_decode.py:186 run(q, k, v, state, A_log, a,
 * dt_bias, b, scale) and its launcher decode_kernel (kernel_decode.py:115-183),
 * whose strides (kernel_decode.py:21-36) it takes the same way.
 *   q, k       [B, 1, num_qk_heads, head_dim]   strides (q_stride_b, q_stride_h)
 *   v          [B, 1, num_v_heads, head_dim]    strides (v_stride_b, v_stride_h)
 *   state      [B, num_v_heads, head_dim, head_dim] fp32 or NULL
 *   a, b       [B, 1, num_v_heads] bf16, head stride 1, batch strides a_stride_b, b_stride_b
 *   A_log, dt_bias  [num_v_heads] fp32
 *   out        [B, 1, num_v_heads, head_dim] bf16   strides (out_stride_b, out_stride_h)
 *   new_state  same shape as state                  strides (new_state_stride_b, new_state_stride_h)
 */
GDN_API int gdn_decode(const void* q, int64_t q_stride_b, int64_t q_stride_h,
                       const void* k, int64_t k_stride_b, int64_t k_stride_h,
               const void* v, int64_t v_stride_b, int64_t v_stride_h,
               const float* state, int64_t state_stride_b, int64_t state_stride_h,
               const float* A_log,
               const void* a, int64_t a_stride_b,
               const float* dt_bias,
               const void* b, int64_t b_stride_b,
               float scale,
               void* out, int64_t out_stride_b, int64_t out_stride_h,
               float* new_state, int64_t new_state_stride_b, int64_t new_state_stride_h,
               int32_t batch, int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
               uint32_t flags, void* stream);

/*
 * Multi-token decode against a pool of states (the serving form: state slots,
 * T >= 1 tokens per sequence, e.g. speculative / multi-token prediction).
 * Follows flashinfer 0.6.11.post2 flashinfer/trace/templates/gdn.py
 * _gdn_mtp_reference (third party; the reference kit's own decode handles one
 * token and a dense state batch): sequence b starts from pool[indices[b]], runs
 * T steps of the decode recurrence of kernel_decode.py:71-103, and writes
 *   out[b, t]              bf16, every token
 *   intermediate[s, t]     the state after token t (optional: NULL skips it)
 *   new_pool[s]            the final state, s = indices[b]
 * new_pool may alias pool exactly (in-place update; slots no index names are left
 * as they are); otherwise its other slots are not written.  indices [B] device
 * int32 (indices_is_int64 = 0) or int64 (= 1), distinct; a negative index skips
 * the sequence (its outputs are zeros); an index >= pool_size sets
 * GDN_DEVERR_BAD_INDEX and is skipped.
 *   q, k       [B, T, num_qk_heads, head_dim]   strides (b, t, h)
 *   v, out     [B, T, num_v_heads, head_dim]    strides (b, t, h)
 *   a, b       [B, T, num_v_heads] bf16, head stride 1, strides (b, t)
 *   pool, new_pool  [pool_size, num_v_heads, head_dim, head_dim] fp32   strides (n, h)
 *   intermediate    [pool_size, T, num_v_heads, head_dim, head_dim] fp32  strides (n, t, h)
 */
GDN_API int gdn_decode_pooled(const void* q, int64_t q_stride_b, int64_t q_stride_t, int64_t q_stride_h,
                const void* k, int64_t k_stride_b, int64_t k_stride_t, int64_t k_stride_h,
                const void* v, int64_t v_stride_b, int64_t v_stride_t, int64_t v_stride_h,
                const float* pool, int64_t pool_stride_n, int64_t pool_stride_h,
                const void* indices, int32_t indices_is_int64,
                const float* A_log,
                const void* a, int64_t a_stride_b, int64_t a_stride_t,
                const float* dt_bias,
                const void* b, int64_t b_stride_b, int64_t b_stride_t,
                float scale,
                void* out, int64_t out_stride_b, int64_t out_stride_t, int64_t out_stride_h,
                float* new_pool, int64_t new_pool_stride_n, int64_t new_pool_stride_h,
                float* intermediate, int64_t inter_stride_n, int64_t inter_stride_t, int64_t inter_stride_h,
                int32_t batch, int32_t tokens, int32_t pool_size,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                uint32_t flags, void* stream);

/*
 * Variable-length prefill.
 * Replaces solution/triton/kernel_prefill.py:234 run(q, k, v, state, A_log, a,
 * dt_bias, b, cu_seqlens, scale) and its launcher run_prefill
 * (kernel_prefill.py:156-231).
 *   q, k       [T, num_qk_heads, head_dim]      strides (q_stride_t, q_stride_h)
 *   v          [T, num_v_heads, head_dim]       strides (v_stride_t, v_stride_h)
 *   state      [N, num_v_heads, head_dim, head_dim] fp32 or NULL
 *   a, b       [T, num_v_heads] bf16, head stride 1
 *   cu_seqlens [N + 1] device int32 (cu_seqlens_is_int64 = 0) or int64 (= 1);
 *              monotone, cu_seqlens[0] >= 0, cu_seqlens[N] <= total_tokens
 *              (checked on the device: GDN_DEVERR_BAD_SEQLENS).
 *   out        [T, num_v_heads, head_dim] bf16
 *   new_state  [N, num_v_heads, head_dim, head_dim] fp32
 *   An empty sequence passes its initial state through (kernel_prefill.py:65-73).
 *   workspace  device scratch of at least gdn_prefill_workspace_size(...) bytes
 *              (may be NULL when that size is 0).
 */
GDN_API int gdn_prefill(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                const void* k, int64_t k_stride_t, int64_t k_stride_h,
                const void* v, int64_t v_stride_t, int64_t v_stride_h,
                const float* state, int64_t state_stride_n, int64_t state_stride_h,
                const float* A_log,
                const void* a, int64_t a_stride_t,
                const float* dt_bias,
                const void* b, int64_t b_stride_t,
                const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                float scale,
                void* out, int64_t out_stride_t, int64_t out_stride_h,
                float* new_state, int64_t new_state_stride_n, int64_t new_state_stride_h,
                int32_t num_seqs, int64_t total_tokens,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                void* workspace, size_t workspace_bytes,
                uint32_t flags, void* stream);

/*
 * Affine state map of each sequence's token range (no counterpart in the reference,
 * whose prefill is token-serial; the building block of context parallelism across
 * GPUs, where a rank holding a later range of a sequence needs its map before the
 * state entering the range is known).  The recurrence is affine in the state: for
 * sequence n and v-head h, running the range from any initial state S gives
 *   S_out = S M + C      (k-last [V x K] states, row vectors; fp32)
 * with M [K x K] the range run from the identity with v taken as 0 and C [V x K]
 * the range run from a zero state.  Inputs as gdn_prefill (no state, no outputs);
 * q/k/v rows and strides 16-byte aligned.  A long range is cut into segments whose
 * maps run on separate SMs and are then multiplied together (fp32; flags may carry
 * GDN_PREFILL_SEGMENTS(n): 0 = automatic, 1 = one chain per map).  Writes
 *   map_m [N, num_v_heads, head_dim, head_dim]   strides (n, h), rows contiguous
 *   map_c [N, num_v_heads, head_dim, head_dim]   strides (n, h), rows contiguous
 * An empty range gives M = I, C = 0.  workspace: at least
 * gdn_prefill_workspace_size(..., GDN_FLAG_STATE_MAP | flags) bytes, 16-byte aligned.
 */
GDN_API int gdn_prefill_state_map(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                const void* k, int64_t k_stride_t, int64_t k_stride_h,
                const void* v, int64_t v_stride_t, int64_t v_stride_h,
                const float* A_log,
                const void* a, int64_t a_stride_t,
                const float* dt_bias,
                const void* b, int64_t b_stride_t,
                const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                float* map_m, int64_t map_m_stride_n, int64_t map_m_stride_h,
                float* map_c, int64_t map_c_stride_n, int64_t map_c_stride_h,
                int32_t num_seqs, int64_t total_tokens,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                void* workspace, size_t workspace_bytes,
                uint32_t flags, void* stream);

/*
 * Context parallelism across GPUs for a rank that holds a later token range of each
 * sequence (no counterpart in the reference, whose prefill is token-serial).  The range's
 * outputs and final state are affine in the state S_in entering it, which the rank learns
 * only from the other ranks' maps, so its prefill is split around that exchange:
 *   gdn_prefill_range_affine  (before): writes out = the range's outputs from a zero initial
 *     state and the range's map, S_out = S_in M + C (map_m, map_c as in
 *     gdn_prefill_state_map); keeps in the workspace the homogeneous outputs (those of the
 *     range run from the identity with v taken as 0) and the maps of its segments.
 *   gdn_prefill_range_finish  (after): given S_in, adds S_in's share to out (the same buffer)
 *     and writes S_out to new_state (may alias state).  S_in is either state (NULL = zero)
 *     or, with num_prev_maps > 0 and state NULL, the fold S = 0, S <- S M_j + C_j over the
 *     preceding ranges' maps prev_maps [num_prev_maps][2 (M, C)][num_seqs][num_v_heads]
 *     [head_dim][head_dim] fp32, contiguous (what an all_gather of (M, C) pairs holds;
 *     the first range's pair may be (0, its final state)), done on the device.
 * No token runs twice.  Inputs as gdn_prefill (q/k/v and out rows 16-byte aligned); q and
 * k are used as given (GDN_FLAG_QK_L2NORM is not supported here).  Both calls take the same
 * num_seqs, total_tokens, head counts, flags (GDN_FLAG_RANGE_AFFINE, optionally
 * GDN_PREFILL_SEGMENTS(n)) and workspace: at least
 * gdn_prefill_workspace_size(..., GDN_FLAG_RANGE_AFFINE | flags) bytes, 16-byte aligned,
 * left untouched between them.
 */
GDN_API int gdn_prefill_range_affine(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                const void* k, int64_t k_stride_t, int64_t k_stride_h,
                const void* v, int64_t v_stride_t, int64_t v_stride_h,
                const float* A_log,
                const void* a, int64_t a_stride_t,
                const float* dt_bias,
                const void* b, int64_t b_stride_t,
                const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                float scale,
                void* out, int64_t out_stride_t, int64_t out_stride_h,
                float* map_m, int64_t map_m_stride_n, int64_t map_m_stride_h,
                float* map_c, int64_t map_c_stride_n, int64_t map_c_stride_h,
                int32_t num_seqs, int64_t total_tokens,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                void* workspace, size_t workspace_bytes,
                uint32_t flags, void* stream);
GDN_API int gdn_prefill_range_finish(const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                const float* state, int64_t state_stride_n, int64_t state_stride_h,
                const float* prev_maps, int32_t num_prev_maps,
                void* out, int64_t out_stride_t, int64_t out_stride_h,
                float* new_state, int64_t new_state_stride_n, int64_t new_state_stride_h,
                int32_t num_seqs, int64_t total_tokens,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                void* workspace, size_t workspace_bytes,
                uint32_t flags, void* stream);

/* Bytes of device workspace gdn_prefill needs for this problem size. */
GDN_API size_t gdn_prefill_workspace_size(int32_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                                  int32_t num_v_heads, int32_t head_dim, uint32_t flags);

/*
 * gdn_prefill without a caller workspace (no counterpart in the reference, whose
 * prefill needs no scratch), for callers that cannot allocate device memory at call
 * time: e.g. code running inside a captured or pre-planned execution graph, or
 * behind an allocator that must not grow.  The chunked prefill's device scratch
 * (the prepared chunk records, and the context-parallel segments' states and maps)
 * lives in a static device array of GDN_PREFILL_NOALLOC_SCRATCH_BYTES inside the
 * library, so the call allocates nothing.  Arguments and semantics are those of gdn_prefill minus the
 * workspace.  A problem whose gdn_prefill_workspace_size(...) exceeds the scratch is
 * rejected with GDN_ERR_WORKSPACE before anything is enqueued.
 * Footprint: the array is part of the library's device module, so every GPU on which
 * the library's kernels are loaded holds those 64 MiB until the process exits,
 * whether or not this entry point is ever called.
 * The scratch is one per device and shared by all calls: calls on that device that
 * overlap in time (other streams or host threads) race on it.  The first call on a
 * device looks its address up (cudaGetSymbolAddress) and caches it; that call should
 * come before any stream capture, and cudaDeviceReset while the library is loaded is
 * not supported (the cached address would outlive the module).  No part of the
 * scratch needs to start at zero.
 */
#define GDN_PREFILL_NOALLOC_SCRATCH_BYTES (64u << 20)
GDN_API int gdn_prefill_noalloc(const void* q, int64_t q_stride_t, int64_t q_stride_h,
                const void* k, int64_t k_stride_t, int64_t k_stride_h,
                const void* v, int64_t v_stride_t, int64_t v_stride_h,
                const float* state, int64_t state_stride_n, int64_t state_stride_h,
                const float* A_log,
                const void* a, int64_t a_stride_t,
                const float* dt_bias,
                const void* b, int64_t b_stride_t,
                const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                float scale,
                void* out, int64_t out_stride_t, int64_t out_stride_h,
                float* new_state, int64_t new_state_stride_n, int64_t new_state_stride_h,
                int32_t num_seqs, int64_t total_tokens,
                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                uint32_t flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H */
