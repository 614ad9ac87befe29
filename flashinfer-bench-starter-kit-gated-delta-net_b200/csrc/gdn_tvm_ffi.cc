// TVM-FFI module of the GDN operators (host C++; built as libgdn_b200_tvm_ffi.so).
//
// The reference's CUDA route binds its kernel through TVM-FFI
// (solution/cuda/binding.py:10-25 registers "flashinfer.kernel"; the harness builds
// `kernel.cu::<fn>` with binding "tvm-ffi", README.md:259-279) and calls it in
// destination-passing style: the definition's inputs, then its outputs.  This module
// exports that form for both definitions, over the C ABI of libgdn_b200.so:
//
//   gdn_decode (q, k, v, state|None, A_log, a, dt_bias, b, scale, output, new_state)
//   gdn_prefill(q, k, v, state|None, A_log, a, dt_bias, b, cu_seqlens, scale, output, new_state)
//
// Shapes, dtypes and the k-last state layout are those of kernel_decode.py:186 /
// kernel_prefill.py:234; new_state may be the state tensor itself (in-place).  Work is
// enqueued on the stream TVM-FFI reports for the output's device
// (TVMFFIEnvGetStream; the caller sets it, e.g. tvm_ffi.use_torch_stream()), nothing is
// synchronised, and a failure raises a TVM-FFI error carrying gdn_last_error().  The
// prefill workspace is a device buffer cached per (device, stream), grown with
// stream-ordered allocation when a larger problem arrives.
#include <cuda_runtime.h>
#include <dlpack/dlpack.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>
#include <tvm/ffi/optional.h>

#include <cmath>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/gdn_b200.h"

namespace {

using tvm::ffi::Optional;
using tvm::ffi::TensorView;

bool is_bf16(const TensorView& t) { return t.dtype().code == kDLBfloat && t.dtype().bits == 16; }
bool is_f32(const TensorView& t) { return t.dtype().code == kDLFloat && t.dtype().bits == 32; }
bool is_int(const TensorView& t) { return t.dtype().code == kDLInt && (t.dtype().bits == 32 || t.dtype().bits == 64); }

void expect(bool cond, const char* what) {
  if (!cond) TVM_FFI_THROW(ValueError) << "gdn_b200: " << what;
}

void check_rc(int rc) {
  if (rc != GDN_OK) TVM_FFI_THROW(RuntimeError) << "gdn_b200 error " << rc << ": " << gdn_last_error();
}

// Pointer to element 0 (DLPack's data + byte_offset).
const void* dptr(const TensorView& t) { return static_cast<const char*>(t.data_ptr()) + t.byte_offset(); }
void* mptr(const TensorView& t) { return static_cast<char*>(t.data_ptr()) + t.byte_offset(); }

void expect_cuda(const TensorView& t, int device_id, const char* name) {
  if (t.device().device_type != kDLCUDA || t.device().device_id != device_id)
    TVM_FFI_THROW(ValueError) << "gdn_b200: " << name << " must be on cuda:" << device_id;
  if (t.ndim() > 0 && t.stride(t.ndim() - 1) != 1)
    TVM_FFI_THROW(ValueError) << "gdn_b200: " << name << " must have a contiguous innermost dimension";
}

void* stream_of(int device_id) { return TVMFFIEnvGetStream(kDLCUDA, device_id); }

// None or 0 selects 1 / sqrt(head_dim) (kernel_decode.py:124-125); the C ABI reads <= 0 as that.
float resolve_scale(const Optional<double>& scale) {
  if (!scale.has_value()) return 0.0f;
  const double s = scale.value();
  return std::isfinite(s) ? (float)s : 0.0f;
}

void decode(TensorView q, TensorView k, TensorView v, Optional<TensorView> state, TensorView A_log, TensorView a,
            TensorView dt_bias, TensorView b, Optional<double> scale, TensorView output, TensorView new_state) {
  expect(q.ndim() == 4 && k.ndim() == 4 && v.ndim() == 4, "q, k, v must be [B, 1, H, 128]");
  expect(is_bf16(q) && is_bf16(k) && is_bf16(v) && is_bf16(a) && is_bf16(b) && is_bf16(output),
         "q, k, v, a, b and output must be bfloat16");
  expect(is_f32(A_log) && is_f32(dt_bias) && is_f32(new_state), "A_log, dt_bias and new_state must be float32");
  expect(q.size(1) == 1, "decode takes one token per sequence");
  expect(a.ndim() == 3 && b.ndim() == 3, "a, b must be [B, 1, HV]");
  expect(new_state.ndim() == 4 && output.ndim() == 4, "output [B, 1, HV, 128], new_state [B, HV, 128, 128]");
  const int dev = output.device().device_id;
  for (const TensorView* t : {&q, &k, &v, &A_log, &a, &dt_bias, &b, &output, &new_state}) expect_cuda(*t, dev, "tensor");
  const float* st = nullptr;
  int64_t ss0 = 0, ss1 = 0;
  if (state.has_value()) {
    TensorView s = state.value();
    expect(is_f32(s) && s.ndim() == 4, "state must be float32 [B, HV, 128, 128]");
    expect_cuda(s, dev, "state");
    st = static_cast<const float*>(dptr(s));
    ss0 = s.stride(0);
    ss1 = s.stride(1);
  }
  const int32_t B = (int32_t)q.size(0), HQ = (int32_t)q.size(2), HV = (int32_t)v.size(2), D = (int32_t)q.size(3);
  check_rc(gdn_decode(dptr(q), q.stride(0), q.stride(2), dptr(k), k.stride(0), k.stride(2), dptr(v), v.stride(0),
                      v.stride(2), st, ss0, ss1, static_cast<const float*>(dptr(A_log)), dptr(a), a.stride(0),
                      static_cast<const float*>(dptr(dt_bias)), dptr(b), b.stride(0), resolve_scale(scale),
                      mptr(output), output.stride(0), output.stride(2), static_cast<float*>(mptr(new_state)),
                      new_state.stride(0), new_state.stride(1), B, HQ, HV, D, 0u, stream_of(dev)));
}

// Workspace per (device, stream): grown by stream-ordered allocation, never shrunk.
std::mutex g_ws_mutex;
std::map<std::pair<int, void*>, std::pair<void*, size_t>> g_ws;

void* workspace(int dev, void* stream, size_t bytes) {
  if (bytes == 0) return nullptr;
  std::lock_guard<std::mutex> lock(g_ws_mutex);
  auto& slot = g_ws[{dev, stream}];
  if (slot.second < bytes) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(dev);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (slot.first) cudaFreeAsync(slot.first, s);
    void* p = nullptr;
    const cudaError_t e = cudaMallocAsync(&p, bytes, s);
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
      slot = {nullptr, 0};
      TVM_FFI_THROW(RuntimeError) << "gdn_b200: workspace allocation of " << bytes
                                  << " bytes failed: " << cudaGetErrorString(e);
    }
    slot = {p, bytes};
  }
  return slot.first;
}

void prefill(TensorView q, TensorView k, TensorView v, Optional<TensorView> state, TensorView A_log, TensorView a,
             TensorView dt_bias, TensorView b, TensorView cu_seqlens, Optional<double> scale, TensorView output,
             TensorView new_state) {
  expect(q.ndim() == 3 && k.ndim() == 3 && v.ndim() == 3, "q, k, v must be [T, H, 128]");
  expect(is_bf16(q) && is_bf16(k) && is_bf16(v) && is_bf16(a) && is_bf16(b) && is_bf16(output),
         "q, k, v, a, b and output must be bfloat16");
  expect(is_f32(A_log) && is_f32(dt_bias) && is_f32(new_state), "A_log, dt_bias and new_state must be float32");
  expect(is_int(cu_seqlens) && cu_seqlens.ndim() == 1 && cu_seqlens.size(0) >= 1, "cu_seqlens must be int32/int64 [N + 1]");
  expect(a.ndim() == 2 && b.ndim() == 2, "a, b must be [T, HV]");
  expect(new_state.ndim() == 4 && output.ndim() == 3, "output [T, HV, 128], new_state [N, HV, 128, 128]");
  const int dev = output.device().device_id;
  for (const TensorView* t : {&q, &k, &v, &A_log, &a, &dt_bias, &b, &cu_seqlens, &output, &new_state})
    expect_cuda(*t, dev, "tensor");
  const float* st = nullptr;
  int64_t ss0 = 0, ss1 = 0;
  if (state.has_value()) {
    TensorView s = state.value();
    expect(is_f32(s) && s.ndim() == 4, "state must be float32 [N, HV, 128, 128]");
    expect_cuda(s, dev, "state");
    st = static_cast<const float*>(dptr(s));
    ss0 = s.stride(0);
    ss1 = s.stride(1);
  }
  const int32_t N = (int32_t)cu_seqlens.size(0) - 1;
  const int64_t T = q.size(0);
  const int32_t HQ = (int32_t)q.size(1), HV = (int32_t)v.size(1), D = (int32_t)q.size(2);
  void* stream = stream_of(dev);
  const size_t ws_bytes = gdn_prefill_workspace_size(N, T, HQ, HV, D, 0u);
  void* ws = workspace(dev, stream, ws_bytes);
  check_rc(gdn_prefill(dptr(q), q.stride(0), q.stride(1), dptr(k), k.stride(0), k.stride(1), dptr(v), v.stride(0),
                       v.stride(1), st, ss0, ss1, static_cast<const float*>(dptr(A_log)), dptr(a), a.stride(0),
                       static_cast<const float*>(dptr(dt_bias)), dptr(b), b.stride(0), dptr(cu_seqlens),
                       cu_seqlens.dtype().bits == 64 ? 1 : 0, resolve_scale(scale), mptr(output),
                       output.stride(0), output.stride(1), static_cast<float*>(mptr(new_state)), new_state.stride(0),
                       new_state.stride(1), N, T, HQ, HV, D, ws, ws_bytes, 0u, stream));
}

int version() { return gdn_version(); }

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_decode, decode);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_prefill, prefill);
TVM_FFI_DLL_EXPORT_TYPED_FUNC(gdn_version, version);
