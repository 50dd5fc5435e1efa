// binding.cu -- TVM-FFI export of the DSA sparse-attention operator for the
// contest's CUDA route (the slot the reference leaves empty in
// solution/cuda/binding.py:10-25 and solution/cuda/kernel.cu; config.toml:7-9
// selects it with language = "cuda").  It wraps the library's C ABI
// (dsa_sparse_attention, include/dsa_b200.h) for tensors that arrive as
// TVM-FFI TensorViews:
//
//   dsa_sparse_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices,
//                        sm_scale, output, lse)
//
// with the shapes and dtypes of the reference kernel() (kernel.py:138-151):
// q_nope [T,H,512] bf16, q_pe [T,H,64] bf16, ckv_cache [P,64,512] bf16,
// kpe_cache [P,64,64] bf16, sparse_indices [T,topk] int32, output [T,H,512]
// bf16, lse [T,H] fp32 (H a multiple of 16, unit stride in the last dim).
// The launch goes to the stream TVM-FFI reports as current for the device.
// The split-K workspace is one zero-filled device buffer per device, grown
// on demand and kept for the life of the process.
#include <cuda_runtime.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <mutex>

#include "include/dsa_b200.h"

namespace {

using tvm::ffi::TensorView;

struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mu;
Workspace g_ws[64];

void* workspace(int dev, size_t need, cudaStream_t stream) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace& w = g_ws[dev];
  if (w.bytes < need) {
    if (w.ptr) {
      // earlier launches on any stream may still use the old buffer
      if (cudaDeviceSynchronize() != cudaSuccess || cudaFree(w.ptr) != cudaSuccess)
        TVM_FFI_THROW(RuntimeError) << "dsa_sparse_attention: cannot release the old workspace";
      w.ptr = nullptr;
      w.bytes = 0;
    }
    const size_t bytes = need < (size_t(1) << 20) ? (size_t(1) << 20) : need;
    if (cudaMalloc(&w.ptr, bytes) != cudaSuccess || cudaMemsetAsync(w.ptr, 0, bytes, stream) != cudaSuccess)
      TVM_FFI_THROW(RuntimeError) << "dsa_sparse_attention: cannot allocate " << bytes
                                  << " bytes of workspace";
    w.bytes = bytes;
  }
  return w.ptr;
}

void check_tensor(const TensorView& t, const char* name, int ndim, uint8_t code, uint8_t bits) {
  TVM_FFI_ICHECK_EQ(t.ndim(), ndim) << name << " must have " << ndim << " dimensions";
  TVM_FFI_ICHECK(t.dtype().code == code && t.dtype().bits == bits && t.dtype().lanes == 1)
      << name << " has the wrong dtype";
  TVM_FFI_ICHECK_EQ(t.device().device_type, kDLCUDA) << name << " must be a CUDA tensor";
  TVM_FFI_ICHECK_EQ(t.stride(-1), 1) << name << " needs a unit stride in its last dimension";
}

char* bytes_of(const TensorView& t) { return static_cast<char*>(t.data_ptr()) + t.byte_offset(); }

void dsa_sparse_attention_ffi(TensorView q_nope, TensorView q_pe, TensorView ckv_cache,
                              TensorView kpe_cache, TensorView sparse_indices, double sm_scale,
                              TensorView output, TensorView lse) {
  check_tensor(q_nope, "q_nope", 3, kDLBfloat, 16);
  check_tensor(q_pe, "q_pe", 3, kDLBfloat, 16);
  check_tensor(ckv_cache, "ckv_cache", 3, kDLBfloat, 16);
  check_tensor(kpe_cache, "kpe_cache", 3, kDLBfloat, 16);
  check_tensor(sparse_indices, "sparse_indices", 2, kDLInt, 32);
  check_tensor(output, "output", 3, kDLBfloat, 16);
  check_tensor(lse, "lse", 2, kDLFloat, 32);
  const int64_t T = q_nope.size(0), H = q_nope.size(1), topk = sparse_indices.size(1);
  // the reference's static shape assertions (kernel.py:147-151), heads any multiple of 16
  TVM_FFI_ICHECK(H % 16 == 0 && q_nope.size(2) == 512 && q_pe.size(2) == 64)
      << "q shapes must be [T, 16k, 512] and [T, 16k, 64]";
  TVM_FFI_ICHECK(q_pe.size(0) == T && q_pe.size(1) == H && sparse_indices.size(0) == T)
      << "q_nope, q_pe and sparse_indices disagree on T or H";
  TVM_FFI_ICHECK(ckv_cache.size(1) == 64 && ckv_cache.size(2) == 512 && kpe_cache.size(0) == ckv_cache.size(0) &&
                 kpe_cache.size(1) == 64 && kpe_cache.size(2) == 64)
      << "caches must be [P, 64, 512] and [P, 64, 64]";
  TVM_FFI_ICHECK(output.size(0) == T && output.size(1) == H && output.size(2) == 512 && lse.size(0) == T &&
                 lse.size(1) == H)
      << "output must be [T, H, 512] and lse [T, H]";
  const int dev = q_nope.device().device_id;
  TVM_FFI_ICHECK(dev >= 0 && dev < 64) << "device id out of range";
  if (cudaSetDevice(dev) != cudaSuccess) TVM_FFI_THROW(RuntimeError) << "cudaSetDevice failed";
  cudaStream_t stream = static_cast<cudaStream_t>(TVMFFIEnvGetStream(kDLCUDA, dev));
  size_t need = 0;
  if (dsa_sparse_attention_workspace_size(T, H, topk, &need) != DSA_OK)
    TVM_FFI_THROW(ValueError) << dsa_last_error_message();
  void* ws = workspace(dev, need, stream);
  const int rc = dsa_sparse_attention(
      bytes_of(q_nope), q_nope.stride(0), q_nope.stride(1), bytes_of(q_pe), q_pe.stride(0), q_pe.stride(1),
      bytes_of(ckv_cache), ckv_cache.stride(0), ckv_cache.stride(1), bytes_of(kpe_cache), kpe_cache.stride(0),
      kpe_cache.stride(1), reinterpret_cast<const int32_t*>(bytes_of(sparse_indices)), sparse_indices.stride(0),
      T, H, ckv_cache.size(0), 64, topk, static_cast<float>(sm_scale), bytes_of(output), output.stride(0),
      output.stride(1), reinterpret_cast<float*>(bytes_of(lse)), lse.stride(0), lse.stride(1), ws,
      g_ws[dev].bytes, stream);
  if (rc != DSA_OK) TVM_FFI_THROW(RuntimeError) << "dsa_sparse_attention: " << dsa_last_error_message();
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(dsa_sparse_attention, dsa_sparse_attention_ffi);
