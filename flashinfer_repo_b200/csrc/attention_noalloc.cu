// attention_noalloc.cu -- dsa_sparse_attention without a caller-provided workspace.
//
// Some callers of this operator cannot allocate device memory at call time:
// serving engines that reserve almost all free HBM for the KV cache at start-up
// and route every later allocation through their own pool (a stray cudaMalloc
// there fails or breaks their accounting), and plugin hosts whose interface
// hands an operator only its input and output buffers, with no workspace
// argument and no allocator to call.  For them this entry point runs the same
// kernel as dsa_sparse_attention with its scratch (error word, split-K
// partials) in a fixed-size array that lives in the
// library's own device memory.
//
// Facts a caller must know:
//  * The array takes kNoAllocScratchBytes (about 20 MiB) on EVERY device that
//    loads this library, for as long as the process runs.
//  * Limits: num_tokens * num_heads / 16 <= kNoAllocMaxVirtualTokens, and the
//    kernel's grid must fit kNoAllocMaxCtas CTAs; larger calls are rejected
//    with DSA_ERR_UNSUPPORTED and a message, nothing is launched.
//  * The first call on a device looks up the array's device address (once per
//    device, with that device current); make that first call before any stream
//    capture begins.
//  * All calls on a device share the one array and it keeps the last call's
//    contents.  Calls whose executions overlap on the GPU (different streams,
//    or several host threads) race on it and give wrong results; serialise
//    them.  Each call clears the error word.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <mutex>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace {

constexpr size_t kNoAllocMaxVirtualTokens = 8192;
constexpr size_t kNoAllocMaxCtas = 320;
constexpr size_t kPartBytes = (16 * 512 + 2 * 16) * sizeof(float);  // one split-K partial
constexpr size_t kCounterBytes = 256;  // error word
constexpr size_t kNoAllocScratchBytes = kCounterBytes + 2 * kNoAllocMaxCtas * kPartBytes;

// Zero-initialised at module load; one instance per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[64] = {};  // device address of g_noalloc_scratch, per device

// Messages go through the library's error channel (dsa_last_error_message).
int dsa_noalloc_fail(int code, const char* msg) { return dsa::report_error(code, msg); }

}  // namespace

extern "C" int dsa_sparse_attention_noalloc(
    const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head, const void* q_pe,
    int64_t q_pe_stride_token, int64_t q_pe_stride_head, const void* ckv_cache,
    int64_t ckv_stride_page, int64_t ckv_stride_row, const void* kpe_cache, int64_t kpe_stride_page,
    int64_t kpe_stride_row, const int32_t* sparse_indices, int64_t indices_stride_token,
    int64_t num_tokens, int64_t num_heads, int64_t num_pages, int64_t page_size, int64_t topk,
    float sm_scale, void* output, int64_t out_stride_token, int64_t out_stride_head, float* lse,
    int64_t lse_stride_token, int64_t lse_stride_head, void* stream) {
  if (num_tokens < 0 || num_heads <= 0 || num_heads % 16)
    return dsa_sparse_attention(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe,
                                q_pe_stride_token, q_pe_stride_head, ckv_cache, ckv_stride_page,
                                ckv_stride_row, kpe_cache, kpe_stride_page, kpe_stride_row,
                                sparse_indices, indices_stride_token, num_tokens, num_heads,
                                num_pages, page_size, topk, sm_scale, output, out_stride_token,
                                out_stride_head, lse, lse_stride_token, lse_stride_head, nullptr, 0,
                                stream);  // reports the argument error
  const int64_t vtokens = num_tokens * (num_heads / 16);
  if ((size_t)vtokens > kNoAllocMaxVirtualTokens) {
    return dsa_noalloc_fail(DSA_ERR_UNSUPPORTED,
                            "dsa_sparse_attention_noalloc: num_tokens*num_heads/16 exceeds the "
                            "8192 the static scratch holds; use dsa_sparse_attention");
  }
  if (num_tokens == 0) return DSA_OK;

  // Once per device: the device address of the scratch array.
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64)
    return dsa_noalloc_fail(DSA_ERR_CUDA, "dsa_sparse_attention_noalloc: no current CUDA device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return dsa_noalloc_fail(DSA_ERR_CUDA, cudaGetErrorString(e));
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }

  size_t need = 0;
  int rc = dsa_sparse_attention_workspace_size(num_tokens, num_heads, topk, &need);
  if (rc != DSA_OK) return rc;
  if (need > kNoAllocScratchBytes)
    return dsa_noalloc_fail(DSA_ERR_UNSUPPORTED,
                            "dsa_sparse_attention_noalloc: this shape needs more split-K scratch "
                            "than the static array holds; use dsa_sparse_attention");

  // The error word starts at zero.
  e = cudaMemsetAsync(scratch, 0, sizeof(int), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return dsa_noalloc_fail(DSA_ERR_CUDA, cudaGetErrorString(e));

  return dsa_sparse_attention(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe,
                              q_pe_stride_token, q_pe_stride_head, ckv_cache, ckv_stride_page,
                              ckv_stride_row, kpe_cache, kpe_stride_page, kpe_stride_row,
                              sparse_indices, indices_stride_token, num_tokens, num_heads, num_pages,
                              page_size, topk, sm_scale, output, out_stride_token, out_stride_head,
                              lse, lse_stride_token, lse_stride_head, scratch,
                              kNoAllocScratchBytes, stream);
}
