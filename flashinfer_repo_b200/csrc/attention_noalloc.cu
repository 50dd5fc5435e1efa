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
//  * The array takes kNoAllocScratchBytes (about 20 MiB) on every device where
//    it is used, for as long as the process runs.  With CUDA's default lazy
//    module loading the array is placed in device memory when this file's code
//    is first used on a device, i.e. by the first call: make that first call
//    (a warm-up call) before the engine reserves its memory pool, or run with
//    CUDA_MODULE_LOADING=EAGER so that it is placed when the library loads.
//  * Limit: the scratch holds the split-K partials of at most kNoAllocMaxCtas
//    CTAs (two slots each).  The default launch plan on a B200 uses at most
//    2 x 148 = 296 CTAs for any batch, so every shape the operator accepts
//    fits; only a plan forced larger through dsa_set_options is rejected with
//    DSA_ERR_UNSUPPORTED and a message, and nothing is launched.
//  * The first call on a device looks up the array's device address (once per
//    device, with that device current); make that first call before any stream
//    capture begins.
//  * All calls on a device share the one array and it keeps the last call's
//    contents.  Calls whose executions overlap on the GPU (different streams,
//    or several host threads) race on it and give wrong results; serialise
//    them.
//  * Device errors (a bad index, a timed-out wait) accumulate in the array's
//    error word across calls until dsa_sparse_attention_noalloc_read_error
//    reads (and optionally clears) it; it starts at zero.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <mutex>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace {

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

// Device address of the scratch array on the current device, looked up once
// per device (cudaGetSymbolAddress with that device current).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64)
    return dsa_noalloc_fail(DSA_ERR_CUDA, "dsa_sparse_attention_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return dsa_noalloc_fail(DSA_ERR_CUDA, cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return DSA_OK;
}

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
  if (num_tokens == 0) return DSA_OK;
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != DSA_OK) return rc;

  size_t need = 0;
  rc = dsa_sparse_attention_workspace_size(num_tokens, num_heads, topk, &need);
  if (rc != DSA_OK) return rc;
  if (need > kNoAllocScratchBytes)
    return dsa_noalloc_fail(DSA_ERR_UNSUPPORTED,
                            "dsa_sparse_attention_noalloc: the launch plan has more than the 320 "
                            "CTAs whose split-K partials the static array holds; use "
                            "dsa_sparse_attention");

  return dsa_sparse_attention(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe,
                              q_pe_stride_token, q_pe_stride_head, ckv_cache, ckv_stride_page,
                              ckv_stride_row, kpe_cache, kpe_stride_page, kpe_stride_row,
                              sparse_indices, indices_stride_token, num_tokens, num_heads, num_pages,
                              page_size, topk, sm_scale, output, out_stride_token, out_stride_head,
                              lse, lse_stride_token, lse_stride_head, scratch,
                              kNoAllocScratchBytes, stream);
}

extern "C" int dsa_sparse_attention_noalloc_read_error(int clear, int* bits, void* stream) {
  if (!bits) return dsa_noalloc_fail(DSA_ERR_INVALID_ARG, "bits is NULL");
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != DSA_OK) return rc;
  return dsa_read_device_error(scratch, clear, bits, stream);
}
