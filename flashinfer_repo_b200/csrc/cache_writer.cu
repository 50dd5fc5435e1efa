// cache_writer.cu -- quantise new index keys to FP8 e4m3 and append them to
// the paged index-key cache that dsa_indexer_scores reads.
//
// The reference only reads this cache (solution/triton/indexer_kernel.py:
// 163-201: fp8 key rows plus a per-token scale, found through the block
// table); this is the producer side of that format.  Per token:
//   scale = max|k| / 448 (1 if the row is all zero), k8 = e4m3(k / scale),
// written as 128 key bytes at k_cache + page*k_page_stride + slot*128 and the
// fp32 scale at scale + page*s_page_stride + slot*4, where (page, slot) =
// (id >> 6, id & 63) of the token's flat slot id.  One warp per token, four
// elements per lane, warp-shuffle max; HBM-bound (256 B in, 132 B out).
#include <cuda_fp8.h>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {
namespace {

__global__ void __launch_bounds__(256)
    dsa_index_cache_append_kernel(const __nv_bfloat16* __restrict__ keys, int64_t n,
                                  const int32_t* __restrict__ slot_ids, uint8_t* k_cache,
                                  int64_t k_page_stride, uint8_t* scales, int64_t s_page_stride,
                                  int64_t num_pages, int* err) {
  const int64_t tok = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= n) return;
  const int32_t id = slot_ids[tok];
  if (id < 0) return;  // padding token: nothing to write
  const int64_t page = id >> 6, slot = id & 63;
  if (page >= num_pages) {
    if (lane == 0) set_error(err, kErrBadIndex);
    return;
  }
  const uint2 raw = *reinterpret_cast<const uint2*>(keys + tok * 128 + lane * 4);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  float v[4] = {__low2float(a), __high2float(a), __low2float(b), __high2float(b)};
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = amax > 0.f ? amax / 448.f : 1.f;
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(v[j] / scale, __NV_SATFINITE, __NV_E4M3);
    packed |= (uint32_t)q << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(k_cache + page * k_page_stride + slot * 128 + lane * 4) = packed;
  if (lane == 0) *reinterpret_cast<float*>(scales + page * s_page_stride + slot * 4) = scale;
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_index_cache_append(const void* keys_bf16, int64_t num_tokens,
                                      const int32_t* slot_ids, void* k_cache_fp8,
                                      int64_t k_page_stride, void* k_scale,
                                      int64_t scale_page_stride, int64_t num_pages,
                                      int* device_error, void* stream) {
  if (num_tokens < 0 || num_pages < 0) return report_error(DSA_ERR_INVALID_ARG, "negative size");
  if (num_tokens == 0) return DSA_OK;
  if (!keys_bf16 || !slot_ids || !k_cache_fp8 || !k_scale)
    return report_error(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  if ((reinterpret_cast<uintptr_t>(keys_bf16) & 7) || (reinterpret_cast<uintptr_t>(k_cache_fp8) & 3) ||
      (reinterpret_cast<uintptr_t>(k_scale) & 3) || k_page_stride % 4 || scale_page_stride % 4)
    return report_error(DSA_ERR_INVALID_ARG, "misaligned key, cache or scale pointer / stride");
  const int64_t threads = num_tokens * 32;
  dsa_index_cache_append_kernel<<<(unsigned)((threads + 255) / 256), 256, 0,
                                  static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(keys_bf16), num_tokens, slot_ids,
      static_cast<uint8_t*>(k_cache_fp8), k_page_stride, static_cast<uint8_t*>(k_scale),
      scale_page_stride, num_pages, device_error);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  return DSA_OK;
}
