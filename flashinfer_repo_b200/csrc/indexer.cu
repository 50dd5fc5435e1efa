// indexer.cu -- FP8 "lightning indexer" scores on sm_100a tensor cores (tcgen05).
//
// Semantics: the reference indexer (solution/triton/indexer_kernel.py:4-287)
// computes, for request b and each token position t < seq_len[b],
//   score[b,t] = sum_h w[b,h] * ReLU(q[b,h,:] . k_t)  with k_t = fp8 key row
//                 of token t dequantised by its per-token scale (:186-201,
//                 :258-275), the key row found through the block table (:159).
// Because the scale is positive it factors out of the ReLU; this kernel
// computes score = scale_t * sum_h w_h * ReLU(q_h . k8_t), with the fp8 dot
// products exact in fp32 on the tensor cores.
//
// Layout: keys are fp8 e4m3 rows of 128 bytes, 64 tokens per page, at
// k_cache + page*k_page_stride + slot*128 (bytes); the fp32 scale of a token
// at scale + page*s_page_stride + slot*4.  This covers both separate key /
// scale tensors ([P,64,128] + [P,64]) and the page-packed format (each page
// holds 64x128 key bytes followed by 64 fp32 scales).
//
// Design (B200): one CTA works on a run of 128-token tiles of one request.
//  * warp 4 (one lane) loads the request's queries [64 heads x 128 B] once
//    and, per tile, the two key pages with TMA (128-byte swizzle) into a
//    4-stage shared-memory ring;
//  * warp 5 (one lane) issues tcgen05.mma kind::f8f6f4, M=128 tokens, N=64
//    heads, K=128 (4 instructions of K=32), into one of two TMEM accumulators
//    (64 columns each), and commits to mbarriers;
//  * warps 0-3 (thread = token row = TMEM lane) read the 64 head logits with
//    tcgen05.ld, apply ReLU, the head weights and the token scale, and store
//    the fp32 score.
// The path is HBM-bound (132 B per token, 16 KFLOP per token).
#include <cuda.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {
namespace {

constexpr int kIdxHeads = 64;
constexpr int kIdxDim = 128;
constexpr int kTileTokens = 128;
constexpr int kIdxStages = 4;
constexpr int kIdxThreads = 192;

struct IdxParams {
  const uint8_t* scale;  // byte base of the fp32 scales
  int64_t s_page_stride;  // bytes
  const float* w;        // [B, 64]
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* seq_lens;
  float* scores;
  int64_t scores_stride;
  int64_t num_pages;
  int tiles_per_cta;
  int* err;
};

struct __align__(1024) IdxSmem {
  uint8_t kbuf[kIdxStages][kTileTokens * kIdxDim];  // 16 KB each, 128-byte swizzled
  uint8_t qbuf[kIdxHeads * kIdxDim];                 // 8 KB, 128-byte swizzled
  float w[kIdxHeads];
  uint64_t full[kIdxStages], empty[kIdxStages];
  uint64_t tfull[2], tempty[2];
  uint64_t qbar;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kIdxThreads)
    dsa_indexer_kernel(const __grid_constant__ CUtensorMap tmap_k,
                       const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ IdxParams p) {
  extern __shared__ uint8_t smem_raw[];
  IdxSmem& S = *reinterpret_cast<IdxSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int len = p.seq_lens[b];
  const int ntiles = (len + kTileTokens - 1) / kTileTokens;
  const int t0 = blockIdx.x * p.tiles_per_cta;
  const int t1 = min(ntiles, t0 + p.tiles_per_cta);
  if (t0 >= t1) return;  // uniform over the CTA: nothing allocated yet
  const int npages = (len + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kIdxStages; ++s) {
      mbar_init(&S.full[s], 1);
      mbar_init(&S.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S.tfull[a], 1);
      mbar_init(&S.tempty[a], 4);
    }
    mbar_init(&S.qbar, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < kIdxHeads) S.w[threadIdx.x] = p.w[(int64_t)b * kIdxHeads + threadIdx.x];
  if (warp == 5) tmem_alloc(&S.tmem_base, 128);  // two 64-column fp32 accumulators
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&S.qbar, kIdxHeads * kIdxDim);
      tma_load_2d(S.qbuf, &tmap_q, 0, b * kIdxHeads, &S.qbar);
      int li = 0;
      for (int t = t0; t < t1; ++t, ++li) {
        const int s = li % kIdxStages;
        if (!mbar_wait(&S.empty[s], ((li / kIdxStages) & 1) ^ 1)) {
          set_error(p.err, kErrTimeout);
          break;
        }
        int pg[2];
        uint32_t bytes = 0;
        for (int h = 0; h < 2; ++h) {
          const int lp = 2 * t + h;
          pg[h] = -1;
          if (lp < npages) {
            const int phys = p.block_table[(int64_t)b * p.bt_stride + lp];
            if (phys >= 0 && phys < p.num_pages) {
              pg[h] = phys;
              bytes += 64 * kIdxDim;
            } else {
              set_error(p.err, kErrBadIndex);
            }
          }
        }
        mbar_arrive_expect_tx(&S.full[s], bytes);
        for (int h = 0; h < 2; ++h)
          if (pg[h] >= 0) tma_load_3d(S.kbuf[s] + h * 64 * kIdxDim, &tmap_k, 0, 0, pg[h], &S.full[s]);
      }
      // let the last copies land before the CTA can exit
      for (int k = li > kIdxStages ? li - kIdxStages : 0; k < li; ++k)
        mbar_wait(&S.full[k % kIdxStages], (k / kIdxStages) & 1);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0, 0, 0, 0, kTileTokens, kIdxHeads);  // e4m3 x e4m3
      bool ok = mbar_wait(&S.qbar, 0);
      if (!ok) set_error(p.err, kErrTimeout);
      int li = 0;
      for (int t = t0; ok && t < t1; ++t, ++li) {
        const int s = li % kIdxStages, ab = li & 1;
        if (!mbar_wait(&S.full[s], (li / kIdxStages) & 1) ||
            !mbar_wait(&S.tempty[ab], ((li >> 1) & 1) ^ 1)) {
          set_error(p.err, kErrTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(S.kbuf[s]), b0 = smem_u32(S.qbuf);
#pragma unroll
        for (int kk = 0; kk < kIdxDim / 32; ++kk)
          umma_f8(tmem + ab * 64, umma_desc(a0 + kk * 32, 16, 1024, kSwizzle128B),
                  umma_desc(b0 + kk * 32, 16, 1024, kSwizzle128B), idesc, kk > 0);
        umma_commit(&S.empty[s]);   // smem stage free once these MMAs finish
        umma_commit(&S.tfull[ab]);  // accumulator ready for the epilogue
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int row = warp * 32 + lane;  // token row of the tile == TMEM lane
    int li = 0;
    for (int t = t0; t < t1; ++t, ++li) {
      const int ab = li & 1;
      const int tok = t * kTileTokens + row;
      float sc = 0.f;
      if (tok < len) {
        const int phys = p.block_table[(int64_t)b * p.bt_stride + (tok >> 6)];
        if (phys >= 0 && phys < p.num_pages)
          sc = *reinterpret_cast<const float*>(p.scale + phys * p.s_page_stride + (tok & 63) * 4);
      }
      if (!mbar_wait(&S.tfull[ab], (li >> 1) & 1)) {
        set_error(p.err, kErrTimeout);
        break;
      }
      tc_fence_after();
      float acc = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + ab * 64 + half * 32, v);
#pragma unroll
        for (int h = 0; h < 32; ++h) acc += S.w[half * 32 + h] * fmaxf(v[h], 0.f);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.tempty[ab]);
      if (tok < len) p.scores[(int64_t)b * p.scores_stride + tok] = acc * sc;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}


}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_indexer_scores(const void* q_fp8, const void* k_cache_fp8, int64_t k_page_stride,
                                  const void* k_scale, int64_t scale_page_stride, const float* weights,
                                  const int32_t* block_table, int64_t block_table_stride,
                                  const int32_t* seq_lens, int64_t batch, int64_t num_heads,
                                  int64_t head_dim, int64_t num_pages, int64_t max_len,
                                  float* scores, int64_t scores_stride, int* device_error,
                                  void* stream) {
  if (batch < 0 || max_len < 0) return report_error(DSA_ERR_INVALID_ARG, "negative size");
  if (num_heads != kIdxHeads || head_dim != kIdxDim)
    return report_error(DSA_ERR_UNSUPPORTED, "indexer needs 64 heads of dimension 128");
  if (batch == 0 || max_len == 0) return DSA_OK;
  if (!q_fp8 || !k_cache_fp8 || !k_scale || !weights || !block_table || !seq_lens || !scores)
    return report_error(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  if ((reinterpret_cast<uintptr_t>(q_fp8) & 15) || (reinterpret_cast<uintptr_t>(k_cache_fp8) & 15) ||
      k_page_stride % 16 || k_page_stride < 64 * kIdxDim)
    return report_error(DSA_ERR_INVALID_ARG,
                        "keys and queries must be 16-byte aligned, page stride a multiple of 16");
  if ((reinterpret_cast<uintptr_t>(k_scale) & 3) || scale_page_stride % 4)
    return report_error(DSA_ERR_INVALID_ARG, "scales must be 4-byte aligned");
  if (scores_stride < max_len) return report_error(DSA_ERR_INVALID_ARG, "scores_stride < max_len");
  EncodeTiledFn enc = encode_fn();
  if (!enc) return report_error(DSA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");

  CUtensorMap tk, tq;
  {
    cuuint64_t dims[3] = {(cuuint64_t)kIdxDim, 64, (cuuint64_t)num_pages};
    cuuint64_t strides[2] = {(cuuint64_t)kIdxDim, (cuuint64_t)k_page_stride};
    cuuint32_t box[3] = {kIdxDim, 64, 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(k_cache_fp8), dims, strides,
            box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return report_error(DSA_ERR_INVALID_ARG, "cannot encode the key tensor map");
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)kIdxDim, (cuuint64_t)(batch * kIdxHeads)};
    cuuint64_t strides[1] = {(cuuint64_t)kIdxDim};
    cuuint32_t box[2] = {kIdxDim, kIdxHeads};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(q_fp8), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return report_error(DSA_ERR_INVALID_ARG, "cannot encode the query tensor map");
  }
  IdxParams p;
  p.scale = static_cast<const uint8_t*>(k_scale);
  p.s_page_stride = scale_page_stride;
  p.w = weights;
  p.block_table = block_table;
  p.bt_stride = block_table_stride;
  p.seq_lens = seq_lens;
  p.scores = scores;
  p.scores_stride = scores_stride;
  p.num_pages = num_pages;
  dsa_options opt;
  dsa_get_options(&opt);
  // Default 20 tiles (2560 tokens) per CTA.  Measured on a B200 at ctx 32768
  // (fraction of the HBM peak at 16 / 20 / 26 tiles per CTA, L2 flushed):
  // 128 requests 0.78 / 0.81 / 0.83, 64 requests 0.66 / 0.73 / 0.68,
  // 32 requests 0.52 / 0.60 / 0.58 -- fewer, longer CTAs amortise the per-CTA
  // set-up (TMEM allocation, query load, ring fill) until too few remain.
  p.tiles_per_cta = opt.indexer_tiles_per_cta > 0 ? opt.indexer_tiles_per_cta : 20;
  if (p.tiles_per_cta < 1) p.tiles_per_cta = 1;
  p.err = device_error;
  const int smem = (int)sizeof(IdxSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(dsa_indexer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem);
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  const int64_t max_tiles = (max_len + kTileTokens - 1) / kTileTokens;
  dim3 grid((unsigned)((max_tiles + p.tiles_per_cta - 1) / p.tiles_per_cta), (unsigned)batch);
  dsa_indexer_kernel<<<grid, kIdxThreads, smem, static_cast<cudaStream_t>(stream)>>>(tk, tq, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  return DSA_OK;
}
