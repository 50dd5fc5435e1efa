// topk.cu -- exact top-k selection of indexer scores, sm_100a.
//
// Replaces the reference's topk_kernel (solution/triton/indexer_kernel.py:
// 289-343), a register top-k with replace-the-minimum insertion (O(len*k);
// it writes every slot equal to the minimum, so ties create duplicates, and
// it returns logical ids seq_start+pos, :317).  This kernel defines a total
// order and is exact: for each request the min(k, len) positions with the
// largest scores, in descending score, ties toward the lower position; the
// rest of the row is -1.  It also emits the physical slot id
// block_table[b, pos/64]*64 + pos%64 that the attention operator consumes.
//
// One CTA (1024 threads) per request:
//  0. rows up to 40960 scores are read once into shared memory;
//  1. radix select over order-preserving 32-bit keys, digits of 11/11/10
//     bits, with a shared-memory histogram, finds the k-th largest key T;
//  2. one pass in index order keeps every key > T and, among keys == T, the
//     lowest positions (block-wide ballot prefix counts keep index order);
//  3. a bitonic sort of the (key, ~position) pairs in shared memory.
#include <cstdio>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 2048;
constexpr int kTopkCache = 40960;  // rows up to this length are read from HBM once
constexpr int kBins = 2048;

// Order-preserving key: larger float -> larger unsigned key; -0.0 and +0.0
// map to the same key (they compare equal, so position decides).
__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t u = (x == 0.f) ? 0u : __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct TopkSmem {
  unsigned long long buf[kTopkMax];
  uint32_t hist[kBins];
  uint32_t warp_cnt[kTopkThreads / 32];
  uint32_t digit, above;
  float cache[kTopkCache];
};

__global__ void __launch_bounds__(kTopkThreads)
    dsa_topk_kernel(const float* __restrict__ scores, int64_t stride, const int32_t* seq_lens,
                    const int32_t* block_table, int64_t bt_stride, int k, int32_t* positions,
                    int32_t* slots) {
  extern __shared__ __align__(16) uint8_t topk_smem[];
  TopkSmem& S = *reinterpret_cast<TopkSmem*>(topk_smem);
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = max(0, seq_lens[b]);
  const float* sc = scores + (int64_t)b * stride;
  const int n_out = min(k, len);
  const bool cached = len <= kTopkCache;

  for (int i = tid; i < kTopkMax; i += kTopkThreads) S.buf[i] = 0ull;  // sorts last
  if (cached) {  // one pass over HBM/L2, 8 loads in flight per thread
    for (int base = 0; base < len; base += 8 * kTopkThreads) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = base + j * kTopkThreads + tid;
        v[j] = i < len ? __ldcs(sc + i) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = base + j * kTopkThreads + tid;
        if (i < len) S.cache[i] = v[j];
      }
    }
    __syncthreads();
  }
  auto score_at = [&](int i) -> float { return cached ? S.cache[i] : __ldcg(sc + i); };

  uint32_t prefix = 0, mask = 0;
  int need = n_out;  // elements still to take from the class equal to the threshold
  if (len > k) {
    // digits of 11, 11 and 10 bits, most significant first
    for (int pass = 0; pass < 3; ++pass) {
      const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
      const int bits = pass == 2 ? 10 : 11;
      const uint32_t dmask = (1u << bits) - 1u;
      for (int i = tid; i < kBins; i += kTopkThreads) S.hist[i] = 0;
      __syncthreads();
      for (int base = 0; base < len; base += kTopkThreads) {
        const int i = base + tid;
        uint32_t key = 0;
        bool in = false;
        if (i < len) {
          key = ordered_key(score_at(i));
          in = (key & mask) == prefix;
        }
        // warp-aggregated increment: real score distributions pile into a few
        // bins, and per-thread shared atomics on one address serialise
        const unsigned active = __ballot_sync(0xffffffffu, in);
        if (in) {
          const uint32_t bin = (key >> shift) & dmask;
          const unsigned peers = __match_any_sync(active, bin);
          if ((__ffs(peers) - 1) == lane) atomicAdd(&S.hist[bin], (uint32_t)__popc(peers));
        }
      }
      __syncthreads();
      if (warp == 0) {
        // digit d with count(> d) < need <= count(>= d): bins scanned from the
        // top, 64 per lane, warp prefix sum over the lanes
        const int nb = 1 << bits, per = nb / 32;
        uint32_t tot = 0;
        for (int j = 0; j < per; ++j) tot += S.hist[nb - 1 - (lane * per + j)];
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        uint32_t run = incl - tot;
        if (run < (uint32_t)need && incl >= (uint32_t)need) {
          for (int j = 0; j < per; ++j) {
            const int d = nb - 1 - (lane * per + j);
            const uint32_t h = S.hist[d];
            if (run < (uint32_t)need && run + h >= (uint32_t)need) {
              S.digit = d;
              S.above = run;
            }
            run += h;
          }
        }
      }
      __syncthreads();
      need -= (int)S.above;
      prefix |= S.digit << shift;
      mask |= dmask << shift;
      __syncthreads();
    }
  }
  // Threshold key T = prefix (all keys qualify when len <= k).  Keep keys > T
  // and the first `need` keys == T in position order.
  const uint32_t T = prefix;
  const bool all = len <= k;
  int taken_gt = 0, taken_eq = 0;
  const int n_gt = n_out - need;  // slots [0, n_gt) for keys > T, then equal keys
  for (int base = 0; base < len; base += kTopkThreads) {
    const int i = base + tid;
    uint32_t key = 0;
    bool gt = false, eq = false;
    if (i < len) {
      key = ordered_key(score_at(i));
      gt = all || key > T;
      eq = !all && key == T;
    }
    const uint32_t bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) S.warp_cnt[warp] = (__popc(bg) << 16) | __popc(be);
    __syncthreads();
    // exclusive prefix of the per-warp counts (both packed in one word)
    const uint32_t cnt = S.warp_cnt[lane];
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = __shfl_sync(0xffffffffu, incl - cnt, warp);
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    const uint32_t off_g = excl >> 16, off_e = excl & 0xffffu;
    const uint32_t tot_g = total >> 16, tot_e = total & 0xffffu;
    const uint32_t lt = (1u << lane) - 1u;
    const unsigned long long comp =
        ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
    if (gt) {
      const int slot = taken_gt + (int)(off_g + __popc(bg & lt));
      if (slot < kTopkMax) S.buf[slot] = comp;
    }
    if (eq) {
      const int r = taken_eq + (int)(off_e + __popc(be & lt));
      if (r < need) S.buf[n_gt + r] = comp;
    }
    taken_gt += (int)tot_g;
    taken_eq += (int)tot_e;
    __syncthreads();
  }
  // Bitonic sort, descending, over kTopkMax entries.
  for (int size = 2; size <= kTopkMax; size <<= 1) {
    for (int stride2 = size >> 1; stride2 > 0; stride2 >>= 1) {
      for (int i = tid; i < kTopkMax / 2; i += kTopkThreads) {
        const int lo = 2 * i - (i & (stride2 - 1));
        const int hi = lo + stride2;
        const bool desc = ((lo & size) == 0);
        const unsigned long long a = S.buf[lo], c = S.buf[hi];
        if ((a < c) == desc) {
          S.buf[lo] = c;
          S.buf[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  for (int j = tid; j < k; j += kTopkThreads) {
    int32_t pos = -1, slot = -1;
    if (j < n_out) {
      pos = (int32_t)(0xFFFFFFFFu - (uint32_t)(S.buf[j] & 0xFFFFFFFFull));
      if (slots) slot = block_table[(int64_t)b * bt_stride + (pos >> 6)] * 64 + (pos & 63);
    }
    positions[(int64_t)b * k + j] = pos;
    if (slots) slots[(int64_t)b * k + j] = slot;
  }
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" int dsa_topk_select(const float* scores, int64_t scores_stride, const int32_t* seq_lens,
                               const int32_t* block_table, int64_t block_table_stride, int64_t batch,
                               int64_t k, int32_t* positions, int32_t* slots, void* stream) {
  if (batch < 0) return report_error(DSA_ERR_INVALID_ARG, "negative batch");
  if (k <= 0 || k > kTopkMax) return report_error(DSA_ERR_UNSUPPORTED, "k must be in [1, 2048]");
  if (batch == 0) return DSA_OK;
  if (!scores || !seq_lens || !positions || (slots && !block_table))
    return report_error(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  const int smem = (int)sizeof(TopkSmem);
  cudaError_t e = cudaFuncSetAttribute(dsa_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  dsa_topk_kernel<<<(unsigned)batch, kTopkThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      scores, scores_stride, seq_lens, block_table, block_table_stride, (int)k, positions, slots);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  return DSA_OK;
}

extern "C" int dsa_indexer_topk(const void* q_fp8, const void* k_cache_fp8, int64_t k_page_stride,
                                const void* k_scale, int64_t scale_page_stride, const float* weights,
                                const int32_t* block_table, int64_t block_table_stride,
                                const int32_t* seq_lens, int64_t batch, int64_t num_heads,
                                int64_t head_dim, int64_t num_pages, int64_t max_len, int64_t k,
                                float* scores_workspace, int32_t* positions, int32_t* slots,
                                int* device_error, void* stream) {
  int rc = dsa_indexer_scores(q_fp8, k_cache_fp8, k_page_stride, k_scale, scale_page_stride,
                              weights, block_table, block_table_stride, seq_lens, batch, num_heads,
                              head_dim, num_pages, max_len, scores_workspace, max_len, device_error,
                              stream);
  if (rc != DSA_OK) return rc;
  return dsa_topk_select(scores_workspace, max_len, seq_lens, block_table, block_table_stride, batch,
                         k, positions, slots, stream);
}
