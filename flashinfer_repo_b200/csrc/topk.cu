// topk.cu -- exact top-k selection of indexer scores, sm_100a.
//
// Replaces the reference's topk_kernel (solution/triton/indexer_kernel.py:
// 289-343), a register top-k with replace-the-minimum insertion (O(len*k);
// it writes every slot equal to the minimum, so ties create duplicates, and
// it returns logical ids seq_start+pos, :317).  This kernel defines a total
// order and is exact: for each request the min(k, len) positions with the
// largest scores, ties toward the lower position; the rest of the row is -1.
// Emitted in descending score (order 0) or ascending position (order 1).  It
// also emits the physical slot id block_table[b, pos/64]*64 + pos%64 that the
// attention operator consumes.
//
#include <cstdio>
#include <cstdlib>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {
namespace {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMax = 2048;
constexpr int kBins = 2048;

// Order-preserving key: larger float -> larger unsigned key; -0.0 and +0.0
// map to the same key (they compare equal, so position decides).
__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t u = (x == 0.f) ? 0u : __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA (1024 threads) per request:
// 1. The row is read once (float4 loads, 8 in flight per thread), converted to
//    order-preserving keys and kept in shared memory (rows up to kKeyCache;
//    longer rows are re-read from L2 in each pass), while the key range
//    [lo, hi] is reduced.
// 2. Adaptive radix select: bins span the current range (bin = (key - lo) >>
//    shift, at most kBins), so even the first pass spreads a real score
//    distribution; each pass keeps the bin holding the k-th largest key until
//    the range is one key T.  Eight histogram copies (one per four warps) cut
//    atomic contention; the bin is found with one block-wide scan (each thread
//    sums two bins over the copies).  Full passes run only until the kept bin
//    holds at most kMaxCand keys: a candidate pass then counts, per warp, the
//    keys above the kept bin and copies the keys inside it into shared
//    memory, and the remaining passes and the per-warp counts of step 3 run
//    over those candidates.
// 3. Selection in position order without atomics: warp w owns a contiguous
//    chunk, lane l four consecutive keys per round.  Per-warp counts of keys
//    > T and == T (from the candidate path, else a counting pass); one scan over
//    the 32 warps gives each warp its output offset and its share of the
//    wanted equal keys (ties go to the lowest positions); a writing pass
//    places (key << 32 | ~position) words with one warp scan per round.
// 4. Order 0 only: a bitonic sort of those words, descending (score, then
//    lower position): strides below 64 in registers with warp shuffles,
//    larger ones in shared memory.
constexpr int kHistCopies = 8;
constexpr int kFixedShift = 21;  // fixed first-pass bins: key >> 21 (2048 bins)
constexpr int kKeyCache = 32768;

struct TopkSmem {
  unsigned long long buf[kTopkMax];
  uint32_t hist[kHistCopies][kBins];
  uint32_t red_lo[32], red_hi[32];
  uint32_t w_cnt[32], w_off[32], w_eqb[32];
  uint32_t w_gt[32], w_ceq[32], w_cgt[32];  // candidate path: per-warp counts
  uint32_t lo, hi, bstar, above, bcount, ncand;
  uint4 keys[kKeyCache / 4];
};

__device__ __forceinline__ unsigned long long shfl_xor64(unsigned long long v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), m);
  return ((unsigned long long)hi << 32) | lo;
}

// Descending bitonic sort of buf[0, P), P a power of two in [64, 2048];
// 1024 threads, warp w holds words 64w + lane and 64w + 32 + lane.
__device__ void bitonic_desc(unsigned long long* buf, int P, int warp, int lane) {
  const bool active = warp * 64 < P;
  unsigned long long v0 = 0, v1 = 0;
  const int e0 = warp * 64 + lane, e1 = e0 + 32;
  if (active) {
    v0 = buf[e0];
    v1 = buf[e1];
  }
  for (int size = 2; size <= P; size <<= 1) {
    if (size > 64) {
      if (active) {
        buf[e0] = v0;
        buf[e1] = v1;
      }
      __syncthreads();
      for (int st = size >> 1; st >= 64; st >>= 1) {
        for (int i = warp * 32 + lane; i < P / 2; i += kTopkThreads) {
          const int l = 2 * i - (i & (st - 1));
          const int h = l + st;
          const bool desc = (l & size) == 0;
          const unsigned long long a = buf[l], c = buf[h];
          if ((a < c) == desc) {
            buf[l] = c;
            buf[h] = a;
          }
        }
        __syncthreads();
      }
      if (active) {
        v0 = buf[e0];
        v1 = buf[e1];
      }
    }
    for (int st = min(size >> 1, 32); st >= 1; st >>= 1) {
      if (st == 32) {
        const bool desc = (e0 & size) == 0;
        if ((v0 < v1) == desc) {
          const unsigned long long t = v0;
          v0 = v1;
          v1 = t;
        }
      } else {
        const bool low = (lane & st) == 0;
        const unsigned long long p0 = shfl_xor64(v0, st), p1 = shfl_xor64(v1, st);
        const bool d0 = (e0 & size) == 0, d1 = (e1 & size) == 0;
        // the low element of a pair keeps the larger word when descending
        v0 = (low == d0) ? (v0 > p0 ? v0 : p0) : (v0 < p0 ? v0 : p0);
        v1 = (low == d1) ? (v1 > p1 ? v1 : p1) : (v1 < p1 ? v1 : p1);
      }
    }
  }
  if (active) {
    buf[e0] = v0;
    buf[e1] = v1;
  }
  __syncthreads();
}

__device__ __forceinline__ uint4 keys4(const float4 v) {
  return make_uint4(ordered_key(v.x), ordered_key(v.y), ordered_key(v.z), ordered_key(v.w));
}

__global__ void __launch_bounds__(kTopkThreads)
    dsa_topk_kernel(const float* __restrict__ scores, int64_t stride, const int32_t* seq_lens,
                     const int32_t* block_table, int64_t bt_stride, int k, int32_t* positions,
                     int32_t* slots, int order) {
  extern __shared__ __align__(16) uint8_t topk_smem[];
  TopkSmem& S = *reinterpret_cast<TopkSmem*>(topk_smem);
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = max(0, seq_lens[b]);
  const float* sc = scores + (int64_t)b * stride;
  const int n_out = min(k, len);
  // shared-memory keys need 16-byte aligned rows for the vector loads
  const bool cached = len <= kKeyCache && ((reinterpret_cast<uintptr_t>(sc) & 15) == 0);
  const int n4 = (len + 3) >> 2;  // groups of four keys

  // key group g (positions 4g..4g+3; positions >= len read as key 0, never taken)
  auto group_at = [&](int g) -> uint4 {
    if (cached) return S.keys[g];
    uint4 r;
    const int i = 4 * g;
    r.x = i < len ? ordered_key(__ldcg(sc + i)) : 0u;
    r.y = i + 1 < len ? ordered_key(__ldcg(sc + i + 1)) : 0u;
    r.z = i + 2 < len ? ordered_key(__ldcg(sc + i + 2)) : 0u;
    r.w = i + 3 < len ? ordered_key(__ldcg(sc + i + 3)) : 0u;
    return r;
  };

  // ---- 1. load and key range; rows held in shared memory also get the first
  // histogram here, on fixed bins (the top 11 bits of the key)
  const bool fuse = cached && len > k;
  if (fuse) {
    for (int j = tid; j < kHistCopies * kBins; j += kTopkThreads) (&S.hist[0][0])[j] = 0;
    __syncthreads();
  }
  uint32_t tlo = 0xffffffffu, thi = 0u;
  auto fold = [&](uint32_t key, int i) {
    if (i < len) {
      tlo = min(tlo, key);
      thi = max(thi, key);
    }
  };
  if (cached) {
    const float4* s4 = reinterpret_cast<const float4*>(sc);
    for (int base = 0; base < n4; base += 8 * kTopkThreads) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int g = base + j * kTopkThreads + tid;
        v[j] = g < n4 ? __ldcs(s4 + g) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int g = base + j * kTopkThreads + tid;
        if (g < n4) {
          uint4 kk = keys4(v[j]);
          const int i = 4 * g;
          if (i + 1 >= len) kk.y = 0u;  // a partial last group: keys past len are 0
          if (i + 2 >= len) kk.z = 0u;
          if (i + 3 >= len) kk.w = 0u;
          S.keys[g] = kk;
          fold(kk.x, i);
          fold(kk.y, i + 1);
          fold(kk.z, i + 2);
          fold(kk.w, i + 3);
          if (fuse) {
            uint32_t* mine = S.hist[warp & (kHistCopies - 1)];
            atomicAdd(&mine[kk.x >> kFixedShift], 1u);
            if (i + 1 < len) atomicAdd(&mine[kk.y >> kFixedShift], 1u);
            if (i + 2 < len) atomicAdd(&mine[kk.z >> kFixedShift], 1u);
            if (i + 3 < len) atomicAdd(&mine[kk.w >> kFixedShift], 1u);
          }
        }
      }
    }
  } else {
    for (int g = tid; g < n4; g += kTopkThreads) {
      const uint4 kk = group_at(g);
      fold(kk.x, 4 * g);
      fold(kk.y, 4 * g + 1);
      fold(kk.z, 4 * g + 2);
      fold(kk.w, 4 * g + 3);
    }
  }
  tlo = __reduce_min_sync(0xffffffffu, tlo);
  thi = __reduce_max_sync(0xffffffffu, thi);
  if (lane == 0) {
    S.red_lo[warp] = tlo;
    S.red_hi[warp] = thi;
  }
  __syncthreads();
  if (warp == 0) {
    const uint32_t a = __reduce_min_sync(0xffffffffu, S.red_lo[lane]);
    const uint32_t c = __reduce_max_sync(0xffffffffu, S.red_hi[lane]);
    if (lane == 0) {
      S.lo = a;
      S.hi = c;
    }
  }
  __syncthreads();

  // ---- 2. exact threshold key T and how many keys == T are wanted
  uint32_t lo = S.lo, hi = S.hi;
  int need = n_out;
  const bool all = len <= k;
  // warp w owns groups [w*cg, (w+1)*cg) in the selection passes, lane l takes
  // group w*cg + r*32 + l in round r
  const int cg = (((n4 + 31) / 32) + 31) / 32 * 32;
  const int g0 = warp * cg, g1 = min(n4, g0 + cg);
  // Block-wide search of a histogram in top-down order: the bin b* holding
  // the need-th largest key and the count above it (thread t holds bins
  // kBins-1-2t and kBins-2-2t, summed over `copies` copies `cstride` apart).
  auto find_bin = [&](const uint32_t* h, int copies, int cstride, int nb, int want) {
    const int d_hi = kBins - 1 - 2 * tid, d_lo = d_hi - 1;
    uint32_t a = 0, c = 0;
    for (int q = 0; q < copies; ++q) {
      a += h[q * cstride + d_hi];
      c += h[q * cstride + d_lo];
    }
    if (d_hi >= nb) a = 0;
    if (d_lo >= nb) c = 0;
    const uint32_t sum = a + c;
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) S.w_cnt[warp] = incl;
    __syncthreads();
    uint32_t wsum = lane < warp ? S.w_cnt[lane] : 0u;
    wsum = __reduce_add_sync(0xffffffffu, wsum);
    const uint32_t run = wsum + incl - sum;  // keys in bins above d_hi
    if (run < (uint32_t)want && run + a >= (uint32_t)want) {
      S.bstar = (uint32_t)d_hi;
      S.above = run;
      S.bcount = a;
    } else if (run + a < (uint32_t)want && run + sum >= (uint32_t)want) {
      S.bstar = (uint32_t)d_lo;
      S.above = run + a;
      S.bcount = c;
    }
    __syncthreads();
  };
  auto bin_shift = [](uint32_t range) {
    int shift = 0;
    while ((range >> shift) >= (uint32_t)kBins) ++shift;
    return shift;
  };
  // Candidate path: after the first radix pass, one pass over the keys counts,
  // per warp, the keys above the kept bin (all taken) and collects the keys
  // inside it (at most kMaxCand) into shared memory; the rest of the radix
  // select and the per-warp counts of the selection then run over the
  // candidates only, so the later full passes (radix passes 2-3 and the
  // counting pass of step 3) are skipped.  Too many candidates (heavy ties):
  // the full passes run as before.
  constexpr uint32_t kMaxCand = kHistCopies * kBins / 2;
  bool counted = false;
  if (!all) {
    uint32_t* hist0 = &S.hist[0][0];
    uint32_t* mine = S.hist[warp & (kHistCopies - 1)];
    bool fused = fuse;  // the first histogram came with the load
    while (lo != hi) {
      uint32_t kept;
      if (fused) {
        fused = false;
        find_bin(hist0, kHistCopies, kBins, kBins, need);
        const uint32_t d = S.bstar;
        kept = S.bcount;
        need -= (int)S.above;
        lo = max(lo, d << kFixedShift);
        hi = min(hi, (d << kFixedShift) | ((1u << kFixedShift) - 1u));
      } else {
        const int shift = bin_shift(hi - lo);
        const int nb = (int)((hi - lo) >> shift) + 1;
        for (int j = tid; j < kHistCopies * kBins; j += kTopkThreads) hist0[j] = 0;
        __syncthreads();
        for (int g = tid; g < n4; g += kTopkThreads) {
          const uint4 kk = group_at(g);
          const int i = 4 * g;
          if (kk.x >= lo && kk.x <= hi) atomicAdd(&mine[(kk.x - lo) >> shift], 1u);
          if (i + 1 < len && kk.y >= lo && kk.y <= hi) atomicAdd(&mine[(kk.y - lo) >> shift], 1u);
          if (i + 2 < len && kk.z >= lo && kk.z <= hi) atomicAdd(&mine[(kk.z - lo) >> shift], 1u);
          if (i + 3 < len && kk.w >= lo && kk.w <= hi) atomicAdd(&mine[(kk.w - lo) >> shift], 1u);
        }
        __syncthreads();
        find_bin(hist0, kHistCopies, kBins, nb, need);
        const uint32_t d = S.bstar;
        kept = S.bcount;
        need -= (int)S.above;
        const uint32_t nlo = lo + (d << shift);
        hi = (uint32_t)min((unsigned long long)hi, (unsigned long long)nlo + (1ull << shift) - 1ull);
        lo = nlo;
      }
      __syncthreads();  // S.bstar / S.above / the histograms are rewritten next
      if (kept > kMaxCand) continue;  // another full pass narrows the bin first
      // ---- candidate pass over this warp's groups: keys > hi are taken,
      // keys in [lo, hi] are candidates (the histogram memory holds them)
      unsigned long long* cand = reinterpret_cast<unsigned long long*>(hist0);
      if (tid == 0) S.ncand = 0;
      __syncthreads();
      uint32_t n_gt = 0;
      if (cached) {
        // keys in shared memory: four ballots (one per key of a lane's group)
        // give every candidate of 128 keys its slot after one atomic, no scan
        const uint32_t lt = (1u << lane) - 1u;
#pragma unroll 2
        for (int gr = g0; gr < g1; gr += 32) {
          const int g = gr + lane;
          const bool gin = g < g1;
          const uint4 kk = gin ? S.keys[g] : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t v[4] = {kk.x, kk.y, kk.z, kk.w};
          uint32_t bq[4], tot = 0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const bool in = gin && 4 * g + q < len;
            n_gt += (in && v[q] > hi) ? 1u : 0u;
            bq[q] = __ballot_sync(0xffffffffu, in && v[q] >= lo && v[q] <= hi);
            tot += (uint32_t)__popc(bq[q]);
          }
          if (tot) {
            uint32_t base = 0;
            if (lane == 0) base = atomicAdd(&S.ncand, tot);
            base = __shfl_sync(0xffffffffu, base, 0);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              if ((bq[q] >> lane) & 1u) {
                const uint32_t o = base + (uint32_t)__popc(bq[q] & lt);
                if (o < kMaxCand) cand[o] = ((unsigned long long)v[q] << 32) | (uint32_t)(4 * g + q);
              }
              base += (uint32_t)__popc(bq[q]);
            }
          }
        }
      }
      for (int gr = cached ? g1 : g0; gr < g1; gr += 32) {
        const int g = gr + lane;
        const uint4 kk = g < g1 ? group_at(g) : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t v[4] = {kk.x, kk.y, kk.z, kk.w};
        uint32_t cm = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const bool in = g < g1 && 4 * g + q < len;
          n_gt += (in && v[q] > hi) ? 1u : 0u;
          cm |= (uint32_t)(in && v[q] >= lo && v[q] <= hi) << q;
        }
        if (__any_sync(0xffffffffu, cm != 0)) {  // most rounds hold no candidate
          const uint32_t nc_l = __popc(cm);
          uint32_t incl = nc_l;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
          }
          uint32_t base = 0;
          if (lane == 31) base = atomicAdd(&S.ncand, incl);
          base = __shfl_sync(0xffffffffu, base, 31) + incl - nc_l;
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if ((cm >> q) & 1u) {
              if (base < kMaxCand) cand[base] = ((unsigned long long)v[q] << 32) | (uint32_t)(4 * g + q);
              ++base;
            }
        }
      }
      n_gt = __reduce_add_sync(0xffffffffu, n_gt);
      if (lane == 0) {
        S.w_gt[warp] = n_gt;
        S.w_cgt[warp] = 0;
        S.w_ceq[warp] = 0;
      }
      __syncthreads();
      const uint32_t nc = S.ncand;  // == kept <= kMaxCand
      // ---- radix select over the candidates (bins in buf, one copy)
      uint32_t* h1 = reinterpret_cast<uint32_t*>(S.buf);
      while (lo != hi) {
        const int sh = bin_shift(hi - lo);
        const int nb1 = (int)((hi - lo) >> sh) + 1;
        for (int j = tid; j < kBins; j += kTopkThreads) h1[j] = 0;
        __syncthreads();
        for (uint32_t c = tid; c < nc; c += kTopkThreads) {
          const uint32_t key = (uint32_t)(cand[c] >> 32);
          if (key >= lo && key <= hi) atomicAdd(&h1[(key - lo) >> sh], 1u);
        }
        __syncthreads();
        find_bin(h1, 1, 0, nb1, need);
        const uint32_t d1 = S.bstar;
        need -= (int)S.above;
        const uint32_t nlo = lo + (d1 << sh);
        hi = (uint32_t)min((unsigned long long)hi, (unsigned long long)nlo + (1ull << sh) - 1ull);
        lo = nlo;
        __syncthreads();
      }
      // ---- per-warp counts of candidates above / equal to the threshold
      for (uint32_t c = tid; c < nc; c += kTopkThreads) {
        const uint32_t key = (uint32_t)(cand[c] >> 32);
        const int owner = (int)((cand[c] & 0xFFFFFFFFull) >> 2) / cg;
        if (key > lo) atomicAdd(&S.w_cgt[owner], 1u);
        else if (key == lo) atomicAdd(&S.w_ceq[owner], 1u);
      }
      __syncthreads();
      if (tid < 32) S.w_cnt[tid] = ((S.w_gt[tid] + S.w_cgt[tid]) << 16) | S.w_ceq[tid];
      counted = true;
      __syncthreads();
    }
  }
  const uint32_t T = lo;  // with `all`, every key is taken

  // ---- 3. selection in position order
  auto flags = [&](const uint4& kk, int i, uint32_t& gt, uint32_t& eq) {
    const uint32_t v[4] = {kk.x, kk.y, kk.z, kk.w};
    gt = 0;
    eq = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const bool in = i + q < len;
      gt |= (uint32_t)(in && (all || v[q] > T)) << q;
      eq |= (uint32_t)(in && !all && v[q] == T) << q;
    }
  };
  if (!counted) {  // counting pass (the candidate path has the counts already)
    uint32_t n_gt = 0, n_eq = 0;
    for (int g = g0 + lane; g < g1; g += 32) {
      uint32_t gt, eq;
      flags(group_at(g), 4 * g, gt, eq);
      n_gt += __popc(gt);
      n_eq += __popc(eq);
    }
    const uint32_t packed = __reduce_add_sync(0xffffffffu, (n_gt << 16) | n_eq);
    if (lane == 0) S.w_cnt[warp] = packed;
    __syncthreads();
  }
  if (warp == 0) {
    const uint32_t pk = S.w_cnt[lane];
    const uint32_t g = pk >> 16, e = pk & 0xffffu;
    uint32_t eb = e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, eb, o);
      if (lane >= o) eb += y;
    }
    eb -= e;  // equal keys in earlier warps
    const uint32_t want = (uint32_t)need > eb ? min(e, (uint32_t)need - eb) : 0u;
    const uint32_t cnt = g + want;
    uint32_t off = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, off, o);
      if (lane >= o) off += y;
    }
    S.w_off[lane] = off - cnt;
    S.w_eqb[lane] = eb;
  }
  __syncthreads();
  if (cached) {
    // keys in shared memory, one per lane per step: ballots of (key > T) and
    // (key == T) give each taken key its rank in position order; equal keys
    // (rare) are taken while their rank among this row's equal keys is below
    // need.  Unrolled so that several steps' shared-memory loads are in flight.
    uint32_t off = S.w_off[warp], eq_rank = S.w_eqb[warp];
    const uint32_t* K1 = reinterpret_cast<const uint32_t*>(S.keys);
    const int i1 = min(len, 4 * g1);
    const uint32_t lt = (1u << lane) - 1u;
#pragma unroll 4
    for (int i = 4 * g0 + lane; i - lane < i1; i += 32) {
      const bool in = i < i1;
      const uint32_t v = in ? K1[i] : 0u;
      bool take = in && (all || v > T);
      const bool eq = in && !all && v == T;
      const uint32_t be = __ballot_sync(0xffffffffu, eq);
      if (be) {  // uniform over the warp
        const uint32_t room = (uint32_t)need > eq_rank ? (uint32_t)need - eq_rank : 0u;
        take = take || (eq && (uint32_t)__popc(be & lt) < room);
        eq_rank += (uint32_t)__popc(be);
      }
      const uint32_t bt = __ballot_sync(0xffffffffu, take);
      if (take) {
        const uint32_t w = off + (uint32_t)__popc(bt & lt);
        if (w < (uint32_t)kTopkMax) S.buf[w] = ((unsigned long long)v << 32) | (0xFFFFFFFFu - (uint32_t)i);
      }
      off += (uint32_t)__popc(bt);
    }
  } else {
    uint32_t off = S.w_off[warp], eq_rank = S.w_eqb[warp];
    for (int gr = g0; gr < g1; gr += 32) {
      const int g = gr + lane;
      uint4 kk = make_uint4(0u, 0u, 0u, 0u);
      uint32_t gt = 0, eq = 0;
      if (g < g1) {
        kk = group_at(g);
        flags(kk, 4 * g, gt, eq);
      }
      // one lane-exclusive scan of (keys > T, keys == T) packed 16|16, in position order
      const uint32_t ng = __popc(gt), ne = __popc(eq);
      uint32_t pk = (ng << 16) | ne;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, pk, o);
        if (lane >= o) pk += y;
      }
      const uint32_t tot = __shfl_sync(0xffffffffu, pk, 31);
      pk -= (ng << 16) | ne;
      const uint32_t pg = pk >> 16, pe = pk & 0xffffu;
      // equal keys are wanted while their rank (position order) is below need
      const uint32_t room = (uint32_t)need > eq_rank ? (uint32_t)need - eq_rank : 0u;
      const uint32_t eq_before = min(pe, room);  // wanted equal keys in earlier lanes
      uint32_t take = gt;
      {
        uint32_t r = pe;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if ((eq >> q) & 1u) {
            if (r < room) take |= 1u << q;
            ++r;
          }
      }
      const uint32_t pt = pg + eq_before;
      const uint32_t tot_t = (tot >> 16) + min(tot & 0xffffu, room);
      const uint32_t tot_e = tot & 0xffffu;
      const uint32_t v[4] = {kk.x, kk.y, kk.z, kk.w};
      uint32_t w = off + pt;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if ((take >> q) & 1u) {
          if (w < (uint32_t)kTopkMax)
            S.buf[w] = ((unsigned long long)v[q] << 32) | (0xFFFFFFFFu - (uint32_t)(4 * g + q));
          ++w;
        }
      off += tot_t;
      eq_rank += tot_e;
    }
  }
  int P = 64;
  while (P < n_out) P <<= 1;
  __syncthreads();
  for (int j = n_out + tid; j < P; j += kTopkThreads) S.buf[j] = 0ull;  // sorts last
  __syncthreads();

  // ---- 4. order by score (order 0); order 1 keeps position order
  if (order == 0) bitonic_desc(S.buf, P, warp, lane);
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
                               int64_t k, int32_t* positions, int32_t* slots, int order,
                               void* stream) {
  if (batch < 0) return report_error(DSA_ERR_INVALID_ARG, "negative batch");
  if (k <= 0 || k > kTopkMax) return report_error(DSA_ERR_UNSUPPORTED, "k must be in [1, 2048]");
  if (order != 0 && order != 1) return report_error(DSA_ERR_INVALID_ARG, "order must be 0 or 1");
  if (batch == 0) return DSA_OK;
  if (!scores || !seq_lens || !positions || (slots && !block_table))
    return report_error(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  const int smem = (int)sizeof(TopkSmem);
  cudaError_t e = cudaFuncSetAttribute(dsa_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  dsa_topk_kernel<<<(unsigned)batch, kTopkThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      scores, scores_stride, seq_lens, block_table, block_table_stride, (int)k, positions, slots,
      order);
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
                                int order, int* device_error, void* stream) {
  int rc = dsa_indexer_scores(q_fp8, k_cache_fp8, k_page_stride, k_scale, scale_page_stride,
                              weights, block_table, block_table_stride, seq_lens, batch, num_heads,
                              head_dim, num_pages, max_len, scores_workspace, max_len, device_error,
                              stream);
  if (rc != DSA_OK) return rc;
  return dsa_topk_select(scores_workspace, max_len, seq_lens, block_table, block_table_stride, batch,
                         k, positions, slots, order, stream);
}
