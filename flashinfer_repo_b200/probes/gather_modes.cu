// gather_modes.cu -- how fast can random latent-cache rows be gathered into
// shared memory on this GPU, by each copy mechanism?  A measurement probe for
// the data mover of the sparse-attention kernels (no counterpart in the
// reference); it computes nothing on the rows.
//
// Workload: T query tokens x 2048 distinct rows each, a row being the 1024-B
// ckv part plus the 128-B kpe part of one cached token (1152 B), drawn at
// random from a request-sized range of a large cache (HBM mode, about 2.5 GB,
// L2 flushed between launches) or from a 75 MB cache that stays in L2
// (--l2: 1024 tokens).  Mechanisms, each with consumers that only wait for
// a slot and release it:
//   raw ldg       plain 16-B loads into registers, no shared memory (ceiling)
//   bulk          one cp.async.bulk per 1-KB ckv row + 16-B cp.async for kpe
//                 into a padded ring (the mma.sync kernel's mover)
//   gather4       cp.async.bulk.tensor.2d tile::gather4 (4 rows x 64 columns,
//                 128-byte swizzle, box one row high), the UMMA operand layout
//   lsu cp.async  16-B cp.async into the same swizzled layout
// Every swizzled variant is checked once against the source rows.
//
//   python -m flashinfer_repo_b200.build --probes
//   flashinfer_repo_b200/probes/gather_modes [--l2] [--order random|sorted|pages]
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <random>
#include <algorithm>
#include "../csrc/common.cuh"
using namespace dsa;

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e_), __LINE__); exit(1);} } while (0)

constexpr int ROWS = 32;           // rows per slot
constexpr int PANEL = ROWS * 128;  // one 64-col panel of a slot
constexpr int SLOT = 9 * PANEL;    // 36,864 B

struct Args {
  const uint8_t* ckv; const uint8_t* kpe; const int* idx; int nrows_total; int per_cta;
  int* err; unsigned long long* check;
};

__device__ __forceinline__ void g4(uint32_t dst, const CUtensorMap* tm, int x, int r0, int r1, int r2, int r3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst), "l"(tm), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3),
      "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

// MODE 0: gather4 for ckv + kpe; MODE 1: LSU cp.async for everything; MODE 2: gather4 ckv + LSU kpe
template <int MODE, int NST, int PW>
__global__ void __launch_bounds__((PW + 1) * 32, 1) k_swz(const __grid_constant__ CUtensorMap tc, const __grid_constant__ CUtensorMap tp, Args a) {
  extern __shared__ __align__(1024) uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[NST], empty[NST];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s0 = (int)((long)blockIdx.x * (a.per_cta) / gridDim.x), s1 = (int)((long)(blockIdx.x + 1) * a.per_cta / gridDim.x);
  const int r_begin = s0 * ROWS, nslots = s1 - s0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      // MODE 0: one expect_tx arrive per producer warp; LSU modes: + 32 noinc arrivals per warp
      mbar_init(&full[s], MODE == 0 ? PW : MODE == 1 ? PW * 32 : PW * 33);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp < PW) {
    for (int it = 0; it < nslots; ++it) {
      const int s = it % NST;
      if (!mbar_wait(&empty[s], ((it / NST) & 1) ^ 1)) { atomicOr(a.err, 2); break; }
      const uint32_t base = smem_u32(sm + s * SLOT);
      // this warp's rows: ROWS/PW rows
      constexpr int RPW = ROWS / PW;
      const int row0 = warp * RPW;
      const int id = lane < RPW ? a.idx[r_begin + it * ROWS + row0 + lane] : 0;
      uint32_t bytes = 0;
      if (MODE == 0) bytes = RPW * 1152;
      if (MODE == 2) bytes = RPW * 1024;
      if (lane == 0 && MODE != 1) mbar_arrive_expect_tx(&full[s], bytes);
      __syncwarp();
      if (MODE == 0 || MODE == 2) {
        // groups of 4 rows x 9 (or 8) panels; lane j issues items j, j+32, ...
        constexpr int NP = MODE == 0 ? 9 : 8;
        constexpr int ITEMS = (RPW / 4) * NP;
        // shuffles must be warp-uniform: gather the 4 ids of every group first
        int ids[RPW];
#pragma unroll
        for (int k = 0; k < RPW; ++k) ids[k] = __shfl_sync(0xffffffffu, id, k);
#pragma unroll
        for (int j0 = 0; j0 < ITEMS; j0 += 32) {
          const int j = j0 + lane;
          if (j < ITEMS) {
            const int grp = j / NP, pnl = j % NP;
            int rr[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              int v = 0;
#pragma unroll
              for (int k = 0; k < RPW; ++k) if (k == grp * 4 + q) v = ids[k];
              rr[q] = v;
            }
            const uint32_t dst = base + pnl * PANEL + (row0 + grp * 4) * 128;
            if (pnl < 8) g4(dst, &tc, pnl * 64, rr[0], rr[1], rr[2], rr[3], &full[s]);
            else g4(dst, &tp, 0, rr[0], rr[1], rr[2], rr[3], &full[s]);
          }
        }
      }
      if (MODE == 1 || MODE == 2) {
#pragma unroll 2
        for (int k = 0; k < RPW; ++k) {
          const int rid = __shfl_sync(0xffffffffu, id, k);
          const int row = row0 + k;
          const uint8_t* crow = a.ckv + (size_t)rid * 1024;
          const uint8_t* krow = a.kpe + (size_t)rid * 128;
          if (MODE == 1) {
            cp_async16(base + (lane >> 3) * PANEL + swz(row, lane & 7), crow + lane * 16, 16);
            cp_async16(base + ((lane + 32) >> 3) * PANEL + swz(row, lane & 7), crow + (lane + 32) * 16, 16);
          }
          if (lane < 8) cp_async16(base + 8 * PANEL + swz(row, lane), krow + lane * 16, 16);
        }
        cp_async_arrive_noinc(&full[s]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // wait own TMA copies: consumer drains all slots; just wait last NST fulls
    for (int k = nslots > NST ? nslots - NST : 0; k < nslots; ++k) mbar_wait(&full[k % NST], (k / NST) & 1);
  } else {
    for (int it = 0; it < nslots; ++it) {
      const int s = it % NST;
      if (!mbar_wait(&full[s], (it / NST) & 1)) { atomicOr(a.err, 4); break; }
      if (a.check) {  // verify layout: every lane checks some 16-B chunks
        const uint8_t* b = sm + s * SLOT;
        for (int q = lane; q < ROWS * 72; q += 32) {
          const int row = q / 72, c = q % 72;
          const int rid = a.idx[r_begin + it * ROWS + row];
          const uint4* src = c < 64 ? reinterpret_cast<const uint4*>(a.ckv + (size_t)rid * 1024 + c * 16)
                                    : reinterpret_cast<const uint4*>(a.kpe + (size_t)rid * 128 + (c - 64) * 16);
          const uint4* dst = reinterpret_cast<const uint4*>(b + (c >> 3) * PANEL + swz(row, c & 7));
          uint4 x = *src, y = *dst;
          if (x.x != y.x || x.y != y.y || x.z != y.z || x.w != y.w) atomicAdd(a.check, 1ull);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
}

// bulk: one cp.async.bulk per 1 KB ckv row, kpe 16-B cp.async; padded pitch
template <int NST>
__global__ void __launch_bounds__(96, 2) k_bulk(Args a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t full[NST], empty[NST];
  constexpr int CP = 1040, KP = 144;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s0 = (int)((long)blockIdx.x * (a.per_cta) / gridDim.x), s1 = (int)((long)(blockIdx.x + 1) * a.per_cta / gridDim.x);
  const int r_begin = s0 * ROWS, nslots = s1 - s0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) { mbar_init(&full[s], 2 * 33); mbar_init(&empty[s], 1); }
    fence_mbar_init();
  }
  __syncthreads();
  if (warp < 2) {
    for (int it = 0; it < nslots; ++it) {
      const int s = it % NST;
      uint8_t* ck = sm + s * ROWS * (CP + KP);
      uint8_t* kp = ck + ROWS * CP;
      if (!mbar_wait(&empty[s], ((it / NST) & 1) ^ 1)) { atomicOr(a.err, 2); break; }
      const int id = lane < 16 ? a.idx[r_begin + it * ROWS + warp * 16 + lane] : 0;
      if (lane == 0) mbar_arrive_expect_tx(&full[s], 16 * 1024);
      __syncwarp();
      if (lane < 16) bulk_g2s(ck + (warp * 16 + lane) * CP, a.ckv + (size_t)id * 1024, 1024, &full[s]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int q = lane + 32 * j, rr = q >> 3, ch = q & 7;
        const int rid = __shfl_sync(0xffffffffu, id, rr);
        cp_async16(smem_u32(kp + (warp * 16 + rr) * KP + ch * 16), a.kpe + (size_t)rid * 128 + ch * 16, 16);
      }
      cp_async_arrive_noinc(&full[s]);
    }
    for (int k = nslots > NST ? nslots - NST : 0; k < nslots; ++k) mbar_wait(&full[k % NST], (k / NST) & 1);
  } else {
    for (int it = 0; it < nslots; ++it) {
      const int s = it % NST;
      if (!mbar_wait(&full[s], (it / NST) & 1)) { atomicOr(a.err, 4); break; }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
}

// raw ceiling: plain 16-B loads, W warps per CTA, 4 rows in flight per warp
__global__ void __launch_bounds__(1024, 1) k_ldg(Args a, uint4* sink) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const long s0 = (long)blockIdx.x * a.per_cta / gridDim.x, s1 = (long)(blockIdx.x + 1) * a.per_cta / gridDim.x;
  uint4 acc = make_uint4(0, 0, 0, 0);
  for (long r = s0 * ROWS + warp * 4; r < s1 * ROWS; r += nw * 4) {
    uint4 v[4][3];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const long rr = r + q;
      const int rid = rr < s1 * ROWS ? a.idx[rr] : a.idx[s0 * ROWS];
      const uint4* c = reinterpret_cast<const uint4*>(a.ckv + (size_t)rid * 1024);
      v[q][0] = __ldg(c + lane);
      v[q][1] = __ldg(c + lane + 32);
      v[q][2] = lane < 8 ? __ldg(reinterpret_cast<const uint4*>(a.kpe + (size_t)rid * 128) + lane) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int j = 0; j < 3; ++j) { acc.x ^= v[q][j].x; acc.y ^= v[q][j].y; acc.z ^= v[q][j].z; acc.w ^= v[q][j].w; }
  }
  if ((acc.x & 0xFFFFF) == 0x12345) sink[threadIdx.x] = acc;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int main(int argc, char** argv) {
  bool l2 = false;
  const char* order = "random";
  for (int i = 1; i < argc; ++i) {
    if (!strcmp(argv[i], "--l2")) l2 = true;
    else if (!strcmp(argv[i], "--order") && i + 1 < argc) order = argv[++i];
  }
  const int T = l2 ? 1024 : 64, K = 2048;
  const long nrows = l2 ? 65536 : 2200000;  // L2 mode: a 75 MB cache, every row re-read
  const int total = T * K;
  uint8_t *ckv, *kpe; int *idx, *err; unsigned long long* chk;
  CK(cudaMalloc(&ckv, nrows * 1024)); CK(cudaMalloc(&kpe, nrows * 128));
  CK(cudaMalloc(&idx, total * 4)); CK(cudaMalloc(&err, 4)); CK(cudaMalloc(&chk, 8));
  CK(cudaMemset(err, 0, 4)); CK(cudaMemset(chk, 0, 8));
  {  // fill cache with a pattern so the layout check is meaningful
    std::vector<uint32_t> h(1 << 20);
    for (size_t i = 0; i < h.size(); ++i) h[i] = (uint32_t)(i * 2654435761u);
    for (long off = 0; off < nrows * 1024; off += (long)h.size() * 4)
      CK(cudaMemcpy(ckv + off, h.data(), std::min<long>(h.size() * 4, nrows * 1024 - off), cudaMemcpyHostToDevice));
    for (size_t i = 0; i < h.size(); ++i) h[i] = (uint32_t)(i * 40503u + 7);
    for (long off = 0; off < nrows * 128; off += (long)h.size() * 4)
      CK(cudaMemcpy(kpe + off, h.data(), std::min<long>(h.size() * 4, nrows * 128 - off), cudaMemcpyHostToDevice));
  }
  std::vector<int> hidx(total);
  std::mt19937_64 rng(1);
  for (int t = 0; t < T; ++t) {
    // per token: a request of ~33k rows somewhere in the cache; 2048 distinct rows of it
    long ctx = l2 ? nrows : 1024 + rng() % 64512; long base = l2 ? 0 : rng() % (nrows - ctx);
    std::vector<int> pick; pick.reserve(K);
    std::uniform_int_distribution<long> d(0, ctx - 1);
    std::vector<char> used(ctx, 0);
    while ((int)pick.size() < K && (int)pick.size() < ctx) { long p = d(rng); if (!used[p]) { used[p] = 1; pick.push_back((int)(base + p)); } }
    while ((int)pick.size() < K) pick.push_back((int)(base + pick.size() % ctx));
    for (int k = 0; k < K; ++k) hidx[t * K + k] = pick[k];
  }
  if (order[0] == 's') for (int t = 0; t < T; ++t) std::sort(hidx.begin() + t * K, hidx.begin() + (t + 1) * K);
  if (order[0] == 'p') {  // page-grouped shuffle: rows of a 64-row page stay adjacent
    for (int t = 0; t < T; ++t) std::sort(hidx.begin() + t * K, hidx.begin() + (t + 1) * K, [](int x, int y){ unsigned hx = (unsigned)(x >> 6) * 2654435761u, hy = (unsigned)(y >> 6) * 2654435761u; return hx != hy ? hx < hy : x < y; });
  }
  printf("%s cache, index order: %s\n", l2 ? "L2-resident 75 MB" : "2.5 GB HBM", order);
  CK(cudaMemcpy(idx, hidx.data(), total * 4, cudaMemcpyHostToDevice));
  uint8_t* flush; CK(cudaMalloc(&flush, 512 << 20));

  void* f = nullptr; cudaDriverEntryPointQueryResult q;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
  auto enc = reinterpret_cast<EncodeTiledFn>(f);
  CUtensorMap tc, tp;
  {
    cuuint64_t dims[2] = {512, (cuuint64_t)nrows}; cuuint64_t st[1] = {1024};
    cuuint32_t box[2] = {64, 1}; cuuint32_t es[2] = {1, 1};
    if (enc(&tc, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ckv, dims, st, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)) { printf("enc tc failed\n"); return 1; }
    cuuint64_t dims2[2] = {64, (cuuint64_t)nrows}; cuuint64_t st2[1] = {128};
    if (enc(&tp, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kpe, dims2, st2, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)) { printf("enc tp failed\n"); return 1; }
  }
  int sms = 0; CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
  const double bytes = (double)total * 1152;
  cudaEvent_t e0, e1; CK(cudaEventCreate(&e0)); CK(cudaEventCreate(&e1));
  auto run = [&](const char* name, auto launch, int ctas) {
    Args a{ckv, kpe, idx, (int)nrows, total / ROWS, err, nullptr};
    // layout check once
    CK(cudaMemset(chk, 0, 8));
    a.check = chk; launch(a); CK(cudaDeviceSynchronize());
    unsigned long long hc = 0; CK(cudaMemcpy(&hc, chk, 8, cudaMemcpyDeviceToHost));
    a.check = nullptr;
    std::vector<float> ms;
    for (int rep = 0; rep < 3; ++rep) {
      const int fl = l2 ? 0 : (512 << 20);
      for (int r = 0; r < 2; ++r) { CK(cudaMemsetAsync(flush, r, fl)); launch(a); }
      CK(cudaEventRecord(e0));
      for (int r = 0; r < 10; ++r) { CK(cudaMemsetAsync(flush, r, fl)); launch(a); }
      CK(cudaEventRecord(e1)); CK(cudaEventSynchronize(e1));
      float x, y; CK(cudaEventElapsedTime(&x, e0, e1));
      CK(cudaEventRecord(e0));
      for (int r = 0; r < 10; ++r) { CK(cudaMemsetAsync(flush, r, fl)); }
      CK(cudaEventRecord(e1)); CK(cudaEventSynchronize(e1));
      CK(cudaEventElapsedTime(&y, e0, e1));
      ms.push_back((x - y) / 10);
    }
    std::sort(ms.begin(), ms.end());
    int he = 0; CK(cudaMemcpy(&he, err, 4, cudaMemcpyDeviceToHost));
    printf("%-34s ctas %4d  median %.2f us  best %.2f us  %.0f GB/s  layout_mismatch %llu err %d\n", name, ctas,
           ms[ms.size() / 2] * 1e3, ms[0] * 1e3, bytes / (ms[ms.size() / 2] * 1e-3) / 1e9, hc, he);
  };
  // per_cta must be a multiple of 32 rows: choose ctas dividing 4096 slots
  // 4096 slots of 32 rows; ctas = 128 (32 slots each) or 256 (16) or 148 -> not divisible; use 128/256
  uint4* sink; CK(cudaMalloc(&sink, 1 << 16));
  for (int w : {8, 16, 32}) {
    char nm[64]; snprintf(nm, 64, "raw ldg %d warps/SM", w);
    auto l = [&](Args a) { k_ldg<<<sms, w * 32>>>(a, sink); CK(cudaGetLastError()); };
    run(nm, l, sms);
  }
  {
    auto l = [&](Args a) { k_ldg<<<2 * sms, 512>>>(a, sink); CK(cudaGetLastError()); };
    run("raw ldg 2x16 warps/SM", l, 2 * sms);
  }
  {
    const int ctas = 2 * sms;
    auto l = [&](Args a) { constexpr int N = 2; k_bulk<N><<<ctas, 96, N * ROWS * (1040 + 144)>>>(a); CK(cudaGetLastError()); };
    CK(cudaFuncSetAttribute(k_bulk<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * ROWS * (1040 + 144)));
    run("bulk NST2 (2 CTA/SM)", l, ctas);
  }
  {
    const int ctas = sms;
    auto l = [&](Args a) { constexpr int N = 5; k_bulk<N><<<ctas, 96, N * ROWS * (1040 + 144)>>>(a); CK(cudaGetLastError()); };
    CK(cudaFuncSetAttribute(k_bulk<5>, cudaFuncAttributeMaxDynamicSharedMemorySize, 5 * ROWS * (1040 + 144)));
    run("bulk NST5 1CTA", l, ctas);
  }
  const int ctas = sms;
#define SWZ(MODE, NST, PW, NAME)                                                                       \
    {                                                                                                  \
      const int smb = NST * SLOT + 1024;                                                               \
      CK(cudaFuncSetAttribute(k_swz<MODE, NST, PW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smb)); \
      auto l = [&](Args a) { k_swz<MODE, NST, PW><<<ctas, (PW + 1) * 32, smb>>>(tc, tp, a); CK(cudaGetLastError()); }; \
      run(NAME, l, ctas);                                                                              \
    }
  SWZ(0, 5, 4, "gather4 all NST5 PW4");
  SWZ(0, 5, 8, "gather4 all NST5 PW8");
  SWZ(0, 6, 8, "gather4 all NST6 PW8");
  SWZ(1, 5, 8, "lsu cp.async NST5 PW8");
  SWZ(1, 5, 16, "lsu cp.async NST5 PW16");
  SWZ(1, 6, 16, "lsu cp.async NST6 PW16");
  SWZ(2, 5, 8, "gather4 ckv + lsu kpe NST5 PW8");
  printf("done\n");
  return 0;
}
