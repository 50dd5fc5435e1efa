// umma_chain.cu -- issue cost of thin tcgen05.mma (kind::f16) on this GPU, as a
// function of the MMA shape and of how many independent accumulators the
// stream of MMAs rotates over.  A measurement probe for the attention
// kernels (no counterpart in the reference): with 16 heads the attention
// MMAs have N=16, so each one is short and a chain of MMAs that accumulate
// into the same TMEM columns may be paced by the accumulate dependency
// rather than by the tensor pipe.
//
// One CTA per SM; one thread issues R MMAs (operands: one 128-byte-swizzled
// K-major panel of A [M x 64] and of B [N x 64] in shared memory, K=16 per
// MMA, stepping through the panel), MMA r accumulating into accumulator
// r % C (C TMEM regions of N columns), then one commit; the clock64 interval
// from the first issue to the commit's arrival, divided by R, is the cost per
// MMA.  Operand values are zero: timing does not depend on them.
//
//   python -m flashinfer_repo_b200.build --probes
//   flashinfer_repo_b200/probes/umma_chain
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <algorithm>
#include "../csrc/common.cuh"
using namespace dsa;

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { printf("CUDA %s at %d\n", cudaGetErrorString(e_), __LINE__); exit(1);} } while (0)

constexpr int kR = 288;          // MMAs per measurement
constexpr int kSmem = 160 * 1024; // forces one CTA per SM

struct __align__(1024) ProbeSmem {
  uint8_t a[128 * 128];  // A panel: up to 128 rows x 128 B
  uint8_t b[256 * 128];  // B panel: up to 256 rows x 128 B
  uint64_t bar;
  uint32_t tmem;
};

__global__ void __launch_bounds__(128, 1) umma_chain_kernel(int m, int n, int chains, long long* cycles,
                                                            int* err) {
  extern __shared__ uint8_t raw[];
  ProbeSmem& S = *reinterpret_cast<ProbeSmem*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (int)sizeof(S.a) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(S.a)[i] = make_uint4(0, 0, 0, 0);
  for (int i = threadIdx.x; i < (int)sizeof(S.b) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(S.b)[i] = make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) {
    mbar_init(&S.bar, 1);
    fence_mbar_init();
  }
  fence_proxy_async_smem();
  if (warp == 0) tmem_alloc(&S.tmem, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem;
  if (threadIdx.x == 0) {
    const uint32_t idesc = umma_idesc(1, 1, 0, 0, (uint32_t)m, (uint32_t)n);
    const uint32_t ab = smem_u32(S.a), bb = smem_u32(S.b);
    const long long t0 = clock64();
    for (int r = 0; r < kR; ++r) {
      const int j = r & 3;  // K16 step inside the 64-wide panel
      umma_f16(tmem + (uint32_t)((r % chains) * n), umma_desc(ab + j * 32, 16, 1024, kSwizzle128B),
               umma_desc(bb + j * 32, 16, 1024, kSwizzle128B), idesc, r >= chains ? 1u : 0u);
    }
    umma_commit(&S.bar);
    if (!mbar_wait(&S.bar, 0)) atomicOr(err, 1);
    cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int main() {
  int sms = 0;
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
  CK(cudaFuncSetAttribute(umma_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
  long long* d_cyc;
  int* d_err;
  CK(cudaMalloc(&d_cyc, sms * sizeof(long long)));
  CK(cudaMalloc(&d_err, sizeof(int)));
  CK(cudaMemset(d_err, 0, sizeof(int)));
  struct Cfg { int m, n; };
  const Cfg cfgs[] = {{64, 16}, {128, 16}, {128, 32}, {128, 64}, {128, 128}, {128, 256}};
  const int chain_opts[] = {1, 2, 4, 8};
  printf("%-4s %-4s %-6s %-14s %-14s %-12s\n", "M", "N", "chains", "cycles/MMA", "MAC/clk/SM", "grid");
  for (const Cfg& c : cfgs) {
    for (int ch : chain_opts) {
      if (ch * c.n > 512) continue;
      for (int grid : {1, sms}) {
        std::vector<long long> h(grid);
        for (int rep = 0; rep < 3; ++rep) {  // the last repetition is reported
          umma_chain_kernel<<<grid, 128, kSmem>>>(c.m, c.n, ch, d_cyc, d_err);
          CK(cudaGetLastError());
          CK(cudaDeviceSynchronize());
        }
        CK(cudaMemcpy(h.data(), d_cyc, grid * sizeof(long long), cudaMemcpyDeviceToHost));
        std::sort(h.begin(), h.end());
        const double cyc = (double)h[grid / 2] / kR;
        printf("%-4d %-4d %-6d %-14.1f %-14.0f %-12d\n", c.m, c.n, ch, cyc, (double)c.m * c.n * 16 / cyc,
               grid);
      }
    }
  }
  int err = 0;
  CK(cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost));
  printf("wait timeouts: %d\n", err);
  return 0;
}
