// peer.cu -- device buffers shared between the GPUs of one node, and a
// bounded cross-GPU barrier, for the head-parallel decode whose attention
// epilogues store straight into every rank's output (dsa_sparse_attention_scatter).
//
// Buffers are plain cudaMalloc allocations exported with CUDA IPC handles and
// opened by the other processes of the node (peer access over NVLink); no
// multicast object is created, so a rank that leaves never has memory bound
// to one.  The barrier is one small kernel per step: thread q (< world) waits
// until rank q has reached the same epoch; the epoch counter lives in device
// memory, so the launch has no per-step host argument and can be captured in
// a CUDA graph.
//
// Flag buffer layout (int32, one per rank, at least 1 + kMaxRanks entries):
//   [0]      this rank's epoch (written only by this rank)
//   [1 + q]  the latest epoch rank q has announced to this rank
// Each wait is bounded (about two seconds of SM clock); a timeout sets
// kErrTimeout in device_error and the kernel returns, leaving the context usable.
#include <cstring>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {
namespace {

constexpr int kMaxRanks = 8;
constexpr long long kBarrierSpin = 4000000000LL;  // SM clock cycles

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerFlags {
  int* flags[kMaxRanks];  // flags[q]: rank q's flag buffer, as mapped in this process
};

__global__ void __launch_bounds__(32) dsa_peer_barrier_kernel(PeerFlags f, int rank, int world, int* err) {
  const int q = threadIdx.x;
  int* mine = f.flags[rank];
  const int epoch = mine[0] + 1;  // every thread reads the old value before thread 0 bumps it
  __syncwarp();
  // Everything this rank stored before the barrier (earlier kernels on the
  // stream, peer stores included) is made visible system-wide by the release.
  __threadfence_system();
  if (q < world) st_release_sys(f.flags[q] + 1 + rank, epoch);
  if (q < world) {
    const long long t0 = clock64();
    while (ld_acquire_sys(mine + 1 + q) < epoch) {
      if (clock64() - t0 > kBarrierSpin) {
        set_error(err, kErrTimeout);
        break;
      }
    }
  }
  __syncwarp();
  if (q == 0) mine[0] = epoch;
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" {

int dsa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return report_error(DSA_ERR_INVALID_ARG, "bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == DSA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return DSA_OK;
}

int dsa_peer_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return report_error(DSA_ERR_INVALID_ARG, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
  return DSA_OK;
}

int dsa_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? DSA_OK : report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
}

int dsa_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? DSA_OK : report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
}

int dsa_peer_barrier(int* const* flags, int rank, int world, int* device_error, void* stream) {
  if (!flags || world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return report_error(DSA_ERR_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
  PeerFlags f = {};
  for (int q = 0; q < world; ++q) {
    if (!flags[q]) return report_error(DSA_ERR_INVALID_ARG, "NULL flag buffer");
    f.flags[q] = flags[q];
  }
  dsa_peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, rank, world, device_error);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSA_OK : report_error(DSA_ERR_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
