// attention.cu -- DSA sparse-attention decode over a paged MLA latent cache, sm_100a.
//
// Semantics follow the reference operator `kernel` / `dsa_fwd_kernel`
// (solution/triton/kernel.py:9-182) and its split-K variant
// (kernel.py:343-567):  for every query token and each of its 16 heads,
//   s_j   = (q_nope . ckv[row_j] + q_pe . kpe[row_j]) * sm_scale  over the
//           top-k rows (row = flat slot id page*64+offset, -1 = padding)
//   out   = softmax(s) . ckv[rows]      (bf16; 0 when no row is valid)
//   lse   = log2(sum_j exp(s_j))         (fp32, base 2; -inf when no row)
// P is rounded to bf16 before the PV product, as in the reference (:114).
//
// Design (B200):
//  * Work unit = tile of 32 selected rows of one (token, 16-head group).
//    A token's 2048 rows are 64 tiles; the whole batch is one list of tiles
//    split evenly over a persistent grid (one contiguous range per CTA), so
//    any T keeps every SM streaming (stream-K over the top-k dimension).
//  * A producer warp turns indices into row addresses and gathers each
//    1024-B ckv row and 128-B kpe row with one cp.async.bulk each into a
//    padded shared-memory ring (row pitch 1040 / 144 B: conflict-free
//    ldmatrix), completion tracked by mbarrier transaction bytes.
//  * Four consumer warps: QK^T with bf16 tensor-core MMA, the 576-d
//    contraction split in four 144-d quarters (Q fragments stay in
//    registers), partial scores reduced through shared memory; online
//    softmax in registers (base-2, exp2); PV with each warp owning 128 of
//    the 512 output columns; P is re-used from registers as the A operand.
//  * A token split across CTAs writes unnormalised (acc, m, l) partials; a
//    second grid (one CTA per token and head, programmatic dependent launch)
//    merges them (LSE merge of kernel.py:437-493) using every SM.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "../../include/dsa_b200.h"
#include "common.cuh"

namespace dsa {

constexpr int kHeads = 16;
constexpr int kMaxTargets = 8;  // output targets of the scatter entry (GPUs of one node)
constexpr int kDc = 512;
constexpr int kDp = 64;
constexpr int kRows = 32;             // rows per tile
constexpr int kCkvStride = 1040;      // smem pitch of a 1024-B ckv row
constexpr int kKpeStride = 144;       // smem pitch of a 128-B kpe row
constexpr int kPPitch = 40;           // P tile row pitch (bf16): 80 B, conflict-free ldmatrix
constexpr float kLazyLog2 = 8.f;     // lazy-rescale threshold (log2 units)
constexpr int kCWarps = 4;            // consumer warps
constexpr int kPWarps = 2;            // producer warps
constexpr int kThreads = (kCWarps + kPWarps) * 32;
constexpr int kPartFloats = kHeads * kDc + 2 * kHeads;  // acc[16][512], m[16], l[16]
// A cluster-plan partial in shared memory: acc rows of 520 floats (a pitch
// that spreads the 8 heads a warp stores at once over distinct banks), then
// m[16] and l[16]; it overlays the (then idle) stage ring.
constexpr int kClPitch = kDc + 8;
constexpr int kClPartFloats = kHeads * kClPitch + 2 * kHeads;

struct AttnParams {
  const __nv_bfloat16* q_nope;
  const __nv_bfloat16* q_pe;
  const __nv_bfloat16* ckv;
  const __nv_bfloat16* kpe;
  const int32_t* idx;
  __nv_bfloat16* out;
  float* lse;
  int64_t qn_st, qn_sh, qp_st, qp_sh;  // element strides (token, head)
  int64_t ckv_sp, ckv_sr, kpe_sp, kpe_sr;  // (page, row)
  int64_t idx_st;
  int64_t out_st, out_sh, lse_st, lse_sh;
  int64_t num_slots;
  int head_groups;      // heads / 16; virtual token v = t * head_groups + group
  int tiles_per_token;  // topk / 32
  float scale_log2;     // sm_scale * log2(e)
  int tiles_base, tiles_rem;
  // Token-aligned plan when > 0: every virtual token is split over exactly
  // `per_token` CTAs, part j of a token taking its tiles
  // [j*tpt/per_token, (j+1)*tpt/per_token) (integer division); tiles_base /
  // tiles_rem are then unused.  0: the flat split of all tiles above.
  int per_token;
  // Optional extra output targets (fused all-gather of head-sharded outputs):
  // when n_peers > 0, every output / lse store goes to each of the n_peers
  // bases (peer GPUs' buffers over NVLink, this rank's head slice), with the
  // same strides; out / lse are then unused.
  __nv_bfloat16* out_peers[kMaxTargets];
  float* lse_peers[kMaxTargets];
  int n_peers;
  float* part;
  int* err;
  // Cross-GPU barrier after the last store (head-parallel decode), when
  // sync_world > 0: the last CTA to finish in the grid that stores last (the
  // merge grid when one runs, else the attention grid) announces this rank's
  // next epoch to every rank and waits, bounded, until all ranks announced it.
  // sync_flags[q]: rank q's flag buffer as mapped in this process; int32
  // layout [0] this rank's epoch, [1 + q] the epoch rank q announced here,
  // [9] CTAs of the current launch that finished (back to 0 after it).
  int* sync_flags[kMaxTargets];
  int sync_rank, sync_world, sync_in_merge;
  int merge_by_boundary;  // merge grid rows are CTA boundaries instead of tokens
  // Cluster plan: every virtual token's tiles are split evenly over one
  // thread-block cluster of `cluster` CTAs (2, 4 or 8), which merge their
  // partials through distributed shared memory at the end; no merge grid runs.
  // 0: partials of split tokens go to the workspace and the merge grid.
  int cluster;
};

template <int NST>
struct AttnSmem {
  // (the first two stages' ckv buffers also hold the cluster plan's partial)
  uint8_t ckv[NST][kRows * kCkvStride];
  uint8_t kpe[NST][kRows * kKpeStride];
  float4 sred[2][kCWarps][4][32];  // [buf][warp][n-block][lane]: conflict-free
  float smax[2][kHeads][kCWarps];  // [buf][head][warp]: per-warp row-block maxima
  __nv_bfloat16 pbuf[2][kHeads][kPPitch];  // [buf][head][row]: P (bf16) for the PV A operand
  float lred[kCWarps][kHeads];     // per-warp normalisers, summed at segment ends
  uint32_t vmask[NST][kPWarps];  // valid-row bits, one word per producer warp
  uint64_t full[NST];
  uint64_t empty[NST];
};

static_assert(kClPartFloats * 4 <= 2 * kRows * kCkvStride, "cluster partial must fit in two ckv stages");

__device__ __forceinline__ int cta_start(const AttnParams& p, int c) {
  if (p.per_token > 0) {
    const int v = c / p.per_token, j = c - v * p.per_token;
    return v * p.tiles_per_token + (j * p.tiles_per_token) / p.per_token;
  }
  return c * p.tiles_base + min(c, p.tiles_rem);
}
__device__ __forceinline__ int cta_of_tile(const AttnParams& p, int tile) {
  if (p.per_token > 0) {  // the part j with j*tpt/C <= r < (j+1)*tpt/C
    const int v = tile / p.tiles_per_token, r = tile - v * p.tiles_per_token;
    return v * p.per_token + ((r + 1) * p.per_token - 1) / p.tiles_per_token;
  }
  const int big = (p.tiles_base + 1) * p.tiles_rem;
  return tile < big ? tile / (p.tiles_base + 1) : p.tiles_rem + (tile - big) / p.tiles_base;
}
// Only a CTA's first and last token segments can be partial (every token
// strictly inside its range is complete), so two partial slots per CTA.
__device__ __forceinline__ float* part_slot(const AttnParams& p, int c, int v) {
  const int j = (v == cta_start(p, c) / p.tiles_per_token) ? 0 : 1;
  return p.part + (int64_t)(2 * c + j) * kPartFloats;
}

__device__ __forceinline__ void st_release_sys(int* ptr, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* ptr) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

// Called by one thread per CTA after a CTA-wide barrier that follows all of
// the CTA's stores.  The last of the grid's `nctas` CTAs runs the cross-GPU
// barrier: its release stores carry every store the grid (and, through grid
// completion, the attention grid before it) made, peer stores included.
__device__ void grid_done_then_sync(const AttnParams& p, unsigned nctas) {
  __threadfence_system();
  int* mine = p.sync_flags[p.sync_rank];
  const unsigned prev = atomicAdd(reinterpret_cast<unsigned*>(mine + 9), 1u);
  if (prev != nctas - 1) return;
  __threadfence_system();
  mine[9] = 0;
  const int epoch = mine[0] + 1;
  for (int q = 0; q < p.sync_world; ++q) st_release_sys(p.sync_flags[q] + 1 + p.sync_rank, epoch);
  const long long t0 = clock64();
  for (int q = 0; q < p.sync_world; ++q) {
    while (ld_acquire_sys(mine + 1 + q) < epoch) {
      if (clock64() - t0 > kWaitBudgetCycles) {
        set_error(p.err, kErrTimeout);
        break;
      }
    }
  }
  mine[0] = epoch;
}

__device__ __forceinline__ int n_targets(const AttnParams& p) { return p.n_peers > 0 ? p.n_peers : 1; }
__device__ __forceinline__ __nv_bfloat16* out_target(const AttnParams& p, int k) {
  return p.n_peers > 0 ? p.out_peers[k] : p.out;
}
__device__ __forceinline__ float* lse_target(const AttnParams& p, int k) {
  return p.n_peers > 0 ? p.lse_peers[k] : p.lse;
}

// ------------------------------------------------------------------ producer
// Producer warp pw gathers rows pw*16 .. pw*16+15 of every tile: each
// 1024-B ckv row is one bulk copy (lanes 0-15), the 128-B kpe rows are
// 16-byte cp.async chunks spread over all 32 lanes (4 per lane), so the copy
// engine sees one operation per row and two warps issue in parallel.
template <int NST>
__device__ __forceinline__ void attn_producer(const AttnParams& p, AttnSmem<NST>& S, int pw,
                                              int lane, int tile_begin, int tile_end) {
  constexpr int RPW = kRows / kPWarps;  // 16 rows per producer warp
  // Indices are fetched kIdxAhead tiles before use so that the dependent
  // global load is off the critical path of the row copies.
  constexpr int kIdxAhead = 3;
  auto load_idx = [&](int tile) -> int32_t {
    if (tile >= tile_end || lane >= RPW) return -1;
    const int v = tile / p.tiles_per_token;
    const int t = v / p.head_groups;
    const int r0 = (tile - v * p.tiles_per_token) * kRows + pw * RPW;
    return __ldg(p.idx + (int64_t)t * p.idx_st + r0 + lane);
  };
  int32_t ring[kIdxAhead];
#pragma unroll
  for (int k = 0; k < kIdxAhead; ++k) ring[k] = load_idx(tile_begin + k);
  int it = 0;
  for (int tile = tile_begin; tile < tile_end; ++tile, ++it) {
    const int s = it % NST;
    const uint32_t ph = (it / NST) & 1;
    const int32_t id = ring[0];
#pragma unroll
    for (int k = 0; k + 1 < kIdxAhead; ++k) ring[k] = ring[k + 1];
    ring[kIdxAhead - 1] = load_idx(tile + kIdxAhead);
    if (!mbar_wait(&S.empty[s], ph ^ 1)) {
      set_error(p.err, kErrTimeout);
      break;
    }
    const bool mine = lane < RPW;
    const bool valid = mine && id >= 0 && id < p.num_slots;
    if (mine && (id < -1 || id >= p.num_slots)) set_error(p.err, kErrBadIndex);
    const uint32_t mask = __ballot_sync(0xffffffffu, valid);
    const int row = pw * RPW + lane;
    if (mine && !valid) {
      // padding row: zeros, so 0-probability rows contribute exactly 0 to PV
      float4* d = reinterpret_cast<float4*>(S.ckv[s] + row * kCkvStride);
#pragma unroll 8
      for (int k = 0; k < 64; ++k) d[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      fence_proxy_async_smem();
    }
    if (lane == 0) S.vmask[s][pw] = mask << (pw * RPW);
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(&S.full[s], __popc(mask) * (kDc * 2));
    __syncwarp();
    if (valid) {
      const int64_t page = id >> 6, r = id & 63;
      bulk_g2s(S.ckv[s] + row * kCkvStride, p.ckv + page * p.ckv_sp + r * p.ckv_sr, kDc * 2,
               &S.full[s]);
    }
    // kpe: chunk q = lane + 32*j of this warp's 16 rows x 8 chunks
    const uint32_t kpe_s = smem_u32(S.kpe[s]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = lane + 32 * j, rr = q >> 3, ch = q & 7;
      const int32_t rid = __shfl_sync(0xffffffffu, id, rr);
      const bool ok = (mask >> rr) & 1u;
      const int64_t page = ok ? (rid >> 6) : 0, r = ok ? (rid & 63) : 0;
      const char* src = reinterpret_cast<const char*>(p.kpe + page * p.kpe_sp + r * p.kpe_sr) + ch * 16;
      cp_async16(kpe_s + (pw * RPW + rr) * kKpeStride + ch * 16, src, ok ? 16u : 0u);
    }
    cp_async_arrive_noinc(&S.full[s]);
  }
  // Do not leave while copies issued by this warp may still be landing.
  for (int k = it > NST ? it - NST : 0; k < it; ++k) mbar_wait(&S.full[k % NST], (k / NST) & 1);
}

// ------------------------------------------------------------------ merge
// LSE merge of the split-K partials (kernel.py:437-493 / the 3-phase merge
// of :583-704 done in one pass): one CTA per (virtual token, head), launched
// as a programmatic dependent of the attention grid.  Thread i owns output
// columns 4i..4i+3.  Partials are taken 8 at a time and every load of a
// chunk -- each partial's max m, normaliser l and the thread's four columns --
// is issued before any is used, so a token with at most 8 partials costs one
// L2 round trip and no barrier; later chunks rescale the running sums
// (online softmax across chunks).
constexpr int kMergeThreads = 128;
constexpr int kMergeChunk = 8;

__device__ __forceinline__ void merge_token(const AttnParams& p, int h, int v, int i, int c_first,
                                            int c_last) {
  const int tpt = p.tiles_per_token;
  // Slot of partial c: every CTA after c_first starts inside this token (its
  // first segment, slot 0); c_first holds it in slot 1 unless it starts at
  // the token's first tile.
  const int first_slot = 2 * c_first + (cta_start(p, c_first) < v * tpt ? 1 : 0);
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int base = c_first; base <= c_last; base += kMergeChunk) {
    float m[kMergeChunk], l[kMergeChunk];
    float4 a[kMergeChunk];
#pragma unroll
    for (int u = 0; u < kMergeChunk; ++u) {
      m[u] = -INFINITY;
      l[u] = 0.f;
      a[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      const int c = base + u;
      if (c <= c_last) {
        const float* ps = p.part + (int64_t)(c == c_first ? first_slot : 2 * c) * kPartFloats;
        m[u] = __ldcg(ps + kHeads * kDc + h);
        l[u] = __ldcg(ps + kHeads * kDc + kHeads + h);
        a[u] = __ldcg(reinterpret_cast<const float4*>(ps + h * kDc) + i);
      }
    }
    float Mn = M;
#pragma unroll
    for (int u = 0; u < kMergeChunk; ++u) Mn = fmaxf(Mn, m[u]);
    const float scale = (M == -INFINITY) ? 0.f : exp2f(M - Mn);
    L *= scale;
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
#pragma unroll
    for (int u = 0; u < kMergeChunk; ++u) {
      const float w = (m[u] == -INFINITY) ? 0.f : exp2f(m[u] - Mn);
      L += w * l[u];
      acc.x += w * a[u].x;
      acc.y += w * a[u].y;
      acc.z += w * a[u].z;
      acc.w += w * a[u].w;
    }
    M = Mn;
  }
  const int t = v / p.head_groups, grp = v - t * p.head_groups;
  const float inv = (M == -INFINITY) ? 0.f : 1.f / L;
  uint2 pk;
  pk.x = pack_bf16(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16(acc.z * inv, acc.w * inv);
  for (int k = 0; k < n_targets(p); ++k) {
    *reinterpret_cast<uint2*>(out_target(p, k) + t * p.out_st + (int64_t)(grp * kHeads + h) * p.out_sh +
                              4 * i) = pk;
    if (i == 0)
      lse_target(p, k)[t * p.lse_st + (int64_t)(grp * kHeads + h) * p.lse_sh] =
          (M == -INFINITY) ? -INFINITY : M + log2f(L);
  }
}

__global__ void __launch_bounds__(kMergeThreads) dsa_attention_merge_kernel(const __grid_constant__ AttnParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // attention grid done, writes visible
  const int h = blockIdx.x, i = threadIdx.x;
  const int tpt = p.tiles_per_token;
  // Row y of the grid is virtual token y, or -- when there are more tokens than
  // CTAs (prefill-sized batches, where only tokens that straddle a CTA
  // boundary are split) -- the token holding CTA boundary y+1, merged by the
  // first boundary inside it.
  int v = blockIdx.y;
  bool mine = true;
  if (p.merge_by_boundary) {
    const int c = blockIdx.y + 1, tile = cta_start(p, c);
    v = tile / tpt;
    mine = (tile % tpt != 0) && cta_of_tile(p, v * tpt) == c - 1;
  }
  const int c_first = cta_of_tile(p, v * tpt), c_last = cta_of_tile(p, v * tpt + tpt - 1);
  if (mine && c_first != c_last) merge_token(p, h, v, i, c_first, c_last);  // else written by the attention grid
  if (p.sync_world > 0 && p.sync_in_merge) {
    __syncthreads();
    if (i == 0) grid_done_then_sync(p, gridDim.x * gridDim.y);
  }
}

// Merge inside a cluster (cluster plan): each of the token's C CTAs left its
// unnormalised partial (acc, m, l; layout kClPitch) in its own shared memory;
// CTA r of the cluster combines output columns [r*512/C, (r+1)*512/C) of all 16
// heads from the C partials, read through distributed shared memory, with the
// arithmetic and order of merge_token, and CTA 0 writes the LSE.  Thread i of
// the 128 consumers takes head i/8 and one eighth of the CTA's columns.
__device__ void cluster_merge(const AttnParams& p, const float* part_local, int v, int i) {
  const int C = p.cluster;
  const uint32_t r = cluster_ctarank();
  const int h = i >> 3, sub = i & 7;
  const int cols = kDc / C, per = cols / 8;
  const int d0 = (int)r * cols + sub * per;
  const uint32_t loc = smem_u32(part_local);
  uint32_t base[8];
  float mq[8], lq[8], w[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    base[q] = 0;
    mq[q] = -INFINITY;
    lq[q] = 0.f;
    if (q < C) {
      base[q] = cluster_map(loc, (uint32_t)q);
      mq[q] = ld_cluster_f32(base[q] + (uint32_t)(kHeads * kClPitch + h) * 4u);
      lq[q] = ld_cluster_f32(base[q] + (uint32_t)(kHeads * kClPitch + kHeads + h) * 4u);
    }
  }
  float M = -INFINITY, L = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) M = fmaxf(M, mq[q]);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    w[q] = (mq[q] == -INFINITY) ? 0.f : exp2f(mq[q] - M);
    L += w[q] * lq[q];
  }
  const float inv = (M == -INFINITY) ? 0.f : 1.f / L;
  const int t = v / p.head_groups, grp = v - t * p.head_groups;
  for (int j = 0; j < per; j += 2) {
    const int d = d0 + j;
    float ax = 0.f, ay = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q < C) {
        const float2 a = ld_cluster_f32x2(base[q] + (uint32_t)(h * kClPitch + d) * 4u);
        ax += w[q] * a.x;
        ay += w[q] * a.y;
      }
    const uint32_t pk = pack_bf16(ax * inv, ay * inv);
    for (int k = 0; k < n_targets(p); ++k)
      *reinterpret_cast<uint32_t*>(out_target(p, k) + t * p.out_st + (int64_t)(grp * kHeads + h) * p.out_sh +
                                   d) = pk;
  }
  if (r == 0 && sub == 0)
    for (int k = 0; k < n_targets(p); ++k)
      lse_target(p, k)[t * p.lse_st + (int64_t)(grp * kHeads + h) * p.lse_sh] =
          (M == -INFINITY) ? -INFINITY : M + log2f(L);
}

// ------------------------------------------------------------------ kernel
template <int NST>
__global__ void __launch_bounds__(kThreads, (NST == 2 ? 2 : 1)) dsa_attention_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<NST>& S = *reinterpret_cast<AttnSmem<NST>*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int tile_begin = cta_start(p, cta), tile_end = cta_start(p, cta + 1);

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) {
      mbar_init(&S.full[s], kPWarps * 33);  // per producer: expect_tx arrive + 32 cp.async arrivals
      mbar_init(&S.empty[s], kCWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp >= kCWarps) {
    attn_producer<NST>(p, S, warp - kCWarps, lane, tile_begin, tile_end);
    if (p.cluster) {  // every thread of the cluster takes part in both cluster barriers
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int g = lane >> 2, c = lane & 3;
  const int kq0 = warp * 144;  // this warp's quarter of the 576-d contraction
  const int tpt = p.tiles_per_token;
  int it = 0, buf = 0;
  int tile = tile_begin;
  while (tile < tile_end) {
    const int v = tile / tpt;
    const int seg_end = min(tile_end, (v + 1) * tpt);
    const int t = v / p.head_groups, grp = v - t * p.head_groups;

    // Q A-fragments for k-steps kq0 + 16j (m16n8k16 row-major A layout).
    uint32_t qa[9][4];
    {
      const __nv_bfloat16* qn = p.q_nope + t * p.qn_st + (int64_t)grp * kHeads * p.qn_sh;
      const __nv_bfloat16* qp = p.q_pe + t * p.qp_st + (int64_t)grp * kHeads * p.qp_sh;
#pragma unroll
      for (int j = 0; j < 9; ++j) {
        const int kk = kq0 + 16 * j;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int h = g + ((e & 1) ? 8 : 0);
          const int d = kk + 2 * c + ((e & 2) ? 8 : 0);
          const __nv_bfloat16* src = d < kDc ? qn + h * p.qn_sh + d : qp + h * p.qp_sh + (d - kDc);
          qa[j][e] = __ldg(reinterpret_cast<const unsigned int*>(src));
        }
      }
    }

    float o[16][4];
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    bool ok = true;

    for (; tile < seg_end; ++tile, ++it) {
      const int s = it % NST;
      if (!mbar_wait(&S.full[s], (it / NST) & 1)) {
        set_error(p.err, kErrTimeout);
        ok = false;
        break;
      }
      const uint32_t ckv_base = smem_u32(S.ckv[s]);
      const uint32_t kpe_base = smem_u32(S.kpe[s]);

      // ---- partial scores over this warp's 144 dims: [16 heads x 32 rows]
      float sc[4][4];
#pragma unroll
      for (int nb = 0; nb < 4; ++nb) sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
#pragma unroll
      for (int j = 0; j < 9; ++j) {
        const int kk = kq0 + 16 * j;
#pragma unroll
        for (int pr = 0; pr < 2; ++pr) {
          const int mi = lane >> 3;
          const int row = (pr * 2 + (mi >> 1)) * 8 + (lane & 7);
          const int kc = kk + (mi & 1) * 8;
          const uint32_t addr = kc < kDc ? ckv_base + row * kCkvStride + kc * 2
                                         : kpe_base + row * kKpeStride + (kc - kDc) * 2;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(addr, b0, b1, b2, b3);
          mma_bf16_16816(sc[pr * 2], qa[j], b0, b1);
          mma_bf16_16816(sc[pr * 2 + 1], qa[j], b2, b3);
        }
      }
#pragma unroll
      for (int nb = 0; nb < 4; ++nb)
        S.sred[buf][warp][nb][lane] = make_float4(sc[nb][0], sc[nb][1], sc[nb][2], sc[nb][3]);
      named_bar_sync(1, kCWarps * 32);
      // ---- softmax, split by rows: warp w owns rows 8w..8w+7 of the tile (its
      // n-block of S, summed over the four quarters); x[0], x[1] are head g at
      // rows 8w+2c, +1 and x[2], x[3] head g+8
      float x[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < kCWarps; ++q) {
        const float4 a = S.sred[buf][q][warp][lane];
        x[0] += a.x;
        x[1] += a.y;
        x[2] += a.z;
        x[3] += a.w;
      }
      uint32_t vm = 0;
#pragma unroll
      for (int q = 0; q < kPWarps; ++q) vm |= S.vmask[s][q];
      const uint32_t vb = vm >> (8 * warp + 2 * c);
      x[0] = (vb & 1u) ? x[0] * p.scale_log2 : -INFINITY;
      x[1] = (vb & 2u) ? x[1] * p.scale_log2 : -INFINITY;
      x[2] = (vb & 1u) ? x[2] * p.scale_log2 : -INFINITY;
      x[3] = (vb & 2u) ? x[3] * p.scale_log2 : -INFINITY;
      float mx0 = fmaxf(x[0], x[1]), mx1 = fmaxf(x[2], x[3]);
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      if (c == 0) {
        S.smax[buf][g][warp] = mx0;
        S.smax[buf][g + 8][warp] = mx1;
      }
      named_bar_sync(1, kCWarps * 32);
      {
        const float4 a = *reinterpret_cast<const float4*>(&S.smax[buf][g][0]);
        const float4 b = *reinterpret_cast<const float4*>(&S.smax[buf][g + 8][0]);
        mx0 = fmaxf(fmaxf(a.x, a.y), fmaxf(a.z, a.w));
        mx1 = fmaxf(fmaxf(b.x, b.y), fmaxf(b.z, b.w));
      }
      // Lazy rescaling: the maximum used for the exponentials moves only when
      // the tile's maximum exceeds it by more than kLazyLog2 (a factor 2^8), so
      // P stays <= 256 and O, l are rescaled on few tiles.  Every warp sees the
      // same maxima and takes the same decisions.
      const bool up0 = mx0 > m0 + kLazyLog2, up1 = mx1 > m1 + kLazyLog2;
      if (__any_sync(0xffffffffu, up0 || up1)) {
        const float a0 = up0 ? ((m0 == -INFINITY) ? 0.f : ex2_approx(m0 - mx0)) : 1.f;
        const float a1 = up1 ? ((m1 == -INFINITY) ? 0.f : ex2_approx(m1 - mx1)) : 1.f;
        if (up0) m0 = mx0;
        if (up1) m1 = mx1;
        l0 *= a0;
        l1 *= a1;
#pragma unroll
        for (int nb = 0; nb < 16; ++nb) {
          o[nb][0] *= a0;
          o[nb][1] *= a0;
          o[nb][2] *= a1;
          o[nb][3] *= a1;
        }
      }
      x[0] = (m0 == -INFINITY) ? 0.f : ex2_approx(x[0] - m0);
      x[1] = (m0 == -INFINITY) ? 0.f : ex2_approx(x[1] - m0);
      x[2] = (m1 == -INFINITY) ? 0.f : ex2_approx(x[2] - m1);
      x[3] = (m1 == -INFINITY) ? 0.f : ex2_approx(x[3] - m1);
      l0 += x[0] + x[1];  // this thread's rows only; summed at the segment end
      l1 += x[2] + x[3];
      *reinterpret_cast<uint32_t*>(&S.pbuf[buf][g][8 * warp + 2 * c]) = pack_bf16(x[0], x[1]);
      *reinterpret_cast<uint32_t*>(&S.pbuf[buf][g + 8][8 * warp + 2 * c]) = pack_bf16(x[2], x[3]);
      named_bar_sync(1, kCWarps * 32);
      // P [16 heads x 32 rows] as the m16n8k16 A operand, two k-steps of 16 rows
      uint32_t pa[2][4];
      {
        const uint32_t pbase = smem_u32(&S.pbuf[buf][0][0]);
#pragma unroll
        for (int kj = 0; kj < 2; ++kj)
          ldsm_x4(pbase + ((lane & 15) * kPPitch + 16 * kj + (lane >> 4) * 8) * 2, pa[kj][0], pa[kj][1],
                  pa[kj][2], pa[kj][3]);
      }
      buf ^= 1;

      // ---- PV: this warp's 128 output columns
#pragma unroll
      for (int kj = 0; kj < 2; ++kj) {
#pragma unroll
        for (int pr = 0; pr < 8; ++pr) {
          const int mi = lane >> 3;
          const int row = 16 * kj + (mi & 1) * 8 + (lane & 7);
          const int col = 128 * warp + 16 * pr + (mi >> 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(ckv_base + row * kCkvStride + col * 2, b0, b1, b2, b3);
          mma_bf16_16816(o[2 * pr], pa[kj], b0, b1);
          mma_bf16_16816(o[2 * pr + 1], pa[kj], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[s]);
    }
    if (!ok) break;

    // ---- finish this (token, segment): normalisers summed over the quad
    // (rows of this warp) and over the four warps
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (c == 0) {
      S.lred[warp][g] = l0;
      S.lred[warp][g + 8] = l1;
    }
    named_bar_sync(1, kCWarps * 32);
    l0 = S.lred[0][g] + S.lred[1][g] + S.lred[2][g] + S.lred[3][g];
    l1 = S.lred[0][g + 8] + S.lred[1][g + 8] + S.lred[2][g + 8] + S.lred[3][g + 8];
    named_bar_sync(1, kCWarps * 32);  // S.lred is rewritten at the next segment end
    const int c_first = cta_of_tile(p, v * tpt);
    const int c_last = cta_of_tile(p, v * tpt + tpt - 1);
    if (c_first == c_last) {
      const float i0 = (m0 == -INFINITY) ? 0.f : 1.f / l0;
      const float i1 = (m1 == -INFINITY) ? 0.f : 1.f / l1;
      for (int k = 0; k < n_targets(p); ++k) {
        __nv_bfloat16* o0 = out_target(p, k) + t * p.out_st + (int64_t)(grp * kHeads + g) * p.out_sh;
        __nv_bfloat16* o1 = o0 + 8 * p.out_sh;
#pragma unroll
        for (int nb = 0; nb < 16; ++nb) {
          const int d = 128 * warp + 8 * nb + 2 * c;
          *reinterpret_cast<uint32_t*>(o0 + d) = pack_bf16(o[nb][0] * i0, o[nb][1] * i0);
          *reinterpret_cast<uint32_t*>(o1 + d) = pack_bf16(o[nb][2] * i1, o[nb][3] * i1);
        }
        if (warp == 0 && c == 0) {
          float* lp = lse_target(p, k) + t * p.lse_st;
          lp[(int64_t)(grp * kHeads + g) * p.lse_sh] = (m0 == -INFINITY) ? -INFINITY : m0 + log2f(l0);
          lp[(int64_t)(grp * kHeads + g + 8) * p.lse_sh] =
              (m1 == -INFINITY) ? -INFINITY : m1 + log2f(l1);
        }
      }
    } else if (p.cluster) {
      // the CTA's only segment is done, so the stage ring is idle (all warps
      // passed the barriers above after their last PV): the partial goes there
      float* ps = reinterpret_cast<float*>(S.ckv[0]);
#pragma unroll
      for (int nb = 0; nb < 16; ++nb) {
        const int d = 128 * warp + 8 * nb + 2 * c;
        *reinterpret_cast<float2*>(ps + g * kClPitch + d) = make_float2(o[nb][0], o[nb][1]);
        *reinterpret_cast<float2*>(ps + (g + 8) * kClPitch + d) = make_float2(o[nb][2], o[nb][3]);
      }
      if (warp == 0 && c == 0) {
        ps[kHeads * kClPitch + g] = m0;
        ps[kHeads * kClPitch + g + 8] = m1;
        ps[kHeads * kClPitch + kHeads + g] = l0;
        ps[kHeads * kClPitch + kHeads + g + 8] = l1;
      }
    } else {
      float* ps = part_slot(p, cta, v);
#pragma unroll
      for (int nb = 0; nb < 16; ++nb) {
        const int d = 128 * warp + 8 * nb + 2 * c;
        __stcg(reinterpret_cast<float2*>(ps + g * kDc + d), make_float2(o[nb][0], o[nb][1]));
        __stcg(reinterpret_cast<float2*>(ps + (g + 8) * kDc + d), make_float2(o[nb][2], o[nb][3]));
      }
      if (warp == 0 && c == 0) {
        __stcg(ps + kHeads * kDc + g, m0);
        __stcg(ps + kHeads * kDc + g + 8, m1);
        __stcg(ps + kHeads * kDc + kHeads + g, l0);
        __stcg(ps + kHeads * kDc + kHeads + g + 8, l1);
      }
    }
  }
  if (p.cluster) {
    cluster_sync_all();  // every CTA's partial is in its shared memory
    cluster_merge(p, reinterpret_cast<const float*>(S.ckv[0]), tile_begin / p.tiles_per_token,
                  threadIdx.x);
    cluster_sync_all();  // no CTA leaves while another still reads its partial
  }
  if (p.sync_world > 0 && !p.sync_in_merge) {  // no merge grid: this grid stores last
    named_bar_sync(1, kCWarps * 32);
    if (threadIdx.x == 0) grid_done_then_sync(p, gridDim.x);
  }
  // This CTA's results are written: the merge grid (launched as a dependent)
  // may start its prologue; it still waits for this whole grid to finish.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ================================================================== tcgen05 variant
// Same operator, tiles of 64 rows, MMAs on the 5th-generation tensor cores:
//   S^T[64 rows x 16 heads] = K[64 x 576] . Q^T      (M=64, N=16, K=576: 36 x K16)
//   O^T[512 dims x 16 heads] += V^T[512 x 64] . P^T  (4 x M=128, N=16, K=64)
// with S^T and O^T in TMEM.  The ckv tile is stored once, as 128-byte-swizzled
// 64-dim panels: K-major for QK^T and read MN-major as V^T for PV.
//   warps 0-3  softmax + epilogue (TMEM lanes 0-127): read S^T, online
//              softmax (base 2; O rescaled in TMEM only when a head's maximum
//              grows by more than 2^8), P^T (bf16) to shared memory, output
//   warps 4-7  gather: 16-byte cp.async of each selected row into the swizzled
//              panels (zero-fill for padding), queries at segment starts
//   warp 8     tcgen05.alloc / MMA issue (one lane) / commits
constexpr int kTcRows = 64;
constexpr int kTcPanel = kTcRows * 128;  // 64 rows x 64 dims (bf16)
constexpr int kTcTile = 9 * kTcPanel;    // ckv panels 0-7 + kpe panel 8
constexpr int kTcQPanel = kHeads * 128;  // 16 heads x 64 dims
constexpr int kTcQ = 9 * kTcQPanel;
constexpr int kTcThreads = 9 * 32;
constexpr int kTcO = 0, kTcS = 64;       // TMEM columns: O^T blocks 0-63, S^T buffers 64, 80

struct __align__(1024) TcSmem {
  uint8_t kv[2][kTcTile];
  uint8_t q[2][kTcQ];
  uint8_t p[2][2048];  // P^T [64 rows][16 heads], MN-major, 8x8 core matrices
  float red[2][4][kHeads];
  float lsum[4][kHeads];
  unsigned long long vmask[2][4];
  uint64_t kv_full[2], kv_empty[2], q_full[2], q_empty[2], s_full[2], s_empty[2], p_full[2];
  uint64_t pv_done, o_empty;
  uint32_t tmem_base;
};

__device__ __forceinline__ uint32_t tc_swz(int row, int chunk) {
  return row * 128 + ((chunk ^ (row & 7)) << 4);
}

// Per-head reduction of v[16] over the warp: afterwards lane l holds the
// result for head l>>1 (16 shuffles instead of 80).
template <bool kMax>
__device__ __forceinline__ float warp_reduce_heads(const float* v, int lane) {
  auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
  float a[8], b4[4], c2[2], d;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    const float keep = hi ? v[i + 8] : v[i], send = hi ? v[i] : v[i + 8];
    a[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 16));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    const float keep = hi ? a[i + 4] : a[i], send = hi ? a[i] : a[i + 4];
    b4[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    const float keep = hi ? b4[i + 2] : b4[i], send = hi ? b4[i] : b4[i + 2];
    c2[i] = op(keep, __shfl_xor_sync(0xffffffffu, send, 4));
  }
  {
    const bool hi = lane & 2;
    const float keep = hi ? c2[1] : c2[0], send = hi ? c2[0] : c2[1];
    d = op(keep, __shfl_xor_sync(0xffffffffu, send, 2));
  }
  return op(d, __shfl_xor_sync(0xffffffffu, d, 1));
}

__global__ void __launch_bounds__(kTcThreads, 1)
    dsa_attention_tc_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  TcSmem& S = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int tile_begin = cta_start(p, cta), tile_end = cta_start(p, cta + 1);
  const int tpt = p.tiles_per_token;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&S.kv_full[i], 4 * 32 + 4);  // 128 cp.async arrivals + 4 mask arrivals
      mbar_init(&S.kv_empty[i], 1);
      mbar_init(&S.q_full[i], 4 * 32);
      mbar_init(&S.q_empty[i], 1);
      mbar_init(&S.s_full[i], 1);
      mbar_init(&S.s_empty[i], 4);
      mbar_init(&S.p_full[i], 4);
    }
    mbar_init(&S.pv_done, 1);
    mbar_init(&S.o_empty, 4);
    fence_mbar_init();
  }
  if (warp == 8) tmem_alloc(&S.tmem_base, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;

  if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- gather
    const int pw = warp - 4;
    constexpr int kIdxAhead = 3;
    auto load_idx = [&](int tile) -> int32_t {
      if (tile >= tile_end || lane >= 16) return -1;
      const int v = tile / tpt;
      const int t = v / p.head_groups;
      const int r = (tile - v * tpt) * kTcRows + pw * 16 + lane;
      return __ldg(p.idx + (int64_t)t * p.idx_st + r);
    };
    int32_t ring[kIdxAhead];
#pragma unroll
    for (int k = 0; k < kIdxAhead; ++k) ring[k] = load_idx(tile_begin + k);
    int it = 0, seg = 0;
    bool ok = true;
    for (int tile = tile_begin; tile < tile_end && ok; ++tile, ++it) {
      const int v = tile / tpt;
      if (tile == tile_begin || tile % tpt == 0) {  // queries of a new (token, group)
        const int qb = seg & 1;
        if (!mbar_wait(&S.q_empty[qb], ((seg >> 1) & 1) ^ 1)) {
          set_error(p.err, kErrTimeout);
          break;
        }
        const int t = v / p.head_groups, grp = v - t * p.head_groups;
        const uint32_t qs = smem_u32(S.q[qb]);
#pragma unroll
        for (int k = 0; k < 9; ++k) {
          const int e = lane + 32 * k, h = pw * 4 + e / 72, c = e % 72;
          const __nv_bfloat16* src =
              c < 64 ? p.q_nope + t * p.qn_st + (int64_t)(grp * kHeads + h) * p.qn_sh + c * 8
                     : p.q_pe + t * p.qp_st + (int64_t)(grp * kHeads + h) * p.qp_sh + (c - 64) * 8;
          cp_async16(qs + (c >> 3) * kTcQPanel + tc_swz(h, c & 7), src, 16u);
        }
        cp_async_arrive_noinc(&S.q_full[qb]);
        ++seg;
      }
      const int s = it & 1;
      const int32_t id = ring[0];
#pragma unroll
      for (int k = 0; k + 1 < kIdxAhead; ++k) ring[k] = ring[k + 1];
      ring[kIdxAhead - 1] = load_idx(tile + kIdxAhead);
      if (!mbar_wait(&S.kv_empty[s], ((it >> 1) & 1) ^ 1)) {
        set_error(p.err, kErrTimeout);
        ok = false;
        break;
      }
      const bool mine = lane < 16;
      const bool valid = mine && id >= 0 && id < p.num_slots;
      if (mine && (id < -1 || id >= p.num_slots)) set_error(p.err, kErrBadIndex);
      const uint32_t bits = __ballot_sync(0xffffffffu, valid) & 0xffffu;
      const uint32_t kv = smem_u32(S.kv[s]);
#pragma unroll 4
      for (int rr = 0; rr < 16; ++rr) {
        const int row = pw * 16 + rr;
        const int32_t rid = __shfl_sync(0xffffffffu, id, rr);
        const bool rv = (bits >> rr) & 1u;
        const int64_t page = rv ? (rid >> 6) : 0, r6 = rv ? (rid & 63) : 0;
        const char* crow = reinterpret_cast<const char*>(p.ckv + page * p.ckv_sp + r6 * p.ckv_sr);
        const char* krow = reinterpret_cast<const char*>(p.kpe + page * p.kpe_sp + r6 * p.kpe_sr);
        const uint32_t nb = rv ? 16u : 0u;
        cp_async16(kv + (lane >> 3) * kTcPanel + tc_swz(row, lane & 7), crow + lane * 16, nb);
        cp_async16(kv + ((lane + 32) >> 3) * kTcPanel + tc_swz(row, lane & 7), crow + (lane + 32) * 16,
                   nb);
        if (lane < 8) cp_async16(kv + 8 * kTcPanel + tc_swz(row, lane), krow + lane * 16, nb);
      }
      cp_async_arrive_noinc(&S.kv_full[s]);
      if (lane == 0) {
        S.vmask[s][pw] = (unsigned long long)bits << (16 * pw);
        mbar_arrive(&S.kv_full[s]);
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // nothing of this warp still landing
  } else if (warp == 8) {
    // ---------------------------------------------------------------- MMA issue
    if (lane == 0) {
      constexpr uint32_t id_qk = umma_idesc(1, 1, 0, 0, kTcRows, kHeads);
      constexpr uint32_t id_pv = umma_idesc(1, 1, 1, 1, 128, kHeads);
      bool ok = true;
      // QK of the next tile and PV of the oldest finished softmax are issued
      // as soon as each is ready (polled), so a stage is released right after
      // its PV even while the next tile is still landing.
      const int ntiles = tile_end - tile_begin;
      int qk_next = 0, pv_next = 0;       // tile indices (relative) of the next QK / PV
      int qk_seg = -1;
      const long long t_start = clock64();
      while (pv_next < ntiles && ok) {
        bool progressed = false;
        if (qk_next < ntiles && qk_next <= pv_next + 1) {  // at most 2 S buffers in use
          const int tile = tile_begin + qk_next;
          const bool first = (qk_next == 0) || (tile % tpt == 0);
          const int s = qk_next & 1;
          const int sg = first ? qk_seg + 1 : qk_seg;
          if ((!first || mbar_try_wait(&S.q_full[sg & 1], (sg >> 1) & 1)) &&
              mbar_try_wait(&S.kv_full[s], (qk_next >> 1) & 1) &&
              mbar_try_wait(&S.s_empty[s], ((qk_next >> 1) & 1) ^ 1)) {
            qk_seg = sg;
            tc_fence_after();
            const uint32_t kvb = smem_u32(S.kv[s]), qb = smem_u32(S.q[sg & 1]);
#pragma unroll
            for (int j = 0; j < 36; ++j)
              umma_f16(tmem + kTcS + 16 * s,
                       umma_desc(kvb + (j >> 2) * kTcPanel + (j & 3) * 32, 16, 1024, kSwizzle128B),
                       umma_desc(qb + (j >> 2) * kTcQPanel + (j & 3) * 32, 16, 1024, kSwizzle128B),
                       id_qk, j > 0 ? 1u : 0u);
            umma_commit(&S.s_full[s]);
            const bool last = (tile + 1 == tile_end) || ((tile + 1) % tpt == 0);
            if (last) umma_commit(&S.q_empty[sg & 1]);
            ++qk_next;
            progressed = true;
          }
        }
        if (pv_next < qk_next) {
          const int tile = tile_begin + pv_next;
          const bool first = (pv_next == 0) || (tile % tpt == 0);
          // segment index of this tile: count segment starts up to it
          const int sj = (tile / tpt) - (tile_begin / tpt);
          const int pb = pv_next & 1;
          if (mbar_try_wait(&S.p_full[pb], (pv_next >> 1) & 1) &&
              (!(first && sj > 0) || mbar_try_wait(&S.o_empty, (sj - 1) & 1))) {
            tc_fence_after();
            const uint32_t kvb = smem_u32(S.kv[pv_next & 1]), pbuf = smem_u32(S.p[pb]);
#pragma unroll
            for (int blk = 0; blk < 4; ++blk)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                umma_f16(tmem + kTcO + 16 * blk,
                         umma_desc(kvb + 2 * blk * kTcPanel + ks * 2048, kTcPanel, 1024, kSwizzle128B),
                         umma_desc(pbuf + ks * 256, 128, 1024, 0), id_pv, (ks > 0 || !first) ? 1u : 0u);
            umma_commit(&S.kv_empty[pv_next & 1]);
            umma_commit(&S.pv_done);
            ++pv_next;
            progressed = true;
          }
        }
        if (!progressed && clock64() - t_start > kWaitBudgetCycles * 8) ok = false;
      }
      if (!ok) set_error(p.err, kErrTimeout);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    const int tid = threadIdx.x;  // 0..127 == TMEM lane
    const int row = warp * 16 + lane;  // S^T row held by this thread (lanes 0-15)
    float m_used[kHeads], lp[kHeads];
    int it = 0, pv_seen = 0;
    bool ok = true;
    auto wait_pv = [&](int j) -> bool {  // PV of tile j (and all before) complete
      while (pv_seen <= j) {
        if (!mbar_wait(&S.pv_done, pv_seen & 1)) return false;
        ++pv_seen;
      }
      return true;
    };
    for (int tile = tile_begin; tile < tile_end && ok; ++tile, ++it) {
      const int v = tile / tpt;
      const bool first = (tile == tile_begin) || (tile % tpt == 0);
      const bool last = (tile + 1 == tile_end) || ((tile + 1) % tpt == 0);
      if (first) {
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          m_used[h] = -INFINITY;
          lp[h] = 0.f;
        }
      }
      const int s = it & 1;
      if (!mbar_wait(&S.s_full[s], (it >> 1) & 1) || !mbar_wait(&S.kv_full[s], (it >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[kHeads];
      tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + kTcS + 16 * s, x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.s_empty[s]);
      const unsigned long long vm = S.vmask[s][0] | S.vmask[s][1] | S.vmask[s][2] | S.vmask[s][3];
      const bool valid = lane < 16 && ((vm >> row) & 1ull);
#pragma unroll
      for (int h = 0; h < kHeads; ++h) x[h] = valid ? x[h] * p.scale_log2 : -INFINITY;
      // tile maximum per head over the 64 rows
      const float wm = warp_reduce_heads<true>(x, lane);
      if ((lane & 1) == 0) S.red[it & 1][warp][lane >> 1] = wm;
      named_bar_sync(1, 128);
      float nm[kHeads];
      bool grow = false;
#pragma unroll
      for (int h = 0; h < kHeads; ++h) {
        const float mt = fmaxf(fmaxf(S.red[it & 1][0][h], S.red[it & 1][1][h]),
                               fmaxf(S.red[it & 1][2][h], S.red[it & 1][3][h]));
        nm[h] = fmaxf(m_used[h], mt);
        grow |= (mt > m_used[h] + 8.f) || (m_used[h] == -INFINITY && mt != -INFINITY);
      }
      if (it > 0 && !wait_pv(it - 1)) {  // P buffer free; O settled before a rescale
        ok = false;
        break;
      }
      if (grow) {  // uniform over the 128 threads
        float alpha[kHeads];
#pragma unroll
        for (int h = 0; h < kHeads; ++h) {
          alpha[h] = (m_used[h] == -INFINITY) ? 0.f : exp2f(m_used[h] - nm[h]);
          lp[h] *= alpha[h];
          m_used[h] = nm[h];
        }
        if (!first) {
          tc_fence_after();
#pragma unroll
          for (int blk = 0; blk < 4; ++blk) {
            float o[kHeads];
            const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + kTcO + 16 * blk;
            tmem_ld16(ta, o);
#pragma unroll
            for (int h = 0; h < kHeads; ++h) o[h] *= alpha[h];
            tmem_st16(ta, o);
          }
        }
      }
      uint32_t pk[8];
#pragma unroll
      for (int h = 0; h < kHeads; h += 2) {
        const float p0 = (x[h] == -INFINITY) ? 0.f : exp2f(x[h] - m_used[h]);
        const float p1 = (x[h + 1] == -INFINITY) ? 0.f : exp2f(x[h + 1] - m_used[h + 1]);
        lp[h] += p0;
        lp[h + 1] += p1;
        pk[h >> 1] = pack_bf16(p0, p1);
      }
      if (lane < 16) {
        uint8_t* pb = S.p[it & 1] + (row >> 3) * 128 + (row & 7) * 16;
        *reinterpret_cast<uint4*>(pb) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(pb + 1024) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.p_full[it & 1]);

      if (last) {
        // ------------------------------------------------------------ epilogue
        const float wl = warp_reduce_heads<false>(lp, lane);
        if ((lane & 1) == 0) S.lsum[warp][lane >> 1] = wl;
        if (!wait_pv(it)) {
          ok = false;
          break;
        }
        named_bar_sync(1, 128);
        tc_fence_after();
        float L[kHeads];
#pragma unroll
        for (int h = 0; h < kHeads; ++h) L[h] = S.lsum[0][h] + S.lsum[1][h] + S.lsum[2][h] + S.lsum[3][h];
        const int t = v / p.head_groups, grp = v - t * p.head_groups;
        const int c_first = cta_of_tile(p, v * tpt), c_last = cta_of_tile(p, v * tpt + tpt - 1);
        const bool direct = c_first == c_last;
        float* ps = direct ? nullptr : part_slot(p, cta, v);
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
          float o[kHeads];
          tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + kTcO + 16 * blk, o);
          const int d = 128 * blk + tid;
#pragma unroll
          for (int h = 0; h < kHeads; ++h) {
            if (direct) {
              const float inv = (m_used[h] == -INFINITY) ? 0.f : 1.f / L[h];
              const __nv_bfloat16 ov = __float2bfloat16_rn(o[h] * inv);
              for (int k = 0; k < n_targets(p); ++k)
                out_target(p, k)[t * p.out_st + (int64_t)(grp * kHeads + h) * p.out_sh + d] = ov;
            } else {
              __stcg(ps + h * kDc + d, o[h]);
            }
          }
        }
        if (tid < kHeads) {
          float m = m_used[0], l = L[0];
#pragma unroll
          for (int h = 1; h < kHeads; ++h)
            if (h == tid) {
              m = m_used[h];
              l = L[h];
            }
          if (direct) {
            for (int k = 0; k < n_targets(p); ++k)
              lse_target(p, k)[t * p.lse_st + (int64_t)(grp * kHeads + tid) * p.lse_sh] =
                  (m == -INFINITY) ? -INFINITY : m + log2f(l);
          } else {
            __stcg(ps + kHeads * kDc + tid, m);
            __stcg(ps + kHeads * kDc + kHeads + tid, l);
          }
        }
        tc_fence_before();
        named_bar_sync(1, 128);  // lsum / O reads done before the next segment
        if (lane == 0) mbar_arrive(&S.o_empty);
      }
    }
    if (!ok) set_error(p.err, kErrTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ host side
namespace {

thread_local char g_errmsg[512] = "";

int fail(int code, const char* msg) {
  snprintf(g_errmsg, sizeof(g_errmsg), "%s", msg);
  return code;
}

struct DevInfo {
  int sms = 0;
  int occ[5] = {0, 0, 0, 0, 0};
  int clusters[5][9] = {};  // [stages][cluster size]: resident clusters (-1: none)
};
std::mutex g_mu;
DevInfo g_dev[64];

// Tuning / profiling options, process-wide, set only through dsa_set_options
// (nothing is read from the environment).  Each call takes a copy.
std::mutex g_opt_mu;
dsa_options g_opt = {0, 0, 0, 0, 0, 1, 0, 0};

dsa_options current_options() {
  std::lock_guard<std::mutex> lk(g_opt_mu);
  return g_opt;
}

int stages_choice(const dsa_options& o) {
  const int s = o.attention_stages ? o.attention_stages : 2;
  return (s >= 2 && s <= 4) ? s : 2;
}

template <int NST>
int smem_bytes() {
  return (int)sizeof(AttnSmem<NST>);
}

template <int NST>
cudaError_t ensure_attr() {
  return cudaFuncSetAttribute(dsa_attention_kernel<NST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              smem_bytes<NST>());
}

// SM count and resident CTAs per SM for the given stage count (cached per device).
int device_slots(int nst, int* sms_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  std::lock_guard<std::mutex> lk(g_mu);
  DevInfo& d = g_dev[dev];
  if (d.sms == 0) {
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return -1;
  }
  if (d.occ[nst] == 0) {
    cudaError_t e;
    int occ = 0;
    switch (nst) {
      case 2:
        e = ensure_attr<2>();
        if (e == cudaSuccess)
          e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dsa_attention_kernel<2>, kThreads,
                                                            smem_bytes<2>());
        break;
      case 3:
        e = ensure_attr<3>();
        if (e == cudaSuccess)
          e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dsa_attention_kernel<3>, kThreads,
                                                            smem_bytes<3>());
        break;
      default:
        e = ensure_attr<4>();
        if (e == cudaSuccess)
          e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, dsa_attention_kernel<4>, kThreads,
                                                            smem_bytes<4>());
        break;
    }
    if (e != cudaSuccess || occ < 1) return -1;
    d.occ[nst] = occ;
  }
  *sms_out = d.sms;
  return d.occ[nst];
}

struct Plan {
  int ctas, base, rem;
  int per_token;  // token-aligned plan: CTAs per virtual token, 0 otherwise
  int cluster;  // CTAs per token in the cluster plan, 0 otherwise
  int64_t vtokens, total_tiles;
  size_t part_off, bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Grid plan: an even split of all tiles over min(slots, tiles/min_tiles) CTAs.
// Which kernel: option attention_kernel 0 (default) or 1: the mma.sync kernel
// (32-row tiles); 2: the tcgen05 kernel (64-row tiles).  With 16 heads every
// tcgen05 MMA has N=16 and a 64-row tile in MMA layout takes 72 KB of shared
// memory (two stages fit); measured on a B200 the tcgen05 kernel was slower on
// both the HBM-bound decode (cfg2: 82 vs 53 us) and the L2-resident prefill
// (cfg5: 3.2 vs 1.6 ms); it is kept as a tested alternative.
bool tc_choice(const dsa_options& o) { return o.attention_kernel == 2; }

int tc_smem_bytes() { return (int)sizeof(TcSmem) + 1024; }

int resident_clusters(int nst, int csize);

// Grid plan.  Stream-K: an even split of all tiles over
// min(slots, tiles/min_tiles) CTAs; tokens split across CTAs are merged by the
// merge grid.  Cluster plan (mma.sync kernel, option attention_cluster = C of
// 2, 4 or 8): when virtual tokens x C CTAs fit in the resident slots and every
// CTA keeps >= min_tiles tiles, every token is split evenly over one cluster
// of C CTAs, which merge inside the attention grid (one launch); otherwise
// stream-K.  Not the default: measured on a B200 at 64 tokens, C=4 (256 CTAs)
// took 47.1 us per call against 43.0 us for stream-K (296 CTAs + merge grid),
// the fewer CTAs gathering costing more than the merge grid.
int make_plan(int64_t num_tokens, int64_t heads, int64_t topk, int nst, Plan* pl, bool tc,
              const dsa_options& o) {
  int sms = 0;
  int occ = 0;
  if (tc) {
    occ = device_slots(2, &sms) > 0 ? 1 : 0;  // SM count; one tcgen05 CTA per SM
  } else {
    occ = device_slots(nst, &sms);
  }
  if (occ < 1) return fail(DSA_ERR_CUDA, "cannot query device / occupancy for the attention kernel");
  const int64_t tpt = topk / (tc ? kTcRows : kRows);
  pl->vtokens = num_tokens * (heads / kHeads);
  pl->total_tiles = pl->vtokens * tpt;
  const int min_tiles = o.attention_min_tiles > 0 ? o.attention_min_tiles : (tc ? 2 : 4);
  int64_t ctas = (int64_t)sms * occ;
  if (o.attention_ctas > 0) ctas = o.attention_ctas;
  const int64_t slots = ctas;
  ctas = std::min<int64_t>(ctas, (pl->total_tiles + min_tiles - 1) / min_tiles);
  if (ctas < 1) ctas = 1;
  // Token-aligned split: when there are fewer (token, head group) pairs than
  // resident CTAs, every pair gets the same number C of CTAs, so no CTA
  // straddles two pairs and each pair has exactly C partials.  C is the
  // largest divisor of the pair's tile count that fits (the flat split above
  // then yields this partition) when that fills >= 80% of the slots; else
  // C = floor(slots / pairs) when C >= 4 and it fills >= 80% (part j of a pair
  // takes tiles [j*tpt/C, (j+1)*tpt/C)); else stream-K.  Measured on B200s
  // (300-400-step means, same process): T=64 (C=4) 42.0 vs 43.1 us stream-K;
  // T=24 (C=12) 26.8 vs 28.5; T=48 (C=6) 34.8 vs 36.8; 48/64-head cfg3 shards
  // 2 us faster; C=3 (T=80) lost 1 us; the per-token closed form costs ~1 us
  // more than the flat one for the same partition, so divisors come first.
  pl->per_token = 0;
  if (!tc && o.attention_ctas == 0 && pl->vtokens < slots) {
    const int64_t cmax = std::min<int64_t>(tpt / min_tiles, slots / pl->vtokens);
    int64_t cd = cmax;
    while (cd >= 2 && tpt % cd) --cd;
    if (cd >= 2 && pl->vtokens * cd * 10 >= slots * 8) {
      ctas = pl->vtokens * cd;
    } else if (cmax >= 4 && pl->vtokens * cmax * 10 >= slots * 8) {
      ctas = pl->vtokens * cmax;
      pl->per_token = (int)cmax;
    }
  }
  pl->cluster = 0;
  if (!tc && o.attention_ctas == 0 && o.attention_cluster >= 2) {
    const int c = o.attention_cluster;
    const int64_t n = pl->vtokens * c;
    if (tpt % c == 0 && tpt / c >= min_tiles && n <= slots && pl->vtokens <= resident_clusters(nst, c)) {
      pl->cluster = c;
      pl->per_token = 0;
      ctas = n;
    }
  }
  pl->ctas = (int)ctas;
  pl->base = (int)(pl->total_tiles / ctas);
  pl->rem = (int)(pl->total_tiles % ctas);
  pl->part_off = 256;  // error word, then the split-K partials
  pl->bytes = pl->part_off + (size_t)pl->ctas * 2 * kPartFloats * sizeof(float);
  return DSA_OK;
}

template <int NST>
cudaError_t launch(const AttnParams& p, int ctas, cudaStream_t st) {
  cudaError_t e = ensure_attr<NST>();
  if (e != cudaSuccess) return e;
  if (p.cluster) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)smem_bytes<NST>();
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dsa_attention_kernel<NST>, p);
  }
  dsa_attention_kernel<NST><<<ctas, kThreads, smem_bytes<NST>(), st>>>(p);
  return cudaGetLastError();
}

// Clusters of `csize` CTAs of the mma.sync kernel that can be resident at
// once on the current device; 0 when none (or the query fails).
template <int NST>
int resident_clusters_q(int csize) {
  if (ensure_attr<NST>() != cudaSuccess) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)csize);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes<NST>();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, dsa_attention_kernel<NST>, &cfg) != cudaSuccess) {
    cudaGetLastError();  // a failed query leaves no error behind for the next launch
    return 0;
  }
  return n;
}

// Cached per device, stage count and cluster size.
int resident_clusters(int nst, int csize) {
  if (nst < 2 || nst > 4 || csize < 1 || csize > 8) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    const int c = g_dev[dev].clusters[nst][csize];
    if (c != 0) return c < 0 ? 0 : c;
  }
  const int n = nst == 2 ? resident_clusters_q<2>(csize)
                         : nst == 3 ? resident_clusters_q<3>(csize) : resident_clusters_q<4>(csize);
  std::lock_guard<std::mutex> lk(g_mu);
  g_dev[dev].clusters[nst][csize] = n > 0 ? n : -1;
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int report_error(int code, const char* msg) { return fail(code, msg); }

}  // namespace dsa

using namespace dsa;

static int attention_impl(const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head,
                         const void* q_pe, int64_t q_pe_stride_token, int64_t q_pe_stride_head,
                         const void* ckv_cache, int64_t ckv_stride_page, int64_t ckv_stride_row,
                         const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
                         const int32_t* sparse_indices, int64_t indices_stride_token,
                         int64_t num_tokens, int64_t num_heads, int64_t num_pages, int64_t page_size,
                         int64_t topk, float sm_scale, void* output, int64_t out_stride_token,
                         int64_t out_stride_head, float* lse, int64_t lse_stride_token,
                         int64_t lse_stride_head, void* workspace, size_t workspace_bytes,
                         void* stream, void* const* out_peers, float* const* lse_peers, int n_peers,
                         int* const* sync_flags = nullptr, int sync_rank = 0, int sync_world = 0) {
  if (num_tokens < 0) return fail(DSA_ERR_INVALID_ARG, "num_tokens < 0");
  if (num_heads <= 0 || num_heads % kHeads)
    return fail(DSA_ERR_UNSUPPORTED, "num_heads must be a positive multiple of 16");
  if (page_size != 64) return fail(DSA_ERR_UNSUPPORTED, "page_size must be 64");
  if (topk <= 0 || topk % kRows || topk > (1 << 20))
    return fail(DSA_ERR_UNSUPPORTED, "topk must be a positive multiple of 32");
  if (num_pages < 0 || num_pages * 64 > INT32_MAX)
    return fail(DSA_ERR_INVALID_ARG, "num_pages out of range for int32 slot ids");
  if (num_tokens == 0) return DSA_OK;
  if (n_peers > 0) {  // stores go to the targets; output / lse are unused
    if (!out_peers || !lse_peers) return fail(DSA_ERR_INVALID_ARG, "NULL target pointer array");
    for (int k = 0; k < n_peers; ++k)
      if (!out_peers[k] || !lse_peers[k] || (reinterpret_cast<uintptr_t>(out_peers[k]) & 7))
        return fail(DSA_ERR_INVALID_ARG, "output targets must be non-NULL and 8-byte aligned");
    output = out_peers[0];
    lse = lse_peers[0];
  }
  if (!q_nope || !q_pe || !ckv_cache || !kpe_cache || !sparse_indices || !output || !lse ||
      !workspace)
    return fail(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  // 16-byte row gathers / fragment loads need aligned rows.
  if (!aligned16(ckv_cache) || !aligned16(kpe_cache) || ckv_stride_page % 8 || ckv_stride_row % 8 ||
      kpe_stride_page % 8 || kpe_stride_row % 8)
    return fail(DSA_ERR_INVALID_ARG, "cache rows must be 16-byte aligned (strides multiple of 8)");
  if ((reinterpret_cast<uintptr_t>(q_nope) & 3) || (reinterpret_cast<uintptr_t>(q_pe) & 3) ||
      q_nope_stride_token % 2 || q_nope_stride_head % 2 || q_pe_stride_token % 2 ||
      q_pe_stride_head % 2)
    return fail(DSA_ERR_INVALID_ARG, "q rows must be 4-byte aligned");
  if ((reinterpret_cast<uintptr_t>(output) & 7) || out_stride_token % 4 || out_stride_head % 4)
    return fail(DSA_ERR_INVALID_ARG, "output rows must be 8-byte aligned");
  const dsa_options opt = current_options();
  const int nst = stages_choice(opt);
  // the tcgen05 kernel gathers queries with 16-byte copies
  const bool q16 = !(reinterpret_cast<uintptr_t>(q_nope) & 15) && !(reinterpret_cast<uintptr_t>(q_pe) & 15) &&
                   q_nope_stride_token % 8 == 0 && q_nope_stride_head % 8 == 0 &&
                   q_pe_stride_token % 8 == 0 && q_pe_stride_head % 8 == 0;
  if (sync_world > 0) {
    if (!sync_flags || sync_world > kMaxTargets || sync_rank < 0 || sync_rank >= sync_world)
      return fail(DSA_ERR_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
    for (int q = 0; q < sync_world; ++q)
      if (!sync_flags[q] || (reinterpret_cast<uintptr_t>(sync_flags[q]) & 3))
        return fail(DSA_ERR_INVALID_ARG, "NULL or misaligned flag buffer");
  }
  // the cross-GPU barrier runs inside the mma.sync kernel's grids only
  const bool tc = tc_choice(opt) && topk % kTcRows == 0 && q16 && sync_world == 0;
  Plan pl;
  int rc = make_plan(num_tokens, num_heads, topk, nst, &pl, tc, opt);
  if (rc) return rc;
  if (workspace_bytes < pl.bytes || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(DSA_ERR_WORKSPACE, "workspace too small or not 256-byte aligned");

  AttnParams p;
  p.q_nope = static_cast<const __nv_bfloat16*>(q_nope);
  p.q_pe = static_cast<const __nv_bfloat16*>(q_pe);
  p.ckv = static_cast<const __nv_bfloat16*>(ckv_cache);
  p.kpe = static_cast<const __nv_bfloat16*>(kpe_cache);
  p.idx = sparse_indices;
  p.out = static_cast<__nv_bfloat16*>(output);
  p.lse = lse;
  p.n_peers = n_peers;
  for (int k = 0; k < kMaxTargets; ++k) {
    p.out_peers[k] = k < n_peers ? static_cast<__nv_bfloat16*>(out_peers[k]) : nullptr;
    p.lse_peers[k] = k < n_peers ? lse_peers[k] : nullptr;
  }
  p.qn_st = q_nope_stride_token;
  p.qn_sh = q_nope_stride_head;
  p.qp_st = q_pe_stride_token;
  p.qp_sh = q_pe_stride_head;
  p.ckv_sp = ckv_stride_page;
  p.ckv_sr = ckv_stride_row;
  p.kpe_sp = kpe_stride_page;
  p.kpe_sr = kpe_stride_row;
  p.idx_st = indices_stride_token;
  p.out_st = out_stride_token;
  p.out_sh = out_stride_head;
  p.lse_st = lse_stride_token;
  p.lse_sh = lse_stride_head;
  p.num_slots = num_pages * 64;
  p.head_groups = (int)(num_heads / kHeads);
  p.tiles_per_token = (int)(topk / (tc ? kTcRows : kRows));
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.tiles_base = pl.base;
  p.tiles_rem = pl.rem;
  p.per_token = pl.per_token;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.err = reinterpret_cast<int*>(ws);
  p.part = reinterpret_cast<float*>(ws + pl.part_off);
  p.sync_world = sync_world;
  p.sync_rank = sync_rank;
  p.cluster = pl.cluster;
  p.sync_in_merge = (pl.ctas > 1 && !pl.cluster) ? 1 : 0;
  p.merge_by_boundary = 0;
  for (int q = 0; q < kMaxTargets; ++q) p.sync_flags[q] = q < sync_world ? sync_flags[q] : nullptr;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Profiling option attention_grids: 1 = attention grid only, 2 = merge grid
  // only (on the partials of an earlier call with the same shapes); 0 both.
  const int stage = sync_world > 0 ? 0 : opt.attention_grids;  // the barrier needs both grids
  cudaError_t e = cudaSuccess;
  if (stage != 2) {
    if (tc) {
      e = cudaFuncSetAttribute(dsa_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               tc_smem_bytes());
      if (e == cudaSuccess) {
        dsa_attention_tc_kernel<<<pl.ctas, kTcThreads, tc_smem_bytes(), st>>>(p);
        e = cudaGetLastError();
      }
    } else {
      e = nst == 2 ? launch<2>(p, pl.ctas, st)
                   : nst == 3 ? launch<3>(p, pl.ctas, st) : launch<4>(p, pl.ctas, st);
    }
  }
  if (e != cudaSuccess) return fail(DSA_ERR_CUDA, cudaGetErrorString(e));
  if (pl.ctas > 1 && !pl.cluster && stage != 1) {  // split tokens: merge grid as a programmatic dependent
    cudaLaunchConfig_t cfg = {};
    p.merge_by_boundary = pl.vtokens > pl.ctas - 1 ? 1 : 0;
    cfg.gridDim = dim3(kHeads, (unsigned)(p.merge_by_boundary ? pl.ctas - 1 : pl.vtokens));
    cfg.blockDim = dim3(kMergeThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = opt.merge_pdl ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, dsa_attention_merge_kernel, p);
    if (e != cudaSuccess) return fail(DSA_ERR_CUDA, cudaGetErrorString(e));
  }
  return DSA_OK;
}

extern "C" {

const char* dsa_last_error_message(void) { return g_errmsg; }

int dsa_sparse_attention_workspace_size(int64_t num_tokens, int64_t num_heads, int64_t topk,
                                        size_t* bytes) {
  if (!bytes) return fail(DSA_ERR_INVALID_ARG, "bytes is NULL");
  if (num_tokens < 0 || num_heads <= 0 || num_heads % kHeads || topk <= 0 || topk % kRows)
    return fail(DSA_ERR_INVALID_ARG, "num_heads must be a multiple of 16 and topk of 32");
  Plan pl;
  const dsa_options opt = current_options();
  // q alignment is unknown here: size for the larger of the two plans
  Plan pl_tc;
  int rc = make_plan(num_tokens > 0 ? num_tokens : 1, num_heads, topk, stages_choice(opt), &pl, false,
                     opt);
  if (rc) return rc;
  if (tc_choice(opt) && topk % kTcRows == 0) {
    rc = make_plan(num_tokens > 0 ? num_tokens : 1, num_heads, topk, stages_choice(opt), &pl_tc, true,
                   opt);
    if (rc) return rc;
    if (pl_tc.bytes > pl.bytes) pl = pl_tc;
  }
  *bytes = pl.bytes;
  return DSA_OK;
}

int dsa_set_options(const dsa_options* options) {
  dsa_options o = {0, 0, 0, 0, 0, 1, 0, 0};
  if (options) {
    o = *options;
    if (o.attention_kernel < 0 || o.attention_kernel > 2 || o.attention_stages < 0 ||
        o.attention_stages > 4 || o.attention_stages == 1 || o.attention_ctas < 0 ||
        o.attention_min_tiles < 0 || o.attention_grids < 0 || o.attention_grids > 2 ||
        o.merge_pdl < 0 || o.merge_pdl > 1 || o.indexer_tiles_per_cta < 0 ||
        !(o.attention_cluster == 0 || o.attention_cluster == 1 || o.attention_cluster == 2 ||
          o.attention_cluster == 4 || o.attention_cluster == 8))
      return fail(DSA_ERR_INVALID_ARG, "dsa_set_options: a field is out of range");
  }
  std::lock_guard<std::mutex> lk(g_opt_mu);
  g_opt = o;
  return DSA_OK;
}

int dsa_get_options(dsa_options* options) {
  if (!options) return fail(DSA_ERR_INVALID_ARG, "options is NULL");
  *options = current_options();
  return DSA_OK;
}

int dsa_sparse_attention(const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head,
                         const void* q_pe, int64_t q_pe_stride_token, int64_t q_pe_stride_head,
                         const void* ckv_cache, int64_t ckv_stride_page, int64_t ckv_stride_row,
                         const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
                         const int32_t* sparse_indices, int64_t indices_stride_token,
                         int64_t num_tokens, int64_t num_heads, int64_t num_pages, int64_t page_size,
                         int64_t topk, float sm_scale, void* output, int64_t out_stride_token,
                         int64_t out_stride_head, float* lse, int64_t lse_stride_token,
                         int64_t lse_stride_head, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return attention_impl(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe, q_pe_stride_token,
                        q_pe_stride_head, ckv_cache, ckv_stride_page, ckv_stride_row, kpe_cache,
                        kpe_stride_page, kpe_stride_row, sparse_indices, indices_stride_token,
                        num_tokens, num_heads, num_pages, page_size, topk, sm_scale, output,
                        out_stride_token, out_stride_head, lse, lse_stride_token, lse_stride_head,
                        workspace, workspace_bytes, stream, nullptr, nullptr, 0);
}

int dsa_sparse_attention_scatter(const void* q_nope, int64_t q_nope_stride_token,
                                 int64_t q_nope_stride_head, const void* q_pe,
                                 int64_t q_pe_stride_token, int64_t q_pe_stride_head,
                                 const void* ckv_cache, int64_t ckv_stride_page, int64_t ckv_stride_row,
                                 const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
                                 const int32_t* sparse_indices, int64_t indices_stride_token,
                                 int64_t num_tokens, int64_t num_heads, int64_t num_pages,
                                 int64_t page_size, int64_t topk, float sm_scale,
                                 void* const* out_targets, int64_t out_stride_token,
                                 int64_t out_stride_head, float* const* lse_targets,
                                 int64_t lse_stride_token, int64_t lse_stride_head, int num_targets,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  if (num_targets <= 0 || num_targets > kMaxTargets)
    return fail(DSA_ERR_INVALID_ARG, "num_targets must be in 1..8");
  return attention_impl(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe, q_pe_stride_token,
                        q_pe_stride_head, ckv_cache, ckv_stride_page, ckv_stride_row, kpe_cache,
                        kpe_stride_page, kpe_stride_row, sparse_indices, indices_stride_token,
                        num_tokens, num_heads, num_pages, page_size, topk, sm_scale, nullptr,
                        out_stride_token, out_stride_head, nullptr, lse_stride_token, lse_stride_head,
                        workspace, workspace_bytes, stream, out_targets, lse_targets, num_targets);
}

int dsa_sparse_attention_scatter_sync(
    const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head, const void* q_pe,
    int64_t q_pe_stride_token, int64_t q_pe_stride_head, const void* ckv_cache, int64_t ckv_stride_page,
    int64_t ckv_stride_row, const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
    const int32_t* sparse_indices, int64_t indices_stride_token, int64_t num_tokens, int64_t num_heads,
    int64_t num_pages, int64_t page_size, int64_t topk, float sm_scale, void* const* out_targets,
    int64_t out_stride_token, int64_t out_stride_head, float* const* lse_targets,
    int64_t lse_stride_token, int64_t lse_stride_head, int num_targets, int* const* flags, int rank,
    int world, void* workspace, size_t workspace_bytes, void* stream) {
  if (num_targets <= 0 || num_targets > kMaxTargets)
    return fail(DSA_ERR_INVALID_ARG, "num_targets must be in 1..8");
  if (world <= 0) return fail(DSA_ERR_INVALID_ARG, "world must be 1..8 and 0 <= rank < world");
  if (num_tokens == 0)  // nothing to store: the ranks still meet
    return dsa_peer_barrier(flags, rank, world, reinterpret_cast<int*>(workspace), stream);
  return attention_impl(q_nope, q_nope_stride_token, q_nope_stride_head, q_pe, q_pe_stride_token,
                        q_pe_stride_head, ckv_cache, ckv_stride_page, ckv_stride_row, kpe_cache,
                        kpe_stride_page, kpe_stride_row, sparse_indices, indices_stride_token,
                        num_tokens, num_heads, num_pages, page_size, topk, sm_scale, nullptr,
                        out_stride_token, out_stride_head, nullptr, lse_stride_token, lse_stride_head,
                        workspace, workspace_bytes, stream, out_targets, lse_targets, num_targets,
                        flags, rank, world);
}

int dsa_read_device_error(const void* workspace, int clear, int* bits, void* stream) {
  if (!workspace || !bits) return fail(DSA_ERR_INVALID_ARG, "NULL pointer argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && clear && h)
    e = cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int), st);
  if (e != cudaSuccess) return fail(DSA_ERR_CUDA, cudaGetErrorString(e));
  *bits = h;
  return DSA_OK;
}

}  // extern "C"
