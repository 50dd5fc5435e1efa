/*
 * dsa_b200.h -- C ABI of the B200 (sm_100a) DeepSeek-sparse-attention library.
 *
 * Plain pointers, sizes and element strides; no framework types.  Every call
 * is asynchronous on the given CUDA stream (a cudaStream_t passed as void*,
 * NULL = legacy default stream) and returns a dsa_status code; the message of
 * the last failing call on the calling host thread is available from
 * dsa_last_error_message().  Device pointers must be on the current device.
 *
 * Reference interfaces replaced (Starkdoorstep12/flashinfer-repo):
 *   dsa_sparse_attention      <- solution/triton/kernel.py:138-182 `kernel`
 *                                (and the split-K variants kernel.py:496-567,
 *                                707-799, which compute the same function);
 *                                the CUDA/TVM-FFI slot the reference leaves
 *                                empty is solution/cuda/binding.py:14-25 and
 *                                solution/cuda/kernel.cu:13-20.
 *   dsa_indexer_scores        <- solution/triton/indexer_kernel.py:4-287
 *                                `indexer_kernel` (+ launch at :386-409)
 *   dsa_topk_select           <- solution/triton/indexer_kernel.py:289-343
 *                                `topk_kernel` (+ launch at :422-431)
 *   dsa_indexer_topk          <- solution/triton/indexer_kernel.py:345-433
 *                                `run_indexer_and_topk`
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
enum dsa_status {
  DSA_OK = 0,
  DSA_ERR_INVALID_ARG = 1, /* NULL pointer, negative size, misaligned row */
  DSA_ERR_UNSUPPORTED = 2, /* shape outside what the kernels implement */
  DSA_ERR_WORKSPACE = 3,   /* workspace too small or misaligned */
  DSA_ERR_CUDA = 4         /* a CUDA runtime call failed (message has details) */
};

/* Bits of the device error word (first int of a workspace). */
enum dsa_device_error {
  DSA_DEVERR_BAD_INDEX = 1, /* an index outside [-1, num_pages*64): row skipped */
  DSA_DEVERR_TIMEOUT = 2    /* a bounded wait inside a kernel gave up */
};

/* Message of the last failing call on this host thread ("" if none). */
const char* dsa_last_error_message(void);

/*
 * Tuning and profiling options, process-wide (no counterpart in the
 * reference, whose kernels take their block sizes as Triton constexprs).
 * The library reads no environment variable; these values are the only way
 * to change a launch plan.  Zero selects the default of a field.
 *   attention_kernel   0 default; 1 the mma.sync kernel (32-row tiles);
 *                      2 the tcgen05 kernel (64-row tiles, TMEM accumulators)
 *   attention_stages   shared-memory ring depth of the mma.sync kernel, 2..4
 *   attention_ctas     grid size (0: resident CTAs per SM x SMs)
 *   attention_min_tiles  fewest 32-row tiles per CTA (0: 4)
 *   attention_grids    PROFILING ONLY: 1 launches the attention grid alone
 *                      (outputs of tokens split across CTAs are then not
 *                      written), 2 the merge grid alone; 0 both
 *   merge_pdl          1 (default) launches the merge grid as a programmatic
 *                      dependent of the attention grid; 0 a plain launch
 *   indexer_tiles_per_cta  128-token tiles per indexer CTA (0: 20)
 *   attention_cluster  2, 4 or 8: where (token, 16-head group) pairs x C
 *                      CTAs fit on the GPU at once, each pair is split over a
 *                      thread-block cluster of C CTAs that merge through
 *                      distributed shared memory (one launch, no merge grid);
 *                      0 or 1 (default): stream-K + merge grid
 * dsa_set_options(NULL) restores every default.  Changing options while
 * other host threads launch gives each launch either the old or the new set.
 */
typedef struct dsa_options {
  int attention_kernel;
  int attention_stages;
  int attention_ctas;
  int attention_min_tiles;
  int attention_grids;
  int merge_pdl;
  int indexer_tiles_per_cta;
  int attention_cluster;
} dsa_options;
int dsa_set_options(const dsa_options* options);
int dsa_get_options(dsa_options* options);

/*
 * Workspace bytes dsa_sparse_attention needs for this shape on the current
 * device.  Layout: the device error word (first 256 bytes), then two split-K
 * partial slots per CTA of the launch plan (acc[16][512], m[16], l[16] fp32).
 */
int dsa_sparse_attention_workspace_size(int64_t num_tokens, int64_t num_heads, int64_t topk,
                                        size_t* bytes);

/*
 * Sparse MLA attention over a paged latent cache (one decode step).
 * Replaces kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale)
 * -> (output, lse) of solution/triton/kernel.py:138-182.
 *
 *   q_nope  [T, H, 512] bf16     q_pe [T, H, 64] bf16        (H = 16*k)
 *   ckv     [num_pages, 64, 512] bf16, kpe [num_pages, 64, 64] bf16
 *   sparse_indices [T, topk] int32: flat slot ids page*64+offset, -1 = pad
 *   output  [T, H, 512] bf16     lse [T, H] fp32 (base-2 log-sum-exp)
 * Strides are in elements; the last dimension of every tensor is contiguous.
 * Cache rows must be 16-byte aligned, q rows 4-byte, output rows 8-byte.
 * A token with no valid index gets output 0 and lse -inf (kernel.py:118-136).
 * page_size must be 64 and topk a multiple of 32 (the reference asserts
 * H=16, page_size=64, topk=2048, kernel.py:147-151; H>16 is handled as
 * independent 16-head groups sharing the same indices).
 *
 * workspace: >= dsa_sparse_attention_workspace_size() bytes, 256-byte aligned,
 * its first int zero before the first use (the device error word, cleared by
 * dsa_read_device_error; the rest holds split-K partials and needs no
 * initialisation).  The same workspace can be reused by later calls of any
 * size on the same stream; calls that share one workspace must not overlap
 * in time.
 */
int dsa_sparse_attention(const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head,
                         const void* q_pe, int64_t q_pe_stride_token, int64_t q_pe_stride_head,
                         const void* ckv_cache, int64_t ckv_stride_page, int64_t ckv_stride_row,
                         const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
                         const int32_t* sparse_indices, int64_t indices_stride_token,
                         int64_t num_tokens, int64_t num_heads, int64_t num_pages, int64_t page_size,
                         int64_t topk, float sm_scale, void* output, int64_t out_stride_token,
                         int64_t out_stride_head, float* lse, int64_t lse_stride_token,
                         int64_t lse_stride_head, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * dsa_sparse_attention_scatter -- dsa_sparse_attention whose epilogues store
 * the result straight into num_targets (1..8) output/lse buffers instead of
 * one: out_targets[k] / lse_targets[k] are HOST arrays of device pointers,
 * each already offset to where this call's heads belong, all with the given
 * strides.  Replaces the gather step of head-parallel decoding: with the
 * targets set to every GPU's symmetric output buffer (peer pointers over
 * NVLink, plain stores, no multicast), each rank computes its head slice and
 * writes it into every rank's full [T, H_total, 512] output, so the separate
 * all-gather (and its pack/unpack) disappears.  The caller orders the stores
 * with its own barrier after the call (the library does not synchronise
 * ranks).  No counterpart in the reference, whose decode runs on one GPU
 * (solution/triton/kernel.py:138-182 is the single-GPU operator this splits).
 */
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
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * dsa_sparse_attention_scatter_sync -- dsa_sparse_attention_scatter followed by
 * the cross-GPU barrier of dsa_peer_barrier, run inside the operator: the last
 * CTA to finish in the grid that stores last announces this rank's next epoch
 * to every rank (release stores at system scope, after all of the call's
 * stores, peer stores included) and waits, bounded, until every rank has
 * announced it.  When it completes on the stream, every rank's stores of this
 * step are visible in every target buffer.  flags[q] is rank q's flag buffer
 * (>= 10 int32, zeroed, from dsa_peer_alloc) as mapped in this process; the
 * same buffers serve dsa_peer_barrier, and the two can be mixed as long as
 * every rank issues the same sequence.  A timed-out wait sets
 * DSA_DEVERR_TIMEOUT in the workspace's error word.  No counterpart in the
 * single-GPU reference.
 */
int dsa_sparse_attention_scatter_sync(
    const void* q_nope, int64_t q_nope_stride_token, int64_t q_nope_stride_head, const void* q_pe,
    int64_t q_pe_stride_token, int64_t q_pe_stride_head, const void* ckv_cache, int64_t ckv_stride_page,
    int64_t ckv_stride_row, const void* kpe_cache, int64_t kpe_stride_page, int64_t kpe_stride_row,
    const int32_t* sparse_indices, int64_t indices_stride_token, int64_t num_tokens, int64_t num_heads,
    int64_t num_pages, int64_t page_size, int64_t topk, float sm_scale, void* const* out_targets,
    int64_t out_stride_token, int64_t out_stride_head, float* const* lse_targets,
    int64_t lse_stride_token, int64_t lse_stride_head, int num_targets, int* const* flags, int rank,
    int world, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Peer buffers and the cross-GPU barrier used with dsa_sparse_attention_scatter
 * (one process per GPU on one node; no counterpart in the single-GPU reference).
 *   dsa_peer_alloc  -- cudaMalloc `bytes` (zeroed) and export a CUDA IPC handle
 *                      (DSA_IPC_HANDLE_BYTES bytes written to ipc_handle);
 *   dsa_peer_open   -- map another process's buffer from its handle;
 *   dsa_peer_close / dsa_peer_free -- undo open / alloc;
 *   dsa_peer_barrier -- one launch on `stream`: rank `rank` of `world` (<= 8)
 *                      announces its next epoch to every rank and waits until
 *                      all have announced it.  flags[q] is rank q's flag
 *                      buffer (>= 9 int32, zeroed, from dsa_peer_alloc) as
 *                      mapped in this process.  Stores issued before the
 *                      barrier on the stream are visible to every rank after
 *                      it.  Waits are bounded (about 2 s); a timeout sets
 *                      DSA_DEVERR_TIMEOUT in *device_error (if not NULL).
 */
#define DSA_IPC_HANDLE_BYTES 64
int dsa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int dsa_peer_open(const void* ipc_handle, void** ptr);
int dsa_peer_close(void* ptr);
int dsa_peer_free(void* ptr);
int dsa_peer_barrier(int* const* flags, int rank, int world, int* device_error, void* stream);

/*
 * dsa_sparse_attention_noalloc -- the same operation, arguments and results as
 * dsa_sparse_attention, without the workspace arguments.  This entry point has
 * no counterpart in the reference.  It exists for callers that cannot
 * allocate device memory when they call the operator: engines that reserve
 * nearly all free HBM for the KV cache at start-up and pass every later
 * allocation through their own pool, and plugin hosts that hand an operator
 * only its inputs and outputs, with no workspace and no allocator.  The
 * scratch lives in a static device array of the library (about 20 MiB per
 * device, held until the process exits).  Under CUDA's default lazy module
 * loading that array takes its device memory at the first call on a device,
 * so make a first (warm-up) call before the engine reserves its memory, or
 * set CUDA_MODULE_LOADING=EAGER.  Limit: the split-K partials of at most 320
 * CTAs, which every default launch plan on a B200 (at most 296 CTAs) fits;
 * a plan forced larger through dsa_set_options returns DSA_ERR_UNSUPPORTED
 * without launching.  The first call on a device also looks up the array's
 * address (do it before any stream capture).  All calls on a device share the
 * array: calls that overlap on the GPU race and must be serialised by the
 * caller.  Device errors accumulate in the array's error word until
 * dsa_sparse_attention_noalloc_read_error reads it.  No cudaMalloc/cudaFree
 * is called.
 */
int dsa_sparse_attention_noalloc(const void* q_nope, int64_t q_nope_stride_token,
                                 int64_t q_nope_stride_head, const void* q_pe,
                                 int64_t q_pe_stride_token, int64_t q_pe_stride_head,
                                 const void* ckv_cache, int64_t ckv_stride_page,
                                 int64_t ckv_stride_row, const void* kpe_cache,
                                 int64_t kpe_stride_page, int64_t kpe_stride_row,
                                 const int32_t* sparse_indices, int64_t indices_stride_token,
                                 int64_t num_tokens, int64_t num_heads, int64_t num_pages,
                                 int64_t page_size, int64_t topk, float sm_scale, void* output,
                                 int64_t out_stride_token, int64_t out_stride_head, float* lse,
                                 int64_t lse_stride_token, int64_t lse_stride_head, void* stream);

/*
 * Read (and, with clear != 0, reset) the DSA_DEVERR_* bits that calls of
 * dsa_sparse_attention_noalloc on the current device have raised since the
 * last clear.  Synchronises the stream.  No counterpart in the reference.
 */
int dsa_sparse_attention_noalloc_read_error(int clear, int* bits, void* stream);

/*
 * FP8 lightning-indexer scores.  Replaces indexer_kernel
 * (solution/triton/indexer_kernel.py:4-287, launched at :386-409):
 *   scores[b*scores_stride + t] = scale(t) * sum_h w[b,h] * ReLU(q[b,h,:] . k8(t))
 * for every token position t < seq_lens[b] (other entries are not written).
 *   q_fp8        [batch, 64, 128] e4m3, contiguous, 16-byte aligned
 *   k_cache_fp8  key row of (page, slot) at k_cache_fp8 + page*k_page_stride
 *                + slot*128 bytes (e4m3), 64 slots per page
 *   k_scale      fp32 scale of (page, slot) at k_scale + page*scale_page_stride
 *                + slot*4 bytes (split [P,64] tensor or page-packed layout)
 *   weights      [batch, 64] fp32; block_table [batch, *] int32 logical page ->
 *                physical page; seq_lens [batch] int32 (device pointers)
 * num_heads must be 64 and head_dim 128.  max_len bounds every seq_len (e.g.
 * block-table width * 64).  device_error (may be NULL) receives DSA_DEVERR_*
 * bits (a page id outside [0, num_pages) is flagged and its rows skipped).
 */
int dsa_indexer_scores(const void* q_fp8, const void* k_cache_fp8, int64_t k_page_stride,
                       const void* k_scale, int64_t scale_page_stride, const float* weights,
                       const int32_t* block_table, int64_t block_table_stride,
                       const int32_t* seq_lens, int64_t batch, int64_t num_heads, int64_t head_dim,
                       int64_t num_pages, int64_t max_len, float* scores, int64_t scores_stride,
                       int* device_error, void* stream);

/*
 * Exact top-k of each request's scores.  Replaces topk_kernel
 * (solution/triton/indexer_kernel.py:289-343, launched at :422-431): the
 * min(k, seq_lens[b]) positions with the largest scores (ties toward the
 * lower position), then -1.  order 0: emitted in descending score, ties by
 * ascending position; order 1: emitted in ascending position (no sort; the
 * attention operator does not depend on the order, and the reference's
 * replace-the-minimum loop leaves it unspecified).  positions[b, j] is the
 * token position inside the request; slots[b, j] (optional, NULL to skip) is
 * the flat physical slot block_table[b, pos/64]*64 + pos%64 that
 * dsa_sparse_attention consumes.  1 <= k <= 2048.
 */
int dsa_topk_select(const float* scores, int64_t scores_stride, const int32_t* seq_lens,
                    const int32_t* block_table, int64_t block_table_stride, int64_t batch, int64_t k,
                    int32_t* positions, int32_t* slots, int order, void* stream);

/*
 * Indexer scores followed by top-k (replaces run_indexer_and_topk,
 * solution/triton/indexer_kernel.py:345-433, without its two device-to-host
 * synchronisations).  scores_workspace holds batch*max_len floats.
 */
int dsa_indexer_topk(const void* q_fp8, const void* k_cache_fp8, int64_t k_page_stride,
                     const void* k_scale, int64_t scale_page_stride, const float* weights,
                     const int32_t* block_table, int64_t block_table_stride, const int32_t* seq_lens,
                     int64_t batch, int64_t num_heads, int64_t head_dim, int64_t num_pages,
                     int64_t max_len, int64_t k, float* scores_workspace, int32_t* positions,
                     int32_t* slots, int order, int* device_error, void* stream);

/*
 * Quantise new index keys and append them to the paged FP8 index-key cache
 * read by dsa_indexer_scores (the reference only reads this format,
 * solution/triton/indexer_kernel.py:163-201).  For token i with flat slot id
 * slot_ids[i] (page*64+slot; -1 = skip): scale = max|k|/448 (1 for an all-zero
 * row), 128 e4m3 bytes of k/scale (round to nearest even, saturating) at
 * k_cache_fp8 + page*k_page_stride + slot*128 and the fp32 scale at
 * k_scale + page*scale_page_stride + slot*4.  keys_bf16 is [num_tokens, 128].
 */
int dsa_index_cache_append(const void* keys_bf16, int64_t num_tokens, const int32_t* slot_ids,
                           void* k_cache_fp8, int64_t k_page_stride, void* k_scale,
                           int64_t scale_page_stride, int64_t num_pages, int* device_error,
                           void* stream);

/*
 * Read (and optionally clear) the device error word of a workspace.
 * Synchronises the stream.  *bits receives DSA_DEVERR_* flags.
 */
int dsa_read_device_error(const void* workspace, int clear, int* bits, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
