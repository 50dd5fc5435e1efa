/*
 * dsa_oracle.c -- CPU restatement of the reference's DSA sparse-attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in flashinfer_repo_b200/csrc.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it; the product path never does.
 *
 * Pinning status:
 *   - Attention (oracle_dsa_attention): restates the reference golden
 *     function `run` (solution/triton/indexer_kernel.py:436-497) and is pinned
 *     against fixtures produced by that function (tests/golden/make_golden.py).
 *   - Indexer scores + top-k (oracle_indexer_scores / oracle_topk): the
 *     reference has no golden function, test or published vector for this
 *     step, so this part is PARITY UNPINNED.  It restates the scoring formula
 *     of solution/triton/indexer_kernel.py:258-275 (sum over heads of
 *     w_h * ReLU(q_h . k_t), keys dequantised by a per-token scale,
 *     :186-201) with an explicit total order for selection: descending score,
 *     ties broken toward the lower token position (the reference's
 *     topk_kernel, :289-343, leaves tie order unspecified).
 *
 * All arithmetic is done in double and rounded once to fp32 (scores, lse) or
 * bf16 (attention output, round-to-nearest-even), which is at least as
 * accurate as the reference's fp32 torch math.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* OCP FP8 E4M3 ("fn" variant): 1 sign, 4 exponent bits (bias 7), 3 mantissa
 * bits, no infinities, S.1111.111 is NaN.  Decoded from the format definition. */
static inline float e4m3_to_f32(uint8_t v) {
  int s = v >> 7, e = (v >> 3) & 0xf, m = v & 7;
  float r;
  if (e == 0xf && m == 7) return NAN;
  if (e == 0) r = ldexpf((float)m, -9);           /* subnormal: m/8 * 2^-6 */
  else r = ldexpf((float)(8 + m), e - 10);        /* (1 + m/8) * 2^(e-7) */
  return s ? -r : r;
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#else
  (void)nthreads;
#endif
}

/*
 * oracle_dsa_attention -- restates `run` (indexer_kernel.py:437-497).
 *
 * Layouts (all contiguous):
 *   q_nope [T,16,512] bf16, q_pe [T,16,64] bf16,
 *   ckv [P,64,512] bf16, kpe [P,64,64] bf16 (flattened to P*64 slots, :458-459),
 *   idx [T,topk] int32 flat slot ids, -1 = padding (:469-471),
 *   out [T,16,512] bf16, lse [T,16] fp32 base-2 (:490).
 * A token with no valid index keeps out = 0 and lse = -inf (:473-475).
 * Returns 0, or -1 if an index is outside [-1, P*64).
 */
int oracle_dsa_attention(const uint16_t* q_nope, const uint16_t* q_pe, const uint16_t* ckv,
                         const uint16_t* kpe, const int32_t* idx, int64_t T, int64_t P,
                         int64_t topk, float sm_scale, uint16_t* out, float* lse, int nthreads) {
  const int H = 16, DC = 512, DP = 64;
  const int64_t slots = P * 64;
  int bad = 0;
  for (int64_t i = 0; i < T * topk; ++i)
    if (idx[i] < -1 || idx[i] >= slots) bad = 1;
  if (bad) return -1;
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t t = 0; t < T; ++t) {
    const int32_t* it = idx + t * topk;
    double* logit = (double*)malloc(sizeof(double) * (size_t)topk * H);
    int32_t* rows = (int32_t*)malloc(sizeof(int32_t) * (size_t)topk);
    int nv = 0;
    for (int64_t j = 0; j < topk; ++j)
      if (it[j] != -1) rows[nv++] = it[j];
    for (int h = 0; h < H; ++h) {
      uint16_t* o = out + (t * H + h) * DC;
      if (nv == 0) {
        memset(o, 0, DC * sizeof(uint16_t));
        lse[t * H + h] = -INFINITY;
        continue;
      }
      const uint16_t* qn = q_nope + (t * H + h) * DC;
      const uint16_t* qp = q_pe + (t * H + h) * DP;
      double mx = -INFINITY;
      for (int j = 0; j < nv; ++j) {
        const uint16_t* kc = ckv + (int64_t)rows[j] * DC;
        const uint16_t* kp = kpe + (int64_t)rows[j] * DP;
        double s = 0.0;
        for (int d = 0; d < DC; ++d) s += (double)bf16_to_f32(qn[d]) * bf16_to_f32(kc[d]);
        for (int d = 0; d < DP; ++d) s += (double)bf16_to_f32(qp[d]) * bf16_to_f32(kp[d]);
        s *= (double)sm_scale;
        logit[j] = s;
        if (s > mx) mx = s;
      }
      double l = 0.0;
      for (int j = 0; j < nv; ++j) {
        logit[j] = exp(logit[j] - mx);
        l += logit[j];
      }
      lse[t * H + h] = (float)((mx + log(l)) / log(2.0));
      double acc[512];
      for (int d = 0; d < DC; ++d) acc[d] = 0.0;
      for (int j = 0; j < nv; ++j) {
        const uint16_t* kc = ckv + (int64_t)rows[j] * DC;
        double p = logit[j] / l;
        for (int d = 0; d < DC; ++d) acc[d] += p * bf16_to_f32(kc[d]);
      }
      for (int d = 0; d < DC; ++d) o[d] = f32_to_bf16((float)acc[d]);
    }
    free(logit);
    free(rows);
  }
  return 0;
}

/*
 * oracle_indexer_scores -- FP8 lightning-indexer scores (PARITY UNPINNED).
 *
 * For request b and token position t < seq_lens[b]:
 *   page = block_table[b, t/64], row = page*64 + t%64
 *   logit_h = sum_d q[b,h,d] * k[row,d]                  (fp8 values, exact products)
 *   score   = scale[row] * sum_h w[b,h] * max(0, logit_h)
 * Key bytes of `row` live at k_cache + page*k_page_stride + (t%64)*128 and its
 * fp32 scale at scale_base + page*s_page_stride + (t%64)*4 (byte strides), so
 * both the split layout (keys [P,64,128] + scales [P,64]) and the page-packed
 * layout (per page 64*128 key bytes followed by 64 fp32 scales) are covered.
 * scores is [B, max_len] fp32; entries t >= seq_lens[b] are set to -inf.
 * Reference: indexer_kernel.py:120-201 (page mapping, dequant), :258-275 (sum).
 */
int oracle_indexer_scores(const uint8_t* q, const uint8_t* k_cache, int64_t k_page_stride,
                          const uint8_t* scale_base, int64_t s_page_stride, const float* w,
                          const int32_t* block_table, int64_t bt_stride, const int32_t* seq_lens,
                          int64_t B, int64_t H, int64_t max_len, float* scores, int nthreads) {
  const int D = 128;
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t b = 0; b < B; ++b) {
    float qf[64 * 128];
    for (int64_t i = 0; i < H * D; ++i) qf[i] = e4m3_to_f32(q[b * H * D + i]);
    int64_t len = seq_lens[b];
    for (int64_t t = 0; t < max_len; ++t) {
      if (t >= len) {
        scores[b * max_len + t] = -INFINITY;
        continue;
      }
      int64_t page = block_table[b * bt_stride + t / 64];
      const uint8_t* kr = k_cache + page * k_page_stride + (t % 64) * D;
      float sc;
      memcpy(&sc, scale_base + page * s_page_stride + (t % 64) * 4, 4);
      float kf[128];
      for (int d = 0; d < D; ++d) kf[d] = e4m3_to_f32(kr[d]);
      double acc = 0.0;
      for (int64_t h = 0; h < H; ++h) {
        double lg = 0.0;
        for (int d = 0; d < D; ++d) lg += (double)qf[h * D + d] * kf[d];
        if (lg > 0) acc += (double)w[b * H + h] * lg;
      }
      scores[b * max_len + t] = (float)(acc * (double)sc);
    }
  }
  return 0;
}

typedef struct {
  float s;
  int32_t i;
} scored_t;

static int cmp_scored(const void* a, const void* b) {
  const scored_t* x = (const scored_t*)a;
  const scored_t* y = (const scored_t*)b;
  if (x->s > y->s) return -1;
  if (x->s < y->s) return 1;
  return (x->i < y->i) ? -1 : (x->i > y->i);
}

/*
 * oracle_topk -- exact top-k with a total order (PARITY UNPINNED).
 * For each request: the min(k, seq_len) positions with the largest scores,
 * emitted in descending score, ties toward the lower position; remaining
 * entries -1.  positions[b,j] is the token position inside the request;
 * slots[b,j] = block_table[b, pos/64]*64 + pos%64 is the flat physical slot id
 * that the attention operator consumes.  Replaces topk_kernel
 * (indexer_kernel.py:289-343), whose replace-the-min loop duplicates ids on
 * ties and returns logical concatenated ids (:317).
 */
int oracle_topk(const float* scores, int64_t B, int64_t max_len, const int32_t* seq_lens,
                const int32_t* block_table, int64_t bt_stride, int64_t k, int32_t* positions,
                int32_t* slots, int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t b = 0; b < B; ++b) {
    int64_t len = seq_lens[b];
    scored_t* v = (scored_t*)malloc(sizeof(scored_t) * (size_t)(len > 0 ? len : 1));
    for (int64_t t = 0; t < len; ++t) {
      v[t].s = scores[b * max_len + t];
      v[t].i = (int32_t)t;
    }
    qsort(v, (size_t)len, sizeof(scored_t), cmp_scored);
    for (int64_t j = 0; j < k; ++j) {
      if (j < len) {
        int32_t p = v[j].i;
        positions[b * k + j] = p;
        slots[b * k + j] = block_table[b * bt_stride + p / 64] * 64 + p % 64;
      } else {
        positions[b * k + j] = -1;
        slots[b * k + j] = -1;
      }
    }
    free(v);
  }
  return 0;
}
