/*
 * oracle.c — multi-threaded CPU port of the reference's decode attention math.
 * TEST INFRASTRUCTURE: used only as the parity checker's fast twin and as bench.py's
 * timed CPU baseline ("port"); never linked into the product library.
 *
 * oracle_paged_attn : speech_serving/models.py:140-164 over the paged gather of
 *                     speech_serving/phase_aware_scheduler.py:617-622 (one query per
 *                     sequence, fp32 arithmetic, max-subtracted softmax);
 *                     context <= 0 gives zeros like scripts/evaluate_paging_variants.py:78-80.
 * oracle_cross_attn : speech_serving/models.py:184-202 with the bool length mask.
 * Inputs are fp32, fp16 or bf16 (dtype 0/1/2), decoded to fp32 by bit manipulation.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float bf16_to_f32(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline void load_row(const void* base, size_t off, int D, int dtype, float* dst) {
  if (dtype == 0) {
    memcpy(dst, (const float*)base + off, (size_t)D * 4);
  } else if (dtype == 1) {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int d = 0; d < D; ++d) dst[d] = f16_to_f32(p[d]);
  } else {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int d = 0; d < D; ++d) dst[d] = bf16_to_f32(p[d]);
  }
}

/* softmax(q k^T scale) v over T rows given by row offsets computed by `row_off`. */
typedef size_t (*row_fn)(const void* ctx, int t);

static void attend(const float* q, const void* k, const void* v, int T, int D, float scale, int dtype,
                   row_fn row_off, const void* ctx, float* scores, float* krow, float* out) {
  float m = -INFINITY;
  for (int t = 0; t < T; ++t) {
    load_row(k, row_off(ctx, t), D, dtype, krow);
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += q[d] * krow[d];
    s *= scale;
    scores[t] = s;
    if (s > m) m = s;
  }
  float l = 0.f;
  for (int t = 0; t < T; ++t) {
    scores[t] = expf(scores[t] - m);
    l += scores[t];
  }
  for (int d = 0; d < D; ++d) out[d] = 0.f;
  for (int t = 0; t < T; ++t) {
    load_row(v, row_off(ctx, t), D, dtype, krow);
    const float p = scores[t] / l;
    for (int d = 0; d < D; ++d) out[d] += p * krow[d];
  }
}

typedef struct {
  const int* table;
  int bs, H, D, h;
} paged_ctx;

static size_t paged_row(const void* c, int t) {
  const paged_ctx* p = (const paged_ctx*)c;
  const size_t blk = (size_t)p->table[t / p->bs];
  return ((blk * p->bs + (size_t)(t % p->bs)) * p->H + p->h) * p->D;
}

typedef struct {
  size_t base;
  int D;
} cross_ctx;

static size_t cross_row(const void* c, int t) {
  const cross_ctx* p = (const cross_ctx*)c;
  return p->base + (size_t)t * p->D;
}

void oracle_paged_attn(const void* q, const void* kpool, const void* vpool, const int32_t* tables,
                       const int32_t* ctx_lens, float* out, int B, int H, int D, int bs, int max_blocks,
                       float scale, int dtype, int nthreads) {
  int max_t = 1;
  for (int b = 0; b < B; ++b) if (ctx_lens[b] > max_t) max_t = ctx_lens[b];
#pragma omp parallel num_threads(nthreads)
  {
    float* scores = (float*)malloc(sizeof(float) * (size_t)max_t);
    float* row = (float*)malloc(sizeof(float) * (size_t)D);
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(dynamic, 4)
    for (int bh = 0; bh < B * H; ++bh) {
      const int b = bh / H, h = bh % H;
      float* o = out + (size_t)bh * D;
      const int T = ctx_lens[b];
      if (T <= 0) {
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        continue;
      }
      load_row(q, (size_t)bh * D, D, dtype, qf);
      paged_ctx c = {tables + (size_t)b * max_blocks, bs, H, D, h};
      attend(qf, kpool, vpool, T, D, scale, dtype, paged_row, &c, scores, row, o);
    }
    free(scores);
    free(row);
    free(qf);
  }
}

void oracle_cross_attn(const void* q, const void* k, const void* v, const int32_t* valid, float* out, int B,
                       int H, int D, int T_max, long long batch_stride, long long head_stride, float scale,
                       int dtype, int nthreads) {
#pragma omp parallel num_threads(nthreads)
  {
    float* scores = (float*)malloc(sizeof(float) * (size_t)T_max);
    float* row = (float*)malloc(sizeof(float) * (size_t)D);
    float* qf = (float*)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(dynamic, 4)
    for (int bh = 0; bh < B * H; ++bh) {
      const int b = bh / H, h = bh % H;
      float* o = out + (size_t)bh * D;
      int T = valid[b] < T_max ? valid[b] : T_max;
      if (T <= 0) {
        for (int d = 0; d < D; ++d) o[d] = 0.f;
        continue;
      }
      load_row(q, (size_t)bh * D, D, dtype, qf);
      cross_ctx c = {(size_t)b * batch_stride + (size_t)h * head_stride, D};
      attend(qf, k, v, T, D, scale, dtype, cross_row, &c, scores, row, o);
    }
    free(scores);
    free(row);
    free(qf);
  }
}
