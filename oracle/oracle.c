/*
 * oracle.c -- CPU restatement of the open-cuda reference's hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libopencuda_cuda.so and the
 * timed CPU baseline.  Nothing in the product path links or calls it.
 *
 * Each routine cites the reference loop it restates (paths relative to the
 * reference workspace).  Arithmetic is f32 in the reference's order; build
 * with -ffp-contract=off so that no a*b+c is fused (Rust never fuses).
 * Math functions: the reference's f32::exp / f64::tanh / f32::sqrt /
 * f32::powf lower to the platform libm, as expf / tanh / sqrtf / powf here.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* A persistent worker pool: the rayon global pool the reference runs its   */
/* parallel loops on (cpu:191 `into_par_iter` over blocks).                 */
/* ------------------------------------------------------------------------ */
typedef void (*task_fn)(void *ctx, size_t begin, size_t end);

static struct {
  pthread_mutex_t mu;
  pthread_cond_t cv_start, cv_done;
  int nthreads;    /* workers incl. the caller */
  int started;     /* workers spawned */
  unsigned long gen;
  task_fn fn;
  void *ctx;
  size_t ntasks, chunk;
  atomic_size_t next;
  int active;      /* workers still running the current job */
} pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER,
          PTHREAD_COND_INITIALIZER, 0, 0, 0, 0, 0, 0, 0, 0, 0};

static int default_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

void ocr_set_threads(int n) {
  pthread_mutex_lock(&pool.mu);
  if (pool.started == 0) pool.nthreads = n > 0 ? n : default_threads();
  pthread_mutex_unlock(&pool.mu);
}

int ocr_get_threads(void) {
  if (pool.nthreads == 0) ocr_set_threads(0);
  return pool.nthreads;
}

static void run_chunks(void) {
  for (;;) {
    size_t i = atomic_fetch_add(&pool.next, 1);
    size_t b = i * pool.chunk;
    if (b >= pool.ntasks) break;
    size_t e = b + pool.chunk;
    if (e > pool.ntasks) e = pool.ntasks;
    pool.fn(pool.ctx, b, e);
  }
}

static void *worker_main(void *arg) {
  (void)arg;
  unsigned long seen = 0;
  pthread_mutex_lock(&pool.mu);
  for (;;) {
    while (pool.gen == seen) pthread_cond_wait(&pool.cv_start, &pool.mu);
    seen = pool.gen;
    pthread_mutex_unlock(&pool.mu);
    run_chunks();
    pthread_mutex_lock(&pool.mu);
    if (--pool.active == 0) pthread_cond_signal(&pool.cv_done);
  }
  return NULL;
}

/* Runs fn over [0, ntasks) in chunks of `chunk` tasks on all workers. */
static void parallel_for(size_t ntasks, size_t chunk, task_fn fn, void *ctx) {
  if (ntasks == 0) return;
  if (chunk == 0) chunk = 1;
  int nt = ocr_get_threads();
  if (nt <= 1 || ntasks <= chunk) {
    fn(ctx, 0, ntasks);
    return;
  }
  pthread_mutex_lock(&pool.mu);
  while (pool.started < nt - 1) {
    pthread_t t;
    pthread_attr_t at;
    pthread_attr_init(&at);
    pthread_attr_setdetachstate(&at, PTHREAD_CREATE_DETACHED);
    pthread_create(&t, &at, worker_main, NULL);
    pthread_attr_destroy(&at);
    pool.started++;
  }
  pool.fn = fn;
  pool.ctx = ctx;
  pool.ntasks = ntasks;
  pool.chunk = chunk;
  atomic_store(&pool.next, 0);
  pool.active = pool.started;
  pool.gen++;
  pthread_cond_broadcast(&pool.cv_start);
  pthread_mutex_unlock(&pool.mu);
  run_chunks();
  pthread_mutex_lock(&pool.mu);
  while (pool.active > 0) pthread_cond_wait(&pool.cv_done, &pool.mu);
  pthread_mutex_unlock(&pool.mu);
}

/* ------------------------------------------------------------------------ */
/* GEMM: blas:148-237 (launch_naive_gemm) and blas:260-295 (sgemm).         */
/* ------------------------------------------------------------------------ */
typedef struct {
  size_t m, k, n;
  float alpha, beta;
  const float *a, *b;
  float *c;
  int tb;
} gemm_ctx;

/* blas:183-216: one output element per thread; acc += a*b ascending k;
 * c = alpha*acc + beta*old_c.  Tasks are 256-element blocks (blas:218)
 * spread over the pool (cpu:191), threads inside a block run serially. */
static void gemm_faithful_blocks(void *p, size_t b0, size_t b1) {
  gemm_ctx *g = (gemm_ctx *)p;
  size_t total = g->m * g->n;
  for (size_t blk = b0; blk < b1; blk++) {
    for (size_t t = 0; t < 256; t++) {
      size_t idx = blk * 256 + t;
      if (idx >= total) break;
      size_t row = idx / g->n, col = idx % g->n;
      float acc = 0.0f;
      for (size_t kk = 0; kk < g->k; kk++) {
        float bv = g->tb ? g->b[col * g->k + kk] : g->b[kk * g->n + col];
        acc += g->a[row * g->k + kk] * bv;
      }
      float old = g->c[idx];
      g->c[idx] = g->alpha * acc + g->beta * old;
    }
  }
}

/* Same per-element expression, blocked over 64 columns so the compiler can
 * keep 64 independent accumulators (each still summed in ascending k).
 * Task t covers row t / ncb, column block t % ncb. */
#define GB 64
static void gemm_fast_tiles(void *p, size_t t0, size_t t1) {
  gemm_ctx *g = (gemm_ctx *)p;
  size_t ncb = (g->n + GB - 1) / GB;
  float acc[GB];
  for (size_t t = t0; t < t1; t++) {
    size_t row = t / ncb, c0 = (t % ncb) * GB;
    const float *arow = g->a + row * g->k;
    size_t nc = g->n - c0 < GB ? g->n - c0 : GB;
    for (size_t j = 0; j < GB; j++) acc[j] = 0.0f;
    if (!g->tb) {
      for (size_t kk = 0; kk < g->k; kk++) {
        float av = arow[kk];
        const float *brow = g->b + kk * g->n + c0;
        if (nc == GB) {
          for (size_t j = 0; j < GB; j++) acc[j] += av * brow[j];
        } else {
          for (size_t j = 0; j < nc; j++) acc[j] += av * brow[j];
        }
      }
    } else {
      for (size_t j = 0; j < nc; j++) {
        const float *bcol = g->b + (c0 + j) * g->k;
        float s = 0.0f;
        for (size_t kk = 0; kk < g->k; kk++) s += arow[kk] * bcol[kk];
        acc[j] = s;
      }
    }
    float *crow = g->c + row * g->n + c0;
    for (size_t j = 0; j < nc; j++) crow[j] = g->alpha * acc[j] + g->beta * crow[j];
  }
}

int ocr_sgemm(size_t m, size_t k, size_t n, float alpha, const float *a,
              const float *b, int transpose_b, float beta, float *c,
              int faithful) {
  if (!a || !b || !c) return 1;
  gemm_ctx g = {m, k, n, alpha, beta, a, b, c, transpose_b};
  if (faithful) {
    /* blas:174-181: ScopedAlloc for A, B, C and host->device copies (the
     * CPU backend's "device" memory is host heap, cpu:80-125), then the
     * launch, then the device->host copy of C and the frees (blas:233). */
    size_t ba = m * k * sizeof(float), bb = k * n * sizeof(float),
           bc = m * n * sizeof(float);
    float *da = (float *)aligned_alloc(16, ba ? (ba + 15) & ~15ul : 16);
    float *db = (float *)aligned_alloc(16, bb ? (bb + 15) & ~15ul : 16);
    float *dc = (float *)aligned_alloc(16, bc ? (bc + 15) & ~15ul : 16);
    if (!da || !db || !dc) {
      free(da); free(db); free(dc);
      return 2;
    }
    memcpy(da, a, ba);
    memcpy(db, b, bb);
    memcpy(dc, c, bc);
    gemm_ctx gd = {m, k, n, alpha, beta, da, db, dc, transpose_b};
    size_t nblk = (m * n + 255) / 256;
    parallel_for(nblk, 1, gemm_faithful_blocks, &gd);
    memcpy(c, dc, bc);
    free(da); free(db); free(dc);
    return 0;
  }
  parallel_for(m * ((n + GB - 1) / GB), 4, gemm_fast_tiles, &g);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Quantization: blas:777-1012.                                             */
/* ------------------------------------------------------------------------ */

/* blas:797-809: per contiguous group, max_abs = fold(0, max(|x|)); scale =
 * max_abs==0 ? 0 : max_abs / q_max. */
void ocr_group_scales(const float *in, size_t len, size_t group, float qmax,
                      float *scales) {
  size_t ng = (len + group - 1) / group;
  for (size_t gi = 0; gi < ng; gi++) {
    size_t b = gi * group, e = b + group < len ? b + group : len;
    float mx = 0.0f;
    for (size_t i = b; i < e; i++) mx = fmaxf(mx, fabsf(in[i]));
    scales[gi] = mx == 0.0f ? 0.0f : mx / qmax;
  }
}

/* blas:834-852: q = scale==0 ? 0 : clamp(round(x/scale), qmin, qmax) as i8.
 * Rust f32::round rounds half away from zero, as C roundf does. */
void ocr_quantize_symmetric(const float *in, size_t len, const float *scales,
                            size_t group, float qmin, float qmax,
                            int8_t *out) {
  for (size_t i = 0; i < len; i++) {
    float s = scales[i / group];
    float q;
    if (s == 0.0f) {
      q = 0.0f;
    } else {
      q = roundf(in[i] / s);
      /* Rust f32::clamp: max(min) ordering; NaN stays NaN -> `as i8` = 0 */
      if (q < qmin) q = qmin;
      if (q > qmax) q = qmax;
    }
    out[i] = isnan(q) ? 0 : (int8_t)q;
  }
}

/* blas:867-872 validate_quantize_args */
static int validate_quant(size_t len, size_t group) {
  if (len == 0) return 1;
  if (group == 0) return 1;
  return 0;
}

/* blas:935-940 */
int ocr_quantize_int8(const float *in, size_t len, size_t group, int8_t *data,
                      float *scales) {
  if (validate_quant(len, group)) return 1;
  ocr_group_scales(in, len, group, 127.0f, scales);
  ocr_quantize_symmetric(in, len, scales, group, -127.0f, 127.0f, data);
  return 0;
}

/* blas:901-919: even index -> low nibble, odd -> high nibble, nibble=q+8,
 * odd length leaves the last high nibble 0. */
int ocr_quantize_int4(const float *in, size_t len, size_t group,
                      uint8_t *data, float *scales) {
  if (validate_quant(len, group)) return 1;
  ocr_group_scales(in, len, group, 7.0f, scales);
  int8_t *q = (int8_t *)malloc(len);
  if (!q) return 2;
  ocr_quantize_symmetric(in, len, scales, group, -7.0f, 7.0f, q);
  memset(data, 0, (len + 1) / 2);
  for (size_t i = 0; i < len; i++) {
    uint8_t nib = (uint8_t)(q[i] + 8) & 0x0F;
    if (i % 2 == 0)
      data[i / 2] |= nib;
    else
      data[i / 2] |= (uint8_t)(nib << 4);
  }
  free(q);
  return 0;
}

/* blas:943-945 */
void ocr_dequantize_int8(const int8_t *data, const float *scales, size_t len,
                         size_t group, float *out) {
  for (size_t i = 0; i < len; i++) out[i] = (float)data[i] * scales[i / group];
}

/* blas:922-931 */
void ocr_dequantize_int4(const uint8_t *data, const float *scales, size_t len,
                         size_t group, float *out) {
  for (size_t i = 0; i < len; i++) {
    uint8_t byte = data[i / 2];
    uint8_t nib = (i % 2 == 0) ? (byte & 0x0F) : (byte >> 4);
    int q = (int)nib - 8;
    out[i] = (float)q * scales[i / group];
  }
}

/* blas:958-989 */
int ocr_quantize_int4_awq(const float *weight, size_t rows, size_t cols,
                          const float *act_scale, size_t group, float alpha,
                          uint8_t *data, float *scales, float *awq_scale) {
  if (rows == 0 || cols == 0) return 1;
  for (size_t c = 0; c < cols; c++)
    awq_scale[c] = act_scale[c] <= 0.0f ? 1.0f : powf(act_scale[c], alpha);
  float *scaled = (float *)malloc(rows * cols * sizeof(float));
  if (!scaled) return 2;
  for (size_t r = 0; r < rows; r++)
    for (size_t c = 0; c < cols; c++)
      scaled[r * cols + c] = weight[r * cols + c] * awq_scale[c];
  int rc = ocr_quantize_int4(scaled, rows * cols, group, data, scales);
  free(scaled);
  return rc;
}

/* blas:993-1003 */
void ocr_dequantize_int4_awq(const uint8_t *data, const float *scales,
                             size_t rows, size_t cols, size_t group,
                             const float *awq_scale, float *out) {
  ocr_dequantize_int4(data, scales, rows * cols, group, out);
  for (size_t r = 0; r < rows; r++)
    for (size_t c = 0; c < cols; c++) {
      float s = awq_scale[c];
      out[r * cols + c] = s == 0.0f ? 0.0f : out[r * cols + c] / s;
    }
}

/* ------------------------------------------------------------------------ */
/* Attention: blas:411-678.                                                 */
/* ------------------------------------------------------------------------ */

/* blas:545-562 */
static void softmax_row(const float *in, float *out, size_t cols) {
  float mx = -INFINITY;
  for (size_t j = 0; j < cols; j++) mx = fmaxf(mx, in[j]);
  float sum = 0.0f;
  for (size_t j = 0; j < cols; j++) {
    float e = expf(in[j] - mx);
    out[j] = e;
    sum += e;
  }
  if (sum > 0.0f)
    for (size_t j = 0; j < cols; j++) out[j] /= sum;
}

void ocr_row_softmax(const float *scores, size_t rows, size_t cols,
                     float *probs) {
  for (size_t r = 0; r < rows; r++)
    softmax_row(scores + r * cols, probs + r * cols, cols);
}

/* blas:475-540 with the CpuNaive GEMM: scores via launch_naive_gemm
 * (transpose_b, alpha = 1/sqrt(d), beta 0), row softmax, then P.V via sgemm.
 */
int ocr_sdpa(const float *q, const float *k, const float *v, size_t seq,
             size_t d, float *out) {
  float scale = 1.0f / sqrtf((float)d);
  float *scores = (float *)calloc(seq * seq, sizeof(float));
  float *probs = (float *)calloc(seq * seq, sizeof(float));
  if (!scores || !probs) {
    free(scores); free(probs);
    return 2;
  }
  ocr_sgemm(seq, d, seq, scale, q, k, 1, 0.0f, scores, 0);
  ocr_row_softmax(scores, seq, seq, probs);
  memset(out, 0, seq * d * sizeof(float));
  ocr_sgemm(seq, seq, d, 1.0f, probs, v, 0, 0.0f, out, 0);
  free(scores);
  free(probs);
  return 0;
}

/* blas:618-675: one query row, K/V blocks of `block` rows, online softmax. */
static void flash_row(const float *qrow, const float *k, const float *v,
                      size_t seq, size_t d, size_t block, float *orow,
                      float *acc, float *bscore) {
  float scale = 1.0f / sqrtf((float)d);
  float m_i = -INFINITY, l_i = 0.0f;
  for (size_t j = 0; j < d; j++) acc[j] = 0.0f;
  for (size_t kv0 = 0; kv0 < seq; kv0 += block) {
    size_t kv1 = kv0 + block < seq ? kv0 + block : seq;
    size_t bc = kv1 - kv0;
    for (size_t j = 0; j < bc; j++) {
      const float *krow = k + (kv0 + j) * d;
      float dot = -0.0f; /* Rust f32 Sum starts from -0.0 */
      for (size_t t = 0; t < d; t++) dot += qrow[t] * krow[t];
      bscore[j] = dot * scale;
    }
    float bmax = -INFINITY;
    for (size_t j = 0; j < bc; j++) bmax = fmaxf(bmax, bscore[j]);
    float new_m = fmaxf(m_i, bmax);
    float corr = (m_i == -INFINITY) ? 0.0f : expf(m_i - new_m);
    l_i *= corr;
    for (size_t t = 0; t < d; t++) acc[t] *= corr;
    float bl = 0.0f;
    for (size_t j = 0; j < bc; j++) {
      float p = expf(bscore[j] - new_m);
      bl += p;
      const float *vrow = v + (kv0 + j) * d;
      for (size_t t = 0; t < d; t++) acc[t] += p * vrow[t];
    }
    l_i += bl;
    m_i = new_m;
  }
  if (l_i > 0.0f)
    for (size_t t = 0; t < d; t++) orow[t] = acc[t] / l_i;
}

typedef struct {
  const float *q, *k, *v;
  size_t seq, d, block;
  float *out;
} flash_ctx;

static void flash_rows(void *p, size_t r0, size_t r1) {
  flash_ctx *f = (flash_ctx *)p;
  float *acc = (float *)malloc(f->d * sizeof(float));
  float *bs = (float *)malloc(f->block * sizeof(float));
  for (size_t r = r0; r < r1; r++)
    flash_row(f->q + r * f->d, f->k, f->v, f->seq, f->d, f->block,
              f->out + r * f->d, acc, bs);
  free(acc);
  free(bs);
}

/* blas:589-678 */
int ocr_flash_attention(const float *q, const float *k, const float *v,
                        size_t seq, size_t d, size_t block, float *out) {
  if (block == 0) return 1;
  memset(out, 0, seq * d * sizeof(float));
  flash_ctx f = {q, k, v, seq, d, block, out};
  parallel_for(seq, 1, flash_rows, &f);
  return 0;
}

void ocr_attend_one(const float *q, const float *k, const float *v, size_t n,
                    size_t d, int flash, size_t block, float *out) {
  if (flash) {
    float *acc = (float *)malloc(d * sizeof(float));
    float *bs = (float *)malloc(block * sizeof(float));
    memset(out, 0, d * sizeof(float));
    flash_row(q, k, v, n, d, block, out, acc, bs);
    free(acc);
    free(bs);
    return;
  }
  /* SDPA row 0: scores_j = scale*acc_j + 0*0 (blas:517 via blas:200-214);
   * softmax; out_c = 1*sum_j p_j v_jc + 0*0 (blas:537). */
  float scale = 1.0f / sqrtf((float)d);
  float *s = (float *)malloc(n * sizeof(float));
  float *p = (float *)malloc(n * sizeof(float));
  for (size_t j = 0; j < n; j++) {
    float acc = 0.0f;
    for (size_t t = 0; t < d; t++) acc += q[t] * k[j * d + t];
    s[j] = scale * acc + 0.0f * 0.0f;
  }
  softmax_row(s, p, n);
  for (size_t c = 0; c < d; c++) {
    float acc = 0.0f;
    for (size_t j = 0; j < n; j++) acc += p[j] * v[j * d + c];
    out[c] = 1.0f * acc + 0.0f * 0.0f;
  }
  free(s);
  free(p);
}

/* ------------------------------------------------------------------------ */
/* MLA: blas:1045-1078 (two plain sgemm calls).                             */
/* ------------------------------------------------------------------------ */
int ocr_mla_compress_kv(size_t seq, size_t d_h, size_t d_c, const float *kv,
                        const float *down, float *latent) {
  memset(latent, 0, seq * d_c * sizeof(float));
  return ocr_sgemm(seq, d_h, d_c, 1.0f, kv, down, 0, 0.0f, latent, 0);
}

int ocr_mla_decompress_kv(size_t seq, size_t d_c, size_t d_h,
                          const float *latent, const float *up, float *out) {
  memset(out, 0, seq * d_h * sizeof(float));
  return ocr_sgemm(seq, d_c, d_h, 1.0f, latent, up, 0, 0.0f, out, 0);
}

double ocr_mla_memory_reduction_percent(size_t d_h, size_t d_c) {
  if (d_h == 0) return 0.0;
  return (1.0 - ((double)d_c / (double)d_h)) * 100.0;
}

/* ------------------------------------------------------------------------ */
/* Quantized matmul oracles (new API, composed from blas routines).         */
/* ------------------------------------------------------------------------ */

/* quantize_int8(A, group = k): groups are the rows of A (blas:797-852). */
int ocr_quantize_rows_int8(const float *a, size_t m, size_t k, int8_t *qa,
                           float *sa) {
  return ocr_quantize_int8(a, m * k, k, qa, sa);
}

typedef struct {
  size_t m, k, n, group;
  const int8_t *qa;
  const float *sa;
  const void *wq;
  const float *ws, *bias;
  float *y;
  int32_t *acc;
} qg_ctx;

static void w8a8_rows(void *p, size_t r0, size_t r1) {
  qg_ctx *g = (qg_ctx *)p;
  const int8_t *wq = (const int8_t *)g->wq;
  for (size_t r = r0; r < r1; r++) {
    const int8_t *ar = g->qa + r * g->k;
    for (size_t c = 0; c < g->n; c++) {
      const int8_t *wr = wq + c * g->k;
      int32_t acc = 0;
      for (size_t t = 0; t < g->k; t++) acc += (int32_t)ar[t] * (int32_t)wr[t];
      if (g->acc) g->acc[r * g->n + c] = acc;
      float y = (float)acc * g->sa[r];
      y = y * g->ws[c];
      g->y[r * g->n + c] = y + (g->bias ? g->bias[c] : 0.0f);
    }
  }
}

int ocr_qgemm_w8a8(size_t m, size_t k, size_t n, const float *a,
                   const int8_t *wq, const float *wscale, const float *bias,
                   float *y, int32_t *acc_out) {
  if (m == 0 || k == 0 || n == 0) return 1;
  int8_t *qa = (int8_t *)malloc(m * k);
  float *sa = (float *)malloc(m * sizeof(float));
  if (!qa || !sa) {
    free(qa); free(sa);
    return 2;
  }
  ocr_quantize_rows_int8(a, m, k, qa, sa);
  qg_ctx g = {m, k, n, k, qa, sa, wq, wscale, bias, y, acc_out};
  parallel_for(m, 1, w8a8_rows, &g);
  free(qa);
  free(sa);
  return 0;
}

static inline int nib_at(const uint8_t *row, size_t t) {
  uint8_t byte = row[t / 2];
  return (int)((t % 2 == 0) ? (byte & 0x0F) : (byte >> 4)) - 8;
}

static void w4a8_rows(void *p, size_t r0, size_t r1) {
  qg_ctx *g = (qg_ctx *)p;
  const uint8_t *wq = (const uint8_t *)g->wq;
  size_t ng = g->k / g->group;
  for (size_t r = r0; r < r1; r++) {
    const int8_t *ar = g->qa + r * g->k;
    for (size_t c = 0; c < g->n; c++) {
      /* W^T flattened [n][k], packed two per byte over the flat index
       * c*k + t (blas:909-917); k is even so rows start on a byte. */
      const uint8_t *wr = wq + (c * g->k) / 2;
      float s = 0.0f;
      for (size_t j = 0; j < ng; j++) {
        int32_t part = 0;
        for (size_t t = j * g->group; t < (j + 1) * g->group; t++)
          part += (int32_t)ar[t] * nib_at(wr, t);
        if (g->acc) g->acc[(r * g->n + c) * ng + j] = part;
        s = fmaf((float)part, g->ws[c * ng + j], s);
      }
      float y = s * g->sa[r];
      g->y[r * g->n + c] = y + (g->bias ? g->bias[c] : 0.0f);
    }
  }
}

int ocr_qgemm_w4a8(size_t m, size_t k, size_t n, size_t group, const float *a,
                   const uint8_t *wq, const float *wscale, const float *bias,
                   float *y, int32_t *acc_out) {
  if (m == 0 || k == 0 || n == 0 || group == 0 || k % group || k % 2) return 1;
  int8_t *qa = (int8_t *)malloc(m * k);
  float *sa = (float *)malloc(m * sizeof(float));
  if (!qa || !sa) {
    free(qa); free(sa);
    return 2;
  }
  ocr_quantize_rows_int8(a, m, k, qa, sa);
  qg_ctx g = {m, k, n, group, qa, sa, wq, wscale, bias, y, acc_out};
  parallel_for(m, 1, w4a8_rows, &g);
  free(qa);
  free(sa);
  return 0;
}

int ocr_qgemm_weight_only(int bits, size_t m, size_t k, size_t n,
                          size_t group, const float *a, const void *wq,
                          const float *wscale, const float *bias, float *y,
                          int faithful) {
  if (m == 0 || k == 0 || n == 0 || group == 0) return 1;
  float *deq = (float *)malloc(n * k * sizeof(float));
  float *bt = (float *)malloc(n * k * sizeof(float));
  if (!deq || !bt) {
    free(deq); free(bt);
    return 2;
  }
  if (bits == 8)
    ocr_dequantize_int8((const int8_t *)wq, wscale, n * k, group, deq);
  else
    ocr_dequantize_int4((const uint8_t *)wq, wscale, n * k, group, deq);
  /* dequantize gives W^T [n][k]; Linear::forward wants weight_t [k][n]. */
  for (size_t c = 0; c < n; c++)
    for (size_t t = 0; t < k; t++) bt[t * n + c] = deq[c * k + t];
  memset(y, 0, m * n * sizeof(float));
  int rc = ocr_sgemm(m, k, n, 1.0f, a, bt, 0, 0.0f, y, faithful);
  if (bias)
    for (size_t r = 0; r < m; r++)
      for (size_t c = 0; c < n; c++) y[r * n + c] += bias[c];
  free(deq);
  free(bt);
  return rc;
}

/* ------------------------------------------------------------------------ */
/* GPT decoder: llm:45-942.                                                 */
/* ------------------------------------------------------------------------ */

/* llm:178-206 */
uint64_t ocr_splitmix64_next(uint64_t *state) {
  *state += 0x9E3779B97F4A7C15ull;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

float ocr_splitmix64_next_f32(uint64_t *state, float scale) {
  uint32_t bits = (uint32_t)(ocr_splitmix64_next(state) >> 40);
  float unit = (float)bits / (float)(1u << 24);
  return (unit * 2.0f - 1.0f) * scale;
}

void ocr_splitmix64_fill(uint64_t seed, float scale, size_t len, float *out) {
  uint64_t st = seed;
  for (size_t i = 0; i < len; i++) out[i] = ocr_splitmix64_next_f32(&st, scale);
}

typedef struct {
  float *w, *b; /* weight_t [in][out], bias [out] */
  size_t in, out;
} linear_t;

typedef struct {
  float *down, *up; /* [head_dim][d_c], [d_c][head_dim] */
} mla_head;

typedef struct {
  float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  linear_t qkv, attn_out, fc, proj;
  mla_head *mla; /* NULL unless enabled */
} layer_t;

struct ocr_gpt {
  ocr_gpt_config cfg;
  float *wte, *wpe, *lnf_w, *lnf_b;
  layer_t *layers;
  linear_t lm_head;
  int flash, faithful;
  size_t block;
  size_t d_c;
};

static void fill_random(uint64_t *st, float *dst, size_t len, float scale) {
  for (size_t i = 0; i < len; i++) dst[i] = ocr_splitmix64_next_f32(st, scale);
}

/* llm:222-226 Linear::random: scale = 1/sqrt(in_dim), bias 0 */
static int linear_random(uint64_t *st, linear_t *l, size_t in, size_t out) {
  l->in = in;
  l->out = out;
  l->w = (float *)malloc(in * out * sizeof(float));
  l->b = (float *)calloc(out, sizeof(float));
  if (!l->w || !l->b) return 2;
  float scale = 1.0f / sqrtf((float)in);
  fill_random(st, l->w, in * out, scale);
  return 0;
}

static float *ones(size_t n) {
  float *p = (float *)malloc(n * sizeof(float));
  if (p)
    for (size_t i = 0; i < n; i++) p[i] = 1.0f;
  return p;
}

ocr_gpt *ocr_gpt_load_random(const ocr_gpt_config *cfg, uint64_t seed) {
  ocr_gpt *m = (ocr_gpt *)calloc(1, sizeof(ocr_gpt));
  if (!m) return NULL;
  m->cfg = *cfg;
  m->flash = 1;
  m->block = 64;
  size_t h = cfg->hidden_size;
  uint64_t st = seed;
  m->wte = (float *)malloc(cfg->vocab_size * h * sizeof(float));
  m->wpe = (float *)malloc(cfg->max_seq_len * h * sizeof(float));
  m->layers = (layer_t *)calloc(cfg->num_layers, sizeof(layer_t));
  if (!m->wte || !m->wpe || !m->layers) {
    ocr_gpt_free(m);
    return NULL;
  }
  fill_random(&st, m->wte, cfg->vocab_size * h, 0.02f);
  fill_random(&st, m->wpe, cfg->max_seq_len * h, 0.02f);
  for (size_t i = 0; i < cfg->num_layers; i++) {
    layer_t *L = &m->layers[i];
    /* llm:304-314: ln_1 identity, qkv, attn_out, ln_2 identity, fc, proj */
    L->ln1_w = ones(h);
    L->ln1_b = (float *)calloc(h, sizeof(float));
    L->ln2_w = ones(h);
    L->ln2_b = (float *)calloc(h, sizeof(float));
    if (linear_random(&st, &L->qkv, h, 3 * h) ||
        linear_random(&st, &L->attn_out, h, h) ||
        linear_random(&st, &L->fc, h, cfg->intermediate_size) ||
        linear_random(&st, &L->proj, cfg->intermediate_size, h)) {
      ocr_gpt_free(m);
      return NULL;
    }
  }
  m->lnf_w = ones(h);
  m->lnf_b = (float *)calloc(h, sizeof(float));
  if (linear_random(&st, &m->lm_head, h, cfg->vocab_size)) {
    ocr_gpt_free(m);
    return NULL;
  }
  return m;
}

void ocr_gpt_free(ocr_gpt *m) {
  if (!m) return;
  free(m->wte);
  free(m->wpe);
  free(m->lnf_w);
  free(m->lnf_b);
  if (m->layers) {
    for (size_t i = 0; i < m->cfg.num_layers; i++) {
      layer_t *L = &m->layers[i];
      free(L->ln1_w); free(L->ln1_b); free(L->ln2_w); free(L->ln2_b);
      free(L->qkv.w); free(L->qkv.b); free(L->attn_out.w); free(L->attn_out.b);
      free(L->fc.w); free(L->fc.b); free(L->proj.w); free(L->proj.b);
      if (L->mla) {
        for (size_t hh = 0; hh < m->cfg.num_heads; hh++) {
          free(L->mla[hh].down);
          free(L->mla[hh].up);
        }
        free(L->mla);
      }
    }
    free(m->layers);
  }
  free(m->lm_head.w);
  free(m->lm_head.b);
  free(m);
}

void ocr_gpt_set_attention(ocr_gpt *m, int flash, size_t block,
                           int faithful) {
  m->flash = flash;
  m->block = block ? block : 1;
  m->faithful = faithful;
}

/* llm:822-838 */
int ocr_gpt_enable_mla(ocr_gpt *m, size_t d_c, uint64_t seed) {
  size_t hd = m->cfg.hidden_size / m->cfg.num_heads;
  if (!(d_c > 0 && d_c < hd)) return 1;
  uint64_t st = seed;
  for (size_t i = 0; i < m->cfg.num_layers; i++) {
    layer_t *L = &m->layers[i];
    if (!L->mla) L->mla = (mla_head *)calloc(m->cfg.num_heads, sizeof(mla_head));
    for (size_t h = 0; h < m->cfg.num_heads; h++) {
      free(L->mla[h].down);
      free(L->mla[h].up);
      L->mla[h].down = (float *)malloc(hd * d_c * sizeof(float));
      L->mla[h].up = (float *)malloc(d_c * hd * sizeof(float));
      fill_random(&st, L->mla[h].down, hd * d_c, 0.02f);
      fill_random(&st, L->mla[h].up, d_c * hd, 0.02f);
    }
  }
  m->d_c = d_c;
  return 0;
}

const float *ocr_gpt_weight(const ocr_gpt *m, int which, size_t layer,
                            size_t head, size_t *len) {
  const ocr_gpt_config *c = &m->cfg;
  size_t h = c->hidden_size;
  const layer_t *L = layer < c->num_layers ? &m->layers[layer] : NULL;
  size_t hd = c->hidden_size / c->num_heads;
  switch (which) {
    case 0: *len = c->vocab_size * h; return m->wte;
    case 1: *len = c->max_seq_len * h; return m->wpe;
    case 14: *len = h; return m->lnf_w;
    case 15: *len = h; return m->lnf_b;
    case 16: *len = h * c->vocab_size; return m->lm_head.w;
    case 17: *len = c->vocab_size; return m->lm_head.b;
    default: break;
  }
  if (!L) return NULL;
  switch (which) {
    case 2: *len = h * 3 * h; return L->qkv.w;
    case 3: *len = 3 * h; return L->qkv.b;
    case 4: *len = h * h; return L->attn_out.w;
    case 5: *len = h; return L->attn_out.b;
    case 6: *len = h * c->intermediate_size; return L->fc.w;
    case 7: *len = c->intermediate_size; return L->fc.b;
    case 8: *len = c->intermediate_size * h; return L->proj.w;
    case 9: *len = h; return L->proj.b;
    case 10: *len = h; return L->ln1_w;
    case 11: *len = h; return L->ln1_b;
    case 12: *len = h; return L->ln2_w;
    case 13: *len = h; return L->ln2_b;
    case 18: if (!L->mla || head >= c->num_heads) return NULL;
      *len = hd * m->d_c; return L->mla[head].down;
    case 19: if (!L->mla || head >= c->num_heads) return NULL;
      *len = m->d_c * hd; return L->mla[head].up;
    default: return NULL;
  }
}

/* llm:252-262 */
void ocr_layer_norm(float *x, size_t rows, size_t dim, const float *w,
                    const float *b, float eps) {
  for (size_t r = 0; r < rows; r++) {
    float *s = x + r * dim;
    float sum = -0.0f;
    for (size_t i = 0; i < dim; i++) sum += s[i];
    float mean = sum / (float)dim;
    float vs = -0.0f;
    for (size_t i = 0; i < dim; i++) {
      float dv = s[i] - mean;
      vs += dv * dv;
    }
    float var = vs / (float)dim;
    float inv_std = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < dim; i++) s[i] = (s[i] - mean) * inv_std * w[i] + b[i];
  }
}

/* llm:268-275: computed in f64, cast to f32 */
void ocr_gelu(float *x, size_t n) {
  const double k = 0.7978845608028654;
  for (size_t i = 0; i < n; i++) {
    double xf = (double)x[i];
    double inner = k * (xf + 0.044715 * (xf * xf * xf));
    x[i] = (float)(0.5 * xf * (1.0 + tanh(inner)));
  }
}

/* llm:227-238: sgemm(seq, in, out, 1, x, weight_t, 0) then host bias add */
static int linear_forward(const ocr_gpt *m, const linear_t *l, const float *x,
                          size_t seq, float *out) {
  memset(out, 0, seq * l->out * sizeof(float));
  int rc = ocr_sgemm(seq, l->in, l->out, 1.0f, x, l->w, 0, 0.0f, out, m->faithful);
  for (size_t r = 0; r < seq; r++)
    for (size_t c = 0; c < l->out; c++) out[r * l->out + c] += l->b[c];
  return rc;
}

/* KvCacheHead (llm:547-596): append-only host K/V per (layer, head); with
 * MLA the latent rows are stored and the whole cache is decompressed on
 * every read. */
typedef struct {
  float *k, *v; /* [cap][head_dim] or latent [cap][d_c] */
  size_t n;
} kvhead;

struct ocr_gpt_state {
  kvhead *heads; /* layers * heads */
  size_t nheads, cap, width;
  float *scratch_k, *scratch_v; /* decompressed views for MLA */
};

ocr_gpt_state *ocr_gpt_state_new(const ocr_gpt *m) {
  ocr_gpt_state *s = (ocr_gpt_state *)calloc(1, sizeof(ocr_gpt_state));
  if (!s) return NULL;
  size_t nh = m->cfg.num_layers * m->cfg.num_heads;
  size_t hd = m->cfg.hidden_size / m->cfg.num_heads;
  int mla = m->cfg.num_layers && m->layers[0].mla;
  s->cap = m->cfg.max_seq_len + 1;
  s->width = mla ? m->d_c : hd;
  s->heads = (kvhead *)calloc(nh, sizeof(kvhead));
  s->nheads = s->heads ? nh : 0;
  s->scratch_k = (float *)malloc(s->cap * hd * sizeof(float));
  s->scratch_v = (float *)malloc(s->cap * hd * sizeof(float));
  if (!s->heads || !s->scratch_k || !s->scratch_v) {
    ocr_gpt_state_free(s);
    return NULL;
  }
  for (size_t i = 0; i < nh; i++) {
    s->heads[i].k = (float *)malloc(s->cap * s->width * sizeof(float));
    s->heads[i].v = (float *)malloc(s->cap * s->width * sizeof(float));
    if (!s->heads[i].k || !s->heads[i].v) {
      ocr_gpt_state_free(s);
      return NULL;
    }
  }
  return s;
}

void ocr_gpt_state_free(ocr_gpt_state *s) {
  if (!s) return;
  for (size_t i = 0; i < s->nheads; i++) {
    free(s->heads[i].k);
    free(s->heads[i].v);
  }
  free(s->scratch_k);
  free(s->scratch_v);
  free(s->heads);
  free(s);
}

/* One (row, head) attention step of DecoderLayer (llm:348-393): push k/v
 * (compressed with MLA), read back the whole cache, attend q over it. */
static void head_step(const ocr_gpt *m, ocr_gpt_state *s, const layer_t *L,
                      size_t layer, size_t h, const float *q_h,
                      const float *k_h, const float *v_h, float *ctx_out) {
  size_t hd = m->cfg.hidden_size / m->cfg.num_heads;
  kvhead *kv = &s->heads[layer * m->cfg.num_heads + h];
  const float *kall, *vall;
  if (L->mla) {
    /* KvCacheHead::push with MLA: mla_compress_kv(1, hd, d_c) (llm:568-573) */
    size_t dc = m->d_c;
    ocr_mla_compress_kv(1, hd, dc, k_h, L->mla[h].down, kv->k + kv->n * dc);
    ocr_mla_compress_kv(1, hd, dc, v_h, L->mla[h].down, kv->v + kv->n * dc);
    kv->n++;
    /* current_kv: decompress all n rows (llm:586-591) */
    ocr_mla_decompress_kv(kv->n, dc, hd, kv->k, L->mla[h].up, s->scratch_k);
    ocr_mla_decompress_kv(kv->n, dc, hd, kv->v, L->mla[h].up, s->scratch_v);
    kall = s->scratch_k;
    vall = s->scratch_v;
  } else {
    memcpy(kv->k + kv->n * hd, k_h, hd * sizeof(float));
    memcpy(kv->v + kv->n * hd, v_h, hd * sizeof(float));
    kv->n++;
    kall = kv->k;
    vall = kv->v;
  }
  size_t n = kv->n;
  if (m->faithful) {
    /* llm:358-387: q replicated n times, all n rows computed, row 0 kept */
    float *qf = (float *)malloc(n * hd * sizeof(float));
    float *of = (float *)malloc(n * hd * sizeof(float));
    for (size_t r = 0; r < n; r++) memcpy(qf + r * hd, q_h, hd * sizeof(float));
    if (m->flash)
      ocr_flash_attention(qf, kall, vall, n, hd, m->block, of);
    else
      ocr_sdpa(qf, kall, vall, n, hd, of);
    memcpy(ctx_out, of, hd * sizeof(float));
    free(qf);
    free(of);
  } else {
    ocr_attend_one(q_h, kall, vall, n, hd, m->flash, m->block, ctx_out);
  }
}

/* DecoderLayer::forward_prefill (llm:436-521); seq = 1 is forward_step
 * (llm:322-410), which performs the same operations. */
static int layer_forward(const ocr_gpt *m, ocr_gpt_state *s, size_t li,
                         float *hidden, size_t seq) {
  const layer_t *L = &m->layers[li];
  size_t H = m->cfg.hidden_size, nh = m->cfg.num_heads, hd = H / nh;
  size_t I = m->cfg.intermediate_size;
  float *normed = (float *)malloc(seq * H * sizeof(float));
  float *qkv = (float *)malloc(seq * 3 * H * sizeof(float));
  float *ctx = (float *)calloc(seq * H, sizeof(float));
  float *tmp = (float *)malloc(seq * H * sizeof(float));
  float *inter = (float *)malloc(seq * I * sizeof(float));
  if (!normed || !qkv || !ctx || !tmp || !inter) {
    free(normed); free(qkv); free(ctx); free(tmp); free(inter);
    return 2;
  }
  memcpy(normed, hidden, seq * H * sizeof(float));
  ocr_layer_norm(normed, seq, H, L->ln1_w, L->ln1_b, m->cfg.layer_norm_eps);
  linear_forward(m, &L->qkv, normed, seq, qkv);
  for (size_t r = 0; r < seq; r++) {
    const float *row = qkv + r * 3 * H;
    for (size_t h = 0; h < nh; h++)
      head_step(m, s, L, li, h, row + h * hd, row + H + h * hd,
                row + 2 * H + h * hd, ctx + r * H + h * hd);
  }
  linear_forward(m, &L->attn_out, ctx, seq, tmp);
  for (size_t i = 0; i < seq * H; i++) hidden[i] += tmp[i]; /* residual */
  memcpy(normed, hidden, seq * H * sizeof(float));
  ocr_layer_norm(normed, seq, H, L->ln2_w, L->ln2_b, m->cfg.layer_norm_eps);
  linear_forward(m, &L->fc, normed, seq, inter);
  ocr_gelu(inter, seq * I);
  linear_forward(m, &L->proj, inter, seq, tmp);
  for (size_t i = 0; i < seq * H; i++) hidden[i] += tmp[i];
  free(normed); free(qkv); free(ctx); free(tmp); free(inter);
  return 0;
}

/* llm:846-864 */
static int forward_rows(const ocr_gpt *m, ocr_gpt_state *s,
                        const uint32_t *ids, size_t len, size_t pos0,
                        float *logits);

int ocr_gpt_forward_step(const ocr_gpt *m, ocr_gpt_state *s, uint32_t token,
                         size_t pos, float *logits) {
  return forward_rows(m, s, &token, 1, pos, logits);
}

/* llm:869-899 (and llm:846-864 with len = 1 at position = cache length) */
static int forward_rows(const ocr_gpt *m, ocr_gpt_state *s,
                        const uint32_t *ids, size_t len, size_t pos0,
                        float *logits) {
  size_t H = m->cfg.hidden_size;
  if (len == 0) return 1;
  float *hidden = (float *)malloc(len * H * sizeof(float));
  if (!hidden) return 2;
  for (size_t r = 0; r < len; r++) {
    size_t pos = pos0 + r;
    if (pos >= m->cfg.max_seq_len || ids[r] >= m->cfg.vocab_size) {
      free(hidden);
      return 1;
    }
    const float *w = m->wte + (size_t)ids[r] * H, *p = m->wpe + pos * H;
    for (size_t i = 0; i < H; i++) hidden[r * H + i] = w[i] + p[i];
  }
  for (size_t li = 0; li < m->cfg.num_layers; li++)
    if (layer_forward(m, s, li, hidden, len)) {
      free(hidden);
      return 2;
    }
  float *last = hidden + (len - 1) * H;
  ocr_layer_norm(last, 1, H, m->lnf_w, m->lnf_b, m->cfg.layer_norm_eps);
  int rc = linear_forward(m, &m->lm_head, last, 1, logits);
  free(hidden);
  return rc;
}

static size_t state_len(const ocr_gpt_state *s) { return s->heads[0].n; }

int ocr_gpt_forward_prefill(const ocr_gpt *m, ocr_gpt_state *s,
                            const uint32_t *ids, size_t len, float *logits) {
  return forward_rows(m, s, ids, len, state_len(s), logits);
}

/* llm:932-942: strict `>` keeps the first maximum */
uint32_t ocr_argmax(const float *x, size_t n) {
  size_t best = 0;
  float bv = -INFINITY;
  for (size_t i = 0; i < n; i++)
    if (x[i] > bv) {
      bv = x[i];
      best = i;
    }
  return (uint32_t)best;
}

/* llm:910-929 */
long ocr_gpt_generate(const ocr_gpt *m, const uint32_t *prompt, size_t len,
                      size_t max_new, uint32_t *out, float *logits_out) {
  if (len == 0) return -1;
  size_t V = m->cfg.vocab_size;
  ocr_gpt_state *s = ocr_gpt_state_new(m);
  float *logits = (float *)malloc(V * sizeof(float));
  if (!s || !logits) {
    free(logits);
    return -1;
  }
  long produced = -1;
  if (forward_rows(m, s, prompt, len, 0, logits) == 0) {
    produced = 0;
    uint32_t next = ocr_argmax(logits, V);
    for (size_t i = 0; i < max_new; i++) {
      size_t pos_now = len + i;
      if (logits_out) memcpy(logits_out + i * V, logits, V * sizeof(float));
      out[i] = next;
      produced++;
      if (pos_now >= m->cfg.max_seq_len) break;
      if (forward_rows(m, s, &next, 1, pos_now, logits)) {
        produced = -1;
        break;
      }
      next = ocr_argmax(logits, V);
    }
  }
  ocr_gpt_state_free(s);
  free(logits);
  return produced;
}
