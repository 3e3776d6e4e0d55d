/*
 * rowops.c — C restatement of the reference's row kernels — TEST INFRASTRUCTURE ONLY.
 *
 * Built by oracle/Makefile into oracle/_build/liboracle_rowops.so and loaded by tests and
 * by bench.py's CPU-baseline legs (never by the product path).  Rows are independent, so
 * the row loop runs on all host threads (pthreads); inside a row the arithmetic is
 * serial and in the reference's order (compiled with -ffp-contract=off, no fast-math):
 *
 *   cumsum : python/ntilang/scan.py:349-389 — 32-column Hillis-Steele segments (offsets
 *            1,2,4,8,16 on a snapshot of the previous level), then carries from +0:
 *            out = local + carry, carry_next = out[last column of the segment].
 *   softmax: examples/softmax.py:9-25 — fmax row max, expf(x - max), perfect-tree sum over
 *            the row padded to a power of two (python/ntilang/codegen.py:1094-1151), x / sum.
 *   rmsnorm: examples/rmsnorm.py:13-37 — tree sum of squares, 1/sqrtf(ss*inv_n + eps),
 *            (x * inv) * w.
 *   vadd   : examples/vector_add.py:5-10.
 *   layernorm: examples/layernorm.py:18-43.  transpose: examples/transpose.py:5-15.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static int g_threads = 0;

int oracle_threads(void) {
  if (g_threads <= 0) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    g_threads = n > 0 ? (int)n : 1;
  }
  return g_threads;
}
void oracle_set_threads(int n) { g_threads = n > 0 ? n : 1; }

/* Static-schedule parallel for over [0, count): body(ctx, begin, end) on each thread. */
typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);
struct job {
  range_fn fn;
  void* ctx;
  int64_t begin, end;
};
static void* run_job(void* arg) {
  struct job* j = (struct job*)arg;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}
static void parallel_for(int64_t count, range_fn fn, void* ctx) {
  int t = oracle_threads();
  if (t > count) t = (int)(count > 0 ? count : 1);
  if (t > 256) t = 256;
  pthread_t th[256];
  struct job jobs[256];
  int64_t per = (count + t - 1) / t;
  for (int i = 0; i < t; ++i) {
    jobs[i].fn = fn, jobs[i].ctx = ctx;
    jobs[i].begin = i * per < count ? i * per : count;
    jobs[i].end = (i + 1) * per < count ? (i + 1) * per : count;
  }
  for (int i = 1; i < t; ++i) pthread_create(&th[i], NULL, run_job, &jobs[i]);
  run_job(&jobs[0]);
  for (int i = 1; i < t; ++i) pthread_join(th[i], NULL);
}

struct vadd_ctx {
  const float *a, *b;
  float* c;
};
static void vadd_range(void* p, int64_t b, int64_t e) {
  struct vadd_ctx* x = (struct vadd_ctx*)p;
  for (int64_t i = b; i < e; ++i) x->c[i] = x->a[i] + x->b[i];
}
void oracle_vadd_f32(const float* a, const float* b, float* c, int64_t n) {
  struct vadd_ctx x = {a, b, c};
  parallel_for(n, vadd_range, &x);
}

static void scan_row(const float* x, float* y, int64_t n, int reverse, float* work) {
  const int64_t segs = (n + 31) / 32;
  float tmp[32];
  for (int64_t s = 0; s < segs; ++s) {
    float* w = work + s * 32;
    for (int l = 0; l < 32; ++l) {
      int64_t c = s * 32 + l;
      w[l] = c < n ? x[c] : 0.0f;
    }
    for (int o = 1; o <= 16; o <<= 1) {
      memcpy(tmp, w, sizeof(tmp));
      if (reverse) {
        for (int l = 0; l + o < 32; ++l) w[l] = tmp[l] + tmp[l + o];
      } else {
        for (int l = o; l < 32; ++l) w[l] = tmp[l] + tmp[l - o];
      }
    }
  }
  float carry = 0.0f;
  for (int64_t i = 0; i < segs; ++i) {
    const int64_t s = reverse ? segs - 1 - i : i;
    float* w = work + s * 32;
    for (int l = 0; l < 32; ++l) w[l] = w[l] + carry;
    carry = w[reverse ? 0 : 31];
  }
  memcpy(y, work, (size_t)n * sizeof(float));
}

struct row_ctx {
  const float *x, *w;
  float* y;
  int64_t cols;
  int reverse;
  float eps, inv_n;
};

static void cumsum_range(void* p, int64_t b, int64_t e) {
  struct row_ctx* c = (struct row_ctx*)p;
  float* work = (float*)malloc((size_t)((c->cols + 31) / 32 * 32) * sizeof(float));
  for (int64_t r = b; r < e; ++r) scan_row(c->x + r * c->cols, c->y + r * c->cols, c->cols, c->reverse, work);
  free(work);
}

void oracle_cumsum_f32(const float* x, float* y, int64_t rows, int64_t cols, int reverse) {
  struct row_ctx c = {x, NULL, y, cols, reverse, 0.f, 0.f};
  parallel_for(rows, cumsum_range, &c);
}

static int64_t next_pow2(int64_t n) {
  int64_t p = 1;
  while (p < n) p <<= 1;
  return p;
}

/* Perfect binary tree over work[0..p), p a power of two; destroys work. */
static float tree_sum(float* work, int64_t p) {
  for (int64_t w = p; w > 1; w >>= 1)
    for (int64_t i = 0; i < w / 2; ++i) work[i] = work[2 * i] + work[2 * i + 1];
  return work[0];
}

static void softmax_range(void* p, int64_t b, int64_t e) {
  struct row_ctx* c = (struct row_ctx*)p;
  const int64_t cols = c->cols, pw = next_pow2(cols);
  float* work = (float*)malloc((size_t)pw * sizeof(float));
  for (int64_t r = b; r < e; ++r) {
    const float* xr = c->x + r * cols;
    float* yr = c->y + r * cols;
    float m = -INFINITY;
    for (int64_t j = 0; j < cols; ++j) m = fmaxf(m, xr[j]);
    for (int64_t j = 0; j < cols; ++j) yr[j] = expf(xr[j] - m);
    for (int64_t j = 0; j < pw; ++j) work[j] = j < cols ? yr[j] : 0.0f;
    const float s = tree_sum(work, pw);
    for (int64_t j = 0; j < cols; ++j) yr[j] = yr[j] / s;
  }
  free(work);
}

void oracle_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols) {
  struct row_ctx c = {x, NULL, y, cols, 0, 0.f, 0.f};
  parallel_for(rows, softmax_range, &c);
}

static void rmsnorm_range(void* p, int64_t b, int64_t e) {
  struct row_ctx* c = (struct row_ctx*)p;
  const int64_t cols = c->cols, pw = next_pow2(cols);
  float* work = (float*)malloc((size_t)pw * sizeof(float));
  for (int64_t r = b; r < e; ++r) {
    const float* xr = c->x + r * cols;
    float* yr = c->y + r * cols;
    for (int64_t j = 0; j < pw; ++j) work[j] = j < cols ? xr[j] * xr[j] : 0.0f;
    const float ss = tree_sum(work, pw);
    const float t = ss * c->inv_n + c->eps;
    const float inv = (float)(1.0 / sqrt((double)t));
    for (int64_t j = 0; j < cols; ++j) yr[j] = (xr[j] * inv) * c->w[j];
  }
  free(work);
}

void oracle_rmsnorm_f32(const float* x, const float* w, float* y, int64_t rows, int64_t cols, float eps,
                        float inv_n) {
  struct row_ctx c = {x, w, y, cols, 0, eps, inv_n};
  parallel_for(rows, rmsnorm_range, &c);
}

/* examples/layernorm.py:18-43: mean = tree(x) * inv_n; d = x - mean; rstd = 1 / sqrtf(tree(d*d)
 * * inv_n + eps) (the reference evaluator's rsqrt, testing.py:98); y = ((d * rstd) * w) + b. */
struct ln_ctx {
  const float *x, *w, *b;
  float* y;
  int64_t cols;
  float eps, inv_n;
};

static void layernorm_range(void* p, int64_t b, int64_t e) {
  struct ln_ctx* c = (struct ln_ctx*)p;
  const int64_t cols = c->cols, pw = next_pow2(cols);
  float* work = (float*)malloc((size_t)pw * sizeof(float));
  for (int64_t r = b; r < e; ++r) {
    const float* xr = c->x + r * cols;
    float* yr = c->y + r * cols;
    for (int64_t j = 0; j < pw; ++j) work[j] = j < cols ? xr[j] : 0.0f;
    const float mean = tree_sum(work, pw) * c->inv_n;
    for (int64_t j = 0; j < pw; ++j) {
      const float d = j < cols ? xr[j] - mean : 0.0f;
      work[j] = d * d;
    }
    const float var = tree_sum(work, pw) * c->inv_n;
    const float rstd = 1.0f / sqrtf(var + c->eps);
    for (int64_t j = 0; j < cols; ++j) yr[j] = ((xr[j] - mean) * rstd) * c->w[j] + c->b[j];
  }
  free(work);
}

void oracle_layernorm_f32(const float* x, const float* w, const float* b, float* y, int64_t rows, int64_t cols,
                          float eps, float inv_n) {
  struct ln_ctx c = {x, w, b, y, cols, eps, inv_n};
  parallel_for(rows, layernorm_range, &c);
}

struct tr_ctx {
  const float* a;
  float* b;
  int64_t m, n;
};

static void transpose_range(void* p, int64_t b, int64_t e) {
  struct tr_ctx* c = (struct tr_ctx*)p;
  for (int64_t r = b; r < e; ++r)
    for (int64_t j = 0; j < c->n; ++j) c->b[j * c->m + r] = c->a[r * c->n + j];
}

/* examples/transpose.py:5-15: b[n, m] = a[m, n]^T. */
void oracle_transpose_f32(const float* a, float* b, int64_t m, int64_t n) {
  struct tr_ctx c = {a, b, m, n};
  parallel_for(m, transpose_range, &c);
}
