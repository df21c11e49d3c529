/*
 * pool.c -- TEST INFRASTRUCTURE (oracle).  The persistent spin-then-park
 * worker pool of crates/prana-kernels/src/pool.rs:28-311 (epoch publish,
 * atomic chunk claiming, submitter participates), the thread-count default of
 * threading.rs:46-53, and the row-chunking matmul drivers of
 * matmul.rs:150-350 / kquant.rs:323-370 that run on it.
 */
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "prana_oracle.h"

typedef void (*chunk_fn)(void *ctx, size_t chunk);

/* pool.rs:109 */
#define SPIN_ITERS 200000u

static struct {
  int threads;
  int started;
  pthread_mutex_t slot_mu;
  pthread_cond_t work_cv;
  pthread_mutex_t done_mu;
  pthread_cond_t done_cv;
  pthread_mutex_t submit_mu;
  _Atomic uint64_t epoch;
  _Atomic uint32_t parked;
  _Atomic int submitter_waiting;
  /* the published job (written under slot_mu before the epoch bump) */
  chunk_fn fn;
  void *ctx;
  _Atomic uint32_t n_chunks;
  _Atomic uint32_t next;
  _Atomic uint32_t remaining;
} P = {.slot_mu = PTHREAD_MUTEX_INITIALIZER,
       .work_cv = PTHREAD_COND_INITIALIZER,
       .done_mu = PTHREAD_MUTEX_INITIALIZER,
       .done_cv = PTHREAD_COND_INITIALIZER,
       .submit_mu = PTHREAD_MUTEX_INITIALIZER};

static pthread_once_t pool_once = PTHREAD_ONCE_INIT;
static int requested_threads = 0;

/* threading.rs:46-53: PRANA_THREADS, else min(available parallelism, 8) */
static int default_threads(void) {
  const char *e = getenv("PRANA_THREADS");
  if (e && atoi(e) > 0) return atoi(e);
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  return n < 8 ? (int)n : 8;
}

/* pool.rs:54-70 */
static void execute_chunks(void) {
  for (;;) {
    uint32_t i = atomic_fetch_add_explicit(&P.next, 1, memory_order_relaxed);
    if (i >= P.n_chunks) break;
    P.fn(P.ctx, i);
    atomic_fetch_sub_explicit(&P.remaining, 1, memory_order_acq_rel);
  }
}

/* pool.rs:259-296 */
static void *worker_loop(void *arg) {
  (void)arg;
  uint64_t seen = 0;
  for (;;) {
    uint32_t spins = 0;
    for (;;) {
      uint64_t e = atomic_load_explicit(&P.epoch, memory_order_acquire);
      if (e != seen) {
        seen = e;
        break;
      }
      if (spins < SPIN_ITERS) {
        spins++;
        __builtin_ia32_pause();
      } else {
        pthread_mutex_lock(&P.slot_mu);
        atomic_fetch_add(&P.parked, 1);
        if (atomic_load(&P.epoch) == seen) pthread_cond_wait(&P.work_cv, &P.slot_mu);
        atomic_fetch_sub(&P.parked, 1);
        pthread_mutex_unlock(&P.slot_mu);
        spins = 0;
      }
    }
    execute_chunks();
    if (atomic_load(&P.remaining) == 0 && atomic_load(&P.submitter_waiting)) {
      pthread_mutex_lock(&P.done_mu);
      pthread_cond_broadcast(&P.done_cv);
      pthread_mutex_unlock(&P.done_mu);
    }
  }
  return NULL;
}

static void pool_start(void) {
  P.threads = requested_threads > 0 ? requested_threads : default_threads();
  for (int i = 1; i < P.threads; i++) {
    pthread_t t;
    pthread_attr_t at;
    pthread_attr_init(&at);
    pthread_attr_setdetachstate(&at, PTHREAD_CREATE_DETACHED);
    pthread_create(&t, &at, worker_loop, NULL);
    pthread_attr_destroy(&at);
  }
  P.started = 1;
}

int or_pool_threads(void) {
  pthread_once(&pool_once, pool_start);
  return P.threads;
}

void or_pool_set_threads(int n) { requested_threads = n; }

/* pool.rs:169-256: Pool::run / dispatch */
static void pool_run(size_t n_chunks, chunk_fn fn, void *ctx) {
  if (n_chunks == 0) return;
  int threads = or_pool_threads();
  if (n_chunks == 1 || threads == 1) {
    for (size_t i = 0; i < n_chunks; i++) fn(ctx, i);
    return;
  }
  pthread_mutex_lock(&P.submit_mu);
  pthread_mutex_lock(&P.slot_mu);
  P.fn = fn;
  P.ctx = ctx;
  P.n_chunks = (uint32_t)n_chunks;
  /* remaining before next: a straggler that claims index 0 of this job the
   * moment `next` is reset must find the counter it decrements already armed */
  atomic_store(&P.remaining, (uint32_t)n_chunks);
  atomic_store(&P.next, 0);
  atomic_fetch_add_explicit(&P.epoch, 1, memory_order_release);
  pthread_mutex_unlock(&P.slot_mu);
  if (atomic_load(&P.parked) > 0) pthread_cond_broadcast(&P.work_cv);

  execute_chunks();
  uint32_t spins = 0;
  while (atomic_load_explicit(&P.remaining, memory_order_acquire) != 0) {
    if (spins < SPIN_ITERS) {
      spins++;
      __builtin_ia32_pause();
    } else {
      pthread_mutex_lock(&P.done_mu);
      atomic_store(&P.submitter_waiting, 1);
      if (atomic_load(&P.remaining) != 0) {
        struct timespec ts;
        clock_gettime(CLOCK_REALTIME, &ts);
        ts.tv_nsec += 1000000;
        if (ts.tv_nsec >= 1000000000) {
          ts.tv_sec++;
          ts.tv_nsec -= 1000000000;
        }
        pthread_cond_timedwait(&P.done_cv, &P.done_mu, &ts);
      }
      atomic_store(&P.submitter_waiting, 0);
      pthread_mutex_unlock(&P.done_mu);
    }
  }
  pthread_mutex_unlock(&P.submit_mu);
}

/* ---------------- matmul drivers ---------------- */

typedef struct {
  int tier;
  const or_matrix *m;
  const int8_t *aq;
  const float *as;
  const int32_t *asum;
  const float *af; /* dense activation row (F32 matrices) */
  float *out;
  size_t n_rows, n_tokens, row_chunk;
} mm_ctx;

/* Linear::row_dot (checkpoint.rs:131-137) for token t, row r */
static float row_dot(const mm_ctx *c, size_t t, size_t r) {
  const or_matrix *m = c->m;
  size_t k = m->cols, g = k / 32;
  const int8_t *aq = c->aq + t * k;
  const float *as = c->as + t * g;
  const int32_t *asum = c->asum + t * g;
  switch (m->kind) {
    case OR_GGML_F32:
      return or_dot_f32(c->tier, c->af + t * k, m->f32 + r * k, k);
    case OR_GGML_Q8_0:
      return or_dot_q8_q8(c->tier, aq, as, k, m->q + r * k, m->scales + r * g);
    case OR_GGML_Q4_0:
      return or_dot_q40_q8(c->tier, aq, as, asum, k, m->blocks + r * g * 18, m->scales + r * g);
    case OR_GGML_Q4_K:
      return or_dot_q4k_q8(c->tier, aq, as, asum, k, m->blocks + r * (k / 256) * 144,
                           m->scales + r * (k / 256) * 2);
    case OR_GGML_Q6_K:
      return or_dot_q6k_q8(aq, as, k, m->blocks + r * (k / 256) * 210, m->scales + r * (k / 256));
  }
  return 0.0f;
}

static void rows_chunk(void *vc, size_t ci) {
  mm_ctx *c = vc;
  size_t r0 = ci * c->row_chunk, r1 = r0 + c->row_chunk;
  if (r1 > c->n_rows) r1 = c->n_rows;
  for (size_t r = r0; r < r1; r++) c->out[r] = row_dot(c, 0, r);
}

/* matmul.rs:318-350 run_rows: one token's outputs split over the pool */
static void run_rows(mm_ctx *c) {
  int threads = or_pool_threads();
  size_t k = c->m->cols;
  if (k * c->n_rows < 256 * 1024 || threads == 1) {
    for (size_t r = 0; r < c->n_rows; r++) c->out[r] = row_dot(c, 0, r);
    return;
  }
  size_t rc = (c->n_rows + (size_t)threads * 4 - 1) / ((size_t)threads * 4);
  if (rc < 16) rc = 16;
  c->row_chunk = rc;
  pool_run((c->n_rows + rc - 1) / rc, rows_chunk, c);
}

static void f32_decode_chunk(void *vc, size_t ci) {
  mm_ctx *c = vc;
  size_t r0 = ci * c->row_chunk, r1 = r0 + c->row_chunk;
  if (r1 > c->n_rows) r1 = c->n_rows;
  for (size_t r = r0; r < r1; r++) c->out[r] = row_dot(c, 0, r);
}

static void f32_token_chunk(void *vc, size_t t) {
  mm_ctx *c = vc;
  for (size_t r = 0; r < c->n_rows; r++) c->out[t * c->n_rows + r] = row_dot(c, t, r);
}

/* matmul.rs:150-156 + run_matmul 263-311 (dense f32) */
static void matmul_f32(int tier, const or_matrix *m, const float *a, size_t n_tokens, float *out) {
  mm_ctx c = {.tier = tier, .m = m, .af = a, .out = out, .n_rows = m->rows, .n_tokens = n_tokens};
  int threads = or_pool_threads();
  if (n_tokens * m->cols * m->rows < 32 * 1024 || threads == 1) {
    for (size_t t = 0; t < n_tokens; t++)
      for (size_t r = 0; r < m->rows; r++) out[t * m->rows + r] = row_dot(&c, t, r);
    return;
  }
  if (n_tokens == 1) {
    size_t rc = (m->rows + threads - 1) / threads;
    if (rc < 1) rc = 1;
    c.row_chunk = rc;
    pool_run((m->rows + rc - 1) / rc, f32_decode_chunk, &c);
    return;
  }
  pool_run(n_tokens, f32_token_chunk, &c);
}

/* matmul.rs:162-178 / kquant.rs:323-333: quantize each token's row, then run_rows */
void or_matmul(int tier, const or_matrix *m, const float *a, size_t n_tokens, float *out) {
  if (m->kind == OR_GGML_F32) {
    matmul_f32(tier, m, a, n_tokens, out);
    return;
  }
  size_t k = m->cols, g = k / 32;
  int8_t *aq = malloc(k);
  float *as = malloc(sizeof(float) * g);
  int32_t *asum = malloc(sizeof(int32_t) * g);
  for (size_t t = 0; t < n_tokens; t++) {
    or_quantize_acts(a + t * k, k, aq, as, asum);
    mm_ctx c = {.tier = tier, .m = m, .aq = aq, .as = as, .asum = asum, .out = out + t * m->rows,
                .n_rows = m->rows, .n_tokens = 1};
    run_rows(&c);
  }
  free(aq);
  free(as);
  free(asum);
}

static void multi_chunk(void *vc, size_t ci) {
  mm_ctx *c = vc;
  size_t r0 = ci * c->row_chunk, r1 = r0 + c->row_chunk;
  if (r1 > c->n_rows) r1 = c->n_rows;
  for (size_t r = r0; r < r1; r++)
    for (size_t t = 0; t < c->n_tokens; t++) c->out[r * c->n_tokens + t] = row_dot(c, t, r);
}

/* matmul.rs:192-232 run_rows_multi: weight-row-outer, then transpose */
void or_matmul_prefill(int tier, const or_matrix *m, const int8_t *aq, const float *as,
                       const int32_t *asum, size_t n_tokens, float *out) {
  size_t n_rows = m->rows;
  float *out_t = malloc(sizeof(float) * n_rows * n_tokens);
  mm_ctx c = {.tier = tier, .m = m, .aq = aq, .as = as, .asum = asum, .out = out_t,
              .n_rows = n_rows, .n_tokens = n_tokens};
  int threads = or_pool_threads();
  if (n_rows * n_tokens * m->cols < (1u << 20) || threads == 1) {
    for (size_t r = 0; r < n_rows; r++)
      for (size_t t = 0; t < n_tokens; t++) out_t[r * n_tokens + t] = row_dot(&c, t, r);
  } else {
    size_t rc = (n_rows + (size_t)threads * 4 - 1) / ((size_t)threads * 4);
    if (rc < 4) rc = 4;
    c.row_chunk = rc;
    pool_run((n_rows + rc - 1) / rc, multi_chunk, &c);
  }
  for (size_t r = 0; r < n_rows; r++)
    for (size_t t = 0; t < n_tokens; t++) out[t * n_rows + r] = out_t[r * n_tokens + t];
  free(out_t);
}
