/*
 * CPU oracle for the SDPA forward — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may
 * load this library, and only as the checker or the timed CPU baseline; the product
 * path (tiledattention_b200) never calls it.
 *
 * Restates the reference algorithm of thisistaimur/TiledAttention for one query row:
 *   scores_c = (q . k_c) * scale                  src/tiledattention/kernels/flash_fwd.py:412-413
 *   masked (-inf) where c >= S, or causal and c > r (top-left, S_q == S_kv)   :400-423
 *   o = softmax(scores) @ v, normalised by the row sum                        :426-444
 * i.e. the math path the reference benchmarks against
 * (benchmark-gb10/run_study.py:304-335 standard_eager_attention,
 *  :249-271 torch_sdpa_math) and the reference test's comparator
 * (tests/test_sdpa_correctness_small.py:37-39).
 *
 * Inputs are float32 [BH, S, D] contiguous (the caller upcasts fp16/bf16 bit-exactly);
 * output float32 [BH, S, D]; optional lse float32 [BH, S] (natural log).
 *
 * ta_oracle_sdpa_f64: double accumulation everywhere — the parity oracle.
 * ta_oracle_sdpa_f32: float accumulation, vectorisable loops — the timed CPU baseline
 *                     (same role as the reference's fp32 torch math backend).
 * Rows [row_begin, row_end) of every head are computed (row sampling for huge S).
 * Parallel over (head, row) with POSIX threads pulling rows from an atomic counter;
 * ta_oracle_set_threads / ta_oracle_threads set and report the thread count
 * (default: all online host cores).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>

static int g_threads = 0;

int ta_oracle_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

void ta_oracle_set_threads(int n) { g_threads = n > 0 ? n : 0; }

typedef struct {
  const float *q, *k, *v;
  float *o, *lse;
  int BH, S, D, causal, row_begin, nrows;
  double scale;
  int f64;
  long long next; /* shared work counter */
} job_t;

static void row_f64(const job_t* j, int bh, int r, double* sc, double* acc);
static void row_f32(const job_t* j, int bh, int r, float* sc, float* acc);

static void* worker(void* arg) {
  job_t* j = (job_t*)arg;
  void* sc = malloc((j->f64 ? sizeof(double) : sizeof(float)) * (size_t)j->S);
  void* acc = malloc((j->f64 ? sizeof(double) : sizeof(float)) * (size_t)j->D);
  const long long total = (long long)j->BH * j->nrows;
  for (;;) {
    long long idx = __atomic_fetch_add(&j->next, 4, __ATOMIC_RELAXED);
    if (idx >= total) break;
    long long end = idx + 4 < total ? idx + 4 : total;
    for (; idx < end; ++idx) {
      const int bh = (int)(idx / j->nrows);
      const int r = j->row_begin + (int)(idx % j->nrows);
      if (j->f64)
        row_f64(j, bh, r, (double*)sc, (double*)acc);
      else
        row_f32(j, bh, r, (float*)sc, (float*)acc);
    }
  }
  free(sc);
  free(acc);
  return NULL;
}

static void run_job(job_t* j) {
  int n = ta_oracle_threads();
  if (n > 256) n = 256;
  pthread_t tid[256];
  int started = 0;
  for (int i = 1; i < n; ++i)
    if (pthread_create(&tid[started], NULL, worker, j) == 0) ++started;
  worker(j);
  for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
}

static int valid_cols(int row, int S, int causal) { return causal ? (row + 1 < S ? row + 1 : S) : S; }

static void row_f64(const job_t* j, int bh, int r, double* sc, double* acc) {
  const int S = j->S, D = j->D;
  const float* qr = j->q + ((size_t)bh * S + r) * D;
  const float* kb = j->k + (size_t)bh * S * D;
  const float* vb = j->v + (size_t)bh * S * D;
  const int nc = valid_cols(r, S, j->causal);
  double mx = -INFINITY;
  for (int c = 0; c < nc; ++c) {
    const float* kc = kb + (size_t)c * D;
    double dot = 0.0;
    for (int d = 0; d < D; ++d) dot += (double)qr[d] * (double)kc[d];
    sc[c] = dot * j->scale;
    if (sc[c] > mx) mx = sc[c];
  }
  double sum = 0.0;
  for (int d = 0; d < D; ++d) acc[d] = 0.0;
  for (int c = 0; c < nc; ++c) {
    const double p = exp(sc[c] - mx);
    sum += p;
    const float* vc = vb + (size_t)c * D;
    for (int d = 0; d < D; ++d) acc[d] += p * (double)vc[d];
  }
  float* orow = j->o + ((size_t)bh * S + r) * D;
  for (int d = 0; d < D; ++d) orow[d] = (float)(acc[d] / sum);
  if (j->lse) j->lse[(size_t)bh * S + r] = (float)(mx + log(sum));
}

static void row_f32(const job_t* j, int bh, int r, float* sc, float* acc) {
  const int S = j->S, D = j->D;
  const float scale = (float)j->scale;
  const float* qr = j->q + ((size_t)bh * S + r) * D;
  const float* kb = j->k + (size_t)bh * S * D;
  const float* vb = j->v + (size_t)bh * S * D;
  const int nc = valid_cols(r, S, j->causal);
  float mx = -INFINITY;
  for (int c = 0; c < nc; ++c) {
    const float* kc = kb + (size_t)c * D;
    float dot0 = 0.f, dot1 = 0.f, dot2 = 0.f, dot3 = 0.f;
    int d = 0;
    for (; d + 4 <= D; d += 4) {
      dot0 += qr[d] * kc[d];
      dot1 += qr[d + 1] * kc[d + 1];
      dot2 += qr[d + 2] * kc[d + 2];
      dot3 += qr[d + 3] * kc[d + 3];
    }
    for (; d < D; ++d) dot0 += qr[d] * kc[d];
    sc[c] = (dot0 + dot1 + dot2 + dot3) * scale;
    mx = sc[c] > mx ? sc[c] : mx;
  }
  float sum = 0.f;
  for (int d = 0; d < D; ++d) acc[d] = 0.f;
  for (int c = 0; c < nc; ++c) {
    const float p = expf(sc[c] - mx);
    sum += p;
    const float* vc = vb + (size_t)c * D;
    for (int d = 0; d < D; ++d) acc[d] += p * vc[d];
  }
  float* orow = j->o + ((size_t)bh * S + r) * D;
  const float inv = 1.f / sum;
  for (int d = 0; d < D; ++d) orow[d] = acc[d] * inv;
  if (j->lse) j->lse[(size_t)bh * S + r] = mx + logf(sum);
}

static void launch(const float* q, const float* k, const float* v, float* o, float* lse, int BH,
                   int S, int D, int causal, double scale, int row_begin, int row_end, int f64) {
  if (row_begin < 0) row_begin = 0;
  if (row_end > S) row_end = S;
  if (row_end <= row_begin || BH <= 0 || D <= 0) return;
  job_t j = {q, k, v, o, lse, BH, S, D, causal, row_begin, row_end - row_begin, scale, f64, 0};
  run_job(&j);
}

void ta_oracle_sdpa_f64(const float* q, const float* k, const float* v, float* o, float* lse,
                        int BH, int S, int D, int causal, double scale, int row_begin,
                        int row_end) {
  launch(q, k, v, o, lse, BH, S, D, causal, scale, row_begin, row_end, 1);
}

void ta_oracle_sdpa_f32(const float* q, const float* k, const float* v, float* o, float* lse,
                        int BH, int S, int D, int causal, float scale, int row_begin,
                        int row_end) {
  launch(q, k, v, o, lse, BH, S, D, causal, scale, row_begin, row_end, 0);
}
