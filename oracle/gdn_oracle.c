/*
 * CPU oracle for the gated-delta recurrence -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker; the product (gdn_b200) never links
 * it and has no CPU fallback.
 *
 * A plain-C, float64 restatement of the reference's ops path for many
 * sequences at once, used where the numpy oracle (gdn_oracle.py) would be too
 * slow (full-size configurations):
 *   qw/gated_delta.py:24-41   one step: S *= g; r = S k; d = beta (v - r);
 *                             S += d k^T; y = S q   (same operation order)
 *   qw/gated_delta.py:93-109  GQA by repeat-interleave: value head h reads key
 *                             head h / (Hv / Hk); positions run in order.
 * (qw/ = src/mlx_lean_moe/model/qwen3_5/ in the reference project.)
 *
 * Layout (row-major, innermost last): q, k [N, Hk, Dk]; v, y [N, Hv, Dv];
 * g, beta [N, Hv]; states [B, Hv, Dv, Dk]; cu_seqlens [B + 1] (int64).
 * g is the multiplicative decay unless g_is_log != 0, in which case exp(g)
 * is applied (the reference takes the multiplier; the benchmark
 * configurations draw a log-decay).  Each (sequence, value head) pair is
 * independent; units are handed out to n_threads POSIX threads.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  const float *q, *k, *v, *g, *beta, *state_in;
  const int64_t *cu_seqlens;
  int64_t n_seq, hk, hv, dk, dv;
  int g_is_log;
  float *y, *state_out;
  int64_t next; /* next unit to take, guarded by lock */
  int failed;
  pthread_mutex_t lock;
} scan_job;

static void scan_unit(scan_job *J, int64_t u, double *S, double *r) {
  const int64_t hv = J->hv, hk = J->hk, dk = J->dk, dv = J->dv;
  const int64_t b = u / hv, h = u % hv, kh = h / (hv / hk);
  const float *s0 = J->state_in + (b * hv + h) * dv * dk;
  for (int64_t i = 0; i < dv * dk; ++i) S[i] = (double)s0[i];
  for (int64_t t = J->cu_seqlens[b]; t < J->cu_seqlens[b + 1]; ++t) {
    const float *qt = J->q + (t * hk + kh) * dk;
    const float *kt = J->k + (t * hk + kh) * dk;
    const float *vt = J->v + (t * hv + h) * dv;
    double gt = (double)J->g[t * hv + h];
    if (J->g_is_log) gt = exp(gt);
    const double bt = (double)J->beta[t * hv + h];
    /* S *= g; r = S k */
    for (int64_t i = 0; i < dv; ++i) {
      double acc = 0.0;
      double *row = S + i * dk;
      for (int64_t j = 0; j < dk; ++j) {
        row[j] *= gt;
        acc += row[j] * (double)kt[j];
      }
      r[i] = acc;
    }
    /* d = beta (v - r); S += d k^T; y = S q */
    for (int64_t i = 0; i < dv; ++i) {
      const double d = ((double)vt[i] - r[i]) * bt;
      double acc = 0.0;
      double *row = S + i * dk;
      for (int64_t j = 0; j < dk; ++j) {
        row[j] += (double)kt[j] * d;
        acc += row[j] * (double)qt[j];
      }
      J->y[(t * hv + h) * dv + i] = (float)acc;
    }
  }
  float *s1 = J->state_out + (b * hv + h) * dv * dk;
  for (int64_t i = 0; i < dv * dk; ++i) s1[i] = (float)S[i];
}

static void *scan_worker(void *arg) {
  scan_job *J = (scan_job *)arg;
  double *S = (double *)malloc(sizeof(double) * (size_t)(J->dv * J->dk));
  double *r = (double *)malloc(sizeof(double) * (size_t)J->dv);
  const int64_t units = J->n_seq * J->hv;
  for (;;) {
    pthread_mutex_lock(&J->lock);
    const int64_t u = J->next++;
    if (!S || !r) J->failed = 1;
    pthread_mutex_unlock(&J->lock);
    if (u >= units || !S || !r) break;
    scan_unit(J, u, S, r);
  }
  free(S);
  free(r);
  return NULL;
}

int gdn_oracle_scan_varlen(const float *q, const float *k, const float *v,
                           const float *g, const float *beta,
                           const int64_t *cu_seqlens, int64_t n_seq,
                           int64_t hk, int64_t hv, int64_t dk, int64_t dv,
                           int g_is_log, const float *state_in,
                           float *y, float *state_out, int n_threads) {
  if (hk <= 0 || hv <= 0 || dk <= 0 || dv <= 0 || hv % hk || n_seq < 0) return 1;
  if (n_threads < 1) n_threads = 1;
  if (n_threads > 256) n_threads = 256;
  scan_job J = {q, k, v, g, beta, state_in, cu_seqlens, n_seq, hk, hv, dk, dv,
                g_is_log, y, state_out, 0, 0, PTHREAD_MUTEX_INITIALIZER};
  pthread_t tid[256];
  int started = 0;
  for (int i = 0; i < n_threads; ++i) {
    if (pthread_create(&tid[i], NULL, scan_worker, &J) != 0) break;
    ++started;
  }
  if (started == 0) scan_worker(&J);
  for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
  return J.failed ? 2 : 0;
}
