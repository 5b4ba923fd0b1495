/*
 * gdn_oracle.c — TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference's
 * gated delta-rule recurrence, used as the parity checker for the CUDA path
 * and as the timed CPU baseline.  The product never links or calls this file.
 *
 * Restated from (paths inside baladithyab/cuda-oxide-bench):
 *   gdn_step   <- gdn_decode_reference
 *                 analysis/wave15-attention-architecture/reference/pytorch_reference_gdn.py:38-91
 *                 (fp32, operation order of steps (1)-(5) there)
 *   kda_step   <- naive_recurrent_kda_step
 *                 analysis/wave15-attention-architecture/reference/pytorch_reference_kda.py:42-71
 *                 (float64, as the reference computes it)
 *   prefill    <- T sequential applications of gdn_step: the reference has no
 *                 chunked prefill (shapes_gdn.py:17-20), so the sequential
 *                 recurrence defines the result.
 * Adapters (BASELINE semantics): value head h reads q/k head h / (Hv/Hqk)
 * (== torch.repeat_interleave), alpha = exp(g) for a log gate, q scaled by
 * `scale` before the output contraction (pytorch_reference_kda.py:58).
 *
 * Parallelism: pthreads over (batch, head) pairs; each pair's arithmetic is
 * sequential in k, so the result is independent of the thread count.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static int g_threads = 0; /* 0: all online CPUs */

int oracle_num_threads(void) {
  if (g_threads > 0) return g_threads;
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

void oracle_set_num_threads(int n) { g_threads = n > 0 ? n : 0; }

typedef void (*pair_fn)(long bh, void* ctx, void* scratch);

typedef struct {
  pair_fn fn;
  void* ctx;
  long begin, end;
  size_t scratch_bytes;
} range_t;

static void* run_range(void* p) {
  range_t* r = (range_t*)p;
  void* scratch = malloc(r->scratch_bytes);
  for (long bh = r->begin; bh < r->end; ++bh) r->fn(bh, r->ctx, scratch);
  free(scratch);
  return NULL;
}

/* Static partition of [0, n) over the oracle's threads. */
static void parallel_pairs(long n, pair_fn fn, void* ctx, size_t scratch_bytes) {
  int nt = oracle_num_threads();
  if (nt > n) nt = (int)n;
  if (nt < 1) nt = 1;
  pthread_t th[256];
  range_t rs[256];
  if (nt > 256) nt = 256;
  for (int i = 0; i < nt; ++i) {
    rs[i].fn = fn;
    rs[i].ctx = ctx;
    rs[i].begin = n * i / nt;
    rs[i].end = n * (i + 1) / nt;
    rs[i].scratch_bytes = scratch_bytes;
  }
  for (int i = 1; i < nt; ++i) pthread_create(&th[i], NULL, run_range, &rs[i]);
  run_range(&rs[0]);
  for (int i = 1; i < nt; ++i) pthread_join(th[i], NULL);
}

/* One (b, h) head of gdn_decode_reference, in place on S (dk x dv, fp32).
 * work: dv floats. */
static void gdn_head_step(const float* q, const float* k, const float* v, float alpha, float beta,
                          float scale, float* S, float* o, int dk, int dv, float* u) {
  /* (1) S_scaled = alpha * S */
  for (int i = 0; i < dk * dv; ++i) S[i] = alpha * S[i];
  /* (2) u = k^T S_scaled */
  for (int j = 0; j < dv; ++j) u[j] = 0.f;
  for (int i = 0; i < dk; ++i) {
    const float ki = k[i];
    const float* row = S + (size_t)i * dv;
    for (int j = 0; j < dv; ++j) u[j] += ki * row[j];
  }
  /* (3) residual = v - u ; (4) S_out = S_scaled + beta * (k outer residual) */
  for (int j = 0; j < dv; ++j) u[j] = v[j] - u[j];
  for (int i = 0; i < dk; ++i) {
    const float ki = k[i];
    float* row = S + (size_t)i * dv;
    for (int j = 0; j < dv; ++j) row[j] = row[j] + beta * (ki * u[j]);
  }
  /* (5) o = S_out^T (scale * q) */
  for (int j = 0; j < dv; ++j) o[j] = 0.f;
  for (int i = 0; i < dk; ++i) {
    const float qi = q[i] * scale;
    const float* row = S + (size_t)i * dv;
    for (int j = 0; j < dv; ++j) o[j] += qi * row[j];
  }
}

/*
 * GDN decode over `steps` tokens, state updated in place.
 *   q, k  : [steps, B, Hqk, dk]   v, o : [steps, B, Hv, dv]
 *   gate, beta : [steps, B, Hv]   (gate_is_log: alpha = exp(gate))
 *   S     : [B, Hv, dk, dv]
 * The prefill layout [B, T, H, d] is the same loop with the token axis
 * inside the batch axis (see `time_major`).
 */
typedef struct {
  const float *q, *k, *v, *gate, *beta;
  float *S, *o;
  int steps, B, Hqk, Hv, dk, dv, gate_is_log, time_major;
  float scale;
} gdn_ctx;

static void gdn_pair(long bh, void* vctx, void* scratch) {
  const gdn_ctx* c = (const gdn_ctx*)vctx;
  const long b = bh / c->Hv;
  const int h = (int)(bh % c->Hv);
  const int hq = h / (c->Hv / c->Hqk);
  float* Sh = c->S + (size_t)bh * c->dk * c->dv;
  for (int t = 0; t < c->steps; ++t) {
    /* token row index: [t][b] (decode) or [b][t] (prefill) */
    const size_t tb = c->time_major ? (size_t)t * c->B + b : (size_t)b * c->steps + t;
    const size_t qoff = (tb * c->Hqk + hq) * c->dk;
    const size_t voff = (tb * c->Hv + h) * c->dv;
    const size_t soff = tb * c->Hv + h;
    const float a = c->gate_is_log ? expf(c->gate[soff]) : c->gate[soff];
    gdn_head_step(c->q + qoff, c->k + qoff, c->v + voff, a, c->beta[soff], c->scale, Sh,
                  c->o + voff, c->dk, c->dv, (float*)scratch);
  }
}

void oracle_gdn_decode(const float* q, const float* k, const float* v, const float* gate,
                       const float* beta, float* S, float* o, int steps, int B, int Hqk, int Hv,
                       int dk, int dv, int gate_is_log, float scale) {
  gdn_ctx c = {q, k, v, gate, beta, S, o, steps, B, Hqk, Hv, dk, dv, gate_is_log, 1, scale};
  parallel_pairs((long)B * Hv, gdn_pair, &c, sizeof(float) * (size_t)dv);
}

/*
 * GDN prefill oracle: the sequential recurrence over T tokens.
 *   q, k : [B, T, Hqk, dk]  v, o : [B, T, Hv, dv]  g, beta : [B, T, Hv] (log gate)
 *   S    : [B, Hv, dk, dv] initial state in, final state out.
 */
void oracle_gdn_prefill(const float* q, const float* k, const float* v, const float* g,
                        const float* beta, float* S, float* o, int B, int T, int Hqk, int Hv,
                        int dk, int dv, float scale) {
  gdn_ctx c = {q, k, v, g, beta, S, o, T, B, Hqk, Hv, dk, dv, 1, 0, scale};
  parallel_pairs((long)B * Hv, gdn_pair, &c, sizeof(float) * (size_t)dv);
}

/*
 * KDA decode over `steps` tokens in float64 (naive_recurrent_kda_step).
 *   q, k : [steps, B, Hqk, dk]   g : [steps, B, Hv, dk] (log gate)
 *   v, o : [steps, B, Hv, dv]    beta : [steps, B, Hv]
 *   S    : [B, Hv, dk, dv] float64, updated in place.
 */
typedef struct {
  const float *q, *k, *v, *g, *beta;
  double *S, *o;
  int steps, B, Hqk, Hv, dk, dv;
  float scale;
} kda_ctx;

static void kda_pair(long bh, void* vctx, void* scratch) {
  const kda_ctx* c = (const kda_ctx*)vctx;
  double* u = (double*)scratch;
  const int dk = c->dk, dv = c->dv;
  const long b = bh / c->Hv;
  const int h = (int)(bh % c->Hv);
  const int hq = h / (c->Hv / c->Hqk);
  double* Sh = c->S + (size_t)bh * dk * dv;
  for (int t = 0; t < c->steps; ++t) {
    const size_t tb = (size_t)t * c->B + b;
    const float* qq = c->q + (tb * c->Hqk + hq) * dk;
    const float* kk = c->k + (tb * c->Hqk + hq) * dk;
    const float* gg = c->g + (tb * c->Hv + h) * dk;
    const float* vv = c->v + (tb * c->Hv + h) * dv;
    double* oo = c->o + (tb * c->Hv + h) * dv;
    const double bt = (double)c->beta[tb * c->Hv + h];
    /* S = exp(g)[..., None] * S */
    for (int i = 0; i < dk; ++i) {
      const double e = exp((double)gg[i]);
      double* row = Sh + (size_t)i * dv;
      for (int j = 0; j < dv; ++j) row[j] *= e;
    }
    /* u = (k[..., None] * S).sum(axis=-2) ; residual = v - u */
    for (int j = 0; j < dv; ++j) u[j] = 0.0;
    for (int i = 0; i < dk; ++i) {
      const double ki = (double)kk[i];
      const double* row = Sh + (size_t)i * dv;
      for (int j = 0; j < dv; ++j) u[j] += ki * row[j];
    }
    for (int j = 0; j < dv; ++j) u[j] = (double)vv[j] - u[j];
    /* S += (beta * k)[..., None] * residual[..., None, :] */
    for (int i = 0; i < dk; ++i) {
      const double bk = bt * (double)kk[i];
      double* row = Sh + (size_t)i * dv;
      for (int j = 0; j < dv; ++j) row[j] += bk * u[j];
    }
    /* o = einsum("bhk,bhkv->bhv", q * scale, S) */
    for (int j = 0; j < dv; ++j) oo[j] = 0.0;
    for (int i = 0; i < dk; ++i) {
      const double qi = (double)qq[i] * (double)c->scale;
      const double* row = Sh + (size_t)i * dv;
      for (int j = 0; j < dv; ++j) oo[j] += qi * row[j];
    }
  }
}

void oracle_kda_decode(const float* q, const float* k, const float* v, const float* g,
                       const float* beta, double* S, double* o, int steps, int B, int Hqk, int Hv,
                       int dk, int dv, float scale) {
  kda_ctx c = {q, k, v, g, beta, S, o, steps, B, Hqk, Hv, dk, dv, scale};
  parallel_pairs((long)B * Hv, kda_pair, &c, sizeof(double) * (size_t)dv);
}
