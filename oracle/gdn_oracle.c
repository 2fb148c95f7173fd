/*
 * C restatement of the GDN decode and prefill recurrences -- TEST
 * INFRASTRUCTURE ONLY.  Built into oracle/libgdn_oracle.so by oracle/Makefile;
 * loaded by tests/ (as a second checker, cross-checked against
 * oracle/gdn_oracle.py) and by bench.py's cpu_baseline / --impl reference legs
 * as the timed CPU implementation.  The product library never links it.
 *
 * The arithmetic follows the PyTorch definitions literally:
 *   definitions/gdn/gdn_decode_qk4_v8_d128_k_last.md:91-132
 *   definitions/gdn/gdn_prefill_qk4_v8_d128_k_last.md:91-142
 * per (sequence, v-head):  old = g*S;  old_v = k.old;  new_v = beta*v + (1-beta)*old_v;
 * S' = old - k (x) old_v + k (x) new_v;  o = scale * q.S'  (S held as [V][K], k-last).
 * Independent (sequence, v-head) units are spread over POSIX threads that
 * pull unit indices from an atomic counter.
 */
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

#define HEAD 128

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* torch.nn.functional.softplus (beta=1, threshold=20) */
static inline float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

static inline void gate(float A_log, float a, float dt_bias, float b, float *g, float *beta) {
  *g = expf(-expf(A_log) * softplus_f(a + dt_bias));
  *beta = 1.0f / (1.0f + expf(-b));
}

/* One token of the recurrence on the [V][K] state S (in place); writes o[V]. */
static void step(float *S, const uint16_t *q, const uint16_t *k, const uint16_t *v, float g,
                 float beta, float scale, uint16_t *o) {
  float kf[HEAD], qf[HEAD];
  for (int i = 0; i < HEAD; ++i) {
    kf[i] = bf16_to_f32(k[i]);
    qf[i] = bf16_to_f32(q[i]);
  }
  for (int r = 0; r < HEAD; ++r) {
    float *row = S + (size_t)r * HEAD;
    float old_v = 0.0f;
    for (int c = 0; c < HEAD; ++c) {
      row[c] = g * row[c];
      old_v += kf[c] * row[c];
    }
    const float new_v = beta * bf16_to_f32(v[r]) + (1.0f - beta) * old_v;
    float acc = 0.0f;
    for (int c = 0; c < HEAD; ++c) {
      row[c] = row[c] - kf[c] * old_v + kf[c] * new_v;
      acc += qf[c] * row[c];
    }
    o[r] = f32_to_bf16(scale * acc);
  }
}

static float resolve_scale(float s) { return s == 0.0f ? 1.0f / sqrtf((float)HEAD) : s; }

typedef struct {
  const uint16_t *q, *k, *v, *a, *b;
  const float *state, *A_log, *dt_bias;
  const int64_t *cu_seqlens; /* NULL for decode */
  float scale;
  uint16_t *out;
  float *new_state;
  int64_t units, Hq, Hv;
  atomic_llong next;
} job_t;

/* decode unit bh = (batch, v-head); prefill unit nh = (sequence, v-head) */
static void run_unit(job_t *J, int64_t u) {
  const int64_t Hv = J->Hv, h = u % Hv, n = u / Hv, qh = h / (Hv / J->Hq);
  float *S = J->new_state + (size_t)u * HEAD * HEAD;
  int64_t s = n, e = n + 1; /* decode: one token, index n */
  if (J->cu_seqlens) {
    s = J->cu_seqlens[n];
    e = J->cu_seqlens[n + 1];
  }
  if (J->state == NULL || e - s <= 0)
    memset(S, 0, sizeof(float) * HEAD * HEAD);
  else if (J->state != J->new_state)
    memcpy(S, J->state + (size_t)u * HEAD * HEAD, sizeof(float) * HEAD * HEAD);
  for (int64_t t = s; t < e; ++t) {
    float g, beta;
    gate(J->A_log[h], bf16_to_f32(J->a[t * Hv + h]), J->dt_bias[h], bf16_to_f32(J->b[t * Hv + h]),
         &g, &beta);
    step(S, J->q + (t * J->Hq + qh) * HEAD, J->k + (t * J->Hq + qh) * HEAD,
         J->v + (t * Hv + h) * HEAD, g, beta, J->scale, J->out + (t * Hv + h) * HEAD);
  }
}

static void *worker(void *arg) {
  job_t *J = (job_t *)arg;
  for (;;) {
    const int64_t u = atomic_fetch_add(&J->next, 1);
    if (u >= J->units) break;
    run_unit(J, u);
  }
  return NULL;
}

static int default_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

static void run_parallel(job_t *J, int nthreads) {
  if (nthreads <= 0) nthreads = default_threads();
  if (nthreads > 512) nthreads = 512;
  if ((int64_t)nthreads > J->units) nthreads = (int)(J->units > 0 ? J->units : 1);
  atomic_store(&J->next, 0);
  pthread_t tid[512];
  int started = 0;
  for (int i = 1; i < nthreads; ++i)
    if (pthread_create(&tid[started], NULL, worker, J) == 0) ++started;
  worker(J);
  for (int i = 0; i < started; ++i) pthread_join(tid[i], NULL);
}

/* q,k [B,Hq,128] bf16; v [B,Hv,128] bf16; state/new_state [B,Hv,128,128] fp32
 * (state may be NULL = zeros; new_state may alias state); a,b [B,Hv] bf16. */
void gdn_oracle_decode(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *state,
                       const float *A_log, const uint16_t *a, const float *dt_bias,
                       const uint16_t *b, float scale, uint16_t *out, float *new_state, int64_t B,
                       int64_t Hq, int64_t Hv, int nthreads) {
  job_t J = {q, k, v, a, b, state, A_log, dt_bias, NULL, resolve_scale(scale), out, new_state,
             B * Hv, Hq, Hv, 0};
  run_parallel(&J, nthreads);
}

/* q,k [T,Hq,128]; v [T,Hv,128]; a,b [T,Hv]; cu_seqlens [N+1] int64;
 * state/new_state [N,Hv,128,128] (state may be NULL).  A sequence of length 0
 * gets a zero final state, as the definition's loop skips it (prefill def :113-114). */
void gdn_oracle_prefill(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *state,
                        const float *A_log, const uint16_t *a, const float *dt_bias,
                        const uint16_t *b, const int64_t *cu_seqlens, int64_t N, float scale,
                        uint16_t *out, float *new_state, int64_t Hq, int64_t Hv, int nthreads) {
  job_t J = {q, k, v, a, b, state, A_log, dt_bias, cu_seqlens, resolve_scale(scale), out,
             new_state, N * Hv, Hq, Hv, 0};
  run_parallel(&J, nthreads);
}

int gdn_oracle_max_threads(void) { return default_threads(); }
