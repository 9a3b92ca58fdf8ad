/* CPU restatement of the reference's fastest CPU product for a quantized layer (TEST INFRASTRUCTURE: it is the
 * timed CPU baseline of bench.py and a checker in tests/, never part of the product).
 *
 * Reference: ATECTechnologies/apsi, apsi/hub_cpu.py
 *   - the Q8_0 row kernel `apsi_hub_q8_rows` (hub_cpu.py:96-167): for every output row o in [o0, o1) and every
 *     token t, a 32-lane float32 accumulator walks the 32-value blocks b of the row and adds
 *     (float(int8 code) * x) * s[o, b] with one fused multiply-add per lane; the 32 lanes are then summed
 *     (fast-math horizontal reduction) into Y[t, O-major];
 *   - the row split of `matmul` (hub_cpu.py:474-534): parts = max(1, min(threads, O / 64)), a step of
 *     ceil(O / parts) rows rounded up to a multiple of 16, one part per worker of its native thread team
 *     (hub_cpu.py:404-471).  Here the team is a pool of POSIX threads that persists between calls, as the
 *     reference's does: workers spin on a generation counter for a while after a job (the reference spins
 *     APSI_HUB_SPIN iterations), then sleep on a condition variable; parts are handed out with an atomic counter
 *     and the caller works on them too.
 *
 * The Q8_0 layout is the reference's `Q8` (hub_cpu.py:170-194): int8 codes [O, I], one float32 scale per 32
 * values [O, I / 32].  The arithmetic order inside a block differs from the reference's only through the
 * fast-math reassociation both allow, so results agree to float32 rounding, not bit for bit.
 *
 * Built by oracle/Makefile with gcc -O3 -ffast-math -pthread.  The row kernel exists for AVX-512, AVX2 + FMA
 * and any CPU; the widest one the CPU supports is chosen at the first call, as the reference's JIT compiles for
 * the host CPU.
 */
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <unistd.h>

#define QB 32

/* Portable row kernel (any target). */
static void q8_rows_generic(const int8_t* __restrict W, const float* __restrict S, const float* __restrict X,
                            float* __restrict Y, int64_t o0, int64_t o1, int64_t I, int64_t T, int64_t O) {
  const int64_t nb = I / QB;
  for (int64_t o = o0; o < o1; ++o) {
    const int8_t* w = W + o * I;
    const float* s = S + o * nb;
    for (int64_t t = 0; t < T; ++t) {
      const float* x = X + t * I;
      float acc[QB] = {0};
      for (int64_t b = 0; b < nb; ++b)
        for (int j = 0; j < QB; ++j) acc[j] = fmaf((float)w[b * QB + j] * x[b * QB + j], s[b], acc[j]);
      float tot = 0.f;
      for (int j = 0; j < QB; ++j) tot += acc[j];
      Y[t * O + o] = tot;
    }
  }
}

#if defined(__x86_64__) && defined(__GNUC__)
#include <immintrin.h>
/* AVX2 + FMA: the 32 lanes as four 8-float registers; codes sign-extended 8 at a time. */
__attribute__((target("avx2,fma"))) static void q8_rows_avx2(const int8_t* __restrict W, const float* __restrict S,
                                                              const float* __restrict X, float* __restrict Y,
                                                              int64_t o0, int64_t o1, int64_t I, int64_t T,
                                                              int64_t O) {
  const int64_t nb = I / QB;
  for (int64_t o = o0; o < o1; ++o) {
    const int8_t* w = W + o * I;
    const float* s = S + o * nb;
    for (int64_t t = 0; t < T; ++t) {
      const float* x = X + t * I;
      __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps(), a2 = _mm256_setzero_ps(), a3 = _mm256_setzero_ps();
      for (int64_t b = 0; b < nb; ++b) {
        const __m256 sc = _mm256_broadcast_ss(s + b);
        const int8_t* wb = w + b * QB;
        const float* xb = x + b * QB;
        const __m128i c01 = _mm_loadu_si128((const __m128i*)wb), c23 = _mm_loadu_si128((const __m128i*)(wb + 16));
        const __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(c01));
        const __m256 w1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(c01, 8)));
        const __m256 w2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(c23));
        const __m256 w3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(_mm_srli_si128(c23, 8)));
        a0 = _mm256_fmadd_ps(_mm256_mul_ps(w0, _mm256_loadu_ps(xb)), sc, a0);
        a1 = _mm256_fmadd_ps(_mm256_mul_ps(w1, _mm256_loadu_ps(xb + 8)), sc, a1);
        a2 = _mm256_fmadd_ps(_mm256_mul_ps(w2, _mm256_loadu_ps(xb + 16)), sc, a2);
        a3 = _mm256_fmadd_ps(_mm256_mul_ps(w3, _mm256_loadu_ps(xb + 24)), sc, a3);
      }
      const __m256 a = _mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3));
      __m128 h = _mm_add_ps(_mm256_castps256_ps128(a), _mm256_extractf128_ps(a, 1));
      h = _mm_add_ps(h, _mm_movehl_ps(h, h));
      h = _mm_add_ss(h, _mm_shuffle_ps(h, h, 1));
      Y[t * O + o] = _mm_cvtss_f32(h);
    }
  }
}

/* AVX-512: the 32 lanes as two 16-float registers. */
__attribute__((target("avx512f"))) static void q8_rows_avx512(const int8_t* __restrict W, const float* __restrict S,
                                                              const float* __restrict X, float* __restrict Y,
                                                              int64_t o0, int64_t o1, int64_t I, int64_t T,
                                                              int64_t O) {
  const int64_t nb = I / QB;
  for (int64_t o = o0; o < o1; ++o) {
    const int8_t* w = W + o * I;
    const float* s = S + o * nb;
    for (int64_t t = 0; t < T; ++t) {
      const float* x = X + t * I;
      __m512 a0 = _mm512_setzero_ps(), a1 = _mm512_setzero_ps();
      for (int64_t b = 0; b < nb; ++b) {
        const __m512 sc = _mm512_set1_ps(s[b]);
        const int8_t* wb = w + b * QB;
        const float* xb = x + b * QB;
        const __m512 w0 = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i*)wb)));
        const __m512 w1 = _mm512_cvtepi32_ps(_mm512_cvtepi8_epi32(_mm_loadu_si128((const __m128i*)(wb + 16))));
        a0 = _mm512_fmadd_ps(_mm512_mul_ps(w0, _mm512_loadu_ps(xb)), sc, a0);
        a1 = _mm512_fmadd_ps(_mm512_mul_ps(w1, _mm512_loadu_ps(xb + 16)), sc, a1);
      }
      Y[t * O + o] = _mm512_reduce_add_ps(_mm512_add_ps(a0, a1));
    }
  }
}
#endif

typedef void (*rows_fn)(const int8_t*, const float*, const float*, float*, int64_t, int64_t, int64_t, int64_t,
                        int64_t);

/* The widest kernel this CPU runs, as the reference's JIT targets the host CPU. */
static rows_fn pick_rows(void) {
#if defined(__x86_64__) && defined(__GNUC__)
  __builtin_cpu_init();
  if (__builtin_cpu_supports("avx512f")) return q8_rows_avx512;
  if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) return q8_rows_avx2;
#endif
  return q8_rows_generic;
}

static rows_fn q8_rows_fn;

static void q8_rows(const int8_t* W, const float* S, const float* X, float* Y, int64_t o0, int64_t o1, int64_t I,
                    int64_t T, int64_t O) {
  q8_rows_fn(W, S, X, Y, o0, o1, I, T, O);
}

/* Which kernel runs: 512, 256 or 0 (portable). */
int hub_q8_isa(void) {
  if (!q8_rows_fn) q8_rows_fn = pick_rows();
#if defined(__x86_64__) && defined(__GNUC__)
  if (q8_rows_fn == q8_rows_avx512) return 512;
  if (q8_rows_fn == q8_rows_avx2) return 256;
#endif
  return 0;
}

/* ------------------------------------------------------------------------------------------- thread team */
struct job {
  const int8_t* W;
  const float* S;
  const float* X;
  float* Y;
  int64_t I, T, O, step, parts;
};

static struct {
  pthread_mutex_t mu;
  pthread_cond_t cv;
  int n;                     /* workers (threads besides the caller) */
  atomic_long gen;           /* job generation */
  atomic_long next;          /* next part to take */
  atomic_long done;          /* parts finished */
  struct job job;
  pthread_t tid[256];
} team = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, 0};

static void run_parts(void) {
  const struct job* j = &team.job;
  for (;;) {
    const long p = atomic_fetch_add(&team.next, 1);
    if (p >= j->parts) return;
    const int64_t a = p * j->step;
    const int64_t e = a + j->step < j->O ? a + j->step : j->O;
    q8_rows(j->W, j->S, j->X, j->Y, a, e, j->I, j->T, j->O);
    atomic_fetch_add(&team.done, 1);
  }
}

static void* worker(void* arg) {
  (void)arg;
  long seen = atomic_load(&team.gen);
  for (;;) {
    long g;
    int spins = 0;
    while ((g = atomic_load(&team.gen)) == seen && spins < 4000000) {
      ++spins;
      if ((spins & 65535) == 0) sched_yield();
    }
    if (g == seen) {
      pthread_mutex_lock(&team.mu);
      while ((g = atomic_load(&team.gen)) == seen) pthread_cond_wait(&team.cv, &team.mu);
      pthread_mutex_unlock(&team.mu);
    }
    seen = g;
    run_parts();
  }
  return NULL;
}

static void ensure_team(int workers) {
  if (workers > 256) workers = 256;
  while (team.n < workers) {
    if (pthread_create(&team.tid[team.n], NULL, worker, NULL) != 0) break;
    pthread_detach(team.tid[team.n]);
    ++team.n;
  }
}

/* Y[T, O] = X[T, I] . deq(W)[O, I]^T on `threads` threads (0: every CPU this process may use).  I % 32 == 0.
 * One call at a time.  Returns the number of parts the rows were split into. */
int hub_q8_matmul(const int8_t* W, const float* S, const float* X, float* Y, int64_t I, int64_t T, int64_t O,
                  int threads) {
  if (!q8_rows_fn) q8_rows_fn = pick_rows();
  if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (threads < 1) threads = 1;
  int64_t parts = O / 64 ? O / 64 : 1;
  if (parts > threads) parts = threads;
  if (parts == 1) {
    q8_rows(W, S, X, Y, 0, O, I, T, O);
    return 1;
  }
  int64_t step = (O + parts - 1) / parts;
  step = (step + 15) / 16 * 16;
  parts = (O + step - 1) / step;
  ensure_team(threads - 1);
  struct job j = {W, S, X, Y, I, T, O, step, parts};
  pthread_mutex_lock(&team.mu);
  team.job = j;
  atomic_store(&team.next, 0);
  atomic_store(&team.done, 0);
  atomic_fetch_add(&team.gen, 1);
  pthread_cond_broadcast(&team.cv);
  pthread_mutex_unlock(&team.mu);
  run_parts();
  while (atomic_load(&team.done) < parts) {
  }
  return (int)parts;
}
