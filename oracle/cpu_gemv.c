/* CPU W8 group-64 matrix-vector product for the timed CPU baseline.
 * TEST / BENCHMARK INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and --impl reference
 * call it through oracle/cpu_baseline.py; no product code links it.
 *
 * The reference's per-token work on its MLX CPU backend is dominated by quantized
 * matrix-vector products (mlx QuantizedLinear, bits 8, group 64, under
 * src/mlx_dspark/target.py:58-75 for greedy_generate, src/mlx_dspark/generate.py:433-450).
 * MLX's CPU qmv reads each int8 weight once and applies the group's scale and bias to the
 * group's partial dot product. This restates that loop in plain C:
 *   y[n] = sum_g ( scale[n,g] * sum_{k in g} q[n,k] * x[k] + bias[n,g] * sum_{k in g} x[k] )
 * with fp32 arithmetic, each group's dot product in AVX2 (x86-64-v3, the build's target).
 * Rows are split over a persistent pool of POSIX threads (the image's gcc has no OpenMP
 * runtime); scales and biases are bf16 bit patterns (the checkpoint format), weights uint8
 * row-major [N, K], K a multiple of 64. */
#include <immintrin.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

typedef struct {
  const uint8_t* q;
  const uint16_t* scales;
  const uint16_t* biases;
  const float* x;
  const float* xs;
  float* y;
  int N, K;
  int T; /* slices: the caller and T - 1 workers */
} job_t;

static inline float hsum8(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(s);
}

/* One group of 64: 16 codes per load widened to two 8-lane fp32 vectors (AVX2), two
   accumulators, one horizontal sum. */
static inline float group_dot(const uint8_t* qg, const float* xg) {
  __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
  for (int k = 0; k < 64; k += 16) {
    const __m128i b = _mm_loadu_si128((const __m128i*)(qg + k));
    const __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(b));
    const __m256 w1 = _mm256_cvtepi32_ps(_mm256_cvtepu8_epi32(_mm_srli_si128(b, 8)));
    a0 = _mm256_fmadd_ps(w0, _mm256_loadu_ps(xg + k), a0);
    a1 = _mm256_fmadd_ps(w1, _mm256_loadu_ps(xg + k + 8), a1);
  }
  return hsum8(_mm256_add_ps(a0, a1));
}

static void rows(const job_t* j, int n0, int n1) {
  const int G = j->K / 64;
  for (int n = n0; n < n1; ++n) {
    const uint8_t* qr = j->q + (size_t)n * j->K;
    const uint16_t* sr = j->scales + (size_t)n * G;
    const uint16_t* br = j->biases + (size_t)n * G;
    float acc = 0.0f;
    for (int g = 0; g < G; ++g)
      acc += bf16_to_f32(sr[g]) * group_dot(qr + g * 64, j->x + g * 64) +
             bf16_to_f32(br[g]) * j->xs[g];
    j->y[n] = acc;
  }
}

/* ---- persistent pool: worker w handles rows [(w+1)*N/T, (w+2)*N/T) of each published job,
   the caller rows [0, N/T). A decode step is ~250 back-to-back products of 1-50 MB, so waking
   sleeping threads per call (a futex wake and a reschedule each, hundreds of microseconds on
   a virtual machine) would cost as much as the products: workers spin on the job counter for
   a few milliseconds before sleeping on the condition variable, and the caller spins on the
   count of unfinished slices. ---- */
#define MAX_THREADS 256
#define SPIN_LIMIT 200000
static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t go = PTHREAD_COND_INITIALIZER;
static job_t cur;                      /* written before gen is released, read after */
static _Atomic unsigned long gen = 0;  /* job counter */
static _Atomic int pending = 0;        /* worker slices of the current job not yet done */
static int nworkers = 0;
static unsigned long start_gen[MAX_THREADS]; /* job counter when worker w was started */

static void* worker(void* arg) {
  const int w = (int)(intptr_t)arg;
  unsigned long seen = start_gen[w];  /* jobs published before it started are not its own */
  for (;;) {
    unsigned long g;
    int spins = 0;
    while ((g = atomic_load_explicit(&gen, memory_order_acquire)) == seen) {
      if (++spins < SPIN_LIMIT) {
        _mm_pause();
        continue;
      }
      pthread_mutex_lock(&mu);
      while (atomic_load_explicit(&gen, memory_order_acquire) == seen) pthread_cond_wait(&go, &mu);
      pthread_mutex_unlock(&mu);
      spins = 0;
    }
    seen = g;
    const job_t j = cur;
    rows(&j, (int)((long long)(w + 1) * j.N / j.T), (int)((long long)(w + 2) * j.N / j.T));
    atomic_fetch_sub_explicit(&pending, 1, memory_order_acq_rel);
  }
  return NULL;
}

/* the calling thread takes slice 0; threads - 1 workers are started on first use */
static void ensure_pool(int threads) {
  if (threads > MAX_THREADS) threads = MAX_THREADS;
  while (nworkers < threads - 1) {
    pthread_t t;
    start_gen[nworkers] = atomic_load_explicit(&gen, memory_order_relaxed);
    if (pthread_create(&t, NULL, worker, (void*)(intptr_t)nworkers) != 0) break;
    pthread_detach(t);
    ++nworkers;
  }
}

void dspark_cpu_w8_gemv(const uint8_t* q, const uint16_t* scales, const uint16_t* biases,
                        const float* x, float* y, int N, int K, float* xs_scratch, int threads) {
  for (int g = 0; g < K / 64; ++g) {
    float s = 0.0f;
    for (int k = 0; k < 64; ++k) s += x[g * 64 + k];
    xs_scratch[g] = s;
  }
  /* workers are only started between jobs (none is running one now) */
  ensure_pool(threads);
  const int T = nworkers + 1;
  job_t j = {q, scales, biases, x, xs_scratch, y, N, K, T};
  cur = j;
  atomic_store_explicit(&pending, nworkers, memory_order_relaxed);
  pthread_mutex_lock(&mu);
  atomic_fetch_add_explicit(&gen, 1, memory_order_release);
  pthread_cond_broadcast(&go);
  pthread_mutex_unlock(&mu);
  rows(&j, 0, (int)((long long)N / T));
  while (atomic_load_explicit(&pending, memory_order_acquire) > 0) _mm_pause();
}

int dspark_cpu_pool_threads(void) { return nworkers + 1; }
