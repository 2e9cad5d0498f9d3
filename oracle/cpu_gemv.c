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
 * with fp32 arithmetic. Rows are split over a persistent pool of POSIX threads (the image's
 * gcc has no OpenMP runtime); scales and biases are bf16 bit patterns (the checkpoint format),
 * weights uint8 row-major [N, K], K a multiple of 64. */
#include <pthread.h>
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
} job_t;

static void rows(const job_t* j, int n0, int n1) {
  const int G = j->K / 64;
  for (int n = n0; n < n1; ++n) {
    const uint8_t* qr = j->q + (size_t)n * j->K;
    const uint16_t* sr = j->scales + (size_t)n * G;
    const uint16_t* br = j->biases + (size_t)n * G;
    float acc = 0.0f;
    for (int g = 0; g < G; ++g) {
      const uint8_t* qg = qr + g * 64;
      const float* xg = j->x + g * 64;
      /* eight independent lanes (one 8-wide vector): the compiler keeps each lane's sum in
         order, so it vectorises without reassociating */
      float d8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < 64; k += 8)
        for (int l = 0; l < 8; ++l) d8[l] += (float)qg[k + l] * xg[k + l];
      const float d = ((d8[0] + d8[1]) + (d8[2] + d8[3])) + ((d8[4] + d8[5]) + (d8[6] + d8[7]));
      acc += bf16_to_f32(sr[g]) * d + bf16_to_f32(br[g]) * j->xs[g];
    }
    j->y[n] = acc;
  }
}

/* ---- persistent pool: worker w handles rows [w*N/T, (w+1)*N/T) of each published job ---- */
#define MAX_THREADS 256
static pthread_mutex_t mu = PTHREAD_MUTEX_INITIALIZER;
static pthread_cond_t go = PTHREAD_COND_INITIALIZER, done = PTHREAD_COND_INITIALIZER;
static job_t cur;
static unsigned long gen = 0;
static int nworkers = 0, pending = 0;

static void* worker(void* arg) {
  const int w = (int)(intptr_t)arg;
  unsigned long seen = 0;
  for (;;) {
    pthread_mutex_lock(&mu);
    while (gen == seen) pthread_cond_wait(&go, &mu);
    seen = gen;
    const job_t j = cur;
    const int T = nworkers + 1;
    pthread_mutex_unlock(&mu);
    rows(&j, (int)((long long)(w + 1) * j.N / T), (int)((long long)(w + 2) * j.N / T));
    pthread_mutex_lock(&mu);
    if (--pending == 0) pthread_cond_signal(&done);
    pthread_mutex_unlock(&mu);
  }
  return NULL;
}

/* the calling thread takes slice 0; threads - 1 workers are started on first use */
static void ensure_pool(int threads) {
  if (threads > MAX_THREADS) threads = MAX_THREADS;
  while (nworkers < threads - 1) {
    pthread_t t;
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
  job_t j = {q, scales, biases, x, xs_scratch, y, N, K};
  pthread_mutex_lock(&mu);
  ensure_pool(threads);
  const int T = nworkers + 1;
  cur = j;
  pending = nworkers;
  ++gen;
  pthread_cond_broadcast(&go);
  pthread_mutex_unlock(&mu);
  rows(&j, 0, (int)((long long)N / T));
  pthread_mutex_lock(&mu);
  while (pending > 0) pthread_cond_wait(&done, &mu);
  pthread_mutex_unlock(&mu);
}

int dspark_cpu_pool_threads(void) { return nworkers + 1; }
