// K10 — DSpark Markov head with greedy block sampling.
//
// Reference: DSparkDrafter.sample_block (src/mlx_dspark/model.py:398-409), batched form
// _batched_sample_block (src/mlx_dspark/batch_engine.py:414-428), VanillaMarkov
// (model.py:324-336):
//   for i in range(cap): logits_i = base_i + w2(w1[prev]); prev = argmax(logits_i)
// One launch per position i: every CTA computes the Markov bias over a vocabulary slice for
// all rows (one pass over the W8 w2 matrix, which stays L2-resident across the cap steps),
// adds the base logits and keeps a per-slice argmax; the last CTA to finish reduces the
// slices in CTA order and publishes the token that the next launch conditions on.
// Rounding follows a bf16 model: e = bf16(dequant w1[prev]); bias = bf16(w2 . e);
// logit = bf16(base + bias); argmax takes the first index of the maximum.
#include "common.cuh"

namespace dspark {
namespace mk {

constexpr int kThreads = 256;
constexpr int kMaxB = 8;
constexpr int kR = 256;  // Markov rank

struct Best {
  float v;
  int i;
};
__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__global__ void __launch_bounds__(kThreads) markov_step_kernel(
    const __nv_bfloat16* __restrict__ base, int ld, int rows_per_b, int B, int cap, int V, int step,
    const uint8_t* __restrict__ w1q, const uint32_t* __restrict__ w1sb,
    const uint8_t* __restrict__ w2q, const uint32_t* __restrict__ w2sb,
    const int32_t* __restrict__ first_prev, int32_t* __restrict__ draft,
    int32_t* __restrict__ verify_ids, float* __restrict__ part_v, int* __restrict__ part_i,
    int* __restrict__ counter) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float e[kMaxB][kR];
  __shared__ Best red[kMaxB][kThreads / 32];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // e_b = bf16(dequant w1[prev_b])
  for (int idx = threadIdx.x; idx < B * kR; idx += kThreads) {
    const int b = idx / kR, r = idx - b * kR;
    int prev = step == 0 ? first_prev[b] : draft[b * cap + step - 1];
    prev = prev < 0 ? 0 : (prev >= V ? V - 1 : prev);
    const uint32_t sbv = w1sb[(size_t)(r >> 6) * V + prev];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    e[b][r] = bf16_round(fmaf(__low2float(sb), (float)w1q[(size_t)prev * kR + r], __high2float(sb)));
  }
  __syncthreads();
  const int chunk = (V + gridDim.x - 1) / gridDim.x;
  const int v0 = blockIdx.x * chunk, v1 = min(V, v0 + chunk);
  Best best[kMaxB];
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) best[b] = Best{-INFINITY, 0x7fffffff};
  // one warp per vocabulary row: lane l covers dims [8l, 8l+8) (group l/8)
  for (int v = v0 + warp; v < v1; v += kThreads / 32) {
    const uint2 q8 = *reinterpret_cast<const uint2*>(w2q + (size_t)v * kR + lane * 8);
    const uint32_t sbv = w2sb[(size_t)(lane >> 3) * V + v];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    const float s = __low2float(sb), bb = __high2float(sb);
    float w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = fmaf(s, (float)(((j < 4 ? q8.x : q8.y) >> (8 * (j & 3))) & 0xFF), bb);
#pragma unroll
    for (int b = 0; b < kMaxB; ++b) {
      if (b >= B) break;
      float d = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) d += w[j] * e[b][lane * 8 + j];
      d = warp_sum(d);
      const float logit =
          bf16_round(__bfloat162float(base[(size_t)(b * rows_per_b + step) * ld + v]) + bf16_round(d));
      best[b] = better(best[b], Best{logit, v});
    }
  }
#pragma unroll
  for (int b = 0; b < kMaxB; ++b) {
    if (b >= B) break;
    if (lane == 0) red[b][warp] = best[b];
  }
  __syncthreads();
  if (threadIdx.x < B) {
    const int b = threadIdx.x;
    Best t = red[b][0];
    for (int w = 1; w < kThreads / 32; ++w) t = better(t, red[b][w]);
    part_v[(size_t)blockIdx.x * B + b] = t.v;
    part_i[(size_t)blockIdx.x * B + b] = t.i;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (threadIdx.x < B) {
    const int b = threadIdx.x;
    Best t{-INFINITY, 0x7fffffff};
    for (int c = 0; c < (int)gridDim.x; ++c)
      t = better(t, Best{__ldcg(part_v + (size_t)c * B + b), __ldcg(part_i + (size_t)c * B + b)});
    if (t.i == 0x7fffffff) t.i = 0;
    draft[b * cap + step] = t.i;
    if (verify_ids) {
      if (step == 0) verify_ids[b * (cap + 1)] = first_prev[b];
      verify_ids[b * (cap + 1) + 1 + step] = t.i;
    }
  }
  if (threadIdx.x == 0) *counter = 0;
}

static size_t ws(int B, int V, int* grid_out, size_t* off_i, size_t* off_c) {
  int grid = 2 * 148;
  if (V / grid < 64) grid = (V + 63) / 64;
  if (grid_out) *grid_out = grid;
  // counter word first (fixed offset for every shape), then the two partial arrays
  const size_t pv = (((size_t)grid * B * 4) + 255) & ~(size_t)255;
  if (off_c) *off_c = 256;           // start of the value partials
  if (off_i) *off_i = 256 + pv;      // start of the index partials
  return 256 + 2 * pv;
}

}  // namespace mk
}  // namespace dspark

using namespace dspark;

extern "C" size_t dspark_markov_workspace_bytes(int B, int V) {
  if (B <= 0 || V <= 0) return 0;
  return mk::ws(B, V, nullptr, nullptr, nullptr);
}

extern "C" int dspark_markov_sample_block(const void* base, int ld, int rows_per_b, int B, int cap,
                                          int V, int R,
                                          const uint8_t* w1q, const uint32_t* w1sb,
                                          const uint8_t* w2q, const uint32_t* w2sb,
                                          const int32_t* first_prev, int32_t* draft,
                                          int32_t* verify_ids, void* workspace,
                                          size_t workspace_bytes, int* status,
                                          dspark_stream_t stream) {
  (void)status;
  if (!base || !w1q || !w1sb || !w2q || !w2sb || !first_prev || !draft || B <= 0 || cap <= 0 ||
      V <= 0 || ld < V)
    return set_error(DSPARK_ERR_INVALID, "markov_sample_block: bad arguments");
  if (R != mk::kR) return set_error(DSPARK_ERR_UNSUPPORTED, "markov_sample_block: rank %d != 256", R);
  if (B > mk::kMaxB) return set_error(DSPARK_ERR_UNSUPPORTED, "markov_sample_block: B > %d", mk::kMaxB);
  int grid;
  size_t off_i, off_c;
  const size_t need = mk::ws(B, V, &grid, &off_i, &off_c);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "markov_sample_block: workspace %zu < %zu", workspace_bytes, need);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < cap; ++i) {
    int rc = launch_pdl("markov_step", mk::markov_step_kernel, dim3(grid), dim3(mk::kThreads), 0, st,
                        static_cast<const __nv_bfloat16*>(base), ld, rows_per_b, B, cap, V, i, w1q, w1sb, w2q,
                        w2sb, first_prev, draft, verify_ids, reinterpret_cast<float*>(w + off_c),
                        reinterpret_cast<int*>(w + off_i), reinterpret_cast<int*>(w));
    if (rc) return rc;
  }
  return DSPARK_OK;
}
