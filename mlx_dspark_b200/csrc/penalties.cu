// R8 — OpenAI presence / frequency penalties on the verify logits, and the running
// completion-token counts they read.
//
// Reference: _Penalizer (src/mlx_dspark/generate.py:179-228). Row i of a verify block
// [pending, d_1..d_L] is penalized by the completion counts plus the block's own draft prefix
// d_1..d_i: for token v with c = counts[v],
//   pen = c > 0 ? bf16(P + bf16(F * bf16(c))) : 0
//   then for each j < i with d_{j+1} == v: pen = bf16(pen + bf16(F + (seen ? 0 : P))), seen++
//   logit' = bf16(logit - pen)           (unchanged where pen == 0)
// where P, F are the penalties rounded to bf16 (MLX casts a Python scalar to the array dtype)
// and every operation rounds to bf16 as MLX's bf16 arithmetic does. The counts advance by the
// committed tokens of each round (pen.add, generate.py:941-949), read from the acceptance plan.
#include "common.cuh"

namespace dspark {
namespace pen {

constexpr int kThreads = 256;
constexpr int kMaxT = 64;

__global__ void __launch_bounds__(kThreads) apply_kernel(
    __nv_bfloat16* __restrict__ logits, long long ld, int T, int V,
    const int32_t* __restrict__ counts, const int32_t* __restrict__ verify_ids, float P, float F,
    float inc_new, float inc_seen) {
  pdl_enter();
  const int b = blockIdx.y;
  __shared__ int draft[kMaxT];
  for (int i = threadIdx.x; i < T - 1; i += kThreads) draft[i] = verify_ids[(size_t)b * T + 1 + i];
  __syncthreads();
  const int32_t* cnt = counts + (size_t)b * V;
  for (int v = blockIdx.x * kThreads + threadIdx.x; v < V; v += gridDim.x * kThreads) {
    const int c = cnt[v];
    // does v occur in the draft at all? (most tokens: no, and c == 0: nothing to do)
    bool in_draft = false;
    for (int j = 0; j < T - 1; ++j) in_draft |= draft[j] == v;
    if (c == 0 && !in_draft) continue;
    float pen = c > 0 ? bf16_round(P + bf16_round(F * bf16_round((float)c))) : 0.0f;
    int seen = c;
    for (int i = 0; i < T; ++i) {
      if (i > 0 && draft[i - 1] == v) {
        pen = bf16_round(pen + (seen == 0 ? inc_new : inc_seen));
        ++seen;
      }
      if (pen != 0.0f) {
        __nv_bfloat16* p = logits + ((size_t)b * T + i) * ld + v;
        *p = __float2bfloat16_rn(__bfloat162float(*p) - pen);
      }
    }
  }
}

// counts[b][tok] += 1 for the committed tokens plan[b][2 .. 2 + plan[b][1])
__global__ void counts_add_kernel(int32_t* __restrict__ counts, int V,
                                  const int32_t* __restrict__ plan, int plan_stride) {
  pdl_enter();
  const int b = blockIdx.x;
  const int32_t* pl = plan + (size_t)b * plan_stride;
  const int cnt = pl[1];
  for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
    const int t = pl[2 + i];
    if (t >= 0 && t < V) atomicAdd(counts + (size_t)b * V + t, 1);
  }
}

float bf16_host(double x) {
  float f = (float)x;
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return f;
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  memcpy(&f, &u, 4);
  return f;
}

}  // namespace pen
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_apply_penalties(void* logits, long long ld, int B, int T, int V,
                                      const int32_t* counts, const int32_t* verify_ids,
                                      double presence, double frequency, dspark_stream_t stream) {
  if (!logits || !counts || B <= 0 || T <= 0 || V <= 0 || ld < V || (T > 1 && !verify_ids))
    return set_error(DSPARK_ERR_INVALID, "apply_penalties: bad arguments");
  if (T > pen::kMaxT) return set_error(DSPARK_ERR_UNSUPPORTED, "apply_penalties: T > %d", pen::kMaxT);
  if (B > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "apply_penalties: B too large");
  const float P = pen::bf16_host(presence), F = pen::bf16_host(frequency);
  // the increments are Python-float sums rounded to bf16 when added to a bf16 row
  const float inc_new = pen::bf16_host(frequency + presence), inc_seen = pen::bf16_host(frequency);
  int grid = (V + pen::kThreads * 4 - 1) / (pen::kThreads * 4);
  if (grid < 1) grid = 1;
  return launch_pdl("apply_penalties", pen::apply_kernel, dim3(grid, B), dim3(pen::kThreads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(logits), ld, T,
                    V, counts, verify_ids, P, F, inc_new, inc_seen);
}

extern "C" int dspark_penalty_counts_add(int32_t* counts, int B, int V, const int32_t* plan,
                                         int plan_stride, dspark_stream_t stream) {
  if (!counts || !plan || B <= 0 || V <= 0 || plan_stride < 3)
    return set_error(DSPARK_ERR_INVALID, "penalty_counts_add: bad arguments");
  return launch_pdl("penalty_counts_add", pen::counts_add_kernel, dim3(B), dim3(64), 0,
                    static_cast<cudaStream_t>(stream), counts, V, plan, plan_stride);
}
