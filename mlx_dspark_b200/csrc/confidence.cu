// DSpark confidence head: per drafted position, the probability that the position survives
// verification given that the prefix did.
//
// Reference (src/mlx_dspark/model.py:211-217 ConfidenceHead, :311-320 confidence_logits;
// generate.py:875-885 uses sigmoid of it):
//   feats_i = [norm(h_i), w1[prev_i]]   (the Markov embedding part when the head reads it)
//   logit_i = proj(feats_i) = w . feats_i + b;   conf_i = sigmoid(logit_i)
// with prev_0 = the pending token and prev_i = draft[i-1]. Rounding follows a bf16 model:
// norm(h) = bf16(h * rsqrt(mean(h^2) + eps) * w) (fp32 math, one rounding), the Markov
// embedding e = bf16(dequant w1[prev]) as in the Markov head, the projection accumulates in
// fp32 and rounds once with its bias, and the sigmoid is rounded to bf16.
// One CTA per position; the inputs are a few KB per position.
#include "common.cuh"

namespace dspark {
namespace conf {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < kThreads / 32 ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[kThreads / 32] = t;
  }
  __syncthreads();
  return red[kThreads / 32];
}

__global__ void __launch_bounds__(kThreads) confidence_kernel(
    const __nv_bfloat16* __restrict__ hidden, long long ld, int H,
    const __nv_bfloat16* __restrict__ norm_w, float eps, const uint8_t* __restrict__ w1q,
    const uint32_t* __restrict__ w1sb, int V, int R, const int32_t* __restrict__ first_prev,
    const int32_t* __restrict__ prev_rest, const __nv_bfloat16* __restrict__ proj_w,
    const __nv_bfloat16* __restrict__ proj_b, float* __restrict__ logit_out,
    float* __restrict__ conf_out) {
  pdl_enter();
  __shared__ float red[kThreads / 32 + 1];
  const int i = blockIdx.x;
  const __nv_bfloat16* x = hidden + (size_t)i * ld;
  float r = 1.0f;
  if (norm_w) {
    float ss = 0.0f;
    for (int j = threadIdx.x; j < H; j += kThreads) {
      const float v = __bfloat162float(x[j]);
      ss = fmaf(v, v, ss);
    }
    r = rsqrtf(block_sum(ss, red) / (float)H + eps);
  }
  float acc = 0.0f;
  for (int j = threadIdx.x; j < H; j += kThreads) {
    float v = __bfloat162float(x[j]);
    if (norm_w) v = bf16_round((v * r) * __bfloat162float(norm_w[j]));
    acc = fmaf(v, __bfloat162float(proj_w[j]), acc);
  }
  if (w1q) {
    int prev = i == 0 ? first_prev[0] : prev_rest[i - 1];
    prev = prev < 0 ? 0 : (prev >= V ? V - 1 : prev);
    for (int k = threadIdx.x; k < R; k += kThreads) {
      const uint32_t sbv = w1sb[(size_t)(k >> 6) * V + prev];
      const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
      const float e = bf16_round(fmaf(__low2float(sb), (float)w1q[(size_t)prev * R + k],
                                      __high2float(sb)));
      acc = fmaf(e, __bfloat162float(proj_w[H + k]), acc);
    }
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) {
    const float lg = bf16_round(acc + __bfloat162float(proj_b[0]));
    if (logit_out) logit_out[i] = lg;
    conf_out[i] = bf16_round(1.0f / (1.0f + expf(-lg)));
  }
}

}  // namespace conf
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_confidence(const void* hidden, long long ld, int rows, int H,
                                 const void* norm_w, float eps, const uint8_t* w1q,
                                 const uint32_t* w1sb, int V, int R, const int32_t* first_prev,
                                 const int32_t* prev_rest, const void* proj_w, const void* proj_b,
                                 float* logit, float* conf, dspark_stream_t stream) {
  if (!hidden || !proj_w || !proj_b || !conf || rows <= 0 || H <= 0 || ld < H)
    return set_error(DSPARK_ERR_INVALID, "confidence: bad arguments");
  if (w1q && (!w1sb || !first_prev || (rows > 1 && !prev_rest) || V <= 0 || R <= 0 || R % 64))
    return set_error(DSPARK_ERR_INVALID, "confidence: bad Markov embedding arguments");
  if (rows > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "confidence: too many rows");
  return launch_pdl("confidence", conf::confidence_kernel, dim3(rows), dim3(conf::kThreads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(hidden),
                    ld, H, static_cast<const __nv_bfloat16*>(norm_w), eps, w1q, w1sb, V,
                    w1q ? R : 0, first_prev, prev_rest, static_cast<const __nv_bfloat16*>(proj_w),
                    static_cast<const __nv_bfloat16*>(proj_b), logit, conf);
}
