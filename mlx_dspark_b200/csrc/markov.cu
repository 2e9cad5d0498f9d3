// K10 — DSpark Markov head with greedy block sampling.
//
// Reference: DSparkDrafter.sample_block (src/mlx_dspark/model.py:270-281), batched form
// _batched_sample_block (src/mlx_dspark/batch_engine.py:414-428), VanillaMarkov
// (model.py:196-208):
//   for i in range(cap): logits_i = base_i + w2(w1[prev]); prev = argmax(logits_i)
// One launch per position i. Each thread owns vocabulary rows: it issues the row's 256 W8
// bytes as 16 independent 16-byte loads before any arithmetic (memory-level parallelism; the
// W8 w2 matrix, 41 MB at V = 151936, stays L2-resident across the cap steps), forms the
// Markov bias for every batch row, adds the base logits and keeps a running argmax. The last
// CTA to finish reduces the per-CTA results in CTA order and publishes the token that the
// next launch conditions on.
// Rounding follows a bf16 model: e = bf16(dequant w1[prev]); bias = bf16(w2 . e);
// logit = bf16(base + bias); argmax takes the first index of the maximum.
//
// Temperature drafts (sample_block_probs, model.py:283-309) use the same step kernel in its
// SAMPLE form: it writes the biased logits row and the next launch (dspark_sample_rows) draws
// token i from truncate(softmax(logits_i / T)), keeping q_i for the acceptance test.
#include "common.cuh"
#include "tensor_map.cuh"

namespace dspark {
namespace mk {

constexpr int kThreads = 256;
constexpr int kMaxB = 8;
constexpr int kR = 256;  // Markov rank
constexpr int kG = kR / 64;

struct Best {
  float v;
  int i;
};
__device__ __forceinline__ Best better(Best a, Best b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

// NB == B: the batch width is a template parameter so every per-row loop is exact.
// SAMPLE: write logits_i of batch row b to out[b * ld_out + v] instead of the argmax.
template <int NB, bool SAMPLE>
__global__ void __launch_bounds__(kThreads) markov_step_kernel(
    const __nv_bfloat16* __restrict__ base, int ld, int rows_per_b, int cap, int V, int step,
    const uint8_t* __restrict__ w1q, const uint32_t* __restrict__ w1sb,
    const uint8_t* __restrict__ w2q, const uint32_t* __restrict__ w2sb,
    const int32_t* __restrict__ first_prev, int32_t* __restrict__ draft,
    int32_t* __restrict__ verify_ids, float* __restrict__ part_v, int* __restrict__ part_i,
    int* __restrict__ counter, __nv_bfloat16* __restrict__ out, int ld_out) {
  pdl_enter();
  if (SAMPLE && step == 0 && verify_ids && blockIdx.x == 0 && threadIdx.x < NB)
    verify_ids[threadIdx.x * (cap + 1)] = first_prev[threadIdx.x];
  __shared__ __align__(16) float e[NB][kR];
  __shared__ float esum[NB][kG];
  __shared__ Best red[NB][kThreads / 32];
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // e_b = bf16(dequant w1[prev_b])
  for (int idx = threadIdx.x; idx < NB * kR; idx += kThreads) {
    const int b = idx / kR, r = idx - b * kR;
    int prev = step == 0 ? first_prev[b] : draft[b * cap + step - 1];
    prev = prev < 0 ? 0 : (prev >= V ? V - 1 : prev);
    const uint32_t sbv = w1sb[(size_t)(r >> 6) * V + prev];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    e[b][r] = bf16_round(fmaf(__low2float(sb), (float)w1q[(size_t)prev * kR + r], __high2float(sb)));
  }
  __syncthreads();
  // w2 . e = sum_g (s_g * sum_{r in g} q_r e_r + b_g * sum_{r in g} e_r)
  // group sums of e: one warp per (b, g), a fixed tree
  for (int bg = warp; bg < NB * kG; bg += kThreads / 32) {
    const int b = bg / kG, g = bg % kG;
    float s = warp_sum(e[b][g * 64 + lane] + e[b][g * 64 + 32 + lane]);
    if (lane == 0) esum[b][g] = s;
  }
  __syncthreads();
  Best best[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) best[b] = Best{-INFINITY, 0x7fffffff};
  // w2 . e, one warp per 8 vocabulary rows at a time: lane l reads bytes [8l, 8l + 8) of each
  // row (one coalesced 256-byte row per warp load, 8 rows in flight) and forms its 8-term
  // partial; the 8 lanes of each 64-wide group combine by a reduce-scatter (lane k & 7 ends
  // with row k's group sum), and lane k then adds the groups in order:
  //   d = fma(s_g, qsum_g, fma(b_g, esum_g, d)), g = 0..3
  const int lane8 = lane & 7, grp = lane >> 3;
  const int gwarp = blockIdx.x * (kThreads / 32) + warp;
  const int stride = gridDim.x * (kThreads / 32) * 8;
  // the 8 rows' W8 bytes (lane: bytes [8l, 8l + 8) of each) and this lane's (row lane & 7,
  // group lane >> 3) scale/bias; rows past V read any valid row, their result is discarded
  auto load_rows = [&](int vb, uint2 (&q)[8], uint32_t& sb) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int v = min(vb + k, V - 1);
      q[k] = __ldg(reinterpret_cast<const uint2*>(w2q + (size_t)v * kR) + lane);
    }
    sb = __ldg(w2sb + (size_t)grp * V + min(vb + lane8, V - 1));
  };
  uint2 q8[8];
  uint32_t sbk = 0;
  if (gwarp * 8 < V) load_rows(gwarp * 8, q8, sbk);
  for (int v0 = gwarp * 8; v0 < V; v0 += stride) {
    // the warp's next 8 rows are in flight while these are reduced
    uint2 qn[8];
    uint32_t sbn = 0;
    if (v0 + stride < V) load_rows(v0 + stride, qn, sbn);
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      float ev[8];  // this lane's 8 columns of e_b (shared memory; registers stay free at large B)
      {
        const float4 t0 = *reinterpret_cast<const float4*>(&e[b][lane * 8]);
        const float4 t1 = *reinterpret_cast<const float4*>(&e[b][lane * 8 + 4]);
        ev[0] = t0.x; ev[1] = t0.y; ev[2] = t0.z; ev[3] = t0.w;
        ev[4] = t1.x; ev[5] = t1.y; ev[6] = t1.z; ev[7] = t1.w;
      }
      float x[8];  // this lane's partial of every row of the batch
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t w0 = q8[k].x, w1 = q8[k].y;
        float acc = 0.0f;
#pragma unroll
        for (int by = 0; by < 4; ++by) {
          // exact byte -> float: the fp32 bit pattern of 2^23 + q, minus 2^23
          acc = fmaf(__uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7650 + by)) - 8388608.0f, ev[by], acc);
        }
#pragma unroll
        for (int by = 0; by < 4; ++by)
          acc = fmaf(__uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7650 + by)) - 8388608.0f, ev[4 + by], acc);
        x[k] = acc;
      }
      // reduce-scatter over the group's 8 lanes: keep the half of the rows matching each lane bit
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool hi = lane & 4;
        const float send = hi ? x[i] : x[i + 4];
        const float keep = hi ? x[i + 4] : x[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const bool hi = lane & 2;
        const float send = hi ? x[i] : x[i + 2];
        const float keep = hi ? x[i + 2] : x[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      {
        const bool hi = lane & 1;
        const float send = hi ? x[0] : x[1];
        const float keep = hi ? x[1] : x[0];
        x[0] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
      }
      // x[0] = group grp's sum of row v0 + lane8; lane lane8 gathers the 4 groups in order
      float d = 0.0f;
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const float qs = __shfl_sync(0xffffffffu, x[0], g * 8 + lane8);
        const uint32_t sbv = __shfl_sync(0xffffffffu, sbk, g * 8 + lane8);
        const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
        d = fmaf(__low2float(sb), qs, fmaf(__high2float(sb), esum[b][g], d));
      }
      const int v = v0 + lane8;
      if (lane < 8 && v < V) {
        const float logit =
            bf16_round(__bfloat162float(base[(size_t)(b * rows_per_b + step) * ld + v]) + bf16_round(d));
        if (SAMPLE)
          out[(size_t)b * ld_out + v] = __float2bfloat16_rn(logit);
        else
          best[b] = better(best[b], Best{logit, v});
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) q8[k] = qn[k];
    sbk = sbn;
  }
  if (SAMPLE) return;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    Best t = best[b];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best y;
      y.v = __shfl_xor_sync(0xffffffffu, t.v, o);
      y.i = __shfl_xor_sync(0xffffffffu, t.i, o);
      t = better(t, y);
    }
    if (lane == 0) red[b][warp] = t;
  }
  __syncthreads();
  if (threadIdx.x < NB) {
    const int b = threadIdx.x;
    Best t = red[b][0];
    for (int w = 1; w < kThreads / 32; ++w) t = better(t, red[b][w]);
    part_v[(size_t)blockIdx.x * NB + b] = t.v;
    part_i[(size_t)blockIdx.x * NB + b] = t.i;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // final reduction: warp b per batch row, lanes over the CTAs' partials (loads in flight
  // together); the (max value, min index) order makes the result independent of grouping
  if (warp < NB) {
    const int b = warp;
    Best t{-INFINITY, 0x7fffffff};
    for (int c = lane; c < (int)gridDim.x; c += 32)
      t = better(t, Best{__ldcg(part_v + (size_t)c * NB + b), __ldcg(part_i + (size_t)c * NB + b)});
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Best y;
      y.v = __shfl_xor_sync(0xffffffffu, t.v, o);
      y.i = __shfl_xor_sync(0xffffffffu, t.i, o);
      t = better(t, y);
    }
    if (lane == 0) {
      if (t.i == 0x7fffffff) t.i = 0;
      draft[b * cap + step] = t.i;
      if (verify_ids) {
        if (step == 0) verify_ids[b * (cap + 1)] = first_prev[b];
        verify_ids[b * (cap + 1) + 1 + step] = t.i;
      }
    }
  }
  if (threadIdx.x == 0) *counter = 0;
}

// Greedy steps: as many CTAs as the device keeps resident at once (the occupancy of the
// batch width's instance: 4 per SM at B = 1), so every warp walks its rows with the next 8 in
// flight and no CTA waits for a second wave. Measured on B200 with V = 151936 before this
// sizing: 297 CTAs (two per SM), 18.5 us per step.
template <int NB, bool SAMPLE = false>
static int resident_ctas() {
  static int cached = 0;  // a failed query (no device) is retried on the next call
  if (cached) return cached;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, markov_step_kernel<NB, SAMPLE>, kThreads,
                                                    0) != cudaSuccess || n < 1)
    return 2;
  cached = n;
  return n;
}
static int ctas_per_sm(int B) {
  switch (B) {
    case 1: return resident_ctas<1>();
    case 2: return resident_ctas<2>();
    case 3: return resident_ctas<3>();
    case 4: return resident_ctas<4>();
    case 5: return resident_ctas<5>();
    case 6: return resident_ctas<6>();
    case 7: return resident_ctas<7>();
    default: return resident_ctas<8>();
  }
}
// the SAMPLE form (temperature drafts) writes the biased logits and keeps no partials
static int sample_ctas_per_sm(int B) {
  switch (B) {
    case 1: return resident_ctas<1, true>();
    case 2: return resident_ctas<2, true>();
    case 3: return resident_ctas<3, true>();
    case 4: return resident_ctas<4, true>();
    case 5: return resident_ctas<5, true>();
    case 6: return resident_ctas<6, true>();
    case 7: return resident_ctas<7, true>();
    default: return resident_ctas<8, true>();
  }
}
static int sample_grid(int B, int V) {
  const int g = std::min((V + 63) / 64, sm_count() * sample_ctas_per_sm(B));
  return g < 1 ? 1 : g;
}
static int step_grid(int B, int V) {
  const int by_rows = (V + 63) / 64;  // at least 8 rows per warp
  const int g = std::min(by_rows, sm_count() * ctas_per_sm(B));
  return g < 1 ? 1 : g;
}

static size_t ws(int B, int V, int* grid_out, size_t* off_i, size_t* off_c) {
  const int grid = step_grid(B, V);
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
  auto run = [&](auto kern) {
    for (int i = 0; i < cap; ++i) {
      int rc = launch_pdl("markov_step", kern, dim3(grid), dim3(mk::kThreads), 0, st,
                          static_cast<const __nv_bfloat16*>(base), ld, rows_per_b, cap, V, i,
                          w1q, w1sb, w2q, w2sb, first_prev, draft, verify_ids,
                          reinterpret_cast<float*>(w + off_c), reinterpret_cast<int*>(w + off_i),
                          reinterpret_cast<int*>(w), (__nv_bfloat16*)nullptr, 0);
      if (rc) return rc;
    }
    return (int)DSPARK_OK;
  };
  switch (B) {
    case 1: return run(mk::markov_step_kernel<1, false>);
    case 2: return run(mk::markov_step_kernel<2, false>);
    case 3: return run(mk::markov_step_kernel<3, false>);
    case 4: return run(mk::markov_step_kernel<4, false>);
    case 5: return run(mk::markov_step_kernel<5, false>);
    case 6: return run(mk::markov_step_kernel<6, false>);
    case 7: return run(mk::markov_step_kernel<7, false>);
    default: return run(mk::markov_step_kernel<8, false>);
  }
}

extern "C" int dspark_sample_rows(const void* logits, long long ld, int groups, int rows, int V,
                                  float temperature, int temp_mode, double top_p, int top_k,
                                  const unsigned long long* rng, int stream_id, int row_base,
                                  float* probs, long long ld_probs, int32_t* tokens, int tok_stride,
                                  int32_t* tokens2, int tok2_stride, dspark_stream_t stream);

extern "C" size_t dspark_markov_probs_workspace_bytes(int B, int V) {
  if (B <= 0 || V <= 0) return 0;
  return (size_t)B * (size_t)((V + 7) & ~7) * 2;
}

extern "C" int dspark_markov_sample_block_probs(
    const void* base, int ld, int rows_per_b, int B, int cap, int V, int R, const uint8_t* w1q,
    const uint32_t* w1sb, const uint8_t* w2q, const uint32_t* w2sb, const int32_t* first_prev,
    int32_t* draft, int32_t* verify_ids, float temperature, double top_p, int top_k,
    const unsigned long long* rng, float* q_probs, long long ld_q, void* workspace,
    size_t workspace_bytes, dspark_stream_t stream) {
  if (!base || !w1q || !w1sb || !w2q || !w2sb || !first_prev || !draft || !rng || !q_probs ||
      B <= 0 || cap <= 0 || V <= 0 || ld < V || ld_q < V)
    return set_error(DSPARK_ERR_INVALID, "markov_sample_block_probs: bad arguments");
  if (R != mk::kR) return set_error(DSPARK_ERR_UNSUPPORTED, "markov_sample_block_probs: rank %d != 256", R);
  if (B > mk::kMaxB) return set_error(DSPARK_ERR_UNSUPPORTED, "markov_sample_block_probs: B > %d", mk::kMaxB);
  const size_t need = dspark_markov_probs_workspace_bytes(B, V);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "markov_sample_block_probs: workspace %zu < %zu",
                     workspace_bytes, need);
  const int ld_out = (V + 7) & ~7;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(workspace);
  const int grid = mk::sample_grid(B, V);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto run = [&](auto kern) {
    for (int i = 0; i < cap; ++i) {
      int rc = launch_pdl("markov_step_sample", kern, dim3(grid), dim3(mk::kThreads), 0, st,
                          static_cast<const __nv_bfloat16*>(base), ld, rows_per_b, cap, V, i,
                          w1q, w1sb, w2q, w2sb, first_prev, draft, verify_ids, (float*)nullptr,
                          (int*)nullptr, (int*)nullptr, out, ld_out);
      if (rc) return rc;
      // token i of batch row b -> draft[b * cap + i] and verify_ids[b * (cap + 1) + 1 + i];
      // q_i of row b -> q_probs[(b * cap + i) * ld_q]
      rc = dspark_sample_rows(out, ld_out, B, 1, V, temperature, 1, top_p, top_k, rng, 1, i,
                              q_probs + (size_t)i * ld_q, (long long)cap * ld_q, draft + i, cap,
                              verify_ids ? verify_ids + 1 + i : nullptr, cap + 1, stream);
      if (rc) return rc;
    }
    return (int)DSPARK_OK;
  };
  switch (B) {
    case 1: return run(mk::markov_step_kernel<1, true>);
    case 2: return run(mk::markov_step_kernel<2, true>);
    case 3: return run(mk::markov_step_kernel<3, true>);
    case 4: return run(mk::markov_step_kernel<4, true>);
    case 5: return run(mk::markov_step_kernel<5, true>);
    case 6: return run(mk::markov_step_kernel<6, true>);
    case 7: return run(mk::markov_step_kernel<7, true>);
    default: return run(mk::markov_step_kernel<8, true>);
  }
}
