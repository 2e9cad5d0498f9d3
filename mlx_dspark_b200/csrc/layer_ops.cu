// Row-wise layer operations around the W8 GEMMs: embedding dequant-gather, RMSNorm, and
// the per-head q/k norm + RoPE + paged KV write. All of them are HBM/latency-bound and use
// one CTA per token row; they honour programmatic dependent launch so they can be queued
// behind a GEMM without a launch gap.
#include "common.cuh"
#include "rope_kv.cuh"

namespace dspark {

// ------------------------------------------------------------------------------------------
// embedding: out[m, k] = bf16(scale * q[id, k] + bias)   (mlx QuantizedEmbedding)
__global__ void __launch_bounds__(256) embed_w8_kernel(const int32_t* __restrict__ ids,
                                                       const uint8_t* __restrict__ wq,
                                                       const uint32_t* __restrict__ wsb, int V,
                                                       int H, __nv_bfloat16* __restrict__ out,
                                                       int ldo) {
  pdl_enter();
  const int m = blockIdx.x;
  int id = ids[m];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const uint8_t* row = wq + (size_t)id * H;
  for (int k = threadIdx.x * 4; k < H; k += blockDim.x * 4) {
    const uint32_t q4 = *reinterpret_cast<const uint32_t*>(row + k);
    const uint32_t sbv = wsb[(size_t)(k >> 6) * V + id];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    const float s = __low2float(sb), b = __high2float(sb);
    __nv_bfloat16 o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = __float2bfloat16_rn(fmaf(s, (float)((q4 >> (8 * j)) & 0xFF), b));
    *reinterpret_cast<uint2*>(out + (size_t)m * ldo + k) = *reinterpret_cast<const uint2*>(o);
  }
}

// the same gather, plus the per-128-column-tile sums of squares of the bf16 outputs
// (sumsq[m, t]): warp w covers columns [128(w + 8j), 128(w + 8j) + 128) in pass j
__global__ void __launch_bounds__(256) embed_w8_sumsq_kernel(const int32_t* __restrict__ ids,
                                                             const uint8_t* __restrict__ wq,
                                                             const uint32_t* __restrict__ wsb, int V,
                                                             int H, __nv_bfloat16* __restrict__ out,
                                                             int ldo, float* __restrict__ sumsq) {
  pdl_enter();
  const int m = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int id = ids[m];
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  const uint8_t* row = wq + (size_t)id * H;
  for (int k = threadIdx.x * 4; k < H; k += blockDim.x * 4) {
    const uint32_t q4 = *reinterpret_cast<const uint32_t*>(row + k);
    const uint32_t sbv = wsb[(size_t)(k >> 6) * V + id];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    const float s = __low2float(sb), b = __high2float(sb);
    __nv_bfloat16 o[4];
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[j] = __float2bfloat16_rn(fmaf(s, (float)((q4 >> (8 * j)) & 0xFF), b));
      const float v = __bfloat162float(o[j]);
      sq += v * v;
    }
    *reinterpret_cast<uint2*>(out + (size_t)m * ldo + k) = *reinterpret_cast<const uint2*>(o);
    sq = warp_sum(sq);
    if (lane == 0) sumsq[(size_t)m * (H / 128) + (k - lane * 4) / 128] = sq;
  }
  (void)warp;
}

// drafter block embedding: row (b, i) embeds pending[b] for i == 0, else mask_id
// (the block [pending, mask x (k-1)] of src/mlx_dspark/generate.py:848-849)
__global__ void __launch_bounds__(256) embed_block_w8_kernel(const int32_t* __restrict__ pending,
                                                             int k, int mask_id,
                                                             const uint8_t* __restrict__ wq,
                                                             const uint32_t* __restrict__ wsb,
                                                             int V, int H,
                                                             __nv_bfloat16* __restrict__ out,
                                                             int ldo, int32_t* __restrict__ ids_out) {
  pdl_enter();
  const int m = blockIdx.x;
  const int b = m / k, i = m - b * k;
  int id = i == 0 ? pending[b] : mask_id;
  id = id < 0 ? 0 : (id >= V ? V - 1 : id);
  if (ids_out && threadIdx.x == 0) ids_out[m] = id;
  const uint8_t* row = wq + (size_t)id * H;
  for (int kk = threadIdx.x * 4; kk < H; kk += blockDim.x * 4) {
    const uint32_t q4 = *reinterpret_cast<const uint32_t*>(row + kk);
    const uint32_t sbv = wsb[(size_t)(kk >> 6) * V + id];
    const __half2 sb = *reinterpret_cast<const __half2*>(&sbv);
    const float s = __low2float(sb), bb = __high2float(sb);
    __nv_bfloat16 o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = __float2bfloat16_rn(fmaf(s, (float)((q4 >> (8 * j)) & 0xFF), bb));
    *reinterpret_cast<uint2*>(out + (size_t)m * ldo + kk) = *reinterpret_cast<const uint2*>(o);
  }
}

// bf16 -> fp16 copy of a [rows, cols] block (hidden-state taps into the fused GEMM input)
__global__ void __launch_bounds__(256) bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ src,
                                                          int lds, __half* __restrict__ dst,
                                                          int ldd, int cols, int* status) {
  pdl_enter();
  const int r = blockIdx.x;
  for (int c = threadIdx.x * 2; c < cols; c += blockDim.x * 2) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + (size_t)r * lds + c));
    check_f16(v.x, status);
    check_f16(v.y, status);
    *reinterpret_cast<__half2*>(dst + (size_t)r * ldd + c) = __floats2half2_rn(v.x, v.y);
  }
}

// ------------------------------------------------------------------------------------------
// RMSNorm: y = bf16(x * rsqrt(mean(x^2) + eps) * w)
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                      const __nv_bfloat16* __restrict__ w, int H,
                                                      float eps, __nv_bfloat16* __restrict__ y,
                                                      int ldy, __half* __restrict__ y16,
                                                      int ldy16) {
  pdl_enter();
  const int m = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)m * ldx;
  float ss = 0.0f;
  for (int k = threadIdx.x * 2; k < H; k += blockDim.x * 2) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + k));
    ss += v.x * v.x + v.y * v.y;
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)H + eps);
  for (int k = threadIdx.x * 2; k < H; k += blockDim.x * 2) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + k));
    const float2 wv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + k));
    const __nv_bfloat162 o = __floats2bfloat162_rn(v.x * r * wv.x, v.y * r * wv.y);
    if (y) *reinterpret_cast<__nv_bfloat162*>(y + (size_t)m * ldy + k) = o;
    if (y16) {
      const float2 of = __bfloat1622float2(o);
      *reinterpret_cast<__half2*>(y16 + (size_t)m * ldy16 + k) = __floats2half2_rn(of.x, of.y);
    }
  }
}

// One warp per (token, head) (rope_kv_item).
template <int E>
__global__ void __launch_bounds__(256) qkv_rope_kv_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ldqkv, int T, int Hq, int Hkv,
    const __nv_bfloat16* __restrict__ qnw, const __nv_bfloat16* __restrict__ knw, float eps,
    const float* __restrict__ inv_freq, const int32_t* __restrict__ pos0,
    __nv_bfloat16* __restrict__ q_out, dspark_kv_layout kv) {
  constexpr int HD = E * 32;
  pdl_enter();
  const int m = blockIdx.x;
  const int b = m / T, t = m - b * T;
  const int pos = pos0[b] + t;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = Hq + 2 * Hkv;
  for (int h = warp; h < nheads; h += blockDim.x >> 5)
    rope_kv_item<E>(qkv + (size_t)m * ldqkv, Hq, Hkv, h, qnw, knw, eps, inv_freq, b, pos,
                    q_out + (size_t)m * Hq * HD, kv, lane);
}

}  // namespace dspark

using namespace dspark;

extern "C" int dspark_embed_w8(const int32_t* ids, int M, const uint8_t* wq, const uint32_t* wsb,
                               int V, int H, void* out, int ldo, dspark_stream_t stream) {
  if (!ids || !wq || !wsb || !out || M <= 0 || V <= 0 || H <= 0 || H % 64 || ldo < H || ldo % 4)
    return set_error(DSPARK_ERR_INVALID, "embed_w8: bad arguments (M=%d V=%d H=%d ldo=%d)", M, V, H, ldo);
  return launch_pdl("embed_w8", embed_w8_kernel, dim3(M), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), ids, wq, wsb, V, H,
                    static_cast<__nv_bfloat16*>(out), ldo);
}

extern "C" int dspark_embed_w8_sumsq(const int32_t* ids, int M, const uint8_t* wq,
                                     const uint32_t* wsb, int V, int H, void* out, int ldo,
                                     float* sumsq, dspark_stream_t stream) {
  if (!ids || !wq || !wsb || !out || !sumsq || M <= 0 || V <= 0 || H <= 0 || H % 128 || ldo < H ||
      ldo % 4)
    return set_error(DSPARK_ERR_INVALID, "embed_w8_sumsq: bad arguments (M=%d V=%d H=%d ldo=%d)", M,
                     V, H, ldo);
  return launch_pdl("embed_w8_sumsq", embed_w8_sumsq_kernel, dim3(M), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), ids, wq, wsb, V, H,
                    static_cast<__nv_bfloat16*>(out), ldo, sumsq);
}

extern "C" int dspark_rmsnorm(const void* x, int ldx, const void* w, int M, int H, float eps,
                              void* y_bf16, int ldy, void* y_f16, int ldy16,
                              dspark_stream_t stream) {
  if (!x || !w || (!y_bf16 && !y_f16) || M <= 0 || H <= 0 || H % 2 || ldx < H)
    return set_error(DSPARK_ERR_INVALID, "rmsnorm: bad arguments (M=%d H=%d)", M, H);
  const int threads = H >= 2048 ? 256 : 128;
  return launch_pdl("rmsnorm", rmsnorm_kernel, dim3(M), dim3(threads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x), ldx,
                    static_cast<const __nv_bfloat16*>(w), H, eps,
                    static_cast<__nv_bfloat16*>(y_bf16), ldy, static_cast<__half*>(y_f16), ldy16);
}

extern "C" long long dspark_kv_page_bytes(int page_size, int num_kv_heads, int head_dim, int kv8) {
  const long long elems = 2LL * num_kv_heads * page_size * head_dim;
  if (!kv8) return elems * 2;
  return elems + 2LL * num_kv_heads * page_size * (head_dim / 64) * 4;
}

extern "C" int dspark_qkv_rope_kv_write(const void* qkv, int ldqkv, int B, int T, int Hq, int Hkv,
                                        int hd, const void* q_norm_w, const void* k_norm_w,
                                        float eps, const float* inv_freq, const int32_t* pos0,
                                        void* q_out, const dspark_kv_layout* kv,
                                        dspark_stream_t stream) {
  if (!qkv || !kv || !kv->pool || !kv->block_table || !k_norm_w || !inv_freq || !pos0 || B <= 0 ||
      T <= 0 || Hkv <= 0 || Hq < 0)
    return set_error(DSPARK_ERR_INVALID, "qkv_rope_kv_write: bad arguments");
  if (Hq > 0 && (!q_out || !q_norm_w))
    return set_error(DSPARK_ERR_INVALID, "qkv_rope_kv_write: q output/norm missing");
  if (hd != 64 && hd != 128) return set_error(DSPARK_ERR_UNSUPPORTED, "qkv_rope_kv_write: head_dim %d", hd);
  if (kv->head_dim != hd || kv->num_kv_heads != Hkv || kv->page_size <= 0)
    return set_error(DSPARK_ERR_INVALID, "qkv_rope_kv_write: kv layout does not match");
  if (kv->page_bytes != dspark_kv_page_bytes(kv->page_size, Hkv, hd, kv->kv8))
    return set_error(DSPARK_ERR_INVALID, "qkv_rope_kv_write: page_bytes mismatch");
  if (ldqkv < (Hq + 2 * Hkv) * hd) return set_error(DSPARK_ERR_INVALID, "qkv_rope_kv_write: ldqkv");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dspark_kv_layout k = *kv;
  auto args = [&](auto kern) {
    return launch_pdl("qkv_rope_kv_write", kern, dim3(B * T), dim3(256), 0, st,
                      static_cast<const __nv_bfloat16*>(qkv), ldqkv, T, Hq, Hkv,
                      static_cast<const __nv_bfloat16*>(q_norm_w),
                      static_cast<const __nv_bfloat16*>(k_norm_w), eps, inv_freq, pos0,
                      static_cast<__nv_bfloat16*>(q_out), k);
  };
  return hd == 128 ? args(qkv_rope_kv_kernel<4>) : args(qkv_rope_kv_kernel<2>);
}

extern "C" int dspark_embed_block_w8(const int32_t* pending, int B, int k, int mask_id,
                                     const uint8_t* wq, const uint32_t* wsb, int V, int H,
                                     void* out, int ldo, int32_t* ids_out,
                                     dspark_stream_t stream) {
  if (!pending || !wq || !wsb || !out || B <= 0 || k <= 0 || V <= 0 || H <= 0 || H % 64 ||
      ldo < H || ldo % 4)
    return set_error(DSPARK_ERR_INVALID, "embed_block_w8: bad arguments");
  return launch_pdl("embed_block_w8", embed_block_w8_kernel, dim3(B * k), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), pending, k, mask_id, wq, wsb, V, H,
                    static_cast<__nv_bfloat16*>(out), ldo, ids_out);
}

extern "C" int dspark_bf16_to_f16(const void* src, int lds, void* dst, int ldd, int rows, int cols,
                                  int* status, dspark_stream_t stream) {
  if (!src || !dst || rows <= 0 || cols <= 0 || cols % 2 || lds % 2 || ldd % 2)
    return set_error(DSPARK_ERR_INVALID, "bf16_to_f16: bad arguments");
  return launch_pdl("bf16_to_f16", bf16_to_f16_kernel, dim3(rows), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(src), lds,
                    static_cast<__half*>(dst), ldd, cols, status);
}

// h = bf16(h + bf16(sum)): the residual epilogue of a row-split projection whose fp32
// partials were summed across tensor-parallel ranks (the RESIDUAL_BF16 epilogue of the
// W8 GEMM, applied after the all-reduce).
__global__ void residual_add_f32_kernel(__nv_bfloat16* __restrict__ h, int ldh,
                                        const float* __restrict__ sum, int lds, int M, int N) {
  pdl_enter();
  const long long total = (long long)M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    __nv_bfloat16* p = h + (size_t)m * ldh + n;
    *p = __float2bfloat16_rn(__bfloat162float(*p) + bf16_round(sum[(size_t)m * lds + n]));
  }
}

extern "C" int dspark_residual_add_f32(void* h, int ldh, const float* sum, int lds, int M, int N,
                                       dspark_stream_t stream) {
  if (!h || !sum || M <= 0 || N <= 0 || ldh < N || lds < N)
    return set_error(DSPARK_ERR_INVALID, "residual_add_f32: bad arguments");
  const long long total = (long long)M * N;
  int grid = (int)((total + 255) / 256);
  if (grid > 4 * 148) grid = 4 * 148;
  return launch_pdl("residual_add_f32", residual_add_f32_kernel, dim3(grid), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(h), ldh, sum,
                    lds, M, N);
}
