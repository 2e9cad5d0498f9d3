// Shared by the standalone q/k-norm + RoPE + KV-write kernel (layer_ops.cu), the q|k|v GEMM's
// fused RoPE epilogue and the rope phase of the fused layer chain (w8a16_gemm.cu).
#pragma once

#include "common.cuh"

namespace dspark {

// ------------------------------------------------------------------------------------------
// paged cache addressing
struct KvAddr {
  uint8_t* page;  // base of the page holding `pos`
  int slot;       // token slot inside the page
};
__device__ __forceinline__ KvAddr kv_locate(const dspark_kv_layout& kv, int b, int pos) {
  const int pi = pos / kv.page_size;
  const int phys = kv.block_table[(size_t)b * kv.max_pages + pi];
  KvAddr a;
  a.page = static_cast<uint8_t*>(kv.pool) + (size_t)phys * (size_t)kv.page_bytes;
  a.slot = pos - pi * kv.page_size;
  return a;
}

// One warp handles head h of token row m (batch row b, position pos) of a packed [q|k|v] row:
// per-head RMSNorm of q and k, non-interleaved RoPE, then q to q_row or K/V into the paged
// cache (bf16, or affine 8-bit group 64 quantized on write). E = head_dim / 32 contiguous
// elements per lane; lanes l and l + 16 hold the halves RoPE rotates against each other.
// `head` points at the head's HD bf16 inputs, in global or shared memory (the W8 GEMM's fused
// epilogue passes a tile it staged in shared memory).
template <int E>
__device__ __forceinline__ void rope_kv_head(const __nv_bfloat16* head, int Hq, int Hkv, int h,
                                             const __nv_bfloat16* __restrict__ qnw,
                                             const __nv_bfloat16* __restrict__ knw, float eps,
                                             const float* __restrict__ inv_freq, int b, int pos,
                                             __nv_bfloat16* __restrict__ q_row,
                                             const dspark_kv_layout& kv, int lane) {
  constexpr int HD = E * 32;
  const __nv_bfloat16* src = head + lane * E;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = __bfloat162float(src[e]);
  const bool is_v = h >= Hq + Hkv;
  if (!is_v) {
    const __nv_bfloat16* nw = h < Hq ? qnw : knw;
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fmaf_rn(x[e], x[e], ss);
    ss = warp_sum(ss);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)HD), eps));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = bf16_round(__fmul_rn(__fmul_rn(x[e], r), __bfloat162float(nw[lane * E + e])));
    // RoPE (rotate-half): pair element i with i + HD/2
    float other[E];
#pragma unroll
    for (int e = 0; e < E; ++e) other[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const bool upper = lane >= 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int fi = (lane & 15) * E + e;
      float sn, cs;
      sincosf((float)pos * inv_freq[fi], &sn, &cs);
      // explicit roundings: the same bits in every kernel that inlines this
      x[e] = upper ? bf16_round(__fadd_rn(__fmul_rn(x[e], cs), __fmul_rn(other[e], sn)))
                   : bf16_round(__fsub_rn(__fmul_rn(x[e], cs), __fmul_rn(other[e], sn)));
    }
  }
  if (h < Hq) {
    __nv_bfloat16* dst = q_row + (size_t)h * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = __float2bfloat16_rn(x[e]);
    return;
  }
  const int kvh = is_v ? h - Hq - Hkv : h - Hq;
  const int which = is_v ? 1 : 0;
  const KvAddr a = kv_locate(kv, b, pos);
  const size_t row = ((size_t)which * Hkv + kvh) * kv.page_size + a.slot;
  if (!kv.kv8) {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.page) + row * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) dst[e] = __float2bfloat16_rn(x[e]);
  } else {
    // affine 8-bit, group 64 along head_dim, by the rule of MLX's affine quantizer (what
    // QuantizedKVCache(64, 8) applies through mx.quantize): in fp32,
    //   scale = max((max - min) / 255, 1e-7), negated unless |min| > |max|;
    //   edge  = the value of larger magnitude (min or max), made exactly representable:
    //   q0 = round(edge / scale); scale = edge / q0 and bias = edge, or bias = 0 if q0 == 0;
    //   q = min(round((x - bias) / scale), 255)   (round: halves away from zero)
    // with the fp32 scale and bias; both are stored as bf16 (the dequantization operands).
    constexpr int LPG = 64 / E;  // lanes per group
    float mn = x[0], mx = x[0];
#pragma unroll
    for (int e = 1; e < E; ++e) { mn = fminf(mn, x[e]); mx = fmaxf(mx, x[e]); }
#pragma unroll
    for (int o = LPG / 2; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    float sc = fmaxf((mx - mn) / 255.0f, 1e-7f);
    const bool neg_edge = fabsf(mn) > fabsf(mx);
    sc = neg_edge ? sc : -sc;
    const float edge = neg_edge ? mn : mx;
    const float q0 = roundf(edge / sc);
    const bool at_zero = q0 == 0.0f;
    sc = at_zero ? sc : edge / q0;
    const float bi = at_zero ? 0.0f : edge;
    uint8_t* qdst = a.page + row * HD + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      // (x - bias) / scale >= 0 by construction; the lower clamp only guards the cast
      const float qv = fminf(fmaxf(roundf((x[e] - bi) / sc), 0.0f), 255.0f);
      qdst[e] = (uint8_t)qv;
    }
    if ((lane % LPG) == 0) {
      uint32_t* sbdst = reinterpret_cast<uint32_t*>(a.page + (size_t)2 * Hkv * kv.page_size * HD) +
                        row * (HD / 64) + (lane * E) / 64;
      const __nv_bfloat16 s16 = __float2bfloat16_rn(sc), b16 = __float2bfloat16_rn(bi);
      *sbdst = (uint32_t)(*reinterpret_cast<const uint16_t*>(&s16)) |
               ((uint32_t)(*reinterpret_cast<const uint16_t*>(&b16)) << 16);
    }
  }
}

// head h of a packed [q|k|v] row in global memory
template <int E>
__device__ __forceinline__ void rope_kv_item(const __nv_bfloat16* __restrict__ qkv_row, int Hq,
                                             int Hkv, int h, const __nv_bfloat16* __restrict__ qnw,
                                             const __nv_bfloat16* __restrict__ knw, float eps,
                                             const float* __restrict__ inv_freq, int b, int pos,
                                             __nv_bfloat16* __restrict__ q_row,
                                             const dspark_kv_layout& kv, int lane) {
  rope_kv_head<E>(qkv_row + (size_t)h * (E * 32), Hq, Hkv, h, qnw, knw, eps, inv_freq, b, pos,
                  q_row, kv, lane);
}

}  // namespace dspark
