// K2/K4/K5 — GQA attention of a block of T queries per row over the paged KV cache.
//
// One CTA per (split, kv head, row). The G = Hq/Hkv query heads of a kv head and the T block
// tokens form R = G*T query rows, tiled by 16 rows per warp; the warps share each 64-token
// K/V page staged in shared memory (cp.async double buffering; 8-bit pages are dequantized
// to bf16 in shared memory). Scores and P.V run on bf16 m16n8k16 tensor-core MMAs with an
// fp32 online softmax. Splits cover disjoint page ranges whose length is computed on the
// device from kv_len, so the same launch serves every context length inside a CUDA graph.
// The per-split (max, sum, O) partials go to the workspace and attn_combine_kernel merges them,
// in split order, into the bf16-rounded output (written as fp16, the o_proj input); a context
// that fits one split is written directly. (Merging inside the attention kernel, through a
// thread-block cluster or through a bounded wait on sibling splits, measured no faster: the
// second launch hides under programmatic dependent launch.)
//
// Semantics follow mx.fast.scaled_dot_product_attention as called from the reference:
// fp32 scores q.k * scale, fp32 softmax, output rounded to bf16; masks as in
// create_attention_mask / build_batch_mask (src/mlx_dspark/batch_engine.py:170-178) for the
// causal verify, and no mask for the drafter block (src/mlx_dspark/model.py:130-156,
// src/mlx_dspark/dflash_model.py:127-133).
#include <algorithm>

#include "common.cuh"

namespace dspark {
namespace attn {

constexpr int KT = 64;  // keys per tile == page size
constexpr int kMinPagesPerSplit = 1;  // a split is at least this many pages

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int HD, bool KV8>
struct Layout {
  static constexpr int kRow = HD + 8;                          // padded bf16 row (elements)
  static constexpr int kTile = KT * kRow * 2;                  // bytes of one K or V tile
  static constexpr int kRawK = KT * HD + KT * (HD / 64) * 4;   // raw 8-bit K page slice
  static constexpr int kRaw = KV8 ? 2 * kRawK : 0;             // K and V raw per buffer
  static constexpr int kBuf = 2 * kTile + kRaw;
  static constexpr int kBytes = 2 * kBuf + 16;
};

struct Args {
  const __nv_bfloat16* q;
  int B, T, Hq, G, R, nsplit, causal;
  float scale_log2;  // softmax scale * log2(e)
  dspark_kv_layout kv;
  const int32_t* kv_len;
  __half* out;
  int ldo;
  float* ws_o;   // [B*Hkv][nsplit][R][HD]
  float* ws_ml;  // [B*Hkv][nsplit][R][2]
  int* status;   // DSPARK_ERR_RANGE if an output is past the fp16 range (NULL: unchecked)
};

// One query row of the merge: lanes over the head dimension, splits in order (max, then the
// rescaled sums and O), bf16-rounded output written as fp16.
template <int HD>
__device__ __forceinline__ void merge_row(const Args& a, int b, int h, int r, int nsplit, int lane) {
  constexpr int E = HD / 32;
  const int bh = b * a.kv.num_kv_heads + h;
  const size_t base0 = (size_t)bh * a.nsplit * a.R;
  float M = -INFINITY;
  for (int sp = lane; sp < nsplit; sp += 32)
    M = fmaxf(M, __ldcg(a.ws_ml + (base0 + (size_t)sp * a.R + r) * 2));
  M = warp_max(M);
  float Ls = 0.0f;
  for (int sp = lane; sp < nsplit; sp += 32) {
    const float ms = __ldcg(a.ws_ml + (base0 + (size_t)sp * a.R + r) * 2);
    if (ms != -INFINITY) Ls += __ldcg(a.ws_ml + (base0 + (size_t)sp * a.R + r) * 2 + 1) * exp2f(ms - M);
  }
  Ls = warp_sum(Ls);
  float acc[E];
#pragma unroll
  for (int k = 0; k < E; ++k) acc[k] = 0.0f;
#pragma unroll 4
  for (int sp = 0; sp < nsplit; ++sp) {
    const size_t row = base0 + (size_t)sp * a.R + r;
    const float ms = __ldcg(a.ws_ml + row * 2);
    const float e = ms == -INFINITY ? 0.0f : exp2f(ms - M);  // empty splits hold zeros
    const float* src = a.ws_o + row * HD + lane * E;
    float v[E];
    if constexpr (E == 4) {
      const float4 t = __ldcg(reinterpret_cast<const float4*>(src));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
      const float2 t = __ldcg(reinterpret_cast<const float2*>(src));
      v[0] = t.x; v[1] = t.y;
    }
#pragma unroll
    for (int k = 0; k < E; ++k) acc[k] = fmaf(e, v[k], acc[k]);
  }
  const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
  const int t = r % a.T, g = r / a.T;
  __half* dst = a.out + (size_t)(b * a.T + t) * a.ldo + (size_t)(h * a.G + g) * HD + lane * E;
#pragma unroll
  for (int k = 0; k < E; k += 2) {
    const float o0 = bf16_round(acc[k] * inv), o1 = bf16_round(acc[k + 1] * inv);
    check_f16(o0, a.status);
    check_f16(o1, a.status);
    *reinterpret_cast<__half2*>(dst + k) = __floats2half2_rn(o0, o1);
  }
}

template <int HD, bool KV8>
__device__ __forceinline__ void issue_tile(const Args& a, uint8_t* buf, int b, int h, int page) {
  using L = Layout<HD, KV8>;
  const int phys = a.kv.block_table[(size_t)b * a.kv.max_pages + page];
  const uint8_t* pg = static_cast<const uint8_t*>(a.kv.pool) + (size_t)phys * (size_t)a.kv.page_bytes;
  const int Hkv = a.kv.num_kv_heads;
  const int nthr = blockDim.x;
  if (!KV8) {
    constexpr int CPR = HD * 2 / 16;  // 16-byte chunks per key row
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const uint8_t* src = pg + ((size_t)(which * Hkv + h) * KT) * HD * 2;
      const uint32_t dst = smem_u32(buf + which * L::kTile);
      for (int i = threadIdx.x; i < KT * CPR; i += nthr) {
        const int row = i / CPR, c = i - row * CPR;
        cp_async16(dst + (row * L::kRow) * 2 + c * 16, src + (size_t)row * HD * 2 + c * 16);
      }
    }
  } else {
    uint8_t* raw = buf + 2 * L::kTile;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const uint8_t* qsrc = pg + ((size_t)(which * Hkv + h) * KT) * HD;
      const uint8_t* ssrc = pg + (size_t)2 * Hkv * KT * HD + ((size_t)(which * Hkv + h) * KT) * (HD / 64) * 4;
      const uint32_t dq = smem_u32(raw + which * L::kRawK);
      const uint32_t ds = dq + KT * HD;
      for (int i = threadIdx.x; i < KT * HD / 16; i += nthr) cp_async16(dq + i * 16, qsrc + (size_t)i * 16);
      for (int i = threadIdx.x; i < KT * (HD / 64) * 4 / 16; i += nthr) cp_async16(ds + i * 16, ssrc + (size_t)i * 16);
    }
  }
}

template <int HD>
__device__ __forceinline__ void dequant_tile(uint8_t* buf) {
  using L = Layout<HD, true>;
  uint8_t* raw = buf + 2 * L::kTile;
#pragma unroll 1
  for (int which = 0; which < 2; ++which) {
    const uint8_t* qs = raw + which * L::kRawK;
    const uint32_t* sb = reinterpret_cast<const uint32_t*>(qs + KT * HD);
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(buf + which * L::kTile);
    for (int i = threadIdx.x; i < KT * HD / 8; i += blockDim.x) {
      const int key = i / (HD / 8), d0 = (i - key * (HD / 8)) * 8;
      const uint32_t sbv = sb[key * (HD / 64) + d0 / 64];
      const float s = __uint_as_float(sbv << 16), bb = __uint_as_float(sbv & 0xFFFF0000u);
      const uint2 q8 = *reinterpret_cast<const uint2*>(qs + key * HD + d0);
      __nv_bfloat162 o[4];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const uint32_t w = j < 4 ? q8.x : q8.y;
        // a code byte under the exponent of 2^23 reads as 2^23 + code (exact)
        const float c0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440 | (j & 3))) - 8388608.0f;
        const float c1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441 | (j & 3))) - 8388608.0f;
        o[j / 2] = __floats2bfloat162_rn(fmaf(s, c0, bb), fmaf(s, c1, bb));
      }
      *reinterpret_cast<uint4*>(dst + key * L::kRow + d0) = *reinterpret_cast<const uint4*>(o);
    }
  }
}

template <int HD, bool KV8>
__global__ void __launch_bounds__(256) attn_kernel(const Args a) {
  using L = Layout<HD, KV8>;
  extern __shared__ __align__(16) uint8_t smem[];
  pdl_enter();

  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int Hkv = a.kv.num_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvlen = a.kv_len[b];
  const int Ltot = kvlen + a.T;
  const int npages = (Ltot + KT - 1) / KT;
  // Splits actually used for this context: at least kMinPagesPerSplit pages each, so the
  // merge stays cheap at short contexts; CTAs past them leave at once.
  const int nsplit = min(a.nsplit, (npages + kMinPagesPerSplit - 1) / kMinPagesPerSplit);
  if (split >= nsplit) return;
  const int pps = (npages + nsplit - 1) / nsplit;
  const int p_lo = split < nsplit ? split * pps : npages;
  const int p_hi = min(p_lo + pps, npages);

  // this warp's two query rows (of 16) per thread: r0 = lane/4, r1 = r0 + 8
  const int r0 = warp * 16 + (lane >> 2), r1 = r0 + 8;
  const int lim0 = (r0 < a.R && a.causal) ? kvlen + (r0 % a.T) : Ltot - 1;
  const int lim1 = (r1 < a.R && a.causal) ? kvlen + (r1 % a.T) : Ltot - 1;

  // Q fragments (A operand, row-major 16 x HD)
  uint32_t qf[HD / 16][4];
  {
    const __nv_bfloat16* q0 = nullptr;
    const __nv_bfloat16* q1 = nullptr;
    if (r0 < a.R) q0 = a.q + ((size_t)(b * a.T + r0 % a.T) * a.Hq + h * a.G + r0 / a.T) * HD;
    if (r1 < a.R) q1 = a.q + ((size_t)(b * a.T + r1 % a.T) * a.Hq + h * a.G + r1 / a.T) * HD;
    const int c = (lane & 3) * 2;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      qf[kk][0] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + kk * 16 + c) : 0u;
      qf[kk][1] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + kk * 16 + c) : 0u;
      qf[kk][2] = q0 ? *reinterpret_cast<const uint32_t*>(q0 + kk * 16 + 8 + c) : 0u;
      qf[kk][3] = q1 ? *reinterpret_cast<const uint32_t*>(q1 + kk * 16 + 8 + c) : 0u;
    }
  }

  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;

  if (p_lo < p_hi) issue_tile<HD, KV8>(a, smem, b, h, p_lo);
  cp_commit();
  for (int p = p_lo; p < p_hi; ++p) {
    const int buf = (p - p_lo) & 1;
    uint8_t* cur = smem + buf * L::kBuf;
    if (p + 1 < p_hi) issue_tile<HD, KV8>(a, smem + (buf ^ 1) * L::kBuf, b, h, p + 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (KV8) {
      dequant_tile<HD>(cur);
      __syncthreads();
    }
    // warps past the last query row only help stage and dequantise the pages
    if (warp * 16 < a.R) {
      const uint32_t ks = smem_u32(cur), vs = smem_u32(cur + L::kTile);
      // S = Q K^T over 64 keys (8 n-tiles of 8 keys)
      float s[8][4];
#pragma unroll
      for (int jn = 0; jn < 8; ++jn) s[jn][0] = s[jn][1] = s[jn][2] = s[jn][3] = 0.0f;
#pragma unroll
      for (int jn = 0; jn < 8; ++jn) {
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk += 2) {
          uint32_t b0, b1, b2, b3;
          const int row = jn * 8 + (lane & 7);
          const int col = kk * 16 + (lane >> 3) * 8;
          ldsm_x4(ks + (row * L::kRow + col) * 2, b0, b1, b2, b3);
          mma_bf16(s[jn], qf[kk], b0, b1);
          mma_bf16(s[jn], qf[kk + 1], b2, b3);
        }
      }
      // mask + online softmax (rows r0 and r1 of this thread)
      const int kbase = p * KT + (lane & 3) * 2;
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int jn = 0; jn < 8; ++jn) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int key = kbase + jn * 8 + c;
          s[jn][c] = (key <= lim0) ? s[jn][c] * a.scale_log2 : -INFINITY;
          s[jn][2 + c] = (key <= lim1) ? s[jn][2 + c] * a.scale_log2 : -INFINITY;
          mx0 = fmaxf(mx0, s[jn][c]);
          mx1 = fmaxf(mx1, s[jn][2 + c]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float mu0 = mn0 == -INFINITY ? 0.0f : mn0;
      const float mu1 = mn1 == -INFINITY ? 0.0f : mn1;
      const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
      m0 = mn0;
      m1 = mn1;
      float sum0 = 0.0f, sum1 = 0.0f;
#pragma unroll
      for (int jn = 0; jn < 8; ++jn) {
        s[jn][0] = exp2f(s[jn][0] - mu0);
        s[jn][1] = exp2f(s[jn][1] - mu0);
        s[jn][2] = exp2f(s[jn][2] - mu1);
        s[jn][3] = exp2f(s[jn][3] - mu1);
        sum0 += s[jn][0] + s[jn][1];
        sum1 += s[jn][2] + s[jn][3];
      }
      l0 = l0 * al0 + sum0;
      l1 = l1 * al1 + sum1;
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        o[j][0] *= al0;
        o[j][1] *= al0;
        o[j][2] *= al1;
        o[j][3] *= al1;
      }
      // O += P V (P as bf16 A fragments, 4 k-steps of 16 keys)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int jd = 0; jd < HD / 8; jd += 2) {
          uint32_t b0, b1, b2, b3;
          const int mi = lane >> 3;
          const int row = kk * 16 + (mi & 1) * 8 + (lane & 7);
          const int col = (jd + (mi >> 1)) * 8;
          ldsm_x4_t(vs + (row * L::kRow + col) * 2, b0, b1, b2, b3);
          mma_bf16(o[jd], pa, b0, b1);
          mma_bf16(o[jd + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_wait<0>();

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  if (nsplit == 1) {
    // the whole context in one CTA: normalise and write the output directly
    const float inv0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, inv1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
    __half* d0 = r0 < a.R ? a.out + (size_t)(b * a.T + r0 % a.T) * a.ldo + (size_t)(h * a.G + r0 / a.T) * HD : nullptr;
    __half* d1 = r1 < a.R ? a.out + (size_t)(b * a.T + r1 % a.T) * a.ldo + (size_t)(h * a.G + r1 / a.T) * HD : nullptr;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      const int d = j * 8 + (lane & 3) * 2;
      const float v0 = bf16_round(o[j][0] * inv0), v1 = bf16_round(o[j][1] * inv0);
      const float v2 = bf16_round(o[j][2] * inv1), v3 = bf16_round(o[j][3] * inv1);
      if (d0) {
        check_f16(v0, a.status);
        check_f16(v1, a.status);
        *reinterpret_cast<__half2*>(d0 + d) = __floats2half2_rn(v0, v1);
      }
      if (d1) {
        check_f16(v2, a.status);
        check_f16(v3, a.status);
        *reinterpret_cast<__half2*>(d1 + d) = __floats2half2_rn(v2, v3);
      }
    }
    return;
  }
  // per-split partials (unnormalised O, running max, running sum); attn_combine_kernel merges
  const int bh = b * Hkv + h;
  const size_t sbase = ((size_t)bh * a.nsplit + split) * a.R;
  if ((lane & 3) == 0) {
    if (r0 < a.R) { a.ws_ml[(sbase + r0) * 2] = m0; a.ws_ml[(sbase + r0) * 2 + 1] = l0; }
    if (r1 < a.R) { a.ws_ml[(sbase + r1) * 2] = m1; a.ws_ml[(sbase + r1) * 2 + 1] = l1; }
  }
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) {
    const int d = j * 8 + (lane & 3) * 2;
    if (r0 < a.R) *reinterpret_cast<float2*>(a.ws_o + (sbase + r0) * HD + d) = make_float2(o[j][0], o[j][1]);
    if (r1 < a.R) *reinterpret_cast<float2*>(a.ws_o + (sbase + r1) * HD + d) = make_float2(o[j][2], o[j][3]);
  }
}

// Merge of the split partials: one warp per query row (8 rows per CTA), every (row, kv head,
// batch row) in parallel. Lanes range over the splits for the max and the softmax sum, and
// over the head dimension for O, whose splits are summed in split order.
template <int HD>
__global__ void __launch_bounds__(256) attn_combine_kernel(const Args a) {
  pdl_enter();
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvlen = a.kv_len[b];
  const int npages = (kvlen + a.T + KT - 1) / KT;
  const int nsplit = min(a.nsplit, (npages + kMinPagesPerSplit - 1) / kMinPagesPerSplit);
  if (nsplit <= 1) return;  // the attention kernel already wrote this output
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= a.R) return;
  merge_row<HD>(a, b, h, r, nsplit, lane);
}



static size_t ws_layout(int B, int T, int Hq, int Hkv, int hd, int nsplit, size_t* off_ml,
                        size_t* off_o) {
  const int R = (Hq / Hkv) * T;
  const size_t ml = (((size_t)B * Hkv * nsplit * R * 2 * sizeof(float)) + 255) & ~(size_t)255;
  const size_t o = (size_t)B * Hkv * nsplit * R * hd * sizeof(float);
  if (off_ml) *off_ml = 0;
  if (off_o) *off_o = ml;
  return ml + o;
}

}  // namespace attn
}  // namespace dspark

using namespace dspark;

extern "C" size_t dspark_attention_workspace_bytes(int B, int T, int Hq, int Hkv, int hd,
                                                   int max_splits) {
  if (B <= 0 || T <= 0 || Hq <= 0 || Hkv <= 0 || hd <= 0 || max_splits <= 0) return 0;
  return attn::ws_layout(B, T, Hq, Hkv, hd, max_splits, nullptr, nullptr);
}

extern "C" int dspark_attention(const void* q, int B, int T, int Hq, const dspark_kv_layout* kv,
                                const int32_t* kv_len, int causal, float scale, void* out, int ldo,
                                int max_splits, void* workspace, size_t workspace_bytes,
                                int* status, dspark_stream_t stream) {
  if (!q || !kv || !kv->pool || !kv->block_table || !kv_len || !out || B <= 0 || T <= 0 || Hq <= 0)
    return set_error(DSPARK_ERR_INVALID, "attention: bad arguments");
  const int Hkv = kv->num_kv_heads, hd = kv->head_dim;
  if (Hkv <= 0 || Hq % Hkv) return set_error(DSPARK_ERR_INVALID, "attention: Hq %% Hkv != 0");
  if (hd != 64 && hd != 128) return set_error(DSPARK_ERR_UNSUPPORTED, "attention: head_dim %d", hd);
  if (kv->page_size != attn::KT)
    return set_error(DSPARK_ERR_UNSUPPORTED, "attention: page_size must be %d", attn::KT);
  if (kv->page_bytes != dspark_kv_page_bytes(kv->page_size, Hkv, hd, kv->kv8))
    return set_error(DSPARK_ERR_INVALID, "attention: page_bytes mismatch");
  const int G = Hq / Hkv, R = G * T;
  if (R > 128) return set_error(DSPARK_ERR_UNSUPPORTED, "attention: %d query rows per kv head > 128", R);
  if (ldo < Hq * hd || ldo % 4) return set_error(DSPARK_ERR_INVALID, "attention: ldo");
  if (max_splits < 1 || max_splits > 256) return set_error(DSPARK_ERR_INVALID, "attention: max_splits");
  size_t off_ml, off_o;
  const size_t need = attn::ws_layout(B, T, Hq, Hkv, hd, max_splits, &off_ml, &off_o);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "attention: workspace %zu < %zu", workspace_bytes, need);
  attn::Args a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.B = B; a.T = T; a.Hq = Hq; a.G = G; a.R = R; a.nsplit = max_splits; a.causal = causal ? 1 : 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.kv = *kv;
  a.kv_len = kv_len;
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.status = status;
  a.ws_ml = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + off_ml);
  a.ws_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + off_o);
  // (R + 15) / 16 warps hold query rows; 8-bit pages get at least 4 warps to dequantise them
  const int warps = kv->kv8 ? max((R + 15) / 16, 4) : (R + 15) / 16;
  const dim3 grid(max_splits, Hkv, B), block(warps * 32);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kern, auto combine, int smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "attention: cudaFuncSetAttribute failed");
    int rc = launch_pdl("attention", kern, grid, block, (size_t)smem, st, a);
    if (rc || max_splits == 1) return rc;
    return launch_pdl("attention.combine", combine, dim3((R + 7) / 8, Hkv, B), dim3(256), 0, st, a);
  };
  using namespace attn;
  if (hd == 128) {
    if (kv->kv8)
      return go(attn_kernel<128, true>, attn_combine_kernel<128>, Layout<128, true>::kBytes);
    return go(attn_kernel<128, false>, attn_combine_kernel<128>, Layout<128, false>::kBytes);
  }
  if (kv->kv8) return go(attn_kernel<64, true>, attn_combine_kernel<64>, Layout<64, true>::kBytes);
  return go(attn_kernel<64, false>, attn_combine_kernel<64>, Layout<64, false>::kBytes);
}
