// K1 — W8A16 group-64 dequant GEMM for the small-M verify shape (sm_100a).
//
// Y[M,N] = X[M,K] . W[N,K]^T with W = scale * q + bias per 64-wide group along K. This is
// the arithmetic of mlx's affine 8-bit QuantizedLinear (group_size 64) that the Qwen3 layers
// run under src/mlx_dspark/target.py:58-75 and src/mlx_dspark/batch_engine.py:184-206.
//
// Shape of the problem: M = batch x (draft + 1) is 1..64, N and K are thousands, so every
// weight byte is read once and the kernel is HBM-bound. The design streams weights at
// full bandwidth and keeps the tensor cores fed with a swap-AB MMA:
//   - MMA M = 128 weight rows of one N-tile, MMA N = BN (M padded to 16/32/48/64), K = 16.
//   - A TMA producer warp streams, per 128-wide k-block, the uint8 weight tile (128 x 128 B,
//     128-byte swizzle), the packed fp16 (scale, bias) pairs of its two groups, and the fp16
//     activation tile (BN x 128, 128-byte swizzle) into a ring of shared-memory stages.
//   - Four converter warps turn the uint8 tile into fp16 weights (byte-permute into the
//     1024+q fp16 pattern, subtract 1024 and one fused multiply-add with the group scale and
//     bias) and store them straight into tensor memory: each thread owns one weight row,
//     which is one TMEM lane, so the A operand never takes a second trip through shared
//     memory.
//   - One thread issues tcgen05.mma (A from TMEM, B from shared memory) into a double-
//     buffered TMEM accumulator and signals the ring with tcgen05.commit.
//   - Four epilogue warps read the accumulator with tcgen05.ld and apply the epilogue.
// Work split: the flattened (tile, k-block) space is cut into equal contiguous ranges, one
// per CTA (stream-K). A tile covered by several CTAs is finished by the last CTA to arrive
// (fp32 partials in the caller's workspace, one atomic counter per tile, summation in CTA
// order so results do not depend on arrival order). No CTA ever waits for another.
// With programmatic dependent launch the weight stream of a GEMM starts while the kernel
// before it is still finishing; only the activation loads wait for it.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace dspark {
namespace w8 {

constexpr int BM = 128;         // weight rows per tile (MMA M)
constexpr int BK = 128;         // k-block width (bytes of one weight row per stage)
constexpr int kConvWarps = 4;   // warps 0..3
constexpr int kEpiWarps = 4;    // warps 4..7
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kABufs = 2;       // TMEM A ring (64 columns each: 128 fp16 per lane)
constexpr int kTmemCols = 256;  // [0,128) A ring, [128,256) two accumulators of <= 64 columns
constexpr uint32_t kWBytes = BM * BK;   // 16 KB
constexpr uint32_t kSBBytes = 2 * BM * 4;  // 1 KB
// Workspace: a fixed counter region first (one int per N-tile, at most kMaxTiles), then the
// fp32 partials. The fixed offset keeps calls of different N from overlapping one call's
// partials with another call's counters.
constexpr int kMaxTiles = 16384;
constexpr size_t kCounterBytes = kMaxTiles * sizeof(int);

struct Params {
  int M, N, K;
  int tiles;  // N / 128
  int kb;     // K / 128 (k-blocks per tile)
  long long total;
  int ldy, ldr;
  int epilogue;
  void* y;
  const void* residual;
  float* partials;  // [grid][2][BN][128]
  int* counters;    // [tiles]
  int* status;
};

__device__ __forceinline__ long long range_start(long long b, long long total, long long G) {
  return b * total / G;
}
// the CTA whose range contains flattened k-block g
__device__ __forceinline__ long long range_owner(long long g, long long total, long long G) {
  return ((g + 1) * G + total - 1) / total - 1;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

template <int BN>
__device__ __forceinline__ void epilogue_store(const Params& p, int tile, int er, const float* acc,
                                               float* xch) {
  const int n = tile * BM + er;
  switch (p.epilogue) {
    case DSPARK_EPI_STORE_BF16: {
      __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
#pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < p.M) y[(size_t)m * p.ldy + n] = __float2bfloat16_rn(acc[m]);
      break;
    }
    case DSPARK_EPI_STORE_F32: {
      float* y = static_cast<float*>(p.y);
#pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < p.M) y[(size_t)m * p.ldy + n] = acc[m];
      break;
    }
    case DSPARK_EPI_RESIDUAL_BF16: {
      __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
      const __nv_bfloat16* r = static_cast<const __nv_bfloat16*>(p.residual);
#pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < p.M) {
          const float rv = __bfloat162float(r[(size_t)m * p.ldr + n]);
          y[(size_t)m * p.ldy + n] = __float2bfloat16_rn(rv + bf16_round(acc[m]));
        }
      break;
    }
    case DSPARK_EPI_SILU_MUL_F16: {
      // rows [0,64) of the tile are gate rows, [64,128) the matching up rows
      if (er >= 64) {
#pragma unroll
        for (int m = 0; m < BN; ++m) xch[(er - 64) * BN + m] = acc[m];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (er < 64) {
        __half* y = static_cast<__half*>(p.y);
        const int col = tile * 64 + er;
#pragma unroll
        for (int m = 0; m < BN; ++m)
          if (m < p.M) {
            const float g = bf16_round(acc[m]);
            const float u = bf16_round(xch[er * BN + m]);
            const float s = bf16_round(silu_f(g));
            y[(size_t)m * p.ldy + col] = __float2half_rn(bf16_round(s * u));
          }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      break;
    }
    default:
      break;
  }
}

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t kXBytes = 2u * BN * 128u;
  static constexpr uint32_t kStageBytes = kWBytes + kXBytes + kSBBytes;
  static constexpr uint32_t kXchBytes = 64u * BN * 4u;
  static constexpr uint32_t kBarBytes = 256;
  static constexpr uint32_t kTotal = 1024 + STAGES * kStageBytes + kXchBytes + kBarBytes;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, (BN <= 32 ? 2 : 1))
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_sb,
                    const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw);

  const uint32_t w_s = base;
  const uint32_t x_s = base + STAGES * kWBytes;
  const uint32_t sb_s = x_s + STAGES * L::kXBytes;
  float* xch = reinterpret_cast<float*>(sbase + STAGES * L::kStageBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbase + STAGES * L::kStageBytes + L::kXchBytes);
  // barrier map
  auto full = [&](int s) { return smem_u32(bars + s); };
  auto xfull = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto empty = [&](int s) { return smem_u32(bars + 2 * STAGES + s); };
  auto afull = [&](int a) { return smem_u32(bars + 3 * STAGES + a); };
  auto aempty = [&](int a) { return smem_u32(bars + 3 * STAGES + kABufs + a); };
  auto accfull = [&](int b) { return smem_u32(bars + 3 * STAGES + 2 * kABufs + b); };
  auto accempty = [&](int b) { return smem_u32(bars + 3 * STAGES + 2 * kABufs + 2 + b); };
  const uint32_t done_bar = smem_u32(bars + 3 * STAGES + 2 * kABufs + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 2 * kABufs + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_holder + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(xfull(s), 1);
      mbar_init(empty(s), kConvWarps + 1);
    }
    for (int a = 0; a < kABufs; ++a) {
      mbar_init(afull(a), kConvWarps);
      mbar_init(aempty(a), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accfull(b), 1);
      mbar_init(accempty(b), kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_sb);
      tma_prefetch_desc(&tm_x);
    }
    __syncwarp();
    tmem_alloc(smem_u32(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  const long long G = gridDim.x;
  const long long total = p.total;
  const long long start = range_start(blockIdx.x, total, G);
  const long long end = range_start(blockIdx.x + 1, total, G);
  const int n_iter = (int)(end - start);
  const int KB = p.kb;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      const int pre = n_iter < STAGES ? n_iter : STAGES;
      // weights do not depend on the previous kernel: start streaming them at once
      for (int i = 0; i < pre; ++i) {
        const long long g = start + i;
        const int tile = (int)(g / KB), kb = (int)(g % KB);
        mbar_arrive_expect_tx(full(i), kWBytes + kSBBytes);
        tma_load_2d(w_s + i * kWBytes, &tm_w, full(i), kb * BK, tile * BM, pol_w);
        tma_load_2d(sb_s + i * kSBBytes, &tm_sb, full(i), tile * BM, kb * 2, pol_w);
      }
      pdl_wait();  // activations are written by the previous kernel
      for (int i = 0; i < pre; ++i) {
        const long long g = start + i;
        const int kb = (int)(g % KB);
        mbar_arrive_expect_tx(xfull(i), L::kXBytes);
        tma_load_2d(x_s + i * L::kXBytes, &tm_x, xfull(i), kb * BK, 0, pol_x);
        tma_load_2d(x_s + i * L::kXBytes + BN * 128, &tm_x, xfull(i), kb * BK + 64, 0, pol_x);
      }
      int issued = pre;
      for (int i = pre; i < n_iter; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status)) break;
        const long long g = start + i;
        const int tile = (int)(g / KB), kb = (int)(g % KB);
        mbar_arrive_expect_tx(full(s), kWBytes + kSBBytes);
        tma_load_2d(w_s + s * kWBytes, &tm_w, full(s), kb * BK, tile * BM, pol_w);
        tma_load_2d(sb_s + s * kSBBytes, &tm_sb, full(s), tile * BM, kb * 2, pol_w);
        mbar_arrive_expect_tx(xfull(s), L::kXBytes);
        tma_load_2d(x_s + s * L::kXBytes, &tm_x, xfull(s), kb * BK, 0, pol_x);
        tma_load_2d(x_s + s * L::kXBytes + BN * 128, &tm_x, xfull(s), kb * BK + 64, 0, pol_x);
        issued = i + 1;
      }
      // drain: no bulk copy may still be writing into this CTA's shared memory at exit
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int i = first; i < issued; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        volatile int never = 0;
        mbar_wait(full(s), ph, &never, p.status);
        mbar_wait(xfull(s), ph, &never, p.status);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN);
      int seg = 0;
      for (int i = 0; i < n_iter; ++i) {
        const long long g = start + i;
        const int kb = (int)(g % KB);
        const bool seg_first = (i == 0) || (kb == 0);
        const bool seg_last = (i == n_iter - 1) || (kb == KB - 1);
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        const int a = i % kABufs;
        const uint32_t aph = (uint32_t)(i / kABufs) & 1u;
        const int ab = seg & 1;
        const uint32_t abph = (uint32_t)(seg >> 1) & 1u;
        if (seg_first && !mbar_wait(accempty(ab), abph ^ 1u, abort_flag, p.status)) break;
        if (!mbar_wait(afull(a), aph, abort_flag, p.status)) break;
        if (!mbar_wait(xfull(s), ph, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + 128u + (uint32_t)ab * 64u;
#pragma unroll
        for (int j = 0; j < BK / 16; ++j) {
          const uint32_t a_tmem = tmem_base + (uint32_t)a * 64u + (uint32_t)j * 8u;
          const uint32_t b_addr = x_s + s * L::kXBytes + (j >> 2) * (BN * 128) + (j & 3) * 32;
          tc_mma_ts(d_tmem, a_tmem, umma_desc_sw128_kmajor(b_addr), idesc,
                    (seg_first && j == 0) ? 0u : 1u);
        }
        tc_commit(empty(s));
        tc_commit(aempty(a));
        if (seg_last) {
          tc_commit(accfull(ab));
          ++seg;
        }
      }
      // every MMA issued above has finished before TMEM is released
      tc_commit(done_bar);
      volatile int never = 0;
      mbar_wait(done_bar, 0, &never, p.status);
    }
  } else if (warp < kConvWarps) {
    // converters: thread r owns weight row r of the tile == TMEM lane r
    const int r = threadIdx.x;
    const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
    const uint32_t k1024 = 0x64006400u;  // fp16x2 {1024, 1024}
    for (int i = 0; i < n_iter; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      const int a = i % kABufs;
      const uint32_t aph = (uint32_t)(i / kABufs) & 1u;
      if (!mbar_wait(full(s), ph, abort_flag, p.status)) break;
      if (!mbar_wait(aempty(a), aph ^ 1u, abort_flag, p.status)) break;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sbv;
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(sbv) : "r"(sb_s + s * kSBBytes + (h * BM + r) * 4));
        const uint32_t sc2 = __byte_perm(sbv, 0, 0x1010);  // {scale, scale}
        const uint32_t bi2 = __byte_perm(sbv, 0, 0x3232);  // {bias, bias}
        uint32_t out[32];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int chunk = h * 4 + j;
          const uint32_t addr = w_s + s * kWBytes + r * 128 + ((chunk ^ (r & 7)) << 4);
          uint32_t v0, v1, v2, v3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                       : "r"(addr));
          const uint32_t vv[4] = {v0, v1, v2, v3};
#pragma unroll
          for (int w = 0; w < 4; ++w) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t q2 = __byte_perm(vv[w], 0x64646464u, hh ? 0x4342u : 0x4140u);
              __half2 qh = *reinterpret_cast<const __half2*>(&q2);
              qh = __hsub2(qh, *reinterpret_cast<const __half2*>(&k1024));
              const __half2 wv = __hfma2(qh, *reinterpret_cast<const __half2*>(&sc2),
                                         *reinterpret_cast<const __half2*>(&bi2));
              out[j * 8 + w * 2 + hh] = *reinterpret_cast<const uint32_t*>(&wv);
            }
          }
        }
        tmem_st32(lane_base + (uint32_t)a * 64u + (uint32_t)h * 32u, out);
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(empty(s));
        mbar_arrive(afull(a));
      }
    }
  } else if (warp < kConvWarps + kEpiWarps) {
    // epilogue: thread er owns row er of the tile (TMEM lane er)
    const int er = threadIdx.x - kConvWarps * 32;
    const int quad = warp & 3;
    pdl_wait();
    int seg = 0;
    long long g = start;
    while (g < end) {
      const int tile = (int)(g / KB);
      const long long tile_lo = (long long)tile * KB;
      const long long seg_end = (end < tile_lo + KB) ? end : tile_lo + KB;
      const bool whole = (g == tile_lo) && (seg_end == tile_lo + KB);
      const int ab = seg & 1;
      const uint32_t abph = (uint32_t)(seg >> 1) & 1u;
      if (!mbar_wait(accfull(ab), abph, abort_flag, p.status)) break;
      tc_fence_after();
      float acc[BN];
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        uint32_t rr[16];
        tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + 128u + (uint32_t)ab * 64u +
                      (uint32_t)c * 16u,
                  rr);
        tc_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[c * 16 + t] = __uint_as_float(rr[t]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty(ab));

      if (whole) {
        epilogue_store<BN>(p, tile, er, acc, xch);
      } else {
        // partial of this CTA: row er's BN values contiguous, so the finishing CTA reads one
        // run of BN floats per contributor with 16-byte loads
        const int slot = (int)blockIdx.x * 2 + (seg == 0 ? 0 : 1);
        float4* part = reinterpret_cast<float4*>(p.partials + (size_t)slot * BN * BM + er * BN);
#pragma unroll
        for (int j = 0; j < BN / 4; ++j)
          part[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const long long c_lo = range_owner(tile_lo, total, G);
        const long long c_hi = range_owner(tile_lo + KB - 1, total, G);
        if (er == 0) {
          const int contributors = (int)(c_hi - c_lo + 1);
          // One acq_rel gpu-scope atomic per CTA. Release: the partials of all 128 threads
          // (ordered before it by the barrier; release is cumulative) are visible to whoever
          // reads the final count. Acquire: the last arriver sees every partial.
          int old;
          asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                       : "=r"(old)
                       : "l"(p.counters + tile)
                       : "memory");
          *last_flag = (old == contributors - 1) ? 1 : 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int is_last = *last_flag;
        if (is_last) {
          float sum[BN];
#pragma unroll
          for (int m = 0; m < BN; ++m) sum[m] = 0.0f;
          // U contributors' loads in flight at once; the sum stays in contributor order
          constexpr int U = BN <= 16 ? 2 : 1;
          for (long long c = c_lo; c <= c_hi; c += U) {
            float4 t[U][BN / 4];
#pragma unroll
            for (int u = 0; u < U; ++u) {
              if (c + u <= c_hi) {
                const int cj = (range_start(c + u, total, G) >= tile_lo) ? 0 : 1;
                const float4* cp = reinterpret_cast<const float4*>(
                    p.partials + ((size_t)(c + u) * 2 + cj) * BN * BM + er * BN);
#pragma unroll
                for (int j = 0; j < BN / 4; ++j) t[u][j] = __ldcg(cp + j);
              }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
              if (c + u <= c_hi) {
#pragma unroll
                for (int j = 0; j < BN / 4; ++j) {
                  sum[4 * j] += t[u][j].x;
                  sum[4 * j + 1] += t[u][j].y;
                  sum[4 * j + 2] += t[u][j].z;
                  sum[4 * j + 3] += t[u][j].w;
                }
              }
            }
          }
          if (er == 0) p.counters[tile] = 0;
          epilogue_store<BN>(p, tile, er, sum, xch);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      ++seg;
      g = seg_end;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------------------------------
// SIMT cross-check kernel: one warp per output column n, fp32 dequant and accumulation.
// Used by the GPU tests to check the tensor-core path on the device and as a diagnostic.
template <int MT>
__global__ void __launch_bounds__(256) w8a16_simt_kernel(const __half* __restrict__ x, int ldx,
                                                         const uint8_t* __restrict__ wq,
                                                         const uint32_t* __restrict__ wsb,
                                                         Params p) {
  pdl_wait();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.N) return;
  const int n = warp;
  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
  for (int k = lane; k < p.K; k += 32) {
    const uint32_t sbv = wsb[(size_t)(k >> 6) * p.N + n];
    const __half2 sb2 = *reinterpret_cast<const __half2*>(&sbv);
    const float w = __low2float(sb2) * (float)wq[(size_t)n * p.K + k] + __high2float(sb2);
#pragma unroll
    for (int m = 0; m < MT; ++m)
      if (m < p.M) acc[m] += __half2float(x[(size_t)m * ldx + k]) * w;
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = warp_sum(acc[m]);
  if (lane != 0) return;
  // scalar epilogue (one thread per column)
  for (int m = 0; m < p.M; ++m) {
    const float a = acc[m];
    switch (p.epilogue) {
      case DSPARK_EPI_STORE_BF16:
        static_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] = __float2bfloat16_rn(a);
        break;
      case DSPARK_EPI_STORE_F32:
        static_cast<float*>(p.y)[(size_t)m * p.ldy + n] = a;
        break;
      case DSPARK_EPI_RESIDUAL_BF16: {
        const float rv =
            __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[(size_t)m * p.ldr + n]);
        static_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] =
            __float2bfloat16_rn(rv + bf16_round(a));
        break;
      }
      default:
        break;  // the gate/up pairing needs the tiled kernel
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

static int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* ptr,
                       uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto enc = get_encoder();
  if (!enc) return set_error(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || (row_bytes & 15u) != 0)
    return set_error(DSPARK_ERR_ALIGN, "tensor map base/stride not 16-byte aligned");
  if ((box_inner * (uint32_t)elem_bytes) % 16u != 0)
    return set_error(DSPARK_ERR_ALIGN, "tensor map box inner extent not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSPARK_OK;
}

static int sm_count() {
  static int cached = 0;
  if (cached) return cached;
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n > 0) cached = n;
  return n > 0 ? n : 148;
}

static int pick_bn(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 48 ? 48 : 64; }

template <int BN>
struct Cfg;
template <>
struct Cfg<16> { static constexpr int kStages = 4; static constexpr int kCtasPerSm = 2; };
template <>
struct Cfg<32> { static constexpr int kStages = 4; static constexpr int kCtasPerSm = 2; };
template <>
struct Cfg<48> { static constexpr int kStages = 5; static constexpr int kCtasPerSm = 1; };
template <>
struct Cfg<64> { static constexpr int kStages = 5; static constexpr int kCtasPerSm = 1; };

static long long grid_for(long long total, int ctas_per_sm) {
  const long long g = (long long)sm_count() * ctas_per_sm;
  return std::min<long long>(g, total);
}

template <int BN>
static int launch_tc(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, Params p,
                     cudaStream_t st) {
  constexpr int S = Cfg<BN>::kStages;
  using L = Smem<BN, S>;
  CUtensorMap tw, tsb, tx;
  int rc;
  if ((rc = make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wq, (uint64_t)p.K, (uint64_t)p.N,
                        (uint64_t)p.K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_map_2d(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wsb, (uint64_t)p.N,
                        (uint64_t)(p.K / 64), (uint64_t)p.N * 4, BM, 2,
                        CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, (uint64_t)p.K, (uint64_t)p.M,
                        (uint64_t)ldx * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  auto kern = w8a16_tc_kernel<BN, S>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kTotal) !=
        cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "cudaFuncSetAttribute(smem=%u) failed", L::kTotal);
    configured = true;
  }
  const long long grid = grid_for(p.total, Cfg<BN>::kCtasPerSm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tsb, tx, p);
  if (e != cudaSuccess)
    return set_error(DSPARK_ERR_LAUNCH, "w8a16 tc launch failed: %s", cudaGetErrorString(e));
  return DSPARK_OK;
}

static size_t ws_bytes(int M, int N, int K) {
  const int bn = pick_bn(M);
  const int cps = bn <= 32 ? 2 : 1;
  const long long total = (long long)(N / BM) * (K / BK);
  const long long grid = std::min<long long>((long long)sm_count() * cps, std::max(total, 1LL));
  return kCounterBytes + (size_t)grid * 2 * bn * BM * sizeof(float);
}

}  // namespace w8
}  // namespace dspark

using namespace dspark;

extern "C" size_t dspark_w8a16_gemm_workspace_bytes(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return w8::ws_bytes(M, N, K);
}

static int gemm_common_checks(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                              int M, int N, int K, void* y, int epilogue, const void* residual) {
  if (!x || !wq || !wsb || !y) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: null pointer");
  if (M < 1 || M > 64) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: M=%d not in [1,64]", M);
  if (N / 128 > 16384) return set_error(DSPARK_ERR_UNSUPPORTED, "w8a16_gemm: N=%d too large", N);
  if (N % 128 || K % 128 || N <= 0 || K <= 0)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: N=%d, K=%d must be positive multiples of 128", N, K);
  if (ldx < K || ldx % 8) return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: ldx=%d", ldx);
  if (epilogue < 0 || epilogue > 3)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: epilogue %d", epilogue);
  if (epilogue == DSPARK_EPI_RESIDUAL_BF16 && !residual)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: residual epilogue without residual");
  return DSPARK_OK;
}

extern "C" int dspark_w8a16_gemm(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                                 int M, int N, int K, void* y, int ldy, const void* residual,
                                 int ldr, int epilogue, void* workspace, size_t workspace_bytes,
                                 int* status, dspark_stream_t stream) {
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, y, epilogue, residual);
  if (rc) return rc;
  const size_t need = w8::ws_bytes(M, N, K);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "w8a16_gemm: workspace %zu < %zu bytes", workspace_bytes, need);
  w8::Params p{};
  p.M = M; p.N = N; p.K = K;
  p.tiles = N / w8::BM;
  p.kb = K / w8::BK;
  p.total = (long long)p.tiles * p.kb;
  p.ldy = ldy; p.ldr = ldr;
  p.epilogue = epilogue;
  p.y = y;
  p.residual = residual;
  const size_t counters = w8::kCounterBytes;
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + counters);
  p.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (w8::pick_bn(M)) {
    case 16: return w8::launch_tc<16>(x, ldx, wq, wsb, p, st);
    case 32: return w8::launch_tc<32>(x, ldx, wq, wsb, p, st);
    case 48: return w8::launch_tc<48>(x, ldx, wq, wsb, p, st);
    default: return w8::launch_tc<64>(x, ldx, wq, wsb, p, st);
  }
}

// Diagnostic entry point: the same product on CUDA cores (fp32 dequant, one warp per
// column). Not used on the serving path.
extern "C" int dspark_w8a16_gemm_simt(const void* x, int ldx, const uint8_t* wq,
                                      const uint32_t* wsb, int M, int N, int K, void* y, int ldy,
                                      const void* residual, int ldr, int epilogue,
                                      dspark_stream_t stream) {
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, y, epilogue, residual);
  if (rc) return rc;
  if (epilogue == DSPARK_EPI_SILU_MUL_F16)
    return set_error(DSPARK_ERR_UNSUPPORTED, "w8a16_gemm_simt: silu-mul epilogue not supported");
  w8::Params p{};
  p.M = M; p.N = N; p.K = K;
  p.ldy = ldy; p.ldr = ldr; p.epilogue = epilogue; p.y = y; p.residual = residual;
  const int blocks = (N * 32 + 255) / 256;
  w8::w8a16_simt_kernel<64><<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(x), ldx, wq, wsb, p);
  return check_launch("w8a16_gemm_simt");
}
