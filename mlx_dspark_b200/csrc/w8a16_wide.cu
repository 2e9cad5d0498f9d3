// K1w — W8A16 group-64 dequant GEMM for prefill chunks (large M), sm_100a.
//
// Y[M,N] = X[M,K] . W[N,K]^T with W = scale * q + bias per 64-wide group along K: the
// arithmetic of the small-M verify GEMM (w8a16_gemm.cu) at the M of a prefill chunk. The
// reference prefills in chunks of 2048 tokens (src/mlx_dspark/generate.py:613-656, each chunk
// one Target.run, src/mlx_dspark/target.py:51-75); at M in the hundreds to thousands every
// weight byte feeds hundreds of MMA rows and the product is compute-bound.
//
// Design (one CTA per SM, persistent over output tiles):
//   - A tile is 128 weight rows x BN tokens (BN 256, or 128 for short chunks). Tiles are
//     numbered n-major, m-minor, and CTA b takes tiles b, b + grid, ...: the CTAs running at
//     one time share weight tiles, and the activation rows stay in L2 across the n-tiles.
//   - Per 64-wide k-block a TMA producer warp loads the uint8 weight tile (128 x 64 B, 64-byte
//     swizzle), the packed fp16 (scale, bias) pairs of its group and the fp16 activation tile
//     (BN x 64, 128-byte swizzle) into a ring of shared-memory stages.
//   - Four converter warps dequantize the weight tile (byte-permute into the 1024+q fp16
//     pattern, subtract 1024, one fused multiply-add with scale and bias: the verify GEMM's
//     arithmetic, so both paths produce the same fp16 weights) and store it into a ring of
//     tensor-memory A buffers; thread r owns weight row r == TMEM lane r.
//   - One thread issues tcgen05.mma (A from TMEM, B = activations from shared memory) into the
//     TMEM accumulator: one of 256 columns at BN 256, two of 128 at BN 128.
//   - Four epilogue warps read the accumulator, round it to bf16 pairs held in registers,
//     release it to the MMA warp, and only then write the outputs: bf16, bf16 residual add
//     (with an optional fp16 copy), or SiLU(gate) * up as fp16. They fill a ring of shared
//     staging buffers 16 activation rows at a time, and one thread writes each chunk with a
//     TMA tensor store; the residual add reads its chunks through TMA loads issued two chunks
//     ahead. (Per-thread 2-byte global stores and loads measured 17-80 us per tile under the
//     mainloop's L2 traffic, longer than the tile's MMAs.) The fp32 store (a diagnostic)
//     writes from registers before releasing the accumulator.
// Every wait is bounded (DSPARK_ERR_TIMEOUT in the caller's status word, then every role
// unwinds); the roles that later meet at a named barrier first agree on a vote.
#include <algorithm>

#include "common.cuh"
#include "tensor_map.cuh"

namespace dspark {
namespace w8w {

constexpr int BM = 128;              // weight rows per tile (MMA M)
constexpr int BK = 64;               // k-block: one quantization group
constexpr int kConvWarps = 4;        // warps 0..3
constexpr int kEpiWarps = 4;         // warps 4..7
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int AB = 8;                // TMEM A ring depth (32 columns = 64 fp16 per lane each)
constexpr uint32_t kARing0 = 256;    // A ring at columns [256, 512); accumulators in [0, 256)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kWBytes = BM * BK;  // 8 KB
constexpr uint32_t kSBBytes = BM * 4;  // 512 B
constexpr int kXchStride = 12;         // u32 per exchanged row: 8 used, 48-byte rows
constexpr int kNB = 4;                 // output staging ring: 16 activation rows per buffer
constexpr uint32_t kStgBytes = 4096;   // 16 rows x 256 B (bf16 x 128 columns)

struct Params {
  int M, N, K;
  int n_tiles, m_tiles, kb;
  int epilogue;
  void* y;
  int ldy;
  const void* residual;
  int ldr;
  __half* copy16;  // RESIDUAL_BF16: fp16 copy of the output rows, or null
  int copy16_ld;
  int* status;
};

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 5 : 8;
  static constexpr int kAccBufs = BN == 256 ? 1 : 2;
  static constexpr uint32_t kXBytes = (uint32_t)BN * 128u;  // BN rows x 64 fp16
  static constexpr uint32_t kStageBytes = kWBytes + kXBytes + kSBBytes;
  static constexpr uint32_t kXchBytes = 64u * kXchStride * 4u;
  static constexpr uint32_t kBarBytes = 512;
  static constexpr uint32_t kTotal =
      1024 + kStages * kStageBytes + kNB * kStgBytes + kXchBytes + kBarBytes;
};

__device__ __forceinline__ float lo_f(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float hi_f(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// AND of `ok` over the 128 epilogue threads (named barrier 2): the epilogue warps leave their
// loop together, so none waits at the exchange barrier for a warp that has gone.
__device__ __forceinline__ bool epi_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    w8a16_wide_kernel(const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_sb,
                      const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_y,   // output (store)
                      const __grid_constant__ CUtensorMap tm_r,   // residual (load)
                      const __grid_constant__ CUtensorMap tm_c,   // fp16 copy (store)
                      const Params p) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  constexpr int NACC = C::kAccBufs;
  static_assert(NACC * BN <= (int)kARing0, "TMEM layout");
  static_assert(kARing0 + AB * 32 <= kTmemCols, "TMEM layout");
  static_assert((2 * S + 2 * AB + 2 * NACC + kNB + 2) * 8 <= (int)C::kBarBytes, "barrier region");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sbase = smem_raw + (base - raw);
  const uint32_t w_s = base;                    // S x 8 KB, 1024-aligned
  const uint32_t x_s = w_s + S * kWBytes;       // S x BN*128 B, 1024-aligned
  const uint32_t sb_s = x_s + S * C::kXBytes;   // S x 512 B
  const uint32_t stg_s = sb_s + S * kSBBytes;   // kNB x 4 KB output staging, 512-aligned
  uint8_t* stg = sbase + S * C::kStageBytes;
  uint32_t* xch = reinterpret_cast<uint32_t*>(stg + kNB * kStgBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(stg + kNB * kStgBytes + C::kXchBytes);
  auto full = [&](int s) { return smem_u32(bars + s); };
  auto empty = [&](int s) { return smem_u32(bars + S + s); };
  auto afull = [&](int a) { return smem_u32(bars + 2 * S + a); };
  auto aempty = [&](int a) { return smem_u32(bars + 2 * S + AB + a); };
  auto accfull = [&](int b) { return smem_u32(bars + 2 * S + 2 * AB + b); };
  auto accempty = [&](int b) { return smem_u32(bars + 2 * S + 2 * AB + NACC + b); };
  const uint32_t done_bar = smem_u32(bars + 2 * S + 2 * AB + 2 * NACC);
  auto rbar = [&](int b) { return smem_u32(bars + 2 * S + 2 * AB + 2 * NACC + 1 + b); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * S + 2 * AB + 2 * NACC + 1 + kNB);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), kConvWarps + 1);  // the converters' reads of W and the MMAs' of X
    }
    for (int a = 0; a < AB; ++a) {
      mbar_init(afull(a), kConvWarps);
      mbar_init(aempty(a), 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(accfull(b), 1);
      mbar_init(accempty(b), kEpiWarps);
    }
    mbar_init(done_bar, 1);
    for (int b = 0; b < kNB; ++b) mbar_init(rbar(b), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_w);
      tma_prefetch_desc(&tm_sb);
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_y);
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

  const int tiles = p.n_tiles * p.m_tiles;
  const int KB = p.kb;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_normal();  // re-read by the CTAs of one n-tile
      const uint64_t pol_x = policy_evict_last();    // re-read by every n-tile
      pdl_wait();  // activations (and nothing else) come from the previous kernel
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int nt = t / p.m_tiles, mt = t - nt * p.m_tiles;
        for (int kb = 0; kb < KB; ++kb) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          if (it >= S && !mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full(s), kWBytes + kSBBytes + C::kXBytes);
          tma_load_2d(w_s + s * kWBytes, &tm_w, full(s), kb * BK, nt * BM, pol_w);
          tma_load_2d(sb_s + s * kSBBytes, &tm_sb, full(s), nt * BM, kb, pol_w);
          tma_load_2d(x_s + s * C::kXBytes, &tm_x, full(s), kb * BK, mt * BN, pol_x);
          ++it;
        }
      }
      // drain: no bulk copy may still be writing into this CTA's shared memory at exit
      for (int i = it > S ? it - S : 0; i < it; ++i) {
        volatile int never = 0;
        mbar_wait(full(i % S), (uint32_t)(i / S) & 1u, &never, p.status);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN);
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tl) {
        const int ab = tl % NACC;
        const uint32_t abph = (uint32_t)(tl / NACC) & 1u;
        if (!mbar_wait(accempty(ab), abph ^ 1u, abort_flag, p.status)) break;
        const uint32_t d_tmem = tmem_base + (uint32_t)(ab * BN);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          const uint32_t ph = (uint32_t)(it / S) & 1u;
          const int a = it % AB;
          const uint32_t aph = (uint32_t)(it / AB) & 1u;
          if (!mbar_wait(afull(a), aph, abort_flag, p.status) ||
              !mbar_wait(full(s), ph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < BK / 16; ++j)
            tc_mma_ts(d_tmem, tmem_base + kARing0 + (uint32_t)(a * 32 + j * 8),
                      umma_desc_sw128_kmajor(x_s + s * C::kXBytes + j * 32), idesc,
                      (kb | j) ? 1u : 0u);
          tc_commit(empty(s));
          tc_commit(aempty(a));
        }
        if (ok) tc_commit(accfull(ab));
      }
      // every MMA issued above has finished before TMEM is released
      tc_commit(done_bar);
      volatile int never = 0;
      mbar_wait(done_bar, 0, &never, p.status);
    }
  } else if (warp < kConvWarps) {
    // converters: thread r owns weight row r of the tile == TMEM lane r
    const int r = threadIdx.x;
    const uint32_t a_lane = tmem_base + ((uint32_t)(warp * 32) << 16) + kARing0;
    const uint32_t k1024 = 0x64006400u;  // fp16x2 {1024, 1024}
    const int sw = (r >> 1) & 3;         // 64-byte swizzle: 16-byte chunk c sits at c ^ sw
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int s = it % S;
        const uint32_t ph = (uint32_t)(it / S) & 1u;
        const int a = it % AB;
        const uint32_t aph = (uint32_t)(it / AB) & 1u;
        bool w_ok = mbar_wait(full(s), ph, abort_flag, p.status) &&
                    mbar_wait(aempty(a), aph ^ 1u, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, w_ok)) {  // tcgen05.st below is warp-collective
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sbv;
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(sbv) : "r"(sb_s + s * kSBBytes + r * 4));
        const uint32_t sc2 = __byte_perm(sbv, 0, 0x1010);  // {scale, scale}
        const uint32_t bi2 = __byte_perm(sbv, 0, 0x3232);  // {bias, bias}
        uint32_t out[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t addr = w_s + s * kWBytes + r * 64 + ((c ^ sw) << 4);
          uint32_t v[4];
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                       : "r"(addr));
#pragma unroll
          for (int w = 0; w < 4; ++w) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t q2 = __byte_perm(v[w], 0x64646464u, hh ? 0x4342u : 0x4140u);
              __half2 qh = *reinterpret_cast<const __half2*>(&q2);
              qh = __hsub2(qh, *reinterpret_cast<const __half2*>(&k1024));
              const __half2 wv = __hfma2(qh, *reinterpret_cast<const __half2*>(&sc2),
                                         *reinterpret_cast<const __half2*>(&bi2));
              out[c * 8 + w * 2 + hh] = *reinterpret_cast<const uint32_t*>(&wv);
            }
          }
        }
        tmem_st32(a_lane + (uint32_t)(a * 32), out);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(empty(s));
          mbar_arrive(afull(a));
        }
      }
    }
  } else if (warp < kConvWarps + kEpiWarps) {
    // epilogue: thread er owns row er of the tile (TMEM lane er) == column er of each staged
    // chunk; thread 0 issues the chunk's TMA loads and stores. gc counts this CTA's chunks over
    // its tiles (staging buffer gc % kNB, residual-load phase (gc / kNB) & 1); lr counts the
    // residual loads issued (always chunks gc .. lr - 1 in flight).
    const int quad = warp & 3;
    const int er = quad * 32 + lane;
    const bool issuer = er == 0;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const bool res = p.epilogue == DSPARK_EPI_RESIDUAL_BF16;
    const bool silu = p.epilogue == DSPARK_EPI_SILU_MUL_F16;
    const bool cp16 = p.copy16 != nullptr;
    const uint64_t pol_r = policy_evict_normal();
    pdl_wait();  // the residual and the outputs belong to the kernels before this one
    int tl = 0, gc = 0, lr = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
      const int nt = t / p.m_tiles, mt = t - nt * p.m_tiles;
      const int m0 = mt * BN;
      const int nch = min(BN / 16, (p.M - m0 + 15) / 16);
      if (res && issuer) {
        // this tile's first two residual chunks, into buffers last stored from by chunks
        // gc - 4 and gc - 3 (at most gc - 2 and gc - 1 may still be reading)
        bulk_wait_read<2>();
        for (int j = 0; j < 2 && j < nch; ++j, ++lr) {
          const int b = lr % kNB;
          mbar_arrive_expect_tx(rbar(b), kStgBytes);
          tma_load_2d(stg_s + b * kStgBytes, &tm_r, rbar(b), nt * BM, m0 + 16 * j, pol_r);
        }
      }
      const int ab = tl % NACC;
      const uint32_t abph = (uint32_t)(tl / NACC) & 1u;
      const bool w_ok = mbar_wait(accfull(ab), abph, abort_flag, p.status);
      if (!epi_all(w_ok)) break;
      tc_fence_after();
      const uint32_t acc_t = tmem_base + lane_off + (uint32_t)(ab * BN);
      if (p.epilogue == DSPARK_EPI_STORE_F32) {
        const int mc = min(BN, p.M - m0);
        float* y = static_cast<float*>(p.y) + (size_t)m0 * p.ldy + nt * BM + er;
        for (int c = 0; c < BN / 16; ++c) {
          uint32_t rr[16];
          tmem_ld16(acc_t + (uint32_t)(c * 16), rr);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c * 16 + j < mc) y[(size_t)(c * 16 + j) * p.ldy] = __uint_as_float(rr[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accempty(ab));
        continue;
      }
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r0[16], r1[16];
        tmem_ld16(acc_t + (uint32_t)(c * 32), r0);
        tmem_ld16(acc_t + (uint32_t)(c * 32 + 16), r1);
        tc_wait_ld();
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const __nv_bfloat162 v0 = __floats2bfloat162_rn(__uint_as_float(r0[2 * q]), __uint_as_float(r0[2 * q + 1]));
          const __nv_bfloat162 v1 = __floats2bfloat162_rn(__uint_as_float(r1[2 * q]), __uint_as_float(r1[2 * q + 1]));
          pk[c * 16 + q] = *reinterpret_cast<const uint32_t*>(&v0);
          pk[c * 16 + 8 + q] = *reinterpret_cast<const uint32_t*>(&v1);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty(ab));  // the MMA warp may refill it meanwhile

#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        if (c < nch) {  // the same for every epilogue thread
          const int b = gc % kNB;
          uint8_t* bp = stg + b * kStgBytes;
          if (res) {
            if (issuer && c + 2 < nch) {
              bulk_wait_read<1>();  // chunk gc - 2, the last user of that buffer, is done reading
              const int b2 = lr % kNB;
              mbar_arrive_expect_tx(rbar(b2), kStgBytes);
              tma_load_2d(stg_s + b2 * kStgBytes, &tm_r, rbar(b2), nt * BM, m0 + 16 * (c + 2), pol_r);
              ++lr;
            }
            // a timeout records the status and the chunk is still written, so that every
            // thread takes the same barriers
            mbar_wait(rbar(b), (uint32_t)(gc / kNB) & 1u, abort_flag, p.status);
          }
          if (silu) {
            // rows [0,64) of the tile are gate rows, [64,128) the matching up rows. Gate row r
            // and up row r finish output column r together: the gate thread takes activation
            // rows 0-7 of the chunk, the up thread rows 8-15, each handing the other the bf16
            // values it lacks (xch row r: gate words of rows 8-15, then up words of rows 0-7)
            const bool gate = er < 64;
            const int r = gate ? er : er - 64;
            uint4* xr = reinterpret_cast<uint4*>(xch + r * kXchStride);
            if (gate)
              xr[0] = make_uint4(pk[8 * c + 4], pk[8 * c + 5], pk[8 * c + 6], pk[8 * c + 7]);
            else
              xr[1] = make_uint4(pk[8 * c], pk[8 * c + 1], pk[8 * c + 2], pk[8 * c + 3]);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const uint4 o4 = gate ? xr[1] : xr[0];
            const uint32_t other[4] = {o4.x, o4.y, o4.z, o4.w};
            const int row0 = gate ? 0 : 8;  // this thread's activation rows of the chunk
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // compile-time indices on both sides keep pk in registers
              const uint32_t own = gate ? pk[8 * c + (j >> 1)] : pk[8 * c + 4 + (j >> 1)];
              const float a = (j & 1) ? hi_f(own) : lo_f(own);
              const float b2 = (j & 1) ? hi_f(other[j >> 1]) : lo_f(other[j >> 1]);
              const float g = gate ? a : b2, u = gate ? b2 : a;
              const float sg = bf16_round(silu_f(g));
              const float act = bf16_round(sg * u);
              check_f16(act, p.status);
              *reinterpret_cast<__half*>(bp + (row0 + j) * 128 + r * 2) = __float2half_rn(act);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float a = (j & 1) ? hi_f(pk[8 * c + (j >> 1)]) : lo_f(pk[8 * c + (j >> 1)]);
              __nv_bfloat16* sp = reinterpret_cast<__nv_bfloat16*>(bp + j * 256 + er * 2);
              *sp = __float2bfloat16_rn(res ? __bfloat162float(*sp) + a : a);
            }
          }
          fence_proxy_async_smem();
          if (issuer) bulk_wait_read<kNB - 2>();  // frees the next chunk's buffer (chunk gc - 3)
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (issuer) {
            tma_store_2d(&tm_y, stg_s + b * kStgBytes, silu ? nt * 64 : nt * BM, m0 + 16 * c);
            bulk_commit();
          }
          if (cp16) {
            // the fp16 copy of the same chunk, converted in place once the bf16 store has read it
            if (issuer) bulk_wait_read<0>();
            asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              uint16_t* sp = reinterpret_cast<uint16_t*>(bp + j * 256 + er * 2);
              const float tv = __uint_as_float((uint32_t)*sp << 16);
              check_f16(tv, p.status);
              const __half h = __float2half_rn(tv);
              *sp = *reinterpret_cast<const uint16_t*>(&h);
            }
            fence_proxy_async_smem();
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (issuer) {
              tma_store_2d(&tm_c, stg_s + b * kStgBytes, nt * BM, m0 + 16 * c);
              bulk_commit();
            }
          }
          ++gc;
        }
      }
    }
    if (issuer) {
      // residual loads issued but not consumed (only after a timeout), then every store
      for (int i = gc; i < lr; ++i) {
        volatile int never = 0;
        mbar_wait(rbar(i % kNB), (uint32_t)(i / kNB) & 1u, &never, p.status);
      }
      bulk_wait_all();
    }
  }

  // a role that ran on one lane (producer, MMA issuer) rejoins its warp before the CTA
  // barrier: the barrier counts whole warps, and TMEM is freed after it
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Tokens per tile. 256 halves the weight conversions and the shared-memory traffic per token,
// 128 doubles the tiles of a short call. Measured on B200 (Qwen3-8B q|k|v, o, gate|up, down,
// us for the four): M 256: 241 at 128 vs 288 at 256; M 512: o and down faster at 128 (64 tiles
// of 256 for 148 SMs), q|k|v and gate|up at 256; M >= 768: 256 for every shape. Hence 128 when
// M <= 256 or when 256-token tiles would number at most 64. g_force_bn (dspark_w8a16_gemm_wide_bn)
// overrides the choice for measurements and tests.
static int g_force_bn = 0;
static int pick_bn(int M, int N) {
  if (g_force_bn) return g_force_bn;
  const long long tiles256 = (long long)(N / BM) * ((M + 255) / 256);
  return (M <= 256 || tiles256 <= 64) ? 128 : 256;
}

template <int BN>
static int launch_wide(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                       const Params& p, cudaStream_t st) {
  using C = Cfg<BN>;
  CUtensorMap tw, tsb, tx;
  int rc;
  if ((rc = make_map_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wq, (uint64_t)p.K, (uint64_t)p.N,
                        (uint64_t)p.K, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B)))
    return rc;
  if ((rc = make_map_2d(&tsb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, wsb, (uint64_t)p.N,
                        (uint64_t)(p.K / 64), (uint64_t)p.N * 4, BM, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if ((rc = make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x, (uint64_t)p.K, (uint64_t)p.M,
                        (uint64_t)ldx * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  // output, residual and fp16-copy maps: rows of 16 activations, 128 (SiLU: 64) columns
  CUtensorMap ty = tx, tr = tx, tc = tx;  // unused ones stay copies of tx
  if (p.epilogue == DSPARK_EPI_SILU_MUL_F16) {
    if ((rc = make_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.y, (uint64_t)(p.N / 2),
                          (uint64_t)p.M, (uint64_t)p.ldy * 2, 64, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
  } else if (p.epilogue != DSPARK_EPI_STORE_F32) {
    if ((rc = make_map_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.y, (uint64_t)p.N,
                          (uint64_t)p.M, (uint64_t)p.ldy * 2, BM, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
      return rc;
  }
  if (p.epilogue == DSPARK_EPI_RESIDUAL_BF16 &&
      (rc = make_map_2d(&tr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.residual, (uint64_t)p.N,
                        (uint64_t)p.M, (uint64_t)p.ldr * 2, BM, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  if (p.copy16 &&
      (rc = make_map_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.copy16, (uint64_t)p.N,
                        (uint64_t)p.M, (uint64_t)p.copy16_ld * 2, BM, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc;
  auto kern = w8a16_wide_kernel<BN>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kTotal) !=
        cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "w8a16_wide: cudaFuncSetAttribute(smem=%u) failed", C::kTotal);
    configured = true;
  }
  const int grid = std::min(p.n_tiles * p.m_tiles, sm_count());
  return launch_pdl("w8a16_wide", kern, dim3(grid), dim3(kThreads), (size_t)C::kTotal, st, tw, tsb,
                    tx, ty, tr, tc, p);
}

}  // namespace w8w
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_w8a16_gemm_wide_bn(int bn) {
  if (bn != 0 && bn != 128 && bn != 256)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide_bn: %d (0, 128 or 256)", bn);
  w8w::g_force_bn = bn;
  return DSPARK_OK;
}

extern "C" int dspark_w8a16_gemm_wide_plan(int M, int N, int K, int* bn, int* grid) {
  if (M < 1 || N <= 0 || K <= 0 || N % w8w::BM || K % w8w::BK || !bn || !grid)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide_plan: M=%d N=%d K=%d", M, N, K);
  const int b = w8w::pick_bn(M, N);
  const long long tiles = (long long)(N / w8w::BM) * ((M + b - 1) / b);
  *bn = b;
  *grid = (int)std::min<long long>(tiles, sm_count());
  return DSPARK_OK;
}

extern "C" int dspark_w8a16_gemm_wide(const void* x, int ldx, const uint8_t* wq,
                                      const uint32_t* wsb, int M, int N, int K, int epilogue,
                                      void* y, int ldy, const void* residual, int ldr,
                                      void* copy_f16, int copy_f16_ld, int* status,
                                      dspark_stream_t stream) {
  if (!x || !wq || !wsb || !y) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide: null pointer");
  if (M < 1 || N <= 0 || K <= 0 || N % w8w::BM || K % w8w::BK)
    return set_error(DSPARK_ERR_INVALID,
                     "w8a16_gemm_wide: M=%d >= 1, N=%d a multiple of 128, K=%d a multiple of 64", M,
                     N, K);
  if (ldx < K || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15))
    return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm_wide: x rows must be 16-byte aligned (ldx=%d)", ldx);
  if (epilogue < 0 || epilogue > 3)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide: epilogue %d", epilogue);
  const int ncols = epilogue == DSPARK_EPI_SILU_MUL_F16 ? N / 2 : N;
  if (ldy < ncols) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide: ldy=%d < %d", ldy, ncols);
  if (epilogue == DSPARK_EPI_RESIDUAL_BF16 && (!residual || ldr < N))
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide: residual epilogue needs residual, ldr >= N");
  if (copy_f16 && (epilogue != DSPARK_EPI_RESIDUAL_BF16 || copy_f16_ld < N))
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_wide: copy_f16 needs RESIDUAL_BF16 and ld >= N");
  w8w::Params p{};
  p.M = M; p.N = N; p.K = K;
  p.kb = K / w8w::BK;
  p.n_tiles = N / w8w::BM;
  p.epilogue = epilogue;
  p.y = y; p.ldy = ldy;
  p.residual = residual; p.ldr = ldr;
  p.copy16 = static_cast<__half*>(copy_f16);
  p.copy16_ld = copy_f16_ld;
  p.status = status;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w8w::pick_bn(M, N) == 256) {
    p.m_tiles = (M + 255) / 256;
    return w8w::launch_wide<256>(x, ldx, wq, wsb, p, st);
  }
  p.m_tiles = (M + 127) / 128;
  return w8w::launch_wide<128>(x, ldx, wq, wsb, p, st);
}
