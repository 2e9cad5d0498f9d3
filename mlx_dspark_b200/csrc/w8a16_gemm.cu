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
#include "rope_kv.cuh"
#include "tensor_map.cuh"

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

// Fused q|k|v epilogue (dspark_w8a16_gemm_qkv_rope): per-head RMSNorm of q and k, RoPE, q to
// q_out and K/V into the paged cache, instead of storing the raw q|k|v row.
struct RopeEpi {
  const __nv_bfloat16* qnw;
  const __nv_bfloat16* knw;
  const float* inv_freq;
  const int32_t* pos0;  // [B] position of each batch row's first token
  __nv_bfloat16* q_out; // [M, Hq*hd]
  dspark_kv_layout kv;
  float eps;
  int T, Hq, Hkv, hd;
};

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
  // > 1: cluster split-K. CTA b works on tile b / csplit, k-slice b % csplit; the csplit CTAs
  // of a tile form one thread-block cluster and sum their partials through distributed shared
  // memory. 0: stream-K over the whole grid.
  int csplit;
  RopeEpi rope;
  // RMSNorm plumbing between GEMMs (dspark_gemm_opts): the STORE_BF16 / RESIDUAL_BF16 epilogues
  // write per-tile sums of squares of their bf16 outputs to ss_out [M][tiles]; a GEMM with norm_w
  // set reads the raw bf16 row as x and normalises each activation tile in shared memory before
  // the MMA, with r[m] = rsqrt(sum_t ss_in[m][t] / K + eps)
  float* ss_out;
  const float* ss_in;
  const __nv_bfloat16* norm_w;
  int ss_tiles;
  int ss_ld;  // row stride of ss_in in floats (>= ss_tiles)
  float norm_eps;
  __half* copy16;  // RESIDUAL_BF16: fp16 copy of the output rows (tap), or null
  int copy16_ld;
  // L2 prefetch of the next kernel's operands: CTA b warms bytes [b*chunk, (b+1)*chunk) of each
  // range after issuing its last load (16-byte aligned, sizes multiples of 16)
  const char* pf_ptr[2];
  unsigned long long pf_bytes[2];
  // PEER_F32 (dspark_w8a16_gemm_peer): every rank's receive buffer and flags, as mapped here
  float* peer_y[8];
  int* peer_f[8];
  int peer_world, peer_rank, peer_mcap, peer_epoch;
};

__device__ __forceinline__ long long range_start(long long b, long long total, long long G) {
  return b * total / G;
}
// the CTA whose range contains flattened k-block g
__device__ __forceinline__ long long range_owner(long long g, long long total, long long G) {
  return ((g + 1) * G + total - 1) / total - 1;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

// PEER: the instance of the tensor-parallel fused all-reduce (dspark_w8a16_gemm_peer); the
// other instances carry no code for it
template <int BN, bool PEER = false>
__device__ __forceinline__ void epilogue_store(const Params& p, int tile, int er, const float* acc,
                                               float* xch,
                                               const __nv_bfloat162* rpre = nullptr) {
  const int n = tile * BM + er;
  switch (p.epilogue) {
    case DSPARK_EPI_STORE_BF16: {
      __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
      const int lane = er & 31, ew = er >> 5;
#pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < p.M) {
          const __nv_bfloat16 o = __float2bfloat16_rn(acc[m]);
          y[(size_t)m * p.ldy + n] = o;
          if (p.ss_out) {
            const float v = __bfloat162float(o);
            const float w = warp_sum(v * v);
            if (lane == 0) xch[ew * BN + m] = w;
          }
        }
      if (p.ss_out) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (er < p.M)
          p.ss_out[(size_t)er * p.tiles + tile] =
              ((xch[er] + xch[BN + er]) + xch[2 * BN + er]) + xch[3 * BN + er];
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      break;
    }
    case DSPARK_EPI_PEER_F32: {
      if constexpr (PEER) {
        // one-shot all-reduce, send half: this rank's fp32 tile into slot (epoch & 1), source row
        // block `rank`, of every rank's receive buffer (plain stores over NVLink), then, once the
        // tile's 128 threads have stored, the tile's epoch flag on every rank
        const int slot = p.peer_epoch & 1;
        const size_t off = ((size_t)(slot * p.peer_world + p.peer_rank) * p.peer_mcap) * p.N + n;
        for (int r = 0; r < p.peer_world; ++r) {
          float* y = p.peer_y[r] + off;
#pragma unroll
          for (int m = 0; m < BN; ++m)
            if (m < p.M) y[(size_t)m * p.N] = acc[m];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (er == 0) {
          __threadfence_system();
          const size_t fo = (size_t)(slot * p.peer_world + p.peer_rank) * p.tiles + tile;
          for (int r = 0; r < p.peer_world; ++r) st_release_sys(p.peer_f[r] + fo, p.peer_epoch);
        }
      }
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
      // y may be the residual itself (in place): read every row first, then store, so the
      // loads are not ordered one by one behind the stores they might alias
      __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
      const __nv_bfloat16* r = static_cast<const __nv_bfloat16*>(p.residual);
      const int lane = er & 31, ew = er >> 5;
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {  // 16 rows at a time bounds the registers held
        __nv_bfloat16 rv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c0 + j;
          if (rpre)  // read by the caller before it waited on the other contributors
            rv[j] = (m & 1) ? rpre[m >> 1].y : rpre[m >> 1].x;
          else
            rv[j] = m < p.M ? r[(size_t)m * p.ldr + n] : __float2bfloat16_rn(0.0f);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < p.M) {
            const __nv_bfloat16 o = __float2bfloat16_rn(__bfloat162float(rv[j]) + bf16_round(acc[c0 + j]));
            y[(size_t)(c0 + j) * p.ldy + n] = o;
            if (p.copy16) p.copy16[(size_t)(c0 + j) * p.copy16_ld + n] = __float2half_rn(__bfloat162float(o));
            if (p.ss_out) {
              // this row's share of the next RMSNorm: warp sum, then the 4 warps in order
              const float v = __bfloat162float(o);
              const float w = warp_sum(v * v);
              if (lane == 0) xch[ew * BN + c0 + j] = w;
            }
          }
      }
      if (p.ss_out) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (er < p.M)
          p.ss_out[(size_t)er * p.tiles + tile] =
              ((xch[er] + xch[BN + er]) + xch[2 * BN + er]) + xch[3 * BN + er];
        asm volatile("bar.sync 1, 128;" ::: "memory");  // xch is reused by the next tile
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
        for (int c0 = 0; c0 < BN; c0 += 16) {
          // the exchanged values first (xch is a generic pointer the stores may alias)
          float up[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) up[j] = xch[er * BN + c0 + j];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < p.M) {
              const float g = bf16_round(acc[c0 + j]);
              const float u = bf16_round(up[j]);
              const float s = bf16_round(silu_f(g));
              y[(size_t)(c0 + j) * p.ldy + col] = __float2half_rn(bf16_round(s * u));
            }
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      break;
    }
    default:
      break;
  }
}

// One output of the tile from its accumulated value v (and, for SILU_MUL, the matching up-row
// value vu): the same arithmetic as epilogue_store, element by element. `row` is the tile row
// (for SILU_MUL a gate row < 64), m the activation row.
__device__ __forceinline__ void epilogue_one(const Params& p, int tile, int row, int m, float v,
                                             float vu) {
  switch (p.epilogue) {
    case DSPARK_EPI_STORE_BF16:
      static_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + tile * BM + row] = __float2bfloat16_rn(v);
      break;
    case DSPARK_EPI_STORE_F32:
      static_cast<float*>(p.y)[(size_t)m * p.ldy + tile * BM + row] = v;
      break;
    case DSPARK_EPI_RESIDUAL_BF16: {
      const size_t n = (size_t)tile * BM + row;
      const float rv = __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[(size_t)m * p.ldr + n]);
      static_cast<__nv_bfloat16*>(p.y)[(size_t)m * p.ldy + n] = __float2bfloat16_rn(rv + bf16_round(v));
      break;
    }
    case DSPARK_EPI_SILU_MUL_F16: {
      const float g = bf16_round(v);
      const float u = bf16_round(vu);
      const float sg = bf16_round(silu_f(g));
      static_cast<__half*>(p.y)[(size_t)m * p.ldy + tile * 64 + row] = __float2half_rn(bf16_round(sg * u));
      break;
    }
    default:
      break;
  }
}

// The fused q|k|v epilogue of a finished tile: stage the tile's bf16 outputs (the values the
// separate q|k|v GEMM would store) in shared memory as [m][128], then one warp per (token, head
// in the tile) runs the same norm + RoPE + KV write as the standalone kernel. The staging fits
// the exchange buffer: BN x 128 bf16 = 64 x BN fp32.
template <int BN>
__device__ __forceinline__ void rope_epilogue(const Params& p, int tile, int er, const float* acc,
                                              float* xch) {
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xch);
#pragma unroll
  for (int m = 0; m < BN; ++m)
    if (m < p.M) xs[m * BM + er] = __float2bfloat16_rn(acc[m]);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const RopeEpi& r = p.rope;
  const int warp = er >> 5, lane = er & 31;
  const int hpt = BM / r.hd;  // heads per tile
  for (int it = warp; it < p.M * hpt; it += kEpiWarps) {
    const int m = it / hpt, j = it - m * hpt;
    const int h = tile * hpt + j;
    const int b = m / r.T;
    const int pos = r.pos0[b] + (m - b * r.T);
    const __nv_bfloat16* head = xs + m * BM + j * r.hd;
    __nv_bfloat16* q_row = r.q_out + (size_t)m * r.Hq * r.hd;
    if (r.hd == 128)
      rope_kv_head<4>(head, r.Hq, r.Hkv, h, r.qnw, r.knw, r.eps, r.inv_freq, b, pos, q_row, r.kv, lane);
    else
      rope_kv_head<2>(head, r.Hq, r.Hkv, h, r.qnw, r.knw, r.eps, r.inv_freq, b, pos, q_row, r.kv, lane);
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");  // xch is reused by this CTA's next tile
}

template <int BN, int STAGES>
struct Smem {
  static constexpr uint32_t kXBytes = 2u * BN * 128u;
  static constexpr uint32_t kStageBytes = kWBytes + kXBytes + kSBBytes;
  static constexpr uint32_t kXchBytes = 64u * BN * 4u;
  static constexpr uint32_t kBarBytes = 512;
  static constexpr uint32_t kTotal = 1024 + STAGES * kStageBytes + kXchBytes + kBarBytes;
};

template <int BN, int STAGES, bool CS, bool ROPE, bool PEER = false>
__global__ void __launch_bounds__(kThreads, (BN <= 32 && !CS ? 2 : 1))
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_sb,
                    const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Smem<BN, STAGES>;
  // TMEM: [0, AB*64) the converted-weight ring (64 columns = 128 fp16 per lane each), then two
  // fp32 accumulators of ACCS columns. Two CTAs per SM share the 512 columns; one CTA per SM
  // takes all of them for a deeper ring (the ring depth bounds how far conversion runs ahead
  // of MMA completion).
  constexpr bool kTwoPerSm = BN <= 32 && !CS;
  constexpr int AB = kTwoPerSm ? 3 : 6;
  constexpr uint32_t ACCS = BN <= 32 ? 32u : 64u;
  constexpr uint32_t ACC0 = (uint32_t)AB * 64u;
  constexpr uint32_t TC = kTwoPerSm ? 256u : 512u;
  static_assert(ACC0 + 2 * ACCS <= TC, "TMEM layout");
  static_assert(3 * STAGES + 2 * AB + 8 <= (int)(L::kBarBytes / 8), "barrier region");
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
  auto aempty = [&](int a) { return smem_u32(bars + 3 * STAGES + AB + a); };
  auto accfull = [&](int b) { return smem_u32(bars + 3 * STAGES + 2 * AB + b); };
  auto accempty = [&](int b) { return smem_u32(bars + 3 * STAGES + 2 * AB + 2 + b); };
  const uint32_t done_bar = smem_u32(bars + 3 * STAGES + 2 * AB + 4);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 2 * AB + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_holder + 2);
  const uint32_t fix_bar = smem_u32(bars + 3 * STAGES + 2 * AB + 7);  // stream-K fixup copies

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(xfull(s), 1);
      mbar_init(empty(s), kConvWarps + 1);
    }
    for (int a = 0; a < AB; ++a) {
      mbar_init(afull(a), kConvWarps);
      mbar_init(aempty(a), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accfull(b), 1);
      mbar_init(accempty(b), kEpiWarps);
    }
    mbar_init(done_bar, 1);
    mbar_init(fix_bar, 1);
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
    tmem_alloc(smem_u32(tmem_holder), TC);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_launch_dependents();

  const long long G = gridDim.x;
  const long long total = p.total;
  const int KB = p.kb;
  long long start, end;
  if constexpr (CS) {
    const int tile = (int)(blockIdx.x / p.csplit), r = (int)(blockIdx.x % p.csplit);
    start = (long long)tile * KB + (long long)r * KB / p.csplit;
    end = (long long)tile * KB + (long long)(r + 1) * KB / p.csplit;
  } else {
    start = range_start(blockIdx.x, total, G);
    end = range_start(blockIdx.x + 1, total, G);
  }
  const int n_iter = (int)(end - start);

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
      // this CTA's loads are all issued: while they land and the tail runs, warm L2 with its
      // slice of the next GEMM's weights so HBM does not idle through the tail and the small
      // kernels in between
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const unsigned long long nb = p.pf_bytes[r];
        if (nb == 0) continue;
        const unsigned long long chunk = ((nb + (unsigned long long)G - 1) / (unsigned long long)G + 15ull) & ~15ull;
        unsigned long long off = (unsigned long long)blockIdx.x * chunk;
        const unsigned long long stop = off + chunk < nb ? off + chunk : nb;
        for (; off < stop; off += 65536ull) {
          const unsigned long long left = stop - off;
          prefetch_l2_bulk(p.pf_ptr[r] + off, (uint32_t)(left < 65536ull ? left : 65536ull));
        }
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
        const int a = i % AB;
        const uint32_t aph = (uint32_t)(i / AB) & 1u;
        const int ab = seg & 1;
        const uint32_t abph = (uint32_t)(seg >> 1) & 1u;
        if (seg_first && !mbar_wait(accempty(ab), abph ^ 1u, abort_flag, p.status)) break;
        if (!mbar_wait(afull(a), aph, abort_flag, p.status)) break;
        if (!mbar_wait(xfull(s), ph, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ACC0 + (uint32_t)ab * ACCS;
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
    // fused input RMSNorm: thread r normalises 16-byte chunk (r & 7) of activation rows
    // (r >> 3) + 16k of both 64-wide boxes of every stage; rn[k] is that row's 1/rms
    float rn[BN / 16];
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) rn[kk] = 0.0f;
    for (int i = 0; i < n_iter; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
      const int a = i % AB;
      const uint32_t aph = (uint32_t)(i / AB) & 1u;
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
      if (p.norm_w) {
        if (i == 0) {
          pdl_wait();  // the row sums of squares come from the previous kernel
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const int m = (r >> 3) + 16 * kk;
            float sum = 0.0f;
            if (m < p.M) {
              // the row's per-tile sums, contiguous: 16-byte loads, added in tile order
              const float* row = p.ss_in + (size_t)m * p.ss_ld;
              int t = 0;
              if ((p.ss_ld & 3) == 0)
                for (; t + 4 <= p.ss_tiles; t += 4) {
                  const float4 q4 = *reinterpret_cast<const float4*>(row + t);
                  sum = (((sum + q4.x) + q4.y) + q4.z) + q4.w;
                }
              for (; t < p.ss_tiles; ++t) sum += row[t];
            }
            rn[kk] = rsqrtf(sum / (float)p.K + p.norm_eps);
          }
        }
        if (!mbar_wait(xfull(s), ph, abort_flag, p.status)) {
          tc_wait_st();  // no TMEM store of this thread may be in flight at teardown
          break;
        }
        const int kb = (int)((start + i) % KB);
        const int c = r & 7;
#pragma unroll
        for (int bx = 0; bx < 2; ++bx) {
          // the RMSNorm weights of these 8 columns (dspark_rmsnorm: bf16(x * r * w))
          const uint4 wq8 = *reinterpret_cast<const uint4*>(p.norm_w + kb * BK + bx * 64 + c * 8);
          const __nv_bfloat162* wv = reinterpret_cast<const __nv_bfloat162*>(&wq8);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const int m = (r >> 3) + 16 * kk;
            if (m >= p.M) continue;
            const uint32_t addr = x_s + s * L::kXBytes + bx * BN * 128 + m * 128 + ((c ^ (m & 7)) << 4);
            uint32_t v[4];
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                         : "r"(addr));
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 hv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v[q]));
              const float2 wf = __bfloat1622float2(wv[q]);
              const __nv_bfloat162 xn = __floats2bfloat162_rn(hv.x * rn[kk] * wf.x, hv.y * rn[kk] * wf.y);
              const float2 xf = __bfloat1622float2(xn);
              const __half2 x16 = __floats2half2_rn(xf.x, xf.y);
              v[q] = *reinterpret_cast<const uint32_t*>(&x16);
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]),
                         "r"(v[2]), "r"(v[3])
                         : "memory");
          }
        }
        // the MMA reads the tile through the async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
    uint32_t fix_phase = 0;
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
        tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + ACC0 + (uint32_t)ab * ACCS +
                      (uint32_t)c * 16u,
                  rr);
        tc_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[c * 16 + t] = __uint_as_float(rr[t]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty(ab));

      if constexpr (CS) {
        // cluster split-K: this CTA's only segment. Every MMA of the CTA has completed, so no
        // copy or MMA touches the stage ring any more: the partial goes to its start, row er's
        // BN values contiguous, and the cluster sums them after the role loops.
        float4* part = reinterpret_cast<float4*>(reinterpret_cast<float*>(sbase) + er * BN);
#pragma unroll
        for (int j = 0; j < BN / 4; ++j)
          part[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        (void)whole;
      } else if (whole) {
        if constexpr (ROPE)
          rope_epilogue<BN>(p, tile, er, acc, xch);
        else
          epilogue_store<BN, PEER>(p, tile, er, acc, xch);
      } else {
        // partial of this CTA, row-major [128][MP] with MP = M rounded up to 4: thread er's
        // values are 16-byte vectors, and each contributor's partial is one contiguous
        // 128*MP*4-byte block
        const int slot = (int)blockIdx.x * 2 + (seg == 0 ? 0 : 1);
        const int MP = (p.M + 3) & ~3;
        {
          float4* part = reinterpret_cast<float4*>(p.partials + (size_t)slot * BN * BM + er * MP);
#pragma unroll
          for (int j = 0; j < BN / 4; ++j)
            if (4 * j < MP) part[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
        }
        // the residual rows of this tile, read now so that the read overlaps the arrival round
        // trip (only the CTA that finishes the tile writes them): into registers at BN 16, into
        // L1 at the wider shapes, whose registers are taken
        constexpr bool kPre = BN <= 16;
        __nv_bfloat162 rpre[kPre ? BN / 2 : 1];
        const bool res = !ROPE && p.epilogue == DSPARK_EPI_RESIDUAL_BF16;
        if (res) {
          const __nv_bfloat16* rp = static_cast<const __nv_bfloat16*>(p.residual) + tile * BM + er;
          if constexpr (kPre) {
#pragma unroll
            for (int j = 0; j < BN / 2; ++j) {
              const int m = 2 * j;
              rpre[j].x = m < p.M ? rp[(size_t)m * p.ldr] : __float2bfloat16_rn(0.0f);
              rpre[j].y = m + 1 < p.M ? rp[(size_t)(m + 1) * p.ldr] : __float2bfloat16_rn(0.0f);
            }
          } else {
#pragma unroll
            for (int m = 0; m < BN; ++m)
              if (m < p.M) asm volatile("prefetch.global.L1 [%0];" ::"l"(rp + (size_t)m * p.ldr));
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const long long c_lo = range_owner(tile_lo, total, G);
        const long long c_hi = range_owner(tile_lo + KB - 1, total, G);
        const int nctr = (int)(c_hi - c_lo + 1);
        // contributor c keeps this tile in its partial slot 2c + 1 only if the tile is its second
        // segment, which only the first contributor's range can make it (ranges are contiguous)
        const int cj_lo = range_start(c_lo, total, G) >= tile_lo ? 0 : 1;
        const uint32_t blk = (uint32_t)MP * BM * 4u;
        // the stage ring is idle once this CTA's last segment is accumulated (every copy into
        // it has landed and been consumed), so the finishing CTA can stage the partials there
        const bool ring_free = seg_end == end && (uint32_t)nctr * blk <= (uint32_t)STAGES * L::kStageBytes;
        if (er == 0) {
          // One acq_rel gpu-scope atomic per CTA. Release: the partials of all 128 threads
          // (ordered before it by the barrier; release is cumulative) are visible to whoever
          // reads the final count. Acquire: the last arriver sees every partial.
          int old;
          asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                       : "=r"(old)
                       : "l"(p.counters + tile)
                       : "memory");
          const bool last = old == nctr - 1;
          *last_flag = last ? 1 : 0;
          if (last && ring_free) {
            // every contributor's block in flight at once: one bulk copy each into the ring
            fence_proxy_async_global();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(fix_bar, (uint32_t)nctr * blk);
            for (int ci = 0; ci < nctr; ++ci) {
              const long long c = c_lo + ci;
              const int cj = ci == 0 ? cj_lo : 0;
              bulk_load_g2s(base + (uint32_t)ci * blk, p.partials + ((size_t)c * 2 + cj) * BN * BM,
                            blk, fix_bar);
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int is_last = *last_flag;
        if (is_last) {
          float sum[BN];
#pragma unroll
          for (int m = 0; m < BN; ++m) sum[m] = 0.0f;
          if (ring_free) {
            if (!mbar_wait(fix_bar, fix_phase, abort_flag, p.status)) {
              // no copy may still be writing into shared memory when the CTA leaves
              volatile int never = 0;
              mbar_wait(fix_bar, fix_phase, &never, p.status);
            }
            fix_phase ^= 1u;
            // contributor order, as in the register path below; two contributors' vectors are
            // loaded before they are added so the shared-memory loads overlap
            const float4* st = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(sbase) + er * MP);
            const int stride = (int)(blk / 16);  // float4s per contributor block
            int ci = 0;
            for (; ci + 2 <= nctr; ci += 2) {
#pragma unroll
              for (int j = 0; j < BN / 4; ++j)
                if (4 * j < MP) {
                  const float4 v0 = st[ci * stride + j], v1 = st[(ci + 1) * stride + j];
                  sum[4 * j] = (sum[4 * j] + v0.x) + v1.x;
                  sum[4 * j + 1] = (sum[4 * j + 1] + v0.y) + v1.y;
                  sum[4 * j + 2] = (sum[4 * j + 2] + v0.z) + v1.z;
                  sum[4 * j + 3] = (sum[4 * j + 3] + v0.w) + v1.w;
                }
            }
            for (; ci < nctr; ++ci) {
#pragma unroll
              for (int j = 0; j < BN / 4; ++j)
                if (4 * j < MP) {
                  const float4 v0 = st[ci * stride + j];
                  sum[4 * j] += v0.x;
                  sum[4 * j + 1] += v0.y;
                  sum[4 * j + 2] += v0.z;
                  sum[4 * j + 3] += v0.w;
                }
            }
          } else {
            for (long long c = c_lo; c <= c_hi; ++c) {
              const int cj = c == c_lo ? cj_lo : 0;
              const float4* cp = reinterpret_cast<const float4*>(p.partials + ((size_t)c * 2 + cj) * BN * BM + er * MP);
#pragma unroll
              for (int j = 0; j < BN / 4; ++j)
                if (4 * j < MP) {
                  const float4 v0 = __ldcg(cp + j);
                  sum[4 * j] += v0.x;
                  sum[4 * j + 1] += v0.y;
                  sum[4 * j + 2] += v0.z;
                  sum[4 * j + 3] += v0.w;
                }
            }
          }
          if (er == 0) p.counters[tile] = 0;
          if constexpr (ROPE)
            rope_epilogue<BN>(p, tile, er, sum, xch);
          else
            epilogue_store<BN, PEER>(p, tile, er, sum, xch, (kPre && res) ? rpre : nullptr);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      ++seg;
      g = seg_end;
    }
  }

  if constexpr (CS) {
    // Every thread of every CTA of the cluster takes both cluster barriers (no early exits
    // above, and each role loop ends after its bounded waits), so both barriers complete.
    cluster_sync_all();  // release/acquire: every CTA's partial is visible cluster-wide
    if (warp >= kConvWarps && warp < kConvWarps + kEpiWarps && !*abort_flag) {
      // CTA rank r finishes tile rows [r0, r1) for every activation row, summing the csplit
      // partials in rank order (the same order whichever CTA finishes first)
      const int t = threadIdx.x - kConvWarps * 32;
      const int c = p.csplit;
      const int rank = (int)(blockIdx.x % c);  // == %cluster_ctarank: clusters are (c, 1, 1)
      const int tile = (int)(blockIdx.x / c);
      const bool silu = p.epilogue == DSPARK_EPI_SILU_MUL_F16;
      const int rows = silu ? BM / 2 : BM;
      const int r0 = rank * rows / c, r1 = (rank + 1) * rows / c;
      const int nr = r1 - r0;
      uint32_t peer[8];  // shared::cluster address of each slice's partial
#pragma unroll
      for (int q = 0; q < 8; ++q) peer[q] = q < c ? mapa_shared(base, (uint32_t)q) : 0u;
      auto slice_sum = [&](uint32_t off) {
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < c) v[q] = ld_shared_cluster_f32(peer[q] + off);
        float sum = 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < c) sum += v[q];
        return sum;
      };
      for (int o = t; o < nr * p.M; o += kEpiWarps * 32) {
        const int m = o / nr, row = r0 + (o - m * nr);
        const float sv = slice_sum((uint32_t)(row * BN + m) * 4u);
        const float su = silu ? slice_sum((uint32_t)((row + BM / 2) * BN + m) * 4u) : 0.0f;
        epilogue_one(p, tile, row, m, sv, su);
      }
    }
    cluster_sync_all();  // no CTA leaves while a peer still reads its shared memory
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC);
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
// Layer chain: the GEMMs and small ops between two attention kernels as phases of ONE
// persistent launch (cooperative: every CTA resident, so grid-wide waits are safe):
//   o_proj (+residual) -> RMSNorm -> gate|up (SiLU*up) -> down (+residual) [-> tap copy]
//   -> next layer's RMSNorm -> next q|k|v -> q/k norm + RoPE + paged KV write
// The per-launch ramp and tail (~6-9 us a GEMM) are paid once per layer. Warp roles are the
// GEMM's; the producer warp splits in two lanes: lane 0 streams every phase's weight tiles
// without waiting for anything but free ring slots (so the next projection's weights are in
// flight while the previous phase finishes), lane 1 issues a GEMM phase's activation loads
// only once the grid-wide counter of the phase before it is full. The epilogue warps finish
// the GEMM tiles, run the elementwise phases, and arrive on each phase's counter.
constexpr int kChainMaxPhases = 10;
constexpr int kChainMaxGemm = 4;
enum { kPhGemm = 0, kPhNorm = 1, kPhRope = 2, kPhCopy = 3 };
// Grid barriers follow GEMM and NORM phases. A barrier may spread its arrivals over kBarSlots
// counters on separate 128-byte lines (CTA c adds to slot c % kBarSlots; a waiter sums them);
// one slot measured fastest on B200 (16 slots: polling 16 lines costs more than the contention
// it removes).
constexpr int kBarSlots = 1;
constexpr int kBarStride = 32;  // ints between slots (128 bytes)
constexpr int kChainMaxBars = kChainMaxPhases;
constexpr size_t kBarRegion = (((size_t)(kChainMaxBars * kBarSlots + 1) * kBarStride * 4) + 255) & ~(size_t)255;

struct ChainGemm {
  int N, K, tiles, kb;
  long long total;
  int epilogue;
  void* y;
  int ldy;
  const void* residual;
  int ldr;
  int* counters;
  float* partials;
};
struct ChainPhase {
  int kind;
  int gemm;        // GEMM phases: index into ChainParams::g and ChainMaps
  int wait_bar;    // grid barrier to acquire before reading inputs (-1: the previous kernel)
  int arrive_bar;  // grid barrier to arrive on afterwards (-1: none)
  int local_norm;  // GEMM: NORM phase (run by this CTA) whose output is X (-1: none)
  // NORM: x (bf16) -> y16 (fp16) ; COPY: x (bf16) -> y16 (fp16), cols = H
  const __nv_bfloat16* x;
  int ldx;
  const __nv_bfloat16* w;
  int H;
  float eps;
  __half* y16;
  int ldy16;
  // ROPE
  const __nv_bfloat16* qkv;
  int ldqkv, T, Hq, Hkv, hd;
  const __nv_bfloat16* qnw;
  const __nv_bfloat16* knw;
  const float* inv_freq;
  const int32_t* pos0;
  __nv_bfloat16* q_out;
  dspark_kv_layout kv;
};
struct ChainParams {
  int M, nphases, ngemm;
  ChainPhase ph[kChainMaxPhases];
  ChainGemm g[kChainMaxGemm];
  int* bars;  // one arrival counter per phase, then a done counter
  int* status;
};
struct ChainMaps {
  CUtensorMap w[kChainMaxGemm], sb[kChainMaxGemm], x[kChainMaxGemm];
};

__device__ __forceinline__ int bar_count(const int* bar) {
  int sum = 0;
#pragma unroll
  for (int k = 0; k < kBarSlots; ++k) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(bar + k * kBarStride) : "memory");
    sum += v;
  }
  return sum;
}
__device__ __forceinline__ bool grid_wait(const int* bar, int target, volatile int* abort_flag,
                                          int* status) {
  if (bar_count(bar) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    __nanosleep(32);
    if (bar_count(bar) >= target) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kSpinLimitNs) {
      *abort_flag = 1;
      report_error(status, DSPARK_ERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ void grid_arrive(int* bar) {
  int* slot = bar + (int)(blockIdx.x % kBarSlots) * kBarStride;
  asm volatile("fence.acq_rel.gpu;\n\tred.release.gpu.global.add.s32 [%0], 1;" ::"l"(slot) : "memory");
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, (BN <= 32 ? 2 : 1))
    chain_kernel(const __grid_constant__ ChainMaps maps, const __grid_constant__ ChainParams p) {
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
  const long long G = gridDim.x;
  const int Gi = (int)gridDim.x;
  // NORM phases run redundantly in every CTA; this CTA's activation producer waits for its
  // own epilogue warps to finish the rows (one use per launch: parity 0)
  __shared__ uint64_t local_done[kChainMaxPhases];
  auto bar_at = [&](int b) { return p.bars + b * kBarSlots * kBarStride; };

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
    for (int q = 0; q < kChainMaxPhases; ++q) mbar_init(smem_u32(&local_done[q]), 1);
    *abort_flag = 0;
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int j = 0; j < p.ngemm; ++j) {
        tma_prefetch_desc(&maps.w[j]);
        tma_prefetch_desc(&maps.sb[j]);
        tma_prefetch_desc(&maps.x[j]);
      }
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

  // A GEMM phase spreads over Gj = min(G, units) CTAs, so every CTA that owns a range owns at
  // least one unit (the stream-K fixup counts contributors by range); the rest sit it out.
  auto phase_range = [&](const ChainGemm& gj, long long& st, long long& en) {
    const long long Gj = gj.total < G ? gj.total : G;
    if ((long long)blockIdx.x < Gj) {
      st = range_start(blockIdx.x, gj.total, Gj);
      en = range_start(blockIdx.x + 1, gj.total, Gj);
    } else {
      st = en = 0;
    }
  };
  // total units of this CTA over all GEMM phases (phase order)
  int n_units = 0;
  for (int j = 0; j < p.ngemm; ++j) {
    long long st, en;
    phase_range(p.g[j], st, en);
    n_units += (int)(en - st);
  }

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // weights and (scale, bias): depend on nothing, streamed through every phase
      const uint64_t pol_w = policy_evict_first();
      int u = 0;
      bool ok = true;
      for (int j = 0; j < p.ngemm && ok; ++j) {
        const ChainGemm& gj = p.g[j];
        long long st, en;
        phase_range(gj, st, en);
        for (long long g = st; g < en; ++g, ++u) {
          const int s = u % STAGES;
          const uint32_t ph = (uint32_t)(u / STAGES) & 1u;
          if (u >= STAGES && !mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status)) { ok = false; break; }
          const int tile = (int)(g / gj.kb), kb = (int)(g % gj.kb);
          mbar_arrive_expect_tx(full(s), kWBytes + kSBBytes);
          tma_load_2d(w_s + s * kWBytes, &maps.w[j], full(s), kb * BK, tile * BM, pol_w);
          tma_load_2d(sb_s + s * kSBBytes, &maps.sb[j], full(s), tile * BM, kb * 2, pol_w);
        }
      }
      const int issued = u;
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int i = first; i < issued; ++i) {
        volatile int never = 0;
        mbar_wait(full(i % STAGES), (uint32_t)(i / STAGES) & 1u, &never, p.status);
      }
    } else if (lane == 1) {
      // activations: a GEMM phase's X is complete once the counter of the phase before it is
      // full (the first phase's X comes from the previous kernel)
      const uint64_t pol_x = policy_evict_last();
      int u = 0;
      bool ok = true;
      for (int q = 0; q < p.nphases && ok; ++q) {
        if (p.ph[q].kind != kPhGemm) continue;
        const int j = p.ph[q].gemm;
        const ChainGemm& gj = p.g[j];
        long long st, en;
        phase_range(gj, st, en);
        if (st == en) continue;
        if (p.ph[q].wait_bar < 0) pdl_wait();
        else if (!grid_wait(bar_at(p.ph[q].wait_bar), Gi, abort_flag, p.status)) { ok = false; break; }
        if (p.ph[q].local_norm >= 0 &&
            !mbar_wait(smem_u32(&local_done[p.ph[q].local_norm]), 0, abort_flag, p.status)) { ok = false; break; }
        // the phase before wrote X with generic stores; these loads go through the async proxy
        asm volatile("fence.proxy.async.global;" ::: "memory");
        for (long long g = st; g < en; ++g, ++u) {
          const int s = u % STAGES;
          const uint32_t ph = (uint32_t)(u / STAGES) & 1u;
          if (u >= STAGES && !mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status)) { ok = false; break; }
          const int kb = (int)(g % gj.kb);
          mbar_arrive_expect_tx(xfull(s), L::kXBytes);
          tma_load_2d(x_s + s * L::kXBytes, &maps.x[j], xfull(s), kb * BK, 0, pol_x);
          tma_load_2d(x_s + s * L::kXBytes + BN * 128, &maps.x[j], xfull(s), kb * BK + 64, 0, pol_x);
        }
      }
      const int issued = u;
      const int first = issued > STAGES ? issued - STAGES : 0;
      for (int i = first; i < issued; ++i) {
        volatile int never = 0;
        mbar_wait(xfull(i % STAGES), (uint32_t)(i / STAGES) & 1u, &never, p.status);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BM, BN);
      int seg = 0, u = 0;
      bool ok = true;
      for (int j = 0; j < p.ngemm && ok; ++j) {
        const ChainGemm& gj = p.g[j];
        long long st, en;
        phase_range(gj, st, en);
        for (long long g = st; g < en; ++g, ++u) {
          const int kb = (int)(g % gj.kb);
          const bool seg_first = (g == st) || (kb == 0);
          const bool seg_last = (g == en - 1) || (kb == gj.kb - 1);
          const int s = u % STAGES;
          const uint32_t ph = (uint32_t)(u / STAGES) & 1u;
          const int a = u % kABufs;
          const uint32_t aph = (uint32_t)(u / kABufs) & 1u;
          const int ab = seg & 1;
          const uint32_t abph = (uint32_t)(seg >> 1) & 1u;
          if (seg_first && !mbar_wait(accempty(ab), abph ^ 1u, abort_flag, p.status)) { ok = false; break; }
          if (!mbar_wait(afull(a), aph, abort_flag, p.status)) { ok = false; break; }
          if (!mbar_wait(xfull(s), ph, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + 128u + (uint32_t)ab * 64u;
#pragma unroll
          for (int jj = 0; jj < BK / 16; ++jj) {
            const uint32_t a_tmem = tmem_base + (uint32_t)a * 64u + (uint32_t)jj * 8u;
            const uint32_t b_addr = x_s + s * L::kXBytes + (jj >> 2) * (BN * 128) + (jj & 3) * 32;
            tc_mma_ts(d_tmem, a_tmem, umma_desc_sw128_kmajor(b_addr), idesc,
                      (seg_first && jj == 0) ? 0u : 1u);
          }
          tc_commit(empty(s));
          tc_commit(aempty(a));
          if (seg_last) {
            tc_commit(accfull(ab));
            ++seg;
          }
        }
      }
      tc_commit(done_bar);
      volatile int never = 0;
      mbar_wait(done_bar, 0, &never, p.status);
    }
  } else if (warp < kConvWarps) {
    const int r = threadIdx.x;
    const uint32_t lane_base = tmem_base + ((uint32_t)(warp * 32) << 16);
    const uint32_t k1024 = 0x64006400u;
    for (int i = 0; i < n_units; ++i) {
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
        const uint32_t sc2 = __byte_perm(sbv, 0, 0x1010);
        const uint32_t bi2 = __byte_perm(sbv, 0, 0x3232);
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
    const int er = threadIdx.x - kConvWarps * 32;
    const int quad = warp & 3;
    const int ew = warp - kConvWarps;  // 0..3
    pdl_wait();
    int seg = 0;
    bool ok = true;
    for (int q = 0; q < p.nphases && ok; ++q) {
      const ChainPhase& P = p.ph[q];
      if (P.kind == kPhGemm) {
        if (P.wait_bar >= 0) {
          // acquire what earlier phases wrote (the residual of down is written by o's epilogue)
          if (er == 0) *last_flag = grid_wait(bar_at(P.wait_bar), Gi, abort_flag, p.status) ? 1 : 0;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (!*last_flag) { ok = false; break; }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
        const int j = P.gemm;
        const ChainGemm& gj = p.g[j];
        Params pp{};
        pp.M = p.M;
        pp.epilogue = gj.epilogue;
        pp.y = gj.y;
        pp.ldy = gj.ldy;
        pp.residual = gj.residual;
        pp.ldr = gj.ldr;
        const int KB = gj.kb;
        const long long total = gj.total;
        const long long Gj = total < G ? total : G;
        long long start, end;
        phase_range(gj, start, end);
        int lseg = 0;
        long long g = start;
        while (g < end) {
          const int tile = (int)(g / KB);
          const long long tile_lo = (long long)tile * KB;
          const long long seg_end = (end < tile_lo + KB) ? end : tile_lo + KB;
          const bool whole = (g == tile_lo) && (seg_end == tile_lo + KB);
          const int ab = seg & 1;
          const uint32_t abph = (uint32_t)(seg >> 1) & 1u;
          if (!mbar_wait(accfull(ab), abph, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          float acc[BN];
#pragma unroll
          for (int c = 0; c < BN / 16; ++c) {
            uint32_t rr[16];
            tmem_ld16(tmem_base + ((uint32_t)(quad * 32) << 16) + 128u + (uint32_t)ab * 64u + (uint32_t)c * 16u, rr);
            tc_wait_ld();
#pragma unroll
            for (int t = 0; t < 16; ++t) acc[c * 16 + t] = __uint_as_float(rr[t]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(accempty(ab));
          if (whole) {
            epilogue_store<BN>(pp, tile, er, acc, xch);
          } else {
            const int slot = (int)blockIdx.x * 2 + (lseg == 0 ? 0 : 1);
            float4* part = reinterpret_cast<float4*>(gj.partials + (size_t)slot * BN * BM + er * BN);
#pragma unroll
            for (int jj = 0; jj < BN / 4; ++jj)
              part[jj] = make_float4(acc[4 * jj], acc[4 * jj + 1], acc[4 * jj + 2], acc[4 * jj + 3]);
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const long long c_lo = range_owner(tile_lo, total, Gj);
            const long long c_hi = range_owner(tile_lo + KB - 1, total, Gj);
            if (er == 0) {
              const int contributors = (int)(c_hi - c_lo + 1);
              int old;
              asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                           : "=r"(old)
                           : "l"(gj.counters + tile)
                           : "memory");
              *last_flag = (old == contributors - 1) ? 1 : 0;
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (*last_flag) {
              float sum[BN];
#pragma unroll
              for (int m = 0; m < BN; ++m) sum[m] = 0.0f;
              for (long long c = c_lo; c <= c_hi; ++c) {
                const int cj = (range_start(c, total, Gj) >= tile_lo) ? 0 : 1;
                const float4* cp = reinterpret_cast<const float4*>(
                    gj.partials + ((size_t)c * 2 + cj) * BN * BM + er * BN);
#pragma unroll
                for (int jj = 0; jj < BN / 4; ++jj) {
                  const float4 t = __ldcg(cp + jj);
                  sum[4 * jj] += t.x;
                  sum[4 * jj + 1] += t.y;
                  sum[4 * jj + 2] += t.z;
                  sum[4 * jj + 3] += t.w;
                }
              }
              if (er == 0) gj.counters[tile] = 0;
              epilogue_store<BN>(pp, tile, er, sum, xch);
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
          ++seg;
          ++lseg;
          g = seg_end;
        }
      } else {
        if (P.wait_bar >= 0) {
          if (er == 0) *last_flag = grid_wait(bar_at(P.wait_bar), Gi, abort_flag, p.status) ? 1 : 0;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (!*last_flag) { ok = false; break; }
        }
        if (P.kind == kPhNorm) {
          // rows m = blockIdx.x, blockIdx.x + G, ...: y16 = fp16(bf16(x * rsqrt(mean x^2 + eps) * w))
          for (int m = blockIdx.x; m < p.M; m += Gi) {
            const __nv_bfloat16* xr = P.x + (size_t)m * P.ldx;
            float ss = 0.0f;
            for (int k = er * 2; k < P.H; k += 256) {
              const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + k));
              ss += v.x * v.x + v.y * v.y;
            }
            ss = warp_sum(ss);
            if (lane == 0) xch[ew] = ss;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            const float tot = (xch[0] + xch[1]) + (xch[2] + xch[3]);
            const float rr = rsqrtf(tot / (float)P.H + P.eps);
            for (int k = er * 2; k < P.H; k += 256) {
              const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + k));
              const float2 wv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(P.w + k));
              const __nv_bfloat162 o = __floats2bfloat162_rn(v.x * rr * wv.x, v.y * rr * wv.y);
              const float2 of = __bfloat1622float2(o);
              *reinterpret_cast<__half2*>(P.y16 + (size_t)m * P.ldy16 + k) = __floats2half2_rn(of.x, of.y);
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        } else if (P.kind == kPhCopy) {
          const long long n2 = (long long)p.M * (P.H / 2);
          for (long long i = (long long)blockIdx.x * 128 + er; i < n2; i += (long long)Gi * 128) {
            const int m = (int)(i / (P.H / 2)), k = (int)(i % (P.H / 2)) * 2;
            const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(P.x + (size_t)m * P.ldx + k));
            *reinterpret_cast<__half2*>(P.y16 + (size_t)m * P.ldy16 + k) = __floats2half2_rn(v.x, v.y);
          }
        } else if (P.kind == kPhRope) {
          const int nheads = P.Hq + 2 * P.Hkv;
          const int items = p.M * nheads;
          for (int it = blockIdx.x * kEpiWarps + ew; it < items; it += Gi * kEpiWarps) {
            const int m = it / nheads, h = it - m * nheads;
            const int b = m / P.T, t = m - b * P.T;
            const int pos = P.pos0[b] + t;
            if (P.hd == 128)
              rope_kv_item<4>(P.qkv + (size_t)m * P.ldqkv, P.Hq, P.Hkv, h, P.qnw, P.knw, P.eps,
                              P.inv_freq, b, pos, P.q_out + (size_t)m * P.Hq * 128, P.kv, lane);
            else
              rope_kv_item<2>(P.qkv + (size_t)m * P.ldqkv, P.Hq, P.Hkv, h, P.qnw, P.knw, P.eps,
                              P.inv_freq, b, pos, P.q_out + (size_t)m * P.Hq * 64, P.kv, lane);
          }
        }
      }
      // this CTA's share of phase q is written: make it visible to later TMA (async proxy)
      // reads, then one release arrival per CTA
      if (P.arrive_bar >= 0) {
        asm volatile("fence.proxy.async.global;" ::: "memory");
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (er == 0) grid_arrive(bar_at(P.arrive_bar));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  // every thread of every CTA is past its last grid wait once `done` reaches G: the last CTA
  // resets the phase counters for the next launch
  if (threadIdx.x == 0) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(p.bars + kChainMaxBars * kBarSlots * kBarStride)
                 : "memory");
    if (old == Gi - 1) {
      for (int k = 0; k < kChainMaxBars * kBarSlots; ++k) p.bars[k * kBarStride] = 0;
      p.bars[kChainMaxBars * kBarSlots * kBarStride] = 0;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
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
// stage ring of the cluster split-K form (one CTA per SM)
template <int BN>
struct CfgCs { static constexpr int kStages = BN <= 32 ? 8 : 6; };

// Split mode of the small-M GEMM: 0 stream-K for every shape (default), 1 cluster split-K for
// shapes with few tiles where one wave of clusters fits. Measured on B200 in a chain of C2 verify
// GEMMs (us per launch, stream-K vs cluster): q|k|v 12.2 vs 17.6, o 12.3 vs 13.1, down 19.0 vs
// 25.1. The cluster form runs one CTA per SM, and its CTAs cannot start until the previous
// kernel's CTAs have left their SM, so it loses more at the launch boundary than it saves in the
// reduction.
static int g_split_mode = 0;

// Cluster split-K for GEMMs with few 128-row tiles (q|k|v, o, down at Qwen3 widths): every
// tile's K is cut into c slices of one cluster, so no single CTA sums ~10 partials at the end.
// The device keeps about one CTA of a cluster kernel per SM resident, so the cluster form runs
// one CTA per SM with a deeper stage ring (the same bytes in flight per SM as two CTAs of the
// stream-K form). Candidates: tiles <= SMs / 2, the largest c <= 8 with tiles * c <= SMs, at
// least 3/5 of the SMs busy; otherwise stream-K.
static int pick_csplit(int tiles, int kb, int c_max) {
  if (g_split_mode != 1) return 0;
  const int sms = sm_count();
  if (tiles <= 0 || tiles * 2 > sms) return 0;
  int c = std::min(std::min(c_max, kb), sms / tiles);
  if (c < 2 || tiles * c * 5 < sms * 3) return 0;
  return c;
}

static long long grid_for(long long total, int ctas_per_sm) {
  const long long g = (long long)sm_count() * ctas_per_sm;
  return std::min<long long>(g, total);
}

// Max active clusters of c CTAs of the cluster-split kernel (cached per c; a failed query is
// retried on the next call and meanwhile reads as "does not fit"). -1: query failed.
template <int BN>
static int max_clusters(int c) {
  constexpr int S = CfgCs<BN>::kStages;
  using L = Smem<BN, S>;
  static int cache[9] = {0};  // max active clusters + 1
  if (c < 2 || c > 8) return -1;
  if (cache[c]) return cache[c] - 1;
  auto kern_cs = w8a16_tc_kernel<BN, S, true, false>;
  if (cudaFuncSetAttribute(kern_cs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kTotal) !=
      cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  cudaLaunchConfig_t q = {};
  q.blockDim = dim3(kThreads);
  q.dynamicSmemBytes = L::kTotal;
  q.gridDim = dim3((unsigned)(c * 64));
  cudaLaunchAttribute qa[1];
  qa[0].id = cudaLaunchAttributeClusterDimension;
  qa[0].val.clusterDim.x = (unsigned)c;
  qa[0].val.clusterDim.y = 1;
  qa[0].val.clusterDim.z = 1;
  q.attrs = qa;
  q.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern_cs, &q) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  cache[c] = n + 1;
  return n;
}

// cluster size for this GEMM: pick_csplit's choice if one wave of its clusters is resident
// at once, else 0 (stream-K)
template <int BN>
static int plan_csplit(int tiles, int kb) {
  for (int c_max = 8; c_max >= 2;) {
    const int c = pick_csplit(tiles, kb, c_max);
    if (c < 2) return 0;
    if (max_clusters<BN>(c) >= tiles) return c;
    c_max = c - 1;  // fewer, wider slices
  }
  return 0;
}

template <int BN, bool ROPE = false, bool PEER = false>
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
  constexpr int SC = CfgCs<BN>::kStages;
  using LC = Smem<BN, SC>;
  auto kern = w8a16_tc_kernel<BN, S, false, ROPE, PEER>;
  auto kern_cs = w8a16_tc_kernel<BN, SC, true, false>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kTotal) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern_cs, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LC::kTotal) !=
            cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "cudaFuncSetAttribute(smem=%u/%u) failed", L::kTotal, LC::kTotal);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the fused epilogues (RoPE, row sums of squares) are stream-K only
  p.csplit = (ROPE || p.ss_out || p.epilogue == DSPARK_EPI_PEER_F32) ? 0 : plan_csplit<BN>(p.tiles, p.kb);
  long long grid;
  if (p.csplit > 1) {
    grid = (long long)p.tiles * p.csplit;
    cfg.dynamicSmemBytes = LC::kTotal;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = (unsigned)p.csplit;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  } else {
    grid = grid_for(p.total, Cfg<BN>::kCtasPerSm);
  }
  cfg.gridDim = dim3((unsigned)grid);
  cudaError_t e = p.csplit > 1 ? cudaLaunchKernelEx(&cfg, kern_cs, tw, tsb, tx, p)
                               : cudaLaunchKernelEx(&cfg, kern, tw, tsb, tx, p);
  if (e != cudaSuccess)
    return set_error(DSPARK_ERR_LAUNCH, "w8a16 tc launch failed: %s", cudaGetErrorString(e));
  note_launch();
  return DSPARK_OK;
}

// ---- layer chain host side
template <int BN>
static int launch_chain(const ChainMaps& maps, const ChainParams& p, cudaStream_t st) {
  constexpr int S = Cfg<BN>::kStages;
  using L = Smem<BN, S>;
  auto kern = chain_kernel<BN, S>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kTotal) !=
        cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "chain: cudaFuncSetAttribute(smem=%u) failed", L::kTotal);
    configured = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, L::kTotal) != cudaSuccess ||
      per_sm < 1)
    return set_error(DSPARK_ERR_LAUNCH, "chain: no resident CTA fits");
  const int grid = sm_count() * std::min(per_sm, Cfg<BN>::kCtasPerSm);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps, p);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_LAUNCH, "chain launch failed: %s", cudaGetErrorString(e));
  note_launch();
  return DSPARK_OK;
}

static int chain_grid(int M) {
  const int bn = pick_bn(M);
  return sm_count() * (bn <= 32 ? 2 : 1);
}

// workspace: [phase counters + done (256 B)] [stream-K tile counters, a FIXED region of
// kMaxTiles ints for every phase list] [2 partial regions]. The fixed region keeps one chain's
// partials from landing where another chain (a different phase list sharing the workspace)
// keeps its counters.
static size_t chain_ws(int M, const dspark_chain_phase* ph, int n, size_t* off_part) {
  (void)ph;
  (void)n;
  const size_t part = (size_t)chain_grid(M) * 2 * pick_bn(M) * BM * sizeof(float);
  if (off_part) *off_part = kBarRegion + kCounterBytes;
  return kBarRegion + kCounterBytes + 2 * part;
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

// Shared launch path of the W8 GEMM entry points: rope != nullptr selects the fused q|k|v
// epilogue (y unused).
static int gemm_launch(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M, int N,
                       int K, void* y, int ldy, const void* residual, int ldr, int epilogue,
                       void* workspace, size_t workspace_bytes, const void* pf0, size_t pf0_bytes,
                       const void* pf1, size_t pf1_bytes, const w8::RopeEpi* rope,
                       const dspark_gemm_opts* opts, int* status, dspark_stream_t stream,
                       const dspark_peer_ar* peer = nullptr) {
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
  if (rope) p.rope = *rope;
  if (peer) {
    for (int r = 0; r < peer->world; ++r) {
      p.peer_y[r] = static_cast<float*>(peer->recv[r]);
      p.peer_f[r] = static_cast<int*>(peer->flags[r]);
    }
    p.peer_world = peer->world;
    p.peer_rank = peer->rank;
    p.peer_mcap = peer->m_cap;
    p.peer_epoch = peer->epoch;
  }
  if (opts) {
    if (opts->copy_f16) {
      if (epilogue != DSPARK_EPI_RESIDUAL_BF16 || opts->copy_f16_ld < N)
        return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: copy_f16 needs RESIDUAL_BF16 and ld >= N");
      p.copy16 = static_cast<__half*>(opts->copy_f16);
      p.copy16_ld = opts->copy_f16_ld;
    }
    if (opts->row_sumsq) {
      if (epilogue != DSPARK_EPI_RESIDUAL_BF16 && epilogue != DSPARK_EPI_STORE_BF16)
        return set_error(DSPARK_ERR_INVALID,
                         "w8a16_gemm: row_sumsq needs the STORE_BF16 or RESIDUAL_BF16 epilogue");
      p.ss_out = opts->row_sumsq;
    }
    if (opts->norm_w) {
      if (!opts->norm_sumsq || opts->norm_tiles <= 0)
        return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: norm_w without norm_sumsq / norm_tiles");
      if (reinterpret_cast<uintptr_t>(opts->norm_w) & 15)
        return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: norm_w not 16-byte aligned");
      p.norm_w = static_cast<const __nv_bfloat16*>(opts->norm_w);
      p.ss_in = opts->norm_sumsq;
      p.ss_tiles = opts->norm_tiles;
      p.ss_ld = opts->norm_ld > 0 ? opts->norm_ld : opts->norm_tiles;
      if (p.ss_ld < opts->norm_tiles)
        return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: norm_ld %d < norm_tiles %d", p.ss_ld,
                         opts->norm_tiles);
      if ((p.ss_ld & 3) == 0 && (reinterpret_cast<uintptr_t>(opts->norm_sumsq) & 15))
        return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: norm_sumsq not 16-byte aligned");
      p.norm_eps = opts->norm_eps;
    }
  }
  const void* pf[2] = {pf0, pf1};
  const size_t pfb[2] = {pf0_bytes, pf1_bytes};
  for (int r = 0; r < 2; ++r) {
    if (pf[r] && pfb[r] && (reinterpret_cast<uintptr_t>(pf[r]) & 15))
      return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm_pf: prefetch range %d not 16-byte aligned", r);
    p.pf_ptr[r] = static_cast<const char*>(pf[r]);
    p.pf_bytes[r] = pf[r] ? (unsigned long long)(pfb[r] & ~(size_t)15) : 0ull;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (peer) {
    switch (w8::pick_bn(M)) {
      case 16: return w8::launch_tc<16, false, true>(x, ldx, wq, wsb, p, st);
      case 32: return w8::launch_tc<32, false, true>(x, ldx, wq, wsb, p, st);
      case 48: return w8::launch_tc<48, false, true>(x, ldx, wq, wsb, p, st);
      default: return w8::launch_tc<64, false, true>(x, ldx, wq, wsb, p, st);
    }
  }
  if (rope) {
    switch (w8::pick_bn(M)) {
      case 16: return w8::launch_tc<16, true>(x, ldx, wq, wsb, p, st);
      case 32: return w8::launch_tc<32, true>(x, ldx, wq, wsb, p, st);
      case 48: return w8::launch_tc<48, true>(x, ldx, wq, wsb, p, st);
      default: return w8::launch_tc<64, true>(x, ldx, wq, wsb, p, st);
    }
  }
  switch (w8::pick_bn(M)) {
    case 16: return w8::launch_tc<16>(x, ldx, wq, wsb, p, st);
    case 32: return w8::launch_tc<32>(x, ldx, wq, wsb, p, st);
    case 48: return w8::launch_tc<48>(x, ldx, wq, wsb, p, st);
    default: return w8::launch_tc<64>(x, ldx, wq, wsb, p, st);
  }
}

extern "C" int dspark_w8a16_gemm_pf(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                                    int M, int N, int K, void* y, int ldy, const void* residual,
                                    int ldr, int epilogue, void* workspace, size_t workspace_bytes,
                                    const void* pf0, size_t pf0_bytes, const void* pf1,
                                    size_t pf1_bytes, int* status, dspark_stream_t stream) {
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, y, epilogue, residual);
  if (rc) return rc;
  return gemm_launch(x, ldx, wq, wsb, M, N, K, y, ldy, residual, ldr, epilogue, workspace,
                     workspace_bytes, pf0, pf0_bytes, pf1, pf1_bytes, nullptr, nullptr, status,
                     stream);
}

extern "C" size_t dspark_gemm_opts_size(void) { return sizeof(dspark_gemm_opts); }

extern "C" int dspark_w8a16_gemm_ex(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                                    int M, int N, int K, void* y, int ldy, const void* residual,
                                    int ldr, int epilogue, const dspark_gemm_opts* opts,
                                    void* workspace, size_t workspace_bytes, int* status,
                                    dspark_stream_t stream) {
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, y, epilogue, residual);
  if (rc) return rc;
  const dspark_gemm_opts z{};
  const dspark_gemm_opts& o = opts ? *opts : z;
  return gemm_launch(x, ldx, wq, wsb, M, N, K, y, ldy, residual, ldr, epilogue, workspace,
                     workspace_bytes, o.prefetch[0], o.prefetch_bytes[0], o.prefetch[1],
                     o.prefetch_bytes[1], nullptr, &o, status, stream);
}

extern "C" int dspark_w8a16_gemm_qkv_rope(const void* x, int ldx, const uint8_t* wq,
                                          const uint32_t* wsb, int M, int K, int T, int Hq,
                                          int Hkv, int hd, const void* q_norm_w,
                                          const void* k_norm_w, float eps, const float* inv_freq,
                                          const int32_t* pos0, void* q_out,
                                          const dspark_kv_layout* kv,
                                          const dspark_gemm_opts* opts, void* workspace,
                                          size_t workspace_bytes, int* status,
                                          dspark_stream_t stream) {
  if (hd != 64 && hd != 128)
    return set_error(DSPARK_ERR_UNSUPPORTED, "w8a16_gemm_qkv_rope: head_dim %d", hd);
  if (T <= 0 || M % T || Hkv <= 0 || Hq < 0 || !k_norm_w || !inv_freq || !pos0 || !kv ||
      !kv->pool || !kv->block_table || (Hq > 0 && (!q_out || !q_norm_w)))
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_qkv_rope: bad arguments");
  if (kv->head_dim != hd || kv->num_kv_heads != Hkv || kv->page_size <= 0 ||
      kv->page_bytes != dspark_kv_page_bytes(kv->page_size, Hkv, hd, kv->kv8))
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_qkv_rope: kv layout does not match");
  const int N = (Hq + 2 * Hkv) * hd;
  // the row output pointer only feeds the shared checks: the fused epilogue writes q_out / cache
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, q_out ? q_out : kv->pool,
                              DSPARK_EPI_STORE_BF16, nullptr);
  if (rc) return rc;
  w8::RopeEpi r{};
  r.qnw = static_cast<const __nv_bfloat16*>(q_norm_w);
  r.knw = static_cast<const __nv_bfloat16*>(k_norm_w);
  r.inv_freq = inv_freq;
  r.pos0 = pos0;
  r.q_out = static_cast<__nv_bfloat16*>(q_out);
  r.kv = *kv;
  r.eps = eps;
  r.T = T; r.Hq = Hq; r.Hkv = Hkv; r.hd = hd;
  const dspark_gemm_opts z{};
  const dspark_gemm_opts& o = opts ? *opts : z;
  if (o.row_sumsq)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_qkv_rope: row_sumsq is not produced here");
  return gemm_launch(x, ldx, wq, wsb, M, N, K, nullptr, 0, nullptr, 0, -1, workspace,
                     workspace_bytes, o.prefetch[0], o.prefetch_bytes[0], o.prefetch[1],
                     o.prefetch_bytes[1], &r, &o, status, stream);
}

extern "C" int dspark_w8a16_gemm(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                                 int M, int N, int K, void* y, int ldy, const void* residual,
                                 int ldr, int epilogue, void* workspace, size_t workspace_bytes,
                                 int* status, dspark_stream_t stream) {
  return dspark_w8a16_gemm_pf(x, ldx, wq, wsb, M, N, K, y, ldy, residual, ldr, epilogue, workspace,
                              workspace_bytes, nullptr, 0, nullptr, 0, status, stream);
}

extern "C" int dspark_w8a16_gemm_peer(const void* x, int ldx, const uint8_t* wq,
                                      const uint32_t* wsb, int M, int N, int K,
                                      const dspark_peer_ar* ar, void* workspace,
                                      size_t workspace_bytes, int* status, dspark_stream_t stream) {
  if (!ar) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_peer: no peer descriptor");
  if (ar->world < 2 || ar->world > 8 || ar->rank < 0 || ar->rank >= ar->world || ar->n != N ||
      ar->epoch < 1 || M > ar->m_cap)
    return set_error(DSPARK_ERR_INVALID,
                     "w8a16_gemm_peer: world=%d rank=%d n=%d (N=%d) epoch=%d M=%d m_cap=%d",
                     ar->world, ar->rank, ar->n, N, ar->epoch, M, ar->m_cap);
  for (int r = 0; r < ar->world; ++r)
    if (!ar->recv[r] || !ar->flags[r])
      return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_peer: rank %d's buffers missing", r);
  int rc = gemm_common_checks(x, ldx, wq, wsb, M, N, K, ar->recv[ar->rank], DSPARK_EPI_STORE_F32,
                              nullptr);
  if (rc) return rc;
  return gemm_launch(x, ldx, wq, wsb, M, N, K, ar->recv[ar->rank], N, nullptr, 0,
                     DSPARK_EPI_PEER_F32, workspace, workspace_bytes, nullptr, 0, nullptr, 0,
                     nullptr, nullptr, status, stream, ar);
}

extern "C" int dspark_w8a16_gemm_plan(int M, int N, int K, int* grid, int* cluster,
                                      int* max_active) {
  using namespace w8;
  if (M < 1 || M > 64 || N <= 0 || K <= 0 || N % BM || K % BK || !grid || !cluster)
    return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_plan: bad arguments");
  const int tiles = N / BM, kb = K / BK;
  const int bn = pick_bn(M);
  const int cps = bn <= 32 ? 2 : 1;
  int c = 0, mc = 0;
  const int saved = g_split_mode;
  g_split_mode = 1;
  const int c0 = pick_csplit(tiles, kb, 8);  // the cluster size mode 1 would try first
  g_split_mode = saved;
  switch (bn) {
    case 16: c = plan_csplit<16>(tiles, kb); mc = max_clusters<16>(c0); break;
    case 32: c = plan_csplit<32>(tiles, kb); mc = max_clusters<32>(c0); break;
    case 48: c = plan_csplit<48>(tiles, kb); mc = max_clusters<48>(c0); break;
    default: c = plan_csplit<64>(tiles, kb); mc = max_clusters<64>(c0); break;
  }
  *cluster = c;
  *grid = c > 1 ? tiles * c : (int)grid_for((long long)tiles * kb, cps);
  if (max_active) *max_active = mc;
  return DSPARK_OK;
}

extern "C" int dspark_w8a16_gemm_split_mode(int mode) {
  if (mode < 0 || mode > 1) return set_error(DSPARK_ERR_INVALID, "w8a16_gemm_split_mode: %d", mode);
  w8::g_split_mode = mode;
  return DSPARK_OK;
}

extern "C" size_t dspark_chain_phase_size(void) { return sizeof(dspark_chain_phase); }

extern "C" size_t dspark_chain_workspace_bytes(int M, const dspark_chain_phase* phases, int n) {
  if (M <= 0 || M > 64 || !phases || n <= 0) return 0;
  return w8::chain_ws(M, phases, n, nullptr);
}

extern "C" int dspark_run_chain(int M, const dspark_chain_phase* ph, int n, void* workspace,
                                size_t workspace_bytes, int* status, dspark_stream_t stream) {
  using namespace w8;
  if (!ph || n <= 0 || n > kChainMaxPhases) return set_error(DSPARK_ERR_INVALID, "chain: %d phases", n);
  if (M < 1 || M > 64) return set_error(DSPARK_ERR_INVALID, "chain: M=%d not in [1,64]", M);
  size_t off_part = 0;
  const size_t need = chain_ws(M, ph, n, &off_part);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "chain: workspace %zu < %zu bytes", workspace_bytes, need);
  const int BNv = pick_bn(M);
  {
    long long tiles = 0;
    for (int i = 0; i < n; ++i)
      if (ph[i].kind == DSPARK_PHASE_GEMM) tiles += ph[i].N / BM;
    if (tiles > kMaxTiles) return set_error(DSPARK_ERR_UNSUPPORTED, "chain: %lld tiles > %d", tiles, kMaxTiles);
  }
  ChainMaps maps;
  memset(&maps, 0, sizeof(maps));
  ChainParams p;
  memset(&p, 0, sizeof(p));
  p.M = M;
  p.nphases = n;
  p.status = status;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  p.bars = reinterpret_cast<int*>(w);
  int* counters = reinterpret_cast<int*>(w + kBarRegion);
  const size_t part_bytes = (size_t)chain_grid(M) * 2 * BNv * BM * sizeof(float);
  int ng = 0;
  // dependencies: a grid barrier after every GEMM and NORM phase but the last phase; every
  // phase reads what was written before the latest barrier
  int nbar = 0, last_bar = -1;
  for (int i = 0; i < n; ++i) {
    const dspark_chain_phase& q = ph[i];
    ChainPhase& P = p.ph[i];
    P.kind = q.kind;
    P.wait_bar = last_bar;
    P.arrive_bar = -1;
    P.local_norm = -1;
    if ((q.kind == DSPARK_PHASE_GEMM || q.kind == DSPARK_PHASE_NORM) && i < n - 1) {
      P.arrive_bar = nbar++;
      last_bar = P.arrive_bar;
    }
    switch (q.kind) {
      case DSPARK_PHASE_GEMM: {
        if (ng >= kChainMaxGemm) return set_error(DSPARK_ERR_UNSUPPORTED, "chain: more than %d GEMMs", kChainMaxGemm);
        int rc = gemm_common_checks(q.x, q.ldx, q.wq, q.wsb, M, q.N, q.K, q.y, q.epilogue, q.residual);
        if (rc) return rc;
        ChainGemm& g = p.g[ng];
        g.N = q.N; g.K = q.K; g.tiles = q.N / BM; g.kb = q.K / BK;
        g.total = (long long)g.tiles * g.kb;
        g.epilogue = q.epilogue; g.y = q.y; g.ldy = q.ldy; g.residual = q.residual; g.ldr = q.ldr;
        g.counters = counters;
        counters += g.tiles;
        g.partials = reinterpret_cast<float*>(w + off_part + (size_t)(ng & 1) * part_bytes);
        if ((rc = make_map_2d(&maps.w[ng], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q.wq, (uint64_t)q.K,
                              (uint64_t)q.N, (uint64_t)q.K, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
          return rc;
        if ((rc = make_map_2d(&maps.sb[ng], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, q.wsb, (uint64_t)q.N,
                              (uint64_t)(q.K / 64), (uint64_t)q.N * 4, BM, 2, CU_TENSOR_MAP_SWIZZLE_NONE)))
          return rc;
        if ((rc = make_map_2d(&maps.x[ng], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, q.x, (uint64_t)q.K,
                              (uint64_t)M, (uint64_t)q.ldx * 2, 64, BNv, CU_TENSOR_MAP_SWIZZLE_128B)))
          return rc;
        P.gemm = ng++;
        break;
      }
      case DSPARK_PHASE_NORM:
      case DSPARK_PHASE_COPY_F16:
        if (!q.x || !q.y || q.H <= 0 || q.H % 2 || q.ldx < q.H || q.ldy < q.H || q.ldx % 2 || q.ldy % 2 ||
            (q.kind == DSPARK_PHASE_NORM && !q.w))
          return set_error(DSPARK_ERR_INVALID, "chain: bad norm/copy phase %d", i);
        P.x = static_cast<const __nv_bfloat16*>(q.x); P.ldx = q.ldx;
        P.w = static_cast<const __nv_bfloat16*>(q.w); P.H = q.H; P.eps = q.eps;
        P.y16 = static_cast<__half*>(q.y); P.ldy16 = q.ldy;
        break;
      case DSPARK_PHASE_ROPE_KV:
        if (!q.qkv || !q.k_norm || !q.inv_freq || !q.pos0 || (q.Hq > 0 && (!q.q_out || !q.q_norm)) ||
            (q.hd != 64 && q.hd != 128) || q.T <= 0 || M % q.T || q.kv.head_dim != q.hd ||
            q.kv.num_kv_heads != q.Hkv || !q.kv.pool || !q.kv.block_table)
          return set_error(DSPARK_ERR_INVALID, "chain: bad rope phase %d", i);
        P.qkv = static_cast<const __nv_bfloat16*>(q.qkv); P.ldqkv = q.ldqkv; P.T = q.T;
        P.Hq = q.Hq; P.Hkv = q.Hkv; P.hd = q.hd;
        P.qnw = static_cast<const __nv_bfloat16*>(q.q_norm);
        P.knw = static_cast<const __nv_bfloat16*>(q.k_norm);
        P.eps = q.eps; P.inv_freq = q.inv_freq; P.pos0 = q.pos0;
        P.q_out = static_cast<__nv_bfloat16*>(q.q_out); P.kv = q.kv;
        break;
      default:
        return set_error(DSPARK_ERR_INVALID, "chain: phase %d kind %d", i, q.kind);
    }
  }
  p.ngemm = ng;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (BNv) {
    case 16: return launch_chain<16>(maps, p, st);
    case 32: return launch_chain<32>(maps, p, st);
    case 48: return launch_chain<48>(maps, p, st);
    default: return launch_chain<64>(maps, p, st);
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
  const int lrc = check_launch("w8a16_gemm_simt");
  if (lrc == DSPARK_OK) note_launch();
  return lrc;
}
