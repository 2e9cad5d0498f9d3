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
  const int* peer_epoch_dev;  // set: the epoch is peer_epoch_dev[0] + 1 (device-resident)
};

__device__ __forceinline__ long long range_start(long long b, long long total, long long G) {
  return b * total / G;
}
// the CTA whose range contains flattened k-block g
__device__ __forceinline__ long long range_owner(long long g, long long total, long long G) {
  return ((g + 1) * G + total - 1) / total - 1;
}

// The bf16 tile staged in shared memory as [BN][BM] (the exchange buffer) goes out as 16-byte
// vectors: rows < M of y (and their fp16 copy), one vector of 8 columns per thread per step.
// With ss_out, thread m < M then sums the squares of row m's 128 staged values, in column
// order with one rounding per step: the same order for a row whatever its place in the block.
// y, ldy (and the copy) are 16-byte aligned / multiples of 8 (checked on the host).
template <typename PT>
__device__ __forceinline__ void store_staged_rows(const PT& p, int tile, int er,
                                                  const __nv_bfloat16* xs) {
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(p.y);
  constexpr int kVec = BM / 8;  // 16-byte vectors per row
  for (int i = er; i < p.M * kVec; i += kEpiWarps * 32) {
    const int m = i / kVec, c = i - m * kVec;
    const uint4 v = *reinterpret_cast<const uint4*>(xs + m * BM + c * 8);
    *reinterpret_cast<uint4*>(y + (size_t)m * p.ldy + tile * BM + c * 8) = v;
    if (p.copy16) {
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
      uint4 h;
      __half2* h2 = reinterpret_cast<__half2*>(&h);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(b2[k]);
        check_f16(f.x, p.status);
        check_f16(f.y, p.status);
        h2[k] = __float22half2_rn(f);
      }
      *reinterpret_cast<uint4*>(p.copy16 + (size_t)m * p.copy16_ld + tile * BM + c * 8) = h;
    }
  }
  if (p.ss_out && er < p.M) {
    float acc = 0.0f;
    for (int c = 0; c < kVec; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(xs + er * BM + c * 8);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(b2[k]);
        acc = __fmaf_rn(f.x, f.x, acc);
        acc = __fmaf_rn(f.y, f.y, acc);
      }
    }
    p.ss_out[(size_t)er * p.tiles + tile] = acc;
  }
}

// The SiLU epilogue computes all rows of a 16-row chunk that holds any of the M rows without a
// branch per row (rows past M hold zeros: their activations are the tensor map's zero fill), so
// the rows' arithmetic overlaps; only the stores are predicated on m < M.
// PEER: the instance of the tensor-parallel fused all-reduce (dspark_w8a16_gemm_peer); the
// other instances carry no code for it
template <int BN, bool PEER = false, typename PT>
__device__ __forceinline__ void epilogue_store(const PT& p, int tile, int er, const float* acc,
                                               float* xch,
                                               const __nv_bfloat162* rpre = nullptr) {
  const int n = tile * BM + er;
  switch (p.epilogue) {
    case DSPARK_EPI_STORE_BF16: {
      // stage the tile's bf16 rows, then store them as vectors
      __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xch);
#pragma unroll
      for (int m = 0; m < BN; ++m)
        if (m < p.M) xs[m * BM + er] = __float2bfloat16_rn(acc[m]);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      store_staged_rows(p, tile, er, xs);
      asm volatile("bar.sync 1, 128;" ::: "memory");  // xch is reused by the next tile
      break;
    }
    case DSPARK_EPI_PEER_F32: {
      if constexpr (PEER) {
        // one-shot all-reduce, send half: this rank's fp32 tile into slot (epoch & 1), source row
        // block `rank`, of every rank's receive buffer (plain stores over NVLink), then, once the
        // tile's 128 threads have stored, the tile's epoch flag on every rank
        // (a device-resident epoch was stored by the previous call's reduce, which completed
        // before this epilogue's griddepcontrol.wait returned)
        const int epoch = p.peer_epoch_dev ? __ldcg(p.peer_epoch_dev) + 1 : p.peer_epoch;
        const int slot = epoch & 1;
        const size_t off = ((size_t)(slot * p.peer_world + p.peer_rank) * p.peer_mcap) * p.N + n;
        for (int r = 0; r < p.peer_world; ++r) {
          float* y = p.peer_y[r] + off;
#pragma unroll
          for (int m = 0; m < BN; ++m)
            if (m < p.M) y[(size_t)m * p.N] = acc[m];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (er == 0) {
          fence_acq_rel_sys();
          const size_t fo = (size_t)(slot * p.peer_world + p.peer_rank) * p.tiles + tile;
          for (int r = 0; r < p.peer_world; ++r) st_relaxed_sys(p.peer_f[r] + fo, epoch);
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
      // y may be the residual itself (in place): every residual value is read (below, or by
      // the caller into rpre) before the barrier that precedes the first store
      const __nv_bfloat16* r = static_cast<const __nv_bfloat16*>(p.residual);
      __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(xch);
#pragma unroll
      for (int c0 = 0; c0 < BN; c0 += 16) {  // 16 rows at a time bounds the registers held
        if (c0 >= p.M) break;
        __nv_bfloat16 rv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c0 + j;
          if (rpre)  // read by the caller before it waited on the other contributors
            rv[j] = (m & 1) ? rpre[m >> 1].y : rpre[m >> 1].x;
          else
            rv[j] = m < p.M ? __ldcg(r + (size_t)m * p.ldr + n) : __float2bfloat16_rn(0.0f);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < p.M)
            xs[(c0 + j) * BM + er] =
                __float2bfloat16_rn(__bfloat162float(rv[j]) + bf16_round(acc[c0 + j]));
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      // the rows (and their fp16 copy) as vectors; the rows' shares of the next RMSNorm
      store_staged_rows(p, tile, er, xs);
      asm volatile("bar.sync 1, 128;" ::: "memory");  // xch is reused by the next tile
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
          if (c0 >= p.M) break;
          // the exchanged values first (xch is a generic pointer the stores may alias)
          float a[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) a[j] = xch[er * BN + c0 + j];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float g = bf16_round(acc[c0 + j]);
            const float s = bf16_round(silu_f(g));
            a[j] = bf16_round(__fmul_rn(s, bf16_round(a[j])));
          }
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < p.M) {
              check_f16(a[j], p.status);
              y[(size_t)(c0 + j) * p.ldy + col] = __float2half_rn(a[j]);
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

// The fused q|k|v epilogue of a finished tile: stage the tile's bf16 outputs (the values the
// separate q|k|v GEMM would store) in shared memory as [m][128], then one warp per (token, head
// in the tile) runs the same norm + RoPE + KV write as the standalone kernel. The staging fits
// the exchange buffer: BN x 128 bf16 = 64 x BN fp32.
template <int BN, typename PT>
__device__ __forceinline__ void rope_epilogue(const PT& p, int tile, int er, const float* acc,
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

template <int BN, int STAGES, bool ROPE, bool PEER = false>
__global__ void __launch_bounds__(kThreads, (BN <= 32 ? 2 : 1))
    w8a16_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_sb,
                    const __grid_constant__ CUtensorMap tm_x, const Params p) {
  using L = Smem<BN, STAGES>;
  // TMEM: [0, AB*64) the converted-weight ring (64 columns = 128 fp16 per lane each), then two
  // fp32 accumulators of ACCS columns. Two CTAs per SM share the 512 columns; one CTA per SM
  // takes all of them for a deeper ring (the ring depth bounds how far conversion runs ahead
  // of MMA completion).
  constexpr bool kTwoPerSm = BN <= 32;
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
  const long long start = range_start(blockIdx.x, total, G);
  const long long end = range_start(blockIdx.x + 1, total, G);
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
              // (read from L2: written by another grid that may still be running)
              if ((p.ss_ld & 3) == 0)
                for (; t + 4 <= p.ss_tiles; t += 4) {
                  const float4 q4 = __ldcg(reinterpret_cast<const float4*>(row + t));
                  sum = (((sum + q4.x) + q4.y) + q4.z) + q4.w;
                }
              for (; t < p.ss_tiles; ++t) sum += __ldcg(row + t);
            }
            rn[kk] = rsqrtf(__fadd_rn(__fdiv_rn(sum, (float)p.K), p.norm_eps));
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
              const __nv_bfloat162 xn = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(hv.x, rn[kk]), wf.x), __fmul_rn(__fmul_rn(hv.y, rn[kk]), wf.y));
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
    pdl_wait();  // outputs may still be read by the previous kernel
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

      if (whole) {
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
              rpre[j].x = m < p.M ? __ldcg(rp + (size_t)m * p.ldr) : __float2bfloat16_rn(0.0f);
              rpre[j].y = m + 1 < p.M ? __ldcg(rp + (size_t)(m + 1) * p.ldr) : __float2bfloat16_rn(0.0f);
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


  // a role that ran on one lane (producer, MMA issuer) rejoins its warp before the
  // CTA barrier: the barrier counts whole warps, and TMEM is freed after it
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TC);
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
static long long grid_for(long long total, int ctas_per_sm) {
  const long long g = (long long)sm_count() * ctas_per_sm;
  return std::min<long long>(g, total);
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
  auto kern = w8a16_tc_kernel<BN, S, ROPE, PEER>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kTotal) !=
            cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return set_error(DSPARK_ERR_CUDA, "cudaFuncSetAttribute(smem=%u) failed", L::kTotal);
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = L::kTotal;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3((unsigned)grid_for(p.total, Cfg<BN>::kCtasPerSm));
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tsb, tx, p);
  if (e != cudaSuccess)
    return set_error(DSPARK_ERR_LAUNCH, "w8a16 tc launch failed: %s", cudaGetErrorString(e));
  note_launch();
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

// The dspark_gemm_opts fields: the fp16 tap copy, the row sums of squares out of the epilogue,
// and the input RMSNorm fused into the converters.
static int apply_opts(w8::Params& p, const dspark_gemm_opts& o, int epilogue, int N) {
  if (o.copy_f16) {
    if (epilogue != DSPARK_EPI_RESIDUAL_BF16 || o.copy_f16_ld < N)
      return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: copy_f16 needs RESIDUAL_BF16 and ld >= N");
    if ((reinterpret_cast<uintptr_t>(o.copy_f16) & 15) || (o.copy_f16_ld & 7))
      return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: copy_f16 must be 16-byte aligned, ld %% 8 == 0");
    p.copy16 = static_cast<__half*>(o.copy_f16);
    p.copy16_ld = o.copy_f16_ld;
  }
  if (o.row_sumsq) {
    if (epilogue != DSPARK_EPI_RESIDUAL_BF16 && epilogue != DSPARK_EPI_STORE_BF16)
      return set_error(DSPARK_ERR_INVALID,
                       "w8a16_gemm: row_sumsq needs the STORE_BF16 or RESIDUAL_BF16 epilogue");
    p.ss_out = o.row_sumsq;
  }
  if (o.norm_w) {
    if (!o.norm_sumsq || o.norm_tiles <= 0)
      return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: norm_w without norm_sumsq / norm_tiles");
    if (reinterpret_cast<uintptr_t>(o.norm_w) & 15)
      return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: norm_w not 16-byte aligned");
    p.norm_w = static_cast<const __nv_bfloat16*>(o.norm_w);
    p.ss_in = o.norm_sumsq;
    p.ss_tiles = o.norm_tiles;
    p.ss_ld = o.norm_ld > 0 ? o.norm_ld : o.norm_tiles;
    if (p.ss_ld < o.norm_tiles)
      return set_error(DSPARK_ERR_INVALID, "w8a16_gemm: norm_ld %d < norm_tiles %d", p.ss_ld,
                       o.norm_tiles);
    if ((p.ss_ld & 3) == 0 && (reinterpret_cast<uintptr_t>(o.norm_sumsq) & 15))
      return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: norm_sumsq not 16-byte aligned");
    p.norm_eps = o.norm_eps;
  }
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
    p.peer_epoch_dev = peer->epoch_dev;
  }
  if (opts) {
    const int rc = apply_opts(p, *opts, epilogue, N);
    if (rc) return rc;
  }
  // the bf16 epilogues store their staged rows as 16-byte vectors
  if (!rope && !peer && (epilogue == DSPARK_EPI_STORE_BF16 || epilogue == DSPARK_EPI_RESIDUAL_BF16) &&
      ((reinterpret_cast<uintptr_t>(y) & 15) || (ldy & 7)))
    return set_error(DSPARK_ERR_ALIGN, "w8a16_gemm: y must be 16-byte aligned with ldy %% 8 == 0 (ldy=%d)", ldy);
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
      (ar->epoch < 1 && !ar->epoch_dev) || M > ar->m_cap)
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

