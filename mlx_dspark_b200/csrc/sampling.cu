// K9 — lossless speculative sampling on the device: top-k / top-p truncation of
// softmax(logits / T), categorical draws from a Philox4x32-10 stream, and the
// rejection-sampling acceptance with residual resampling.
//
// Reference semantics:
//   truncate_probs                 src/mlx_dspark/sampling.py:18-44
//   sample_probs                   src/mlx_dspark/sampling.py:47-49
//   _spec_sample_accept            src/mlx_dspark/generate.py:659-688
//   DSpark q (sample_block_probs)  src/mlx_dspark/model.py:283-309
//   DFlash q and draft             src/mlx_dspark/generate.py:541-545
//   point-mass q of lookup drafts  src/mlx_dspark/generate.py:815-824
//
// Arithmetic (every step is reproducible bit for bit on a CPU):
//   x_i   = bf16(l_i / bf16(T))  (temp_mode 0)  or  bf16(l_i * bf16(1/T))  (temp_mode 1)
//   key_i = order-preserving 16-bit key of x_i; -0 folds into +0
//   w_i   = floor(2^40 * 2^t), t = (x_i - max x) * log2(e), with 2^t = 2^rint(t) * P7(t - rint(t))
//           and P7 the degree-7 Taylor polynomial of 2^f; multiplies and adds round separately
//           (no FMA contraction) and w_i = 0 below 2^-45
//   top-k: keep key >= the k-th largest key (ties kept)
//   top-p: keep key >= t_p, the smallest key t present with G(t) < top_p * Z, where G(t) is the
//          weight strictly above t after the top-k cut and Z the weight of the whole row
//   p_i   = float(double(w_i) * (1 / double(S))), S = kept weight
//   draws: r = 64-bit Philox word, target = floor(r * S / 2^64), token = the first index (in
//          vocabulary order) whose inclusive weight prefix exceeds target; a zero total draws
//          uniformly over the vocabulary
//   accept row i: u = (Philox word >> 8) * 2^-24; accepted iff u < min(1, p[x] / max(q[x], 1e-9))
//   residual: d_j = p_j - q_j (fp32), weight floor(2^40 * d_j) where d_j > 0
// The reference rounds p to bf16 (MLX softmax output dtype) before truncating; this build keeps
// 2^-40 fixed point, so kept sets can differ only where probabilities tie after bf16 rounding.
//
// Layout: one thread-block cluster of 8 CTAs per row. Each CTA holds 1/8 of the row as 16-bit
// keys in shared memory; the cluster exchanges histograms and partial sums through distributed
// shared memory (barrier.cluster, no spin waits). Thresholds come from two 8-bit radix passes
// over the keys. When at most kCand keys survive the top-k cut, rank 0 gathers them and finishes
// the nucleus, the draw and the residual on that short list.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace dspark {
namespace smp {

constexpr int kCluster = 8;
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxChunk = 32768;
constexpr int kMaxV = kCluster * kMaxChunk;
constexpr int kCand = 512;
constexpr int kBins = 256;
constexpr int kSub = 4;
constexpr int kMbox = 64;
constexpr int kMaxT = 32;
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): counter {offset_lo, offset_hi, row, stream}, key {seed_lo, seed_hi}.
struct U4 {
  uint32_t x, y, z, w;
};
__device__ __forceinline__ U4 philox(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
  }
  return c;
}

// ------------------------------------------------------------------------------------------
// keys and fixed-point weights
__device__ __forceinline__ uint32_t key_of(uint16_t b, float tb, int tmode) {
  if (tmode != 2) {
    const float l = __uint_as_float((uint32_t)b << 16);
    const float x = tmode == 0 ? __fdiv_rn(l, tb) : __fmul_rn(l, tb);
    b = __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  if (b == 0x8000u) b = 0;
  return (b & 0x8000u) ? (uint32_t)(~b & 0xFFFFu) : (uint32_t)(b | 0x8000u);
}
__device__ __forceinline__ float key_val(uint32_t k) {
  const uint32_t b = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
  return __uint_as_float(b << 16);
}
__device__ __forceinline__ unsigned long long wfix(uint32_t key, float m) {
  const float d = __fadd_rn(key_val(key), -m);
  const float t = __fmul_rn(d, __uint_as_float(0x3fb8aa3bu));  // log2(e)
  if (!(t >= -45.0f)) return 0ull;
  const float r = rintf(t);
  const float f = __fadd_rn(t, -r);
  // Taylor coefficients ln(2)^k / k!, k = 7 .. 0, rounded to fp32
  float p = __uint_as_float(0x377fe5feu);
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x39218489u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3aaec3ffu));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3c1d955bu));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3d635847u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3e75fdf0u));
  p = __fadd_rn(__fmul_rn(p, f), __uint_as_float(0x3f317218u));
  p = __fadd_rn(__fmul_rn(p, f), 1.0f);
  const float sc = __int_as_float(((int)r + 40 + 127) << 23);  // 2^(r + 40), r in [-45, 0]
  return __float2ull_rz(__fmul_rn(p, sc));
}
__device__ __forceinline__ float prob_of(unsigned long long w, double inv_s) {
  return __double2float_rn(__dmul_rn((double)w, inv_s));
}
__device__ __forceinline__ unsigned long long fix_diff(float d) {
  return d > 0.0f ? __float2ull_rz(__fmul_rn(d, 1099511627776.0f)) : 0ull;  // 2^40
}

// ------------------------------------------------------------------------------------------
struct Smem {
  uint32_t sub_cnt[kSub][kBins];
  unsigned long long sub_mass[kSub][kBins];
  uint32_t hcnt[2][kBins];
  unsigned long long hmass[2][kBins];
  uint32_t fcnt[kBins];
  unsigned long long fmass[kBins];
  unsigned long long mbox[kMbox];
  unsigned long long gv[kCluster];
  unsigned long long red[kWarps];
  unsigned long long wsum[kWarps];
  // candidate list (filled in rank 0 by every CTA of the cluster)
  uint32_t c_key[kCand];
  uint32_t c_idx[kCand];
  unsigned long long c_w[kCand];
  uint32_t s_key[kCand];           // list sorted by (key desc, index asc)
  unsigned long long s_w[kCand];
  uint32_t o_idx[kCand];           // list sorted by index
  uint32_t o_key[kCand];
  unsigned long long o_w[kCand];   // kept weight in index order (0 when cut)
  unsigned long long px_w;         // kept weight of the draft token (0 when cut)
  int list_fill;
  int sel_bin;
  unsigned long long sel_above;
  int found;
  uint32_t bc_thr;                 // rank 0 -> cluster: final threshold key
  unsigned long long bc_S;         // rank 0 -> cluster: kept weight
};

struct Args {
  const __nv_bfloat16* logits;
  long long ld;
  int rows;                 // rows per group (grid.y)
  int V;
  float tb;                 // bf16(T) or bf16(1/T)
  int tmode;                // 0 divide, 1 multiply, 2 identity
  double top_p;
  int top_k;
  const unsigned long long* rng;  // [groups][2] {seed, offset}
  int stream_id;
  int row_base;
  // sample mode
  float* probs;
  long long ld_probs;
  int* tokens;
  int tok_stride;
  int* tokens2;
  int tok2_stride;
  // accept mode
  const int* verify_ids;    // [groups][rows]
  const float* q;           // [groups][rows - 1][ld_q]
  long long ld_q;
  int q_onehot;
  int* kv_len;
  int commit;
  int* pending;
  int* plan;                // [groups][rows + 2]
  unsigned long long* rng_rw;
  int* flags;               // [groups][rows]
  int* cands;               // [groups][rows]
  int* counters;            // [groups]
};

template <class T>
__device__ __forceinline__ T warp_red_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ unsigned long long block_sum(unsigned long long v, Smem& s) {
  v = warp_red_sum(v);
  if ((threadIdx.x & 31) == 0) s.red[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) r += s.red[i];
  __syncthreads();
  return r;
}
__device__ __forceinline__ uint32_t block_max(uint32_t v, Smem& s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
  if ((threadIdx.x & 31) == 0) s.red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) r = max(r, (uint32_t)s.red[i]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ uint32_t block_min(uint32_t v, Smem& s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(kFull, v, o));
  if ((threadIdx.x & 31) == 0) s.red[threadIdx.x >> 5] = v;
  __syncthreads();
  uint32_t r = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) r = min(r, (uint32_t)s.red[i]);
  __syncthreads();
  return r;
}
// exclusive prefix of v over the block (thread order); *total receives the block sum
__device__ __forceinline__ unsigned long long block_excl_scan(unsigned long long v, Smem& s,
                                                              unsigned long long* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s.wsum[warp] = incl;
  __syncthreads();
  unsigned long long before = 0, tot = 0;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) {
    if (i < warp) before += s.wsum[i];
    tot += s.wsum[i];
  }
  __syncthreads();
  if (total) *total = tot;
  return before + incl - v;
}

// every CTA publishes v; returns the values of all ranks in s.gv (block-visible)
__device__ __forceinline__ void cluster_gather(cg::cluster_group& cl, Smem& s, int slot,
                                               unsigned long long v) {
  if (threadIdx.x == 0) s.mbox[slot] = v;
  cl.sync();
  if (threadIdx.x < kCluster) s.gv[threadIdx.x] = *cl.map_shared_rank(&s.mbox[slot], threadIdx.x);
  __syncthreads();
}

// adds one element per lane (valid lanes only) to sub-histogram `sub`; lanes of the warp that
// share a bin are combined first. Every lane of the warp must call it.
__device__ __forceinline__ void hist_add(Smem& s, int sub, bool valid, uint32_t bin,
                                         unsigned long long w, bool with_mass) {
  const int lane = threadIdx.x & 31;
  const uint32_t tag = valid ? bin : (0x100u + lane);
  const unsigned grp = __match_any_sync(kFull, tag);
  unsigned long long m = w;
  if (with_mass && !__all_sync(kFull, __popc(grp) == 1)) {
    m = 0;
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const unsigned long long o = __shfl_sync(kFull, w, j);
      if ((grp >> j) & 1u) m += o;
    }
  }
  if (valid && lane == __ffs(grp) - 1) {
    atomicAdd(&s.sub_cnt[sub][bin], (uint32_t)__popc(grp));
    if (with_mass && m) atomicAdd(&s.sub_mass[sub][bin], m);
  }
}

// sub-histograms -> this CTA's histogram (buffer buf) -> cluster-wide histogram in fcnt/fmass
__device__ __forceinline__ void hist_reduce(cg::cluster_group& cl, Smem& s, int buf) {
  __syncthreads();
  for (int b = threadIdx.x; b < kBins; b += kThreads) {
    uint32_t c = 0;
    unsigned long long m = 0;
#pragma unroll
    for (int j = 0; j < kSub; ++j) {
      c += s.sub_cnt[j][b];
      m += s.sub_mass[j][b];
    }
    s.hcnt[buf][b] = c;
    s.hmass[buf][b] = m;
  }
  cl.sync();
  for (int b = threadIdx.x; b < kBins; b += kThreads) {
    uint32_t c = 0;
    unsigned long long m = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      c += *cl.map_shared_rank(&s.hcnt[buf][b], r);
      m += *cl.map_shared_rank(&s.hmass[buf][b], r);
    }
    s.fcnt[b] = c;
    s.fmass[b] = m;
  }
  for (int i = threadIdx.x; i < kSub * kBins; i += kThreads) {
    (&s.sub_cnt[0][0])[i] = 0;
    (&s.sub_mass[0][0])[i] = 0;
  }
  __syncthreads();
}

// Scanning bins from 255 down with `above` elements already counted, the first bin at which
// the running count reaches k. Sets s.sel_bin and s.sel_above (count above that bin).
__device__ __forceinline__ void select_count(Smem& s, unsigned long long above, unsigned long long k) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    uint32_t c[8];
    unsigned long long tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = s.fcnt[255 - 8 * lane - j];
      tot += c[j];
    }
    unsigned long long incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += t;
    }
    const unsigned hit = __ballot_sync(kFull, above + incl >= k);
    const int L = hit ? __ffs(hit) - 1 : 31;
    if (lane == L) {
      unsigned long long cum = above + incl - tot;
      int bin = 255 - 8 * lane - 7;
      unsigned long long ab = cum;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (cum + c[j] >= k) {
          bin = 255 - 8 * lane - j;
          ab = cum;
          break;
        }
        cum += c[j];
        ab = cum;
      }
      s.sel_bin = bin;
      s.sel_above = ab;
    }
  }
  __syncthreads();
}

// Scanning bins from 255 down, A_b = above + weight of the bins above b; returns the lowest
// non-empty bin with A_b < thr (s.sel_bin, s.sel_above = A_b), or s.sel_bin = -1 if none.
__device__ __forceinline__ void select_mass(Smem& s, unsigned long long above, double thr) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    unsigned long long m[8];
    uint32_t c[8];
    unsigned long long tot = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = s.fcnt[255 - 8 * lane - j];
      m[j] = s.fmass[255 - 8 * lane - j];
      tot += m[j];
    }
    unsigned long long incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long t = __shfl_up_sync(kFull, incl, o);
      if (lane >= o) incl += t;
    }
    unsigned long long A = above + incl - tot;
    int mine = -1;
    unsigned long long mineA = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (c[j] > 0 && (double)A < thr) {
        mine = 255 - 8 * lane - j;
        mineA = A;
      }
      A += m[j];
    }
    const unsigned has = __ballot_sync(kFull, mine >= 0);
    if (has == 0) {
      if (lane == 0) s.sel_bin = -1;
    } else {
      const int L = 31 - __clz(has);
      if (lane == L) {
        s.sel_bin = mine;
        s.sel_above = mineA;
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ unsigned long long mulhi64(unsigned long long r, unsigned long long S) {
  return __umul64hi(r, S);
}

// Inverse-CDF draw over this CTA's chunk: thread ranges [tid*E, (tid+1)*E) hold `mine` weight;
// `t` is the target within this CTA. Returns the chunk-local index via s.found.
template <class WF>
__device__ __forceinline__ void chunk_draw(Smem& s, int n, unsigned long long mine, unsigned long long t,
                                           WF weight_at) {
  const int E = (n + kThreads - 1) / kThreads;
  const unsigned long long ex = block_excl_scan(mine, s, nullptr);
  if (threadIdx.x == 0) s.found = -1;
  __syncthreads();
  if (mine > 0 && ex <= t && t < ex + mine) {
    unsigned long long cum = ex;
    const int r0 = threadIdx.x * E, r1 = min(n, r0 + E);
    for (int i = r0; i < r1; ++i) {
      cum += weight_at(i);
      if (cum > t) {
        s.found = i;
        break;
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------
template <bool ACCEPT>
__global__ void __launch_bounds__(kThreads, 1) row_kernel(const Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  uint16_t* keys = reinterpret_cast<uint16_t*>(smem_raw + ((sizeof(Smem) + 15) & ~size_t(15)));
  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int y = blockIdx.y, g = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = g * a.rows + y;
  const int V = a.V;
  const int chunk = ((V + kCluster - 1) / kCluster + 7) & ~7;
  const int v0 = min(V, rank * chunk), v1 = min(V, v0 + chunk);
  const int n = v1 - v0;
  int slot = 0;

  pdl_enter();

  for (int i = tid; i < kSub * kBins; i += kThreads) {
    (&s.sub_cnt[0][0])[i] = 0;
    (&s.sub_mass[0][0])[i] = 0;
  }
  if (tid == 0) s.list_fill = 0;

  const unsigned long long seed = a.rng[2 * g], offset = a.rng[2 * g + 1];
  const U4 rnd = philox(U4{(uint32_t)offset, (uint32_t)(offset >> 32), (uint32_t)(a.row_base + y),
                           (uint32_t)a.stream_id},
                        (uint32_t)seed, (uint32_t)(seed >> 32));
  const unsigned long long r64 = ((unsigned long long)rnd.z << 32) | rnd.w;

  // 1. keys and the row maximum
  const __nv_bfloat16* lrow = a.logits + (size_t)row * a.ld + v0;
  const bool vec = ((a.ld & 7) == 0) && ((reinterpret_cast<uintptr_t>(a.logits) & 15) == 0);
  uint32_t kmax = 0;
  for (int i = tid * 8; i < n; i += kThreads * 8) {
    if (vec && i + 8 <= n) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(lrow + i));
      const uint16_t* e = reinterpret_cast<const uint16_t*>(&u);
      uint16_t kk[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        kk[j] = (uint16_t)key_of(e[j], a.tb, a.tmode);
        kmax = max(kmax, (uint32_t)kk[j]);
      }
      *reinterpret_cast<uint4*>(keys + i) = *reinterpret_cast<const uint4*>(kk);
    } else {
      for (int j = i; j < min(i + 8, n); ++j) {
        const uint32_t k = key_of(__bfloat16_as_ushort(lrow[j]), a.tb, a.tmode);
        keys[j] = (uint16_t)k;
        kmax = max(kmax, k);
      }
    }
  }
  kmax = block_max(kmax, s);
  cluster_gather(cl, s, slot++, kmax);
  uint32_t maxkey = 0;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) maxkey = max(maxkey, (uint32_t)s.gv[r]);
  const float m = key_val(maxkey);

  // 2. total weight Z, and the high-byte counts for top-k
  const bool topk = a.top_k > 0 && a.top_k < V;
  const bool topp = a.top_p < 1.0;
  unsigned long long z = 0;
  for (int i = tid; i - lane < n; i += kThreads) {
    const bool valid = i < n;
    const uint32_t k = valid ? keys[i] : 0u;
    if (valid) z += wfix(k, m);
    if (topk) hist_add(s, warp & (kSub - 1), valid, k >> 8, 0, false);
  }
  z = block_sum(z, s);
  cluster_gather(cl, s, slot++, z);
  unsigned long long Z = 0;
#pragma unroll
  for (int r = 0; r < kCluster; ++r) Z += s.gv[r];

  // 3. top-k threshold: two 8-bit count passes
  uint32_t tk = 0;
  unsigned long long n_ge = (unsigned long long)V;
  if (topk) {
    hist_reduce(cl, s, 0);
    select_count(s, 0, (unsigned long long)a.top_k);
    const uint32_t hb = (uint32_t)s.sel_bin;
    const unsigned long long above = s.sel_above;
    for (int i = tid; i - lane < n; i += kThreads) {
      const bool valid = i < n && ((uint32_t)keys[i] >> 8) == hb;
      hist_add(s, warp & (kSub - 1), valid, valid ? (keys[i] & 255u) : 0u, 0, false);
    }
    hist_reduce(cl, s, 1);
    select_count(s, above, (unsigned long long)a.top_k);
    const uint32_t lb = (uint32_t)s.sel_bin;
    tk = (hb << 8) | lb;
    n_ge = s.sel_above + s.fcnt[lb];
  }
  const double thr = a.top_p * (double)Z;
  const bool small = n_ge <= (unsigned long long)kCand;

  uint32_t thrkey = tk;
  unsigned long long S = 0;
  int cand_local = -1;  // chunk-local index of this row's draw, if it fell in this CTA
  // accept-mode row facts
  const int L = a.rows - 1;
  const bool is_draft_row = ACCEPT && y < L;
  const int x = is_draft_row ? a.verify_ids[(size_t)g * a.rows + y + 1] : -1;
  const float* qrow = (ACCEPT && is_draft_row && !a.q_onehot) ? a.q + ((size_t)g * L + y) * a.ld_q : nullptr;
  const float u = (float)(rnd.x >> 8) * (1.0f / 16777216.0f);

  if (small) {
    // ---- short list: every kept candidate goes to rank 0 ----
    unsigned long long mycnt = 0;
    for (int i = tid; i < n; i += kThreads) mycnt += keys[i] >= tk;
    mycnt = block_sum(mycnt, s);
    cluster_gather(cl, s, slot++, mycnt);
    unsigned long long off = 0;
    for (int r = 0; r < rank; ++r) off += s.gv[r];
    uint32_t* rk = cl.map_shared_rank(s.c_key, 0);
    uint32_t* ri = cl.map_shared_rank(s.c_idx, 0);
    unsigned long long* rw = cl.map_shared_rank(s.c_w, 0);
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t k = keys[i];
      if (k >= tk) {
        const int sl = (int)off + atomicAdd(&s.list_fill, 1);
        if (sl < kCand) {  // the counts above make sl < n_ge <= kCand; kept as a bound
          rk[sl] = k;
          ri[sl] = (uint32_t)(v0 + i);
          rw[sl] = wfix(k, m);
        }
      }
    }
    cl.sync();
    if (rank == 0) {
      const int nl = (int)n_ge;
      // ranks: (key desc, index asc) and index asc; all list entries are distinct indices
      if (tid < nl) {
        const uint32_t kj = s.c_key[tid], ij = s.c_idx[tid];
        int r_key = 0, r_idx = 0;
        for (int i = 0; i < nl; ++i) {
          const uint32_t ki = s.c_key[i], ii = s.c_idx[i];
          r_key += (ki > kj) || (ki == kj && ii < ij);
          r_idx += ii < ij;
        }
        s.s_key[r_key] = kj;
        s.s_w[r_key] = s.c_w[tid];
        s.o_idx[r_idx] = ij;
        s.o_key[r_idx] = kj;
        s.o_w[r_idx] = s.c_w[tid];
      }
      __syncthreads();
      uint32_t tp = 0;
      if (topp) {
        const unsigned long long wj = tid < nl ? s.s_w[tid] : 0ull;
        const unsigned long long E = block_excl_scan(wj, s, nullptr);
        uint32_t cand = 0xffffffffu;
        if (tid < nl && (tid == 0 || s.s_key[tid - 1] != s.s_key[tid]) && (double)E < thr)
          cand = s.s_key[tid];
        tp = block_min(cand, s);
        if (tp == 0xffffffffu) tp = 0;
      }
      const uint32_t th = max(tk, tp);
      // kept weights in index order
      const unsigned long long wk = (tid < nl && s.o_key[tid] >= th) ? s.o_w[tid] : 0ull;
      unsigned long long Stot = 0;
      const unsigned long long ex = block_excl_scan(wk, s, &Stot);
      S = Stot;
      const double inv_s = S ? 1.0 / (double)S : 0.0;
      if (tid == 0) {
        s.bc_thr = th;
        s.bc_S = S;
        s.found = -1;
      }
      __syncthreads();
      if (!ACCEPT || !is_draft_row) {
        // draw from p: sample rows and the all-accepted bonus row
        if (S == 0) {
          if (tid == 0) s.found = (int)mulhi64(r64, (unsigned long long)V);
        } else {
          const unsigned long long t = mulhi64(r64, S);
          if (tid < nl && wk > 0 && ex <= t && t < ex + wk) s.found = (int)s.o_idx[tid];
        }
        __syncthreads();
        const int tok = s.found;
        if (tid == 0) {
          if (ACCEPT) {
            a.cands[(size_t)g * a.rows + y] = tok;
            a.flags[(size_t)g * a.rows + y] = 0;
            __threadfence();
          } else {
            a.tokens[(size_t)row * a.tok_stride] = tok;
            if (a.tokens2) a.tokens2[(size_t)row * a.tok2_stride] = tok;
          }
        }
      } else {
        // accept test for draft token x, then the residual draw over the list
        if (tid == 0) s.px_w = 0;
        __syncthreads();
        if (tid < nl && (int)s.o_idx[tid] == x) s.px_w = wk;  // list indices are distinct
        __syncthreads();
        const float pd = prob_of(s.px_w, inv_s);
        unsigned long long rwj = 0;
        if (tid < nl && wk > 0) {
          const int idx = (int)s.o_idx[tid];
          const float qv = a.q_onehot ? (idx == x ? 1.0f : 0.0f) : qrow[idx];
          rwj = fix_diff(__fadd_rn(prob_of(wk, inv_s), -qv));
        }
        unsigned long long Sr = 0;
        const unsigned long long exr = block_excl_scan(rwj, s, &Sr);
        if (Sr == 0) {
          if (tid == 0) s.found = (int)mulhi64(r64, (unsigned long long)V);
        } else {
          const unsigned long long t = mulhi64(r64, Sr);
          if (rwj > 0 && exr <= t && t < exr + rwj) s.found = (int)s.o_idx[tid];
        }
        __syncthreads();
        if (tid == 0) {
          const float qd = a.q_onehot ? 1.0f : (x >= 0 && x < V ? qrow[x] : 0.0f);
          const float ratio = __fdiv_rn(pd, fmaxf(qd, 1e-9f));
          a.flags[(size_t)g * a.rows + y] = u < fminf(1.0f, ratio) ? 1 : 0;
          a.cands[(size_t)g * a.rows + y] = s.found;
          __threadfence();
        }
      }
    }
    cl.sync();
    thrkey = *cl.map_shared_rank(&s.bc_thr, 0);
    S = *cl.map_shared_rank(&s.bc_S, 0);
  } else {
    // ---- long path: nucleus by two 8-bit weight passes, draws by a cluster-wide scan ----
    if (topp) {
      for (int i = tid; i - lane < n; i += kThreads) {
        const bool valid = i < n;
        const uint32_t k = valid ? keys[i] : 0u;
        const unsigned long long w = (valid && k >= tk) ? wfix(k, m) : 0ull;
        hist_add(s, warp & (kSub - 1), valid, k >> 8, w, true);
      }
      hist_reduce(cl, s, 0);
      select_mass(s, 0, thr);
      uint32_t tp = 0;
      if (s.sel_bin >= 0) {
        const uint32_t hb = (uint32_t)s.sel_bin;
        const unsigned long long above = s.sel_above;
        __syncthreads();
        for (int i = tid; i - lane < n; i += kThreads) {
          const bool valid = i < n && ((uint32_t)keys[i] >> 8) == hb;
          const uint32_t k = valid ? keys[i] : 0u;
          const unsigned long long w = (valid && k >= tk) ? wfix(k, m) : 0ull;
          hist_add(s, warp & (kSub - 1), valid, k & 255u, w, true);
        }
        hist_reduce(cl, s, 1);
        select_mass(s, above, thr);
        tp = (hb << 8) | (uint32_t)max(s.sel_bin, 0);
      } else {
        __syncthreads();
      }
      thrkey = max(tk, tp);
    }
    // kept weight per thread range (contiguous ranges, vocabulary order)
    const int E = (n + kThreads - 1) / kThreads;
    const int r0 = min(n, tid * E), r1 = min(n, r0 + E);
    unsigned long long mine = 0;
    for (int i = r0; i < r1; ++i) {
      const uint32_t k = keys[i];
      if (k >= thrkey) mine += wfix(k, m);
    }
    const unsigned long long Sc = block_sum(mine, s);
    cluster_gather(cl, s, slot++, Sc);
    unsigned long long pre = 0;
    S = 0;
#pragma unroll
    for (int r = 0; r < kCluster; ++r) {
      if (r < rank) pre += s.gv[r];
      S += s.gv[r];
    }
    const double inv_s = S ? 1.0 / (double)S : 0.0;
    const uint32_t th = thrkey;
    if (!ACCEPT || !is_draft_row) {
      if (S == 0) {
        if (rank == 0 && tid == 0) {
          const int tok = (int)mulhi64(r64, (unsigned long long)V);
          if (ACCEPT) {
            a.cands[(size_t)g * a.rows + y] = tok;
            a.flags[(size_t)g * a.rows + y] = 0;
            __threadfence();
          } else {
            a.tokens[(size_t)row * a.tok_stride] = tok;
            if (a.tokens2) a.tokens2[(size_t)row * a.tok2_stride] = tok;
          }
        }
      } else {
        const unsigned long long t = mulhi64(r64, S);
        if (t >= pre && t < pre + Sc) {  // block-uniform
          chunk_draw(s, n, mine, t - pre, [&](int i) {
            const uint32_t k = keys[i];
            return k >= th ? wfix(k, m) : 0ull;
          });
          cand_local = s.found;
          if (tid == 0) {
            const int tok = v0 + max(cand_local, 0);
            if (ACCEPT) {
              a.cands[(size_t)g * a.rows + y] = tok;
              a.flags[(size_t)g * a.rows + y] = 0;
              __threadfence();
            } else {
              a.tokens[(size_t)row * a.tok_stride] = tok;
              if (a.tokens2) a.tokens2[(size_t)row * a.tok2_stride] = tok;
            }
          }
        }
      }
    } else {
      // accept flag by the CTA owning x (rank 0 rejects a token outside the vocabulary)
      if ((x < 0 || x >= V) && rank == 0 && tid == 0) {
        a.flags[(size_t)g * a.rows + y] = 0;
        __threadfence();
      }
      if (x >= v0 && x < v1 && tid == 0) {
        const uint32_t kx = keys[x - v0];
        const float pd = kx >= th ? prob_of(wfix(kx, m), inv_s) : 0.0f;
        const float qd = a.q_onehot ? 1.0f : qrow[x];
        const float ratio = __fdiv_rn(pd, fmaxf(qd, 1e-9f));
        a.flags[(size_t)g * a.rows + y] = u < fminf(1.0f, ratio) ? 1 : 0;
        __threadfence();
      }
      // residual weight per thread range
      auto resid_at = [&](int i) -> unsigned long long {
        const uint32_t k = keys[i];
        const float pv = k >= th ? prob_of(wfix(k, m), inv_s) : 0.0f;
        const int idx = v0 + i;
        const float qv = a.q_onehot ? (idx == x ? 1.0f : 0.0f) : __ldg(qrow + idx);
        return fix_diff(__fadd_rn(pv, -qv));
      };
      unsigned long long rmine = 0;
      for (int i = r0; i < r1; ++i) rmine += resid_at(i);
      const unsigned long long Rc = block_sum(rmine, s);
      cluster_gather(cl, s, slot++, Rc);
      unsigned long long rpre = 0, Sr = 0;
#pragma unroll
      for (int r = 0; r < kCluster; ++r) {
        if (r < rank) rpre += s.gv[r];
        Sr += s.gv[r];
      }
      if (Sr == 0) {
        if (rank == 0 && tid == 0) {
          a.cands[(size_t)g * a.rows + y] = (int)mulhi64(r64, (unsigned long long)V);
          __threadfence();
        }
      } else {
        const unsigned long long t = mulhi64(r64, Sr);
        if (t >= rpre && t < rpre + Rc) {
          chunk_draw(s, n, rmine, t - rpre, resid_at);
          if (tid == 0) {
            a.cands[(size_t)g * a.rows + y] = v0 + max(s.found, 0);
            __threadfence();
          }
        }
      }
    }
  }

  // dense truncated distribution (sample mode)
  if (!ACCEPT && a.probs) {
    const double inv_s = S ? 1.0 / (double)S : 0.0;
    float* prow = a.probs + (size_t)row * a.ld_probs + v0;
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t k = keys[i];
      prow[i] = (S && k >= thrkey) ? prob_of(wfix(k, m), inv_s) : 0.0f;
    }
  }
  (void)cand_local;
  cl.sync();  // no CTA leaves while another may still read its shared memory

  if (ACCEPT && rank == 0 && tid == 0) {
    __threadfence();
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(old)
                 : "l"(a.counters + g)
                 : "memory");
    if (old == a.rows - 1) {
      const int T = a.rows;
      const int* fl = a.flags + (size_t)g * T;
      int nacc = 0;
      while (nacc < T - 1 && __ldcg(fl + nacc)) ++nacc;
      const int repl = __ldcg(a.cands + (size_t)g * T + nacc);
      int* pl = a.plan + (size_t)g * (T + 2);
      pl[0] = nacc;
      pl[1] = nacc + 1;
      for (int i = 0; i < nacc; ++i) pl[2 + i] = a.verify_ids[(size_t)g * T + 1 + i];
      pl[2 + nacc] = repl;
      for (int i = nacc + 1; i < T; ++i) pl[2 + i] = -1;
      a.pending[g] = repl;
      if (a.commit) a.kv_len[g] += nacc + 1;
      a.rng_rw[2 * g + 1] += 1ull;
      a.counters[g] = 0;
    }
  }
}

size_t smem_bytes(int V) {
  const int chunk = ((V + kCluster - 1) / kCluster + 7) & ~7;
  return ((sizeof(Smem) + 15) & ~size_t(15)) + (size_t)chunk * 2;
}

template <bool ACCEPT>
int launch(const char* what, const Args& a, int groups, cudaStream_t st) {
  auto kern = row_kernel<ACCEPT>;
  const size_t smem = smem_bytes(a.V);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCluster, a.rows, groups);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1] = pdl_attr();
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  note_launch();
  return DSPARK_OK;
}

float bf16_host(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return x;
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

int fill_temperature(Args& a, float temperature, int temp_mode, const char* what) {
  if (!(temperature > 0.0f) || !(temperature < 1e30f))
    return set_error(DSPARK_ERR_INVALID, "%s: temperature must be > 0", what);
  if (temp_mode != 0 && temp_mode != 1)
    return set_error(DSPARK_ERR_INVALID, "%s: temp_mode must be 0 (divide) or 1 (multiply)", what);
  a.tb = temp_mode == 0 ? bf16_host(temperature) : bf16_host((float)(1.0 / (double)temperature));
  a.tmode = a.tb == 1.0f ? 2 : temp_mode;
  return DSPARK_OK;
}

}  // namespace smp
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_sample_rows(const void* logits, long long ld, int groups, int rows, int V,
                                  float temperature, int temp_mode, double top_p, int top_k,
                                  const unsigned long long* rng, int stream_id, int row_base,
                                  float* probs, long long ld_probs, int32_t* tokens, int tok_stride,
                                  int32_t* tokens2, int tok2_stride, dspark_stream_t stream) {
  if (!logits || !rng || !tokens || groups <= 0 || rows <= 0 || V <= 0 || ld < V || tok_stride < 1 ||
      (tokens2 && tok2_stride < 1) || (probs && ld_probs < V))
    return set_error(DSPARK_ERR_INVALID, "sample_rows: bad arguments");
  if (V > smp::kMaxV) return set_error(DSPARK_ERR_UNSUPPORTED, "sample_rows: V %d > %d", V, smp::kMaxV);
  if (!(top_p > 0.0) || top_k < 0) return set_error(DSPARK_ERR_INVALID, "sample_rows: top_p must be > 0, top_k >= 0");
  if (groups > 65535 || rows > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "sample_rows: grid too large");
  smp::Args a = {};
  if (int rc = smp::fill_temperature(a, temperature, temp_mode, "sample_rows")) return rc;
  a.logits = static_cast<const __nv_bfloat16*>(logits);
  a.ld = ld;
  a.rows = rows;
  a.V = V;
  a.top_p = top_p;
  a.top_k = top_k;
  a.rng = rng;
  a.stream_id = stream_id;
  a.row_base = row_base;
  a.probs = probs;
  a.ld_probs = ld_probs;
  a.tokens = tokens;
  a.tok_stride = tok_stride;
  a.tokens2 = tokens2;
  a.tok2_stride = tok2_stride;
  return smp::launch<false>("sample_rows", a, groups, static_cast<cudaStream_t>(stream));
}

extern "C" size_t dspark_accept_sample_workspace_bytes(int B, int T) {
  if (B <= 0 || T <= 0) return 0;
  // counters first (fixed offset 0), then flags and candidates
  const size_t c = ((size_t)B * 4 + 255) & ~(size_t)255;
  const size_t f = ((size_t)B * T * 4 + 255) & ~(size_t)255;
  return c + 2 * f;
}

extern "C" int dspark_accept_sample(const void* logits, long long ld, int B, int T, int V,
                                    const int32_t* verify_ids, const float* q_probs, long long ld_q,
                                    int q_onehot, float temperature, int temp_mode, double top_p,
                                    int top_k, unsigned long long* rng, int32_t* kv_len, int commit,
                                    int32_t* pending, int32_t* plan, void* workspace,
                                    size_t workspace_bytes, dspark_stream_t stream) {
  if (!logits || !verify_ids || !rng || !pending || !plan || B <= 0 || T <= 0 || V <= 0 || ld < V)
    return set_error(DSPARK_ERR_INVALID, "accept_sample: bad arguments");
  if (T > 1 && !q_onehot && (!q_probs || ld_q < V))
    return set_error(DSPARK_ERR_INVALID, "accept_sample: q_probs required unless q_onehot");
  if (commit && !kv_len) return set_error(DSPARK_ERR_INVALID, "accept_sample: commit without kv_len");
  if (T > smp::kMaxT) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_sample: T %d > %d", T, smp::kMaxT);
  if (V > smp::kMaxV) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_sample: V %d > %d", V, smp::kMaxV);
  if (B > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_sample: B too large");
  if (!(top_p > 0.0) || top_k < 0) return set_error(DSPARK_ERR_INVALID, "accept_sample: top_p must be > 0, top_k >= 0");
  const size_t need = dspark_accept_sample_workspace_bytes(B, T);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "accept_sample: workspace %zu < %zu", workspace_bytes, need);
  smp::Args a = {};
  if (int rc = smp::fill_temperature(a, temperature, temp_mode, "accept_sample")) return rc;
  uint8_t* w = static_cast<uint8_t*>(workspace);
  const size_t c = ((size_t)B * 4 + 255) & ~(size_t)255;
  const size_t f = ((size_t)B * T * 4 + 255) & ~(size_t)255;
  a.logits = static_cast<const __nv_bfloat16*>(logits);
  a.ld = ld;
  a.rows = T;
  a.V = V;
  a.top_p = top_p;
  a.top_k = top_k;
  a.rng = rng;
  a.rng_rw = rng;
  a.stream_id = 0;
  a.row_base = 0;
  a.verify_ids = verify_ids;
  a.q = q_probs;
  a.ld_q = ld_q;
  a.q_onehot = q_onehot;
  a.kv_len = kv_len;
  a.commit = commit;
  a.pending = pending;
  a.plan = plan;
  a.counters = reinterpret_cast<int*>(w);
  a.flags = reinterpret_cast<int*>(w + c);
  a.cands = reinterpret_cast<int*>(w + c + f);
  return smp::launch<true>("accept_sample", a, B, static_cast<cudaStream_t>(stream));
}
