// Per-token logprobs of committed tokens: the raw target log-softmax of a verify row, the
// chosen token's entry and the row's top entries.
//
// Reference semantics (src/mlx_dspark/generate.py:149-176, _logprobs_for_block):
//   x = float32(row);  m = max(x);  logp = x - m - log(sum(exp(x - m)))
//   chosen = logp[token];  top = the top_k (id, logp) pairs in descending logp order
// The committed token of row r is ids[(r / T) * ids_ld + r % T], so a speculative round's
// plan rows (n, n + 1, committed...) serve as the id source without a copy.
//
// One CTA per row. The row (V bf16 values, 300 KB at V = 151936) stays in L2 across the
// passes:
//   1. max, and a histogram of the high byte of each value's order key (per-warp copies);
//   2. sum of exp(x - m), and a histogram of the low byte among the values whose high byte is
//      that of the k-th largest key: this gives the k-th largest key exactly and how many keys
//      lie above it;
//   3. the keys above it and the first (lowest-index) ties at it are gathered, k in all;
//      ties are taken in index order by giving each thread a contiguous slice of the row and
//      an exclusive scan of the per-thread tie counts;
//   4. each candidate's rank is counted against the others (larger value first, equal values
//      by smaller index, the order of a stable descending sort).
#include "common.cuh"

namespace dspark {
namespace lp {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTop = 1024;

// Order key of a bf16 bit pattern: a larger value has a larger key; -0 is keyed as +0.
__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
  bits &= 0xFFFFu;
  if (bits == 0x8000u) bits = 0;
  return (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);
}

__device__ __forceinline__ float bits_to_float(uint32_t bits) { return __uint_as_float(bits << 16); }

// Calls f(index, bf16 bits) for this thread's share of a row: 8 consecutive values per step,
// strided by the block (16-byte loads where the row start allows them).
template <typename F>
__device__ __forceinline__ void for_row(const uint16_t* row, int V, bool vec, F&& f) {
  for (int v = threadIdx.x * 8; v < V; v += kThreads * 8) {
    if (vec && v + 8 <= V) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + v));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) f(v + j, (w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu);
    } else {
      for (int j = v; j < min(v + 8, V); ++j) f(j, (uint32_t)row[j]);
    }
  }
}

// Calls f(index, bf16 bits) for the contiguous slice [lo, hi) of a row (lo a multiple of 8).
template <typename F>
__device__ __forceinline__ void for_slice(const uint16_t* row, int lo, int hi, bool vec, F&& f) {
  for (int v = lo; v < hi; v += 8) {
    if (vec && v + 8 <= hi) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + v));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) f(v + j, (w[j >> 1] >> (16 * (j & 1))) & 0xFFFFu);
    } else {
      for (int j = v; j < min(v + 8, hi); ++j) f(j, (uint32_t)row[j]);
    }
  }
}

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();  // red[] may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < kWarps ? red[lane] : (is_max ? -INFINITY : 0.0f);
    t = is_max ? warp_max(t) : warp_sum(t);
    if (lane == 0) red[kWarps] = t;
  }
  __syncthreads();
  return red[kWarps];
}

struct Smem {
  uint32_t hist[kWarps][256];
  uint32_t hist2[256];
  float red[kWarps + 1];
  int scan[kWarps];
  uint32_t kth_key;
  int above;       // keys strictly above kth_key
  int ncand;
  int cand_idx[kMaxTop];
  uint16_t cand_bits[kMaxTop];
};

__global__ void __launch_bounds__(kThreads) logprobs_kernel(
    const __nv_bfloat16* __restrict__ logits, long long ld, int V, const int32_t* __restrict__ ids,
    int ids_ld, int T, int top_k, float* __restrict__ logp, int32_t* __restrict__ top_ids,
    float* __restrict__ top_logp) {
  pdl_enter();
  __shared__ Smem s;  // 23.6 KB
  const int r = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint16_t* row = reinterpret_cast<const uint16_t*>(logits) + (size_t)r * ld;
  const bool vec = ((ld & 7) == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  const int k = min(top_k, V);

  if (k > 0) {
    for (int i = tid; i < kWarps * 256; i += kThreads) (&s.hist[0][0])[i] = 0;
    for (int i = tid; i < 256; i += kThreads) s.hist2[i] = 0;
    if (tid == 0) s.ncand = 0;
  }
  __syncthreads();

  // 1. max and the high-byte histogram
  float mx = -INFINITY;
  for_row(row, V, vec, [&](int, uint32_t b) {
    mx = fmaxf(mx, bits_to_float(b));
    if (k > 0) atomicAdd(&s.hist[warp][order_key(b) >> 8], 1u);
  });
  const float m = block_reduce(mx, s.red, true);
  if (k > 0) {
    // fold the per-warp copies into copy 0, then find the high byte of the k-th largest key
    for (int i = tid; i < 256; i += kThreads) {
      uint32_t t = 0;
      for (int w = 0; w < kWarps; ++w) t += s.hist[w][i];
      s.hist[0][i] = t;
    }
    __syncthreads();
    if (tid == 0) {
      int cum = 0, hb = 0;
      for (int b = 255; b >= 0; --b) {
        if (cum + (int)s.hist[0][b] >= k) { hb = b; break; }
        cum += (int)s.hist[0][b];
      }
      s.kth_key = (uint32_t)hb << 8;
      s.above = cum;
    }
    __syncthreads();
  }

  // 2. sum of exp(x - m), and the low-byte histogram inside the k-th key's high byte
  const uint32_t hb = s.kth_key >> 8;
  float sum = 0.0f;
  for_row(row, V, vec, [&](int, uint32_t b) {
    sum += expf(bits_to_float(b) - m);
    if (k > 0) {
      const uint32_t key = order_key(b);
      if ((key >> 8) == hb) atomicAdd(&s.hist2[key & 0xFFu], 1u);
    }
  });
  const float ls = logf(block_reduce(sum, s.red, false));

  if (tid == 0 && logp) {
    const int tok = ids[(size_t)(r / T) * ids_ld + r % T];
    logp[r] = (tok >= 0 && tok < V) ? (bits_to_float(row[tok]) - m) - ls : __int_as_float(0x7fc00000);
  }
  if (k == 0) return;

  if (tid == 0) {
    int cum = s.above, lb = 0;
    for (int b = 255; b >= 0; --b) {
      if (cum + (int)s.hist2[b] >= k) { lb = b; break; }
      cum += (int)s.hist2[b];
    }
    s.kth_key |= (uint32_t)lb;
    s.above = cum;
  }
  __syncthreads();
  const uint32_t kth = s.kth_key;
  const int need = k - s.above;  // ties at kth to take, lowest indices first (>= 1)

  // 3. gather: thread t owns the contiguous slice [lo, hi)
  const int chunk = ((V + kThreads - 1) / kThreads + 7) & ~7;
  const int lo = min(V, tid * chunk), hi = min(V, lo + chunk);
  int ties = 0;
  for_slice(row, lo, hi, vec, [&](int, uint32_t b) { ties += order_key(b) == kth; });
  // exclusive scan of the tie counts in thread order
  int incl = ties;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s.scan[warp] = incl;
  __syncthreads();
  int base = incl - ties;
  for (int w = 0; w < warp; ++w) base += s.scan[w];
  int rank_tie = base;
  for_slice(row, lo, hi, vec, [&](int i, uint32_t b) {
    const uint32_t key = order_key(b);
    bool take = key > kth;
    if (key == kth) take = rank_tie++ < need;
    if (take) {
      const int slot = atomicAdd(&s.ncand, 1);
      if (slot < kMaxTop) {
        s.cand_idx[slot] = i;
        s.cand_bits[slot] = (uint16_t)b;
      }
    }
  });
  __syncthreads();

  // 4. rank of each candidate: larger value first, equal values by smaller index
  const int n = min(s.ncand, k);
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t ki = order_key(s.cand_bits[i]);
    const int ii = s.cand_idx[i];
    int rank = 0;
    for (int j = 0; j < n; ++j) {
      const uint32_t kj = order_key(s.cand_bits[j]);
      rank += (kj > ki) || (kj == ki && s.cand_idx[j] < ii);
    }
    if (rank < top_k) {
      top_ids[(size_t)r * top_k + rank] = ii;
      top_logp[(size_t)r * top_k + rank] = (bits_to_float(s.cand_bits[i]) - m) - ls;
    }
  }
}

}  // namespace lp
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_logprobs(const void* logits, long long ld, int rows, int V, const int32_t* ids,
                               int ids_ld, int T, int top_k, float* logp, int32_t* top_ids,
                               float* top_logp, dspark_stream_t stream) {
  if (!logits || !ids || !logp || rows <= 0 || V <= 0 || ld < V || T < 1 || ids_ld < T ||
      top_k < 0 || (top_k > 0 && (!top_ids || !top_logp)))
    return set_error(DSPARK_ERR_INVALID, "logprobs: bad arguments");
  if (rows > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "logprobs: too many rows");
  if (top_k > lp::kMaxTop)
    return set_error(DSPARK_ERR_UNSUPPORTED, "logprobs: top_k %d > %d", top_k, lp::kMaxTop);
  return launch_pdl("logprobs", lp::logprobs_kernel, dim3(rows), dim3(lp::kThreads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(logits),
                    ld, V, ids, ids_ld, T, top_k, logp, top_ids, top_logp);
}
