// K8 — greedy acceptance fused with the row argmax, and the length-only KV commit.
//
// Reference semantics (src/mlx_dspark/generate.py:910-933, batch_engine.py:573-595):
//   tt = argmax(v_logits)  (mx.argmax: first index of the maximum)
//   n  = sum(cumprod(draft == tt[:cap]))
//   committed = draft[:n] + [tt[n]];  cache.trim(len(draft) - n)
// The verify block already wrote K/V for all T positions; keeping n + 1 of them is a length
// update (kv_len += n + 1), so commit and rollback are O(1) on the device.
#include <mutex>

#include "common.cuh"

namespace dspark {
namespace acc {

constexpr int kThreads = 256;

struct Best {
  float v;
  int i;
};
__device__ __forceinline__ Best better(Best a, Best b) {
  // larger value wins; equal values: smaller index (first occurrence)
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ __forceinline__ Best warp_best(Best x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Best y;
    y.v = __shfl_xor_sync(0xffffffffu, x.v, o);
    y.i = __shfl_xor_sync(0xffffffffu, x.i, o);
    x = better(x, y);
  }
  return x;
}

// Each CTA scans a contiguous vocabulary slice of every row; the last CTA to finish
// reduces the per-CTA partials (in CTA order) and runs the acceptance.
__global__ void __launch_bounds__(kThreads) accept_greedy_kernel(
    const __nv_bfloat16* __restrict__ logits, int ld, int B, int T, int V,
    const int32_t* __restrict__ verify_ids, int32_t* __restrict__ argmax_out,
    int32_t* __restrict__ kv_len, int commit, int32_t* __restrict__ pending,
    int32_t* __restrict__ plan, float* __restrict__ part_v, int* __restrict__ part_i,
    int* __restrict__ counter) {
  pdl_enter();
  const int rows = B * T;
  const int chunk = ((V + gridDim.x - 1) / gridDim.x + 7) & ~7;
  const int v0 = blockIdx.x * chunk;
  const int v1 = min(V, v0 + chunk);
  __shared__ int is_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kWarps = kThreads / 32;
  // 16-byte loads only where every row start is 16-byte aligned (a row-major view of any
  // offset or stride still takes the scalar path)
  const bool vec = ((ld & 7) == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  // one warp per row (rows strided over the warps), no block barrier in the scan: every
  // lane's loads of a row are independent, so a row costs about one memory round trip
  for (int r = warp; r < rows; r += kWarps) {
    const __nv_bfloat16* row = logits + (size_t)r * ld;
    Best b{-INFINITY, 0x7fffffff};
    for (int v = v0 + lane * 8; v < v1; v += 32 * 8) {
      if (v + 8 <= v1 && vec) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + v));
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) b = better(b, Best{__bfloat162float(e[j]), v + j});
      } else {
        for (int j = v; j < min(v + 8, v1); ++j) b = better(b, Best{__bfloat162float(row[j]), j});
      }
    }
    b = warp_best(b);
    if (lane == 0) {
      part_v[(size_t)blockIdx.x * rows + r] = b.v;
      part_i[(size_t)blockIdx.x * rows + r] = b.i;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = (atomicAdd(counter, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  __shared__ int tt[64];
  // final reduction: a warp per row, lanes over the CTAs' partials (all loads in flight)
  for (int r = warp; r < rows; r += kWarps) {
    Best t{-INFINITY, 0x7fffffff};
    for (int c = lane; c < (int)gridDim.x; c += 32)
      t = better(t, Best{__ldcg(part_v + (size_t)c * rows + r), __ldcg(part_i + (size_t)c * rows + r)});
    t = warp_best(t);
    if (lane == 0) {
      if (t.i == 0x7fffffff) t.i = 0;  // all-NaN row
      tt[r] = t.i;
      argmax_out[r] = t.i;
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += kThreads) {
    int n = 0;
    while (n < T - 1 && verify_ids[b * T + n + 1] == tt[b * T + n]) ++n;
    int32_t* pl = plan + (size_t)b * (T + 2);
    pl[0] = n;
    pl[1] = n + 1;
    for (int i = 0; i < n; ++i) pl[2 + i] = verify_ids[b * T + i + 1];
    pl[2 + n] = tt[b * T + n];
    for (int i = n + 1; i < T; ++i) pl[2 + i] = -1;
    pending[b] = tt[b * T + n];
    if (commit) kv_len[b] += n + 1;
  }
  if (threadIdx.x == 0) *counter = 0;
}

// kv_len[b] += plan[b * stride + 1] for every length array given
__global__ void commit_lengths_kernel(const int32_t* __restrict__ plan, int stride, int B,
                                      int32_t* __restrict__ a, int32_t* __restrict__ b2) {
  pdl_enter();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int add = plan[(size_t)b * stride + 1];
    if (a) a[b] += add;
    if (b2) b2[b] += add;
  }
}

// Benchmark draft override (greedy configs with a Bernoulli agree mask): draft position i of
// row b proposes ref[b][j] when agree[b][round][i] is set, else (ref[b][j] + 1) mod V, where
// j = kv_len[b] - prompt_len[b] + 1 + i indexes the row's reference greedy continuation.
__global__ void draft_override_kernel(int B, int cap, int V, const int32_t* __restrict__ ref,
                                      int ref_len, const uint8_t* __restrict__ agree,
                                      int rounds, const int32_t* __restrict__ round_ctr,
                                      const int32_t* __restrict__ kv_len,
                                      const int32_t* __restrict__ prompt_len,
                                      int32_t* __restrict__ verify_ids) {
  pdl_enter();
  const int b = blockIdx.x;
  const int rnd = min(round_ctr[b], rounds - 1);
  for (int i = threadIdx.x; i < cap; i += blockDim.x) {
    int j = kv_len[b] - prompt_len[b] + 1 + i;
    j = j < 0 ? 0 : (j >= ref_len ? ref_len - 1 : j);
    const int g = ref[(size_t)b * ref_len + j];
    const bool ok = agree[((size_t)b * rounds + rnd) * cap + i] != 0;
    verify_ids[(size_t)b * (cap + 1) + 1 + i] = ok ? g : (g + 1) % V;
  }
}

// Row argmax (first index of the maximum), one CTA per row: the greedy block draft of a
// drafter without a sequential head (DFlash, generate.py:564; sample_block without a Markov
// head, model.py:272-273). Token of row r -> tokens[r * s1] (and tokens2[r * s2]).
constexpr int kArgThreads = 1024;
__global__ void __launch_bounds__(kArgThreads) argmax_rows_kernel(
    const __nv_bfloat16* __restrict__ logits, long long ld, int V, int32_t* __restrict__ tokens,
    int s1, int32_t* __restrict__ tokens2, int s2, float* __restrict__ values, int index_offset) {
  pdl_enter();
  const int r = blockIdx.x;
  const __nv_bfloat16* row = logits + (size_t)r * ld;
  Best b{-INFINITY, 0x7fffffff};
  const bool vec = ((ld & 7) == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  for (int v = threadIdx.x * 8; v < V; v += kArgThreads * 8) {
    if (vec && v + 8 <= V) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(row + v));
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) b = better(b, Best{__bfloat162float(e[j]), v + j});
    } else {
      for (int j = v; j < min(v + 8, V); ++j) b = better(b, Best{__bfloat162float(row[j]), j});
    }
  }
  b = warp_best(b);
  __shared__ Best red[kArgThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = b;
  __syncthreads();
  if (warp == 0) {
    b = red[lane];
    b = warp_best(b);
    if (lane == 0) {
      const int t = (b.i == 0x7fffffff ? 0 : b.i) + index_offset;
      tokens[(size_t)r * s1] = t;
      if (tokens2) tokens2[(size_t)r * s2] = t;
      if (values) values[r] = b.v;
    }
  }
}

// Greedy acceptance over a vocabulary split across `shards` ranks: row r's argmax is the
// largest of the shards' (value, global index) pairs, ties to the smallest index (the
// mx.argmax rule over the whole row). Then the accepted prefix, plan, pending and commit of
// accept_greedy_kernel. One thread per batch row.
__global__ void accept_sharded_kernel(const float* __restrict__ vals, const int32_t* __restrict__ idx,
                                      int shards, int B, int T, const int32_t* __restrict__ verify_ids,
                                      int32_t* __restrict__ kv_len, int commit,
                                      int32_t* __restrict__ pending, int32_t* __restrict__ plan) {
  pdl_enter();
  const int rows = B * T;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    int tt[64];
    for (int t = 0; t < T; ++t) {
      const int r = b * T + t;
      Best best{-INFINITY, 0x7fffffff};
      for (int s = 0; s < shards; ++s)
        best = better(best, Best{vals[(size_t)s * rows + r], idx[(size_t)s * rows + r]});
      tt[t] = best.i == 0x7fffffff ? 0 : best.i;
    }
    int n = 0;
    while (n < T - 1 && verify_ids[b * T + n + 1] == tt[n]) ++n;
    int32_t* pl = plan + (size_t)b * (T + 2);
    pl[0] = n;
    pl[1] = n + 1;
    for (int i = 0; i < n; ++i) pl[2 + i] = verify_ids[b * T + i + 1];
    pl[2 + n] = tt[n];
    for (int i = n + 1; i < T; ++i) pl[2 + i] = -1;
    pending[b] = tt[n];
    if (commit) kv_len[b] += n + 1;
  }
}

__global__ void bump_kernel(int32_t* __restrict__ ctr, int B) {
  pdl_enter();
  for (int b = threadIdx.x; b < B; b += blockDim.x) ctr[b] += 1;
}

static size_t ws(int rows, int V, int* grid_out, size_t* off_i, size_t* off_c) {
  int grid = 148;
  if (V / grid < 1024) grid = (V + 1023) / 1024;
  if (grid < 1) grid = 1;
  if (grid_out) *grid_out = grid;
  // counter word first (fixed offset for every shape), then the two partial arrays
  const size_t pv = (((size_t)grid * rows * 4) + 255) & ~(size_t)255;
  if (off_c) *off_c = 256;
  if (off_i) *off_i = 256 + pv;
  return 256 + 2 * pv;
}

}  // namespace acc
}  // namespace dspark

using namespace dspark;

extern "C" size_t dspark_accept_workspace_bytes(int rows, int V) {
  if (rows <= 0 || V <= 0) return 0;
  return acc::ws(rows, V, nullptr, nullptr, nullptr);
}

extern "C" int dspark_accept_greedy(const void* logits, int ld, int B, int T, int V,
                                    const int32_t* verify_ids, int32_t* argmax, int32_t* kv_len,
                                    int commit, int32_t* pending, int32_t* plan, void* workspace,
                                    size_t workspace_bytes, dspark_stream_t stream) {
  if (!logits || !verify_ids || !argmax || !pending || !plan || B <= 0 || T <= 0 || V <= 0 || ld < V)
    return set_error(DSPARK_ERR_INVALID, "accept_greedy: bad arguments");
  if (commit && !kv_len) return set_error(DSPARK_ERR_INVALID, "accept_greedy: commit without kv_len");
  if (B * T > 64) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_greedy: more than 64 rows");
  int grid;
  size_t off_i, off_c;
  const size_t need = acc::ws(B * T, V, &grid, &off_i, &off_c);
  if (!workspace || workspace_bytes < need)
    return set_error(DSPARK_ERR_WORKSPACE, "accept_greedy: workspace %zu < %zu", workspace_bytes, need);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  return launch_pdl("accept_greedy", acc::accept_greedy_kernel, dim3(grid), dim3(acc::kThreads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(logits),
                    ld, B, T, V, verify_ids, argmax, kv_len, commit, pending, plan,
                    reinterpret_cast<float*>(w + off_c), reinterpret_cast<int*>(w + off_i),
                    reinterpret_cast<int*>(w));
}

// ------------------------------------------------------------------------------------------
// Allocation-free variant of dspark_accept_greedy.
//
// For callers that are handed only their input and output buffers and may not allocate
// device memory themselves: a serving process whose device memory pool is fixed when it
// starts, or a binding from another language that has no handle on the process's allocator.
// The kernel's scratch (one counter word and the per-CTA partial argmaxes) lives in a
// file-scope device array instead of a caller-provided workspace. Its size serves up to
// kStaticRows verify rows with the kStaticGrid-CTA vocabulary split, about 74 KB, held by
// every GPU that loads this library until the process exits.
//
// The array is shared by every call on a device and keeps the last call's contents: the
// counter is cleared on the stream before each launch, and calls that overlap on the GPU (two
// streams at once) race on it. The first call on a device looks the array's device address
// up with cudaGetSymbolAddress (in host code the array's name is only a host-side stand-in),
// so that first call should come before any stream capture.
namespace dspark {
namespace acc {
constexpr int kStaticRows = 64;   // same row limit as the workspace entry point
constexpr int kStaticGrid = 148;  // ws() never splits the vocabulary over more CTAs
constexpr size_t kStaticScratchBytes =
    256 + 2 * ((((size_t)kStaticGrid * kStaticRows * 4) + 255) & ~(size_t)255);
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
}  // namespace acc
}  // namespace dspark

static std::mutex g_static_scratch_mu;
static void* g_static_scratch_ptr[128] = {};

static int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_error(DSPARK_ERR_CUDA, "accept_greedy_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_greedy_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, acc::g_static_scratch);
    if (e != cudaSuccess || !p)
      return set_error(DSPARK_ERR_CUDA, "accept_greedy_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    g_static_scratch_ptr[dev] = p;
  }
  *out = g_static_scratch_ptr[dev];
  return DSPARK_OK;
}

extern "C" int dspark_accept_greedy_noalloc(const void* logits, int ld, int B, int T, int V,
                                            const int32_t* verify_ids, int32_t* argmax,
                                            int32_t* kv_len, int commit, int32_t* pending,
                                            int32_t* plan, dspark_stream_t stream) {
  if (!logits || !verify_ids || !argmax || !pending || !plan || B <= 0 || T <= 0 || V <= 0 || ld < V)
    return set_error(DSPARK_ERR_INVALID, "accept_greedy_noalloc: bad arguments");
  if (commit && !kv_len)
    return set_error(DSPARK_ERR_INVALID, "accept_greedy_noalloc: commit without kv_len");
  if (B * T > acc::kStaticRows)
    return set_error(DSPARK_ERR_UNSUPPORTED,
                     "accept_greedy_noalloc: %d rows exceed the fixed scratch limit of %d rows",
                     B * T, acc::kStaticRows);
  int grid;
  size_t off_i, off_c;
  const size_t need = acc::ws(B * T, V, &grid, &off_i, &off_c);
  if (grid > acc::kStaticGrid || need > acc::kStaticScratchBytes)
    return set_error(DSPARK_ERR_UNSUPPORTED,
                     "accept_greedy_noalloc: needs %zu scratch bytes, the fixed scratch holds %zu",
                     need, acc::kStaticScratchBytes);
  void* base = nullptr;
  int rc = static_scratch_address(&base);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(base, 0, sizeof(int), st);  // the arrival counter
  if (e != cudaSuccess)
    return set_error(DSPARK_ERR_CUDA, "accept_greedy_noalloc: clearing the counter: %s",
                     cudaGetErrorString(e));
  uint8_t* w = static_cast<uint8_t*>(base);
  return launch_pdl("accept_greedy_noalloc", acc::accept_greedy_kernel, dim3(grid),
                    dim3(acc::kThreads), 0, st, static_cast<const __nv_bfloat16*>(logits), ld, B,
                    T, V, verify_ids, argmax, kv_len, commit, pending, plan,
                    reinterpret_cast<float*>(w + off_c), reinterpret_cast<int*>(w + off_i),
                    reinterpret_cast<int*>(w));
}

extern "C" int dspark_commit_lengths(const int32_t* plan, int plan_stride, int B, int32_t* len_a,
                                     int32_t* len_b, dspark_stream_t stream) {
  if (!plan || B <= 0 || (!len_a && !len_b))
    return set_error(DSPARK_ERR_INVALID, "commit_lengths: bad arguments");
  return launch_pdl("commit_lengths", acc::commit_lengths_kernel, dim3(1), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), plan, plan_stride, B, len_a, len_b);
}

extern "C" int dspark_draft_override(int B, int cap, int V, const int32_t* ref, int ref_len,
                                     const uint8_t* agree, int rounds, int32_t* round_ctr,
                                     const int32_t* kv_len, const int32_t* prompt_len,
                                     int32_t* verify_ids, dspark_stream_t stream) {
  if (!ref || !agree || !round_ctr || !kv_len || !prompt_len || !verify_ids || B <= 0 || cap <= 0 ||
      ref_len <= 0 || rounds <= 0)
    return set_error(DSPARK_ERR_INVALID, "draft_override: bad arguments");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = launch_pdl("draft_override", acc::draft_override_kernel, dim3(B), dim3(32), 0, st, B,
                      cap, V, ref, ref_len, agree, rounds, (const int32_t*)round_ctr, kv_len,
                      prompt_len, verify_ids);
  if (rc) return rc;
  return launch_pdl("draft_override.bump", acc::bump_kernel, dim3(1), dim3(32), 0, st, round_ctr, B);
}

extern "C" int dspark_argmax_rows(const void* logits, long long ld, int rows, int V, int32_t* tokens,
                                  int tok_stride, int32_t* tokens2, int tok2_stride,
                                  float* values, int index_offset, dspark_stream_t stream) {
  if (!logits || !tokens || rows <= 0 || V <= 0 || ld < V || tok_stride < 1 ||
      (tokens2 && tok2_stride < 1) || index_offset < 0)
    return set_error(DSPARK_ERR_INVALID, "argmax_rows: bad arguments");
  if (rows > 65535) return set_error(DSPARK_ERR_UNSUPPORTED, "argmax_rows: too many rows");
  return launch_pdl("argmax_rows", acc::argmax_rows_kernel, dim3(rows), dim3(acc::kArgThreads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(logits),
                    ld, V, tokens, tok_stride, tokens2, tok2_stride, values, index_offset);
}

extern "C" int dspark_accept_greedy_sharded(const float* values, const int32_t* indices, int shards,
                                            int B, int T, const int32_t* verify_ids,
                                            int32_t* kv_len, int commit, int32_t* pending,
                                            int32_t* plan, dspark_stream_t stream) {
  if (!values || !indices || !verify_ids || !pending || !plan || shards <= 0 || B <= 0 || T <= 0)
    return set_error(DSPARK_ERR_INVALID, "accept_greedy_sharded: bad arguments");
  if (commit && !kv_len) return set_error(DSPARK_ERR_INVALID, "accept_greedy_sharded: commit without kv_len");
  if (T > 64) return set_error(DSPARK_ERR_UNSUPPORTED, "accept_greedy_sharded: T > 64");
  return launch_pdl("accept_greedy_sharded", acc::accept_sharded_kernel, dim3(1), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), values, indices, shards, B, T, verify_ids,
                    kv_len, commit, pending, plan);
}
