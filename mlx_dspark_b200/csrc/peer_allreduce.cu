// K1p, receive half — the tensor-parallel one-shot all-reduce that dspark_w8a16_gemm_peer
// starts: the row-split o_proj / down_proj partials of every rank, summed in rank order and
// added to the residual stream (the NCCL all-reduce + residual add after those projections in
// the tensor-parallel target; the reference is single-device). Also the CUDA IPC plumbing that
// maps every rank's receive buffer and flags into every process.
#include <cstring>

#include "common.cuh"

namespace dspark {
namespace par {

constexpr int kCols = 128;  // one output tile of the GEMM per CTA

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// CTA t: wait (bounded) for every rank's flag of tile t at this epoch, then
// h[m, n] = bf16(h + bf16(sum_r recv[slot][r][m][n])), r = 0 .. world-1 in order.
// The kernel does not wait for the GEMM before it to complete: the flags carry every input
// (each tile's partials, this rank's included, behind a system-scope release), and the
// residual rows were last written by a kernel that completed before that GEMM's CTAs started.
// So a tile is summed as soon as every rank has finished it, while the GEMM's last tiles are
// still running.
// With epoch_dev, the GEMMs and the reduces keep separate counts, because the reduce of call
// e runs next to the GEMM of call e and may start before the reduce of call e - 1 is done:
//   [2], [3]: the reduces' count. Every CTA reads [2] + 1 and counts itself in [3]; the last
//     stores the epoch into [2] before triggering the next launch, and a later reduce starts
//     only after that trigger (it follows a GEMM whose CTAs start after it).
//   [0], [1]: the GEMMs' count, which a GEMM reads in its epilogue after the kernel before it
//     completed. Every CTA counts itself in [1] when it is done, and the last stores the
//     epoch into [0]: by then every tile of this rank's GEMM of this call is finished.
__global__ void __launch_bounds__(kCols) peer_reduce_residual_kernel(
    __nv_bfloat16* __restrict__ h, int ldh, int M, int N, const float* __restrict__ recv,
    const int* __restrict__ flags, int world, int mcap, int epoch_arg, int* epoch_dev,
    long long timeout_ns, int* status) {
  __shared__ int s_epoch;
  if (threadIdx.x == 0) {
    int e = epoch_arg;
    if (epoch_dev) {
      e = __ldcg(epoch_dev + 2) + 1;
      int old;
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(epoch_dev + 3)
                   : "memory");
      if (old == (int)gridDim.x - 1) {
        epoch_dev[3] = 0;
        epoch_dev[2] = e;
        __threadfence();
      }
    }
    s_epoch = e;
  }
  __syncthreads();
  pdl_launch_dependents();
  const int epoch = s_epoch;
  const int tile = blockIdx.x, tiles = N / kCols;
  const int slot = epoch & 1;
  if (threadIdx.x < world) {
    const int* f = flags + ((size_t)slot * world + threadIdx.x) * tiles + tile;
    if (ld_acquire_sys(f) != epoch) {
      const unsigned long long t0 = globaltimer_ns();
      while (ld_acquire_sys(f) != epoch) {
        if ((long long)(globaltimer_ns() - t0) > timeout_ns) {
          report_error(status, DSPARK_ERR_TIMEOUT);  // the sums below are then not meaningful
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();  // the acquires above order every thread's reads below
  const int n = tile * kCols + threadIdx.x;
  for (int m = 0; m < M; ++m) {
    float s = 0.0f;
    for (int r = 0; r < world; ++r)
      s += __ldcg(recv + (((size_t)slot * world + r) * mcap + m) * N + n);
    __nv_bfloat16* p = h + (size_t)m * ldh + n;
    *p = __float2bfloat16_rn(__bfloat162float(*p) + bf16r(s));
  }
  if (epoch_dev) {
    __syncthreads();
    if (threadIdx.x == 0) {
      int old;
      asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(epoch_dev + 1)
                   : "memory");
      if (old == (int)gridDim.x - 1) {
        epoch_dev[1] = 0;
        epoch_dev[0] = epoch;
        __threadfence();
      }
    }
  }
}

}  // namespace par
}  // namespace dspark

using namespace dspark;

extern "C" int dspark_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return set_error(DSPARK_ERR_INVALID, "peer_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_CUDA, "peer_alloc: %s", cudaGetErrorString(e));
  e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_CUDA, "peer_alloc memset: %s", cudaGetErrorString(e));
  return DSPARK_OK;
}

extern "C" int dspark_peer_free(void* ptr) {
  if (!ptr) return DSPARK_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? DSPARK_OK : set_error(DSPARK_ERR_CUDA, "peer_free: %s", cudaGetErrorString(e));
}

extern "C" int dspark_ipc_handle(const void* ptr, void* handle64) {
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  if (!ptr || !handle64) return set_error(DSPARK_ERR_INVALID, "ipc_handle: bad arguments");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return set_error(DSPARK_ERR_CUDA, "ipc_handle: %s", cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  return DSPARK_OK;
}

extern "C" int dspark_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return set_error(DSPARK_ERR_INVALID, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(DSPARK_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(e));
  return DSPARK_OK;
}

extern "C" int dspark_ipc_close(void* ptr) {
  if (!ptr) return DSPARK_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? DSPARK_OK : set_error(DSPARK_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
}

extern "C" int dspark_peer_reduce_residual(void* h, int ldh, int M, const dspark_peer_ar* ar,
                                           long long timeout_ns, int* status,
                                           dspark_stream_t stream) {
  if (!h || !ar || M <= 0 || M > ar->m_cap || ar->world < 2 || ar->world > 8 || ar->rank < 0 ||
      ar->rank >= ar->world || ar->n <= 0 || ar->n % par::kCols || ldh < ar->n ||
      (ar->epoch < 1 && !ar->epoch_dev) || timeout_ns <= 0)
    return set_error(DSPARK_ERR_INVALID, "peer_reduce_residual: bad arguments");
  if (!ar->recv[ar->rank] || !ar->flags[ar->rank])
    return set_error(DSPARK_ERR_INVALID, "peer_reduce_residual: own buffers missing");
  return launch_pdl("peer_reduce_residual", par::peer_reduce_residual_kernel,
                    dim3(ar->n / par::kCols), dim3(par::kCols), 0,
                    static_cast<cudaStream_t>(stream), static_cast<__nv_bfloat16*>(h), ldh, M,
                    ar->n, static_cast<const float*>(ar->recv[ar->rank]),
                    static_cast<const int*>(ar->flags[ar->rank]), ar->world, ar->m_cap, ar->epoch,
                    ar->epoch_dev, timeout_ns, status);
}
