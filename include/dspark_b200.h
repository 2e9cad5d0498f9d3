/*
 * dspark_b200.h — C ABI of libdspark_b200.so, the sm_100a kernels under the speculative
 * verify step of mlx-dspark (Qwen3 targets with W8 affine group-64 weights, DSpark and
 * DFlash drafters).
 *
 * Conventions shared by every entry point:
 *   - Pointers are device pointers unless a parameter says "host". Shapes are explicit
 *     ints; leading dimensions are in elements. No torch types cross this boundary.
 *   - Calls are stream-ordered and asynchronous; nothing is allocated inside the library
 *     except by dspark_peer_alloc (the IPC-shareable buffers of the tensor-parallel fused
 *     all-reduce). Scratch memory is passed in by the caller (sizes from the *_workspace_bytes
 *     queries).
 *   - The return value is a status code (DSPARK_OK = 0). On failure the thread-local
 *     message from dspark_last_error() says what was wrong.
 *   - Kernels that wait on the device (pipeline barriers, grid barriers) give up after a
 *     bounded time and write DSPARK_ERR_TIMEOUT into the caller's device status word
 *     (`int* status`, may be NULL); the host reads it at its next synchronisation point.
 *
 * Reference interfaces replaced (paths inside regeter/mlx-dspark):
 *   the mlx-lm Qwen3 forward called by src/mlx_dspark/target.py:58-75 and
 *   src/mlx_dspark/batch_engine.py:184-206; the DSpark drafter src/mlx_dspark/model.py:220-320;
 *   the DFlash drafter src/mlx_dspark/dflash_model.py:100-208; greedy acceptance
 *   src/mlx_dspark/generate.py:905-921 and batch_engine.py:573-595; speculative-sampling
 *   acceptance src/mlx_dspark/generate.py:659-688 with src/mlx_dspark/sampling.py:18-49.
 */
#ifndef DSPARK_B200_H_
#define DSPARK_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* opaque stream handle (a cudaStream_t); NULL means the legacy default stream */
typedef void* dspark_stream_t;

enum {
  DSPARK_OK = 0,
  DSPARK_ERR_INVALID = 1,     /* bad shape, pointer or argument */
  DSPARK_ERR_ALIGN = 2,       /* pointer or leading dimension not aligned as required */
  DSPARK_ERR_LAUNCH = 3,      /* kernel launch failed */
  DSPARK_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up */
  DSPARK_ERR_UNSUPPORTED = 5, /* configuration not compiled in */
  DSPARK_ERR_CUDA = 6,        /* CUDA runtime / driver call failed */
  DSPARK_ERR_WORKSPACE = 7,   /* workspace missing or too small */
  DSPARK_ERR_RANGE = 8        /* a value written as an fp16 GEMM operand (the SiLU*up
                                 activations, the attention output, the fp16 hidden-state
                                 taps) was outside the fp16 range (|x| > 65504) or NaN: the
                                 kernel stores it as fp16 (an infinity) and records this code in
                                 the caller's status word */
};

/* W8A16 GEMM epilogues */
enum {
  DSPARK_EPI_STORE_BF16 = 0,    /* y[m,n] = bf16(acc)                                      */
  DSPARK_EPI_RESIDUAL_BF16 = 1, /* y[m,n] = bf16(r[m,n] + bf16(acc)); y may alias r          */
  DSPARK_EPI_SILU_MUL_F16 = 2,  /* gate/up interleaved in 64-row halves of each 128-row tile;
                                   y[m,j] = fp16(bf16(bf16(silu(g)) * u)), y has N/2 columns */
  DSPARK_EPI_STORE_F32 = 3,     /* y[m,n] = acc (fp32)                                       */
  DSPARK_EPI_PEER_F32 = 4       /* dspark_w8a16_gemm_peer only: acc to every rank's receive
                                   buffer, then the tile's epoch flag (fused all-reduce)      */
};

/* library identity */
int dspark_version(void);
const char* dspark_last_error(void);
/* Kernels this thread has launched through the library so far (monotonic; the difference
 * around a call is what the call launched, e.g. 1 or 2 for dspark_attention). */
long long dspark_launch_count(void);

/* -------------------------------------------------------------------------------------
 * K1 — W8A16 group-64 dequant GEMM for the small-M verify shape.
 * Replaces: mlx nn.QuantizedLinear (bits 8, group 64, affine) inside the mlx-lm Qwen3
 * layers (called from src/mlx_dspark/target.py:67, batch_engine.py:200) and the drafter's
 * quantized linears (src/mlx_dspark/load.py:204-206).
 *
 *   Y[M,N] = X[M,K] . W[N,K]^T,   W[n,k] = scale[n,k/64] * q[n,k] + bias[n,k/64]
 *
 * x   : fp16 [M, ldx] activations (bf16-rounded values stored as fp16, |x| < 65504)
 * wq  : uint8 [N, K] row-major
 * wsb : uint32 [K/64, N]; low half = fp16 scale, high half = fp16 bias of group (n, g)
 * M <= 64, N % 128 == 0, K % 128 == 0, ldx % 8 == 0, 16-byte aligned x / wq / wsb.
 * workspace: dspark_w8a16_gemm_workspace_bytes(M, N, K) bytes, zero-filled once before the
 * first call; every call leaves its counter words at zero again.
 * ------------------------------------------------------------------------------------- */
size_t dspark_w8a16_gemm_workspace_bytes(int M, int N, int K);
int dspark_w8a16_gemm(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M,
                      int N, int K, void* y, int ldy, const void* residual, int ldr, int epilogue,
                      void* workspace, size_t workspace_bytes, int* status,
                      dspark_stream_t stream);
/* The same GEMM, which also warms L2 with up to two byte ranges a later kernel reads (the next
 * projection's weights): each CTA prefetches its slice after issuing its last load, so HBM keeps
 * streaming through the GEMM's tail and the small kernels that follow. Ranges are 16-byte
 * aligned; sizes are rounded down to multiples of 16; NULL / 0 means none. The result is that of
 * dspark_w8a16_gemm. (No reference counterpart: MLX schedules its own memory traffic.) */
int dspark_w8a16_gemm_pf(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M,
                         int N, int K, void* y, int ldy, const void* residual, int ldr,
                         int epilogue, void* workspace, size_t workspace_bytes, const void* pf0,
                         size_t pf0_bytes, const void* pf1, size_t pf1_bytes, int* status,
                         dspark_stream_t stream);
/* Options of dspark_w8a16_gemm_ex (zero-initialise; NULL pointers switch a feature off).
 *   prefetch[2], prefetch_bytes[2]: as dspark_w8a16_gemm_pf.
 *   row_sumsq (STORE_BF16 / RESIDUAL_BF16 epilogues): fp32 [M, N/128] output; entry (m, t) is
 *     the sum of the squares of the bf16 outputs y[m, 128t .. 128t+127] this call writes, summed
 *     in a fixed order — the pieces of the next RMSNorm of that row.
 *   norm_w, norm_sumsq, norm_tiles, norm_eps: fuse the RMSNorm of the GEMM input (mlx.fast.rms_norm,
 *     the input/post-attention/final norms of the Qwen3 layers). x is then the bf16 residual stream
 *     [M, K] itself; the GEMM consumes bf16(x[m,k] * r[m] * w[k]) (as dspark_rmsnorm's output)
 *     with r[m] = rsqrt(sum_t norm_sumsq[m, t] / K + eps), t in order, from the row_sumsq of the
 *     GEMM that wrote x (norm_tiles = its N/128; norm_ld = the row stride in floats, 0 meaning
 *     norm_tiles; 16-byte aligned rows when norm_ld % 4 == 0). The only difference from
 *     dspark_rmsnorm + this GEMM is the fp32 summation order of the squares.
 *   copy_f16, copy_f16_ld: RESIDUAL_BF16 only; the epilogue also stores each bf16 output as fp16
 *     (exact) at copy_f16[m * copy_f16_ld + n] (the drafter's hidden-state tap). */
typedef struct dspark_gemm_opts {
  const void* prefetch[2];
  size_t prefetch_bytes[2];
  float* row_sumsq;
  const float* norm_sumsq;
  const void* norm_w;
  int norm_tiles;
  float norm_eps;
  int norm_ld;
  int reserved;
  void* copy_f16;   /* RESIDUAL_BF16 only: also store fp16(y) here (the hidden-state tap) */
  int copy_f16_ld;  /* its row stride in elements */
  int reserved2;
} dspark_gemm_opts;
int dspark_w8a16_gemm_ex(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M,
                         int N, int K, void* y, int ldy, const void* residual, int ldr,
                         int epilogue, const dspark_gemm_opts* opts, void* workspace,
                         size_t workspace_bytes, int* status, dspark_stream_t stream);
size_t dspark_gemm_opts_size(void); /* sizeof(dspark_gemm_opts), for bindings to check */


/* -------------------------------------------------------------------------------------
 * K1p — tensor-parallel row-split projection with its all-reduce fused into the GEMM: the
 * GEMM-epilogue one-shot all-reduce over NVLink peer memory. Replaces, for the tensor-parallel
 * Qwen3-32B target, the NCCL all-reduce of [M, N] after o_proj and down_proj and the residual
 * add after it (no reference counterpart: the reference runs on one device).
 *
 * Every rank holds a receive buffer recv [2][world][m_cap][N] fp32 and flags [2][world][N/128]
 * int32, both from dspark_peer_alloc, and maps every peer's pair through CUDA IPC handles. For
 * all-reduce number `epoch` (1, 2, ...; slot = epoch & 1):
 *   - dspark_w8a16_gemm_peer: the CTA that finishes output tile t stores its fp32 tile (rows
 *     < M, columns 128t..128t+127) into recv_r[slot][rank] of every rank r with plain
 *     stores over NVLink, then, after a system-scope acq_rel fence, writes epoch into
 *     flags_r[slot][rank][t] with relaxed system-scope stores. No TMA and no multicast.
 *   - dspark_peer_reduce_residual: on each rank, CTA t waits (acquire loads, bounded by
 *     timeout_ns, DSPARK_ERR_TIMEOUT in *status on expiry) until flags[slot][r][t] == epoch for
 *     every r, then h[m, n] = bf16(h[m, n] + bf16(sum over r in rank order of recv[slot][r][m][n])).
 *     It does not wait for the GEMM's grid to complete (the flags carry its inputs), so a tile
 *     is summed as soon as every rank has finished it; it must follow the GEMM on the stream,
 *     with h last written by a kernel that completed before the GEMM started.
 * Two slots keep epoch e + 2's stores out of a slot a peer may still read for epoch e: a rank
 * issues them only after its own reduce for e + 1 has seen every peer's flags for e + 1, which
 * each peer raises after its reduce for e. Every rank calls both, in the same order, every epoch.
 * ------------------------------------------------------------------------------------- */
typedef struct dspark_peer_ar {
  void* recv[8];   /* rank r's receive buffer as mapped in this process (own one at [rank]) */
  void* flags[8];  /* rank r's flag array as mapped in this process */
  int world;       /* ranks, 2..8 */
  int rank;
  int m_cap;       /* rows per rank slot in recv */
  int n;           /* columns (the projection's N, a multiple of 128) */
  int epoch;       /* this all-reduce's number, >= 1 (ignored when epoch_dev is set) */
  int reserved;
  int* epoch_dev;  /* NULL, or 4 zero-initialised ints on this rank's device: the calls then
                    * number themselves on the device ([0] the last all-reduce whose reduce has
                    * finished, read by the GEMM; [2] the last whose reduce has started, read
                    * by the reduce; [1], [3] scratch), so a CUDA graph of the calls replays
                    * with fresh epochs. */
} dspark_peer_ar;
/* cudaMalloc'd, zero-filled memory for recv / flags (IPC needs its own allocation), and its
 * release. These two entry points allocate; nothing else in the library does. */
int dspark_peer_alloc(size_t bytes, void** ptr);
int dspark_peer_free(void* ptr);
/* 64-byte CUDA IPC handle of a dspark_peer_alloc pointer; open a peer's handle in this process
 * (peer access enabled) and close it again. */
int dspark_ipc_handle(const void* ptr, void* handle64);
int dspark_ipc_open(const void* handle64, void** ptr);
int dspark_ipc_close(void* ptr);
/* y = x . W^T of this rank's K-slice, all-reduced as described above (M <= min(64, m_cap)). */
int dspark_w8a16_gemm_peer(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M,
                           int N, int K, const dspark_peer_ar* ar, void* workspace,
                           size_t workspace_bytes, int* status, dspark_stream_t stream);
int dspark_peer_reduce_residual(void* h, int ldh, int M, const dspark_peer_ar* ar,
                                long long timeout_ns, int* status, dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K1w — the same W8A16 product for prefill chunks (large M). Replaces the QuantizedLinear
 * calls of Target.run over one prefill chunk (src/mlx_dspark/generate.py:613-656 ->
 * src/mlx_dspark/target.py:51-75) and of the drafter's update_context over the chunk's tapped
 * hidden states (src/mlx_dspark/model.py:253-256).
 *   x fp16 [M, K] (16-byte aligned rows), any M >= 1; N a multiple of 128, K of 64;
 *   epilogue STORE_BF16, RESIDUAL_BF16 (y may alias residual; copy_f16 optional, as in
 *   dspark_gemm_opts), SILU_MUL_F16 (interleaved gate/up pack, y [M, N/2]) or STORE_F32.
 * Outputs are the verify GEMM's: the same fp16 weights, fp32 accumulation (in another order)
 * and the same epilogue roundings. Persistent tcgen05 kernel, one CTA per SM, tiles of 128
 * weight rows x 256 tokens (128 tokens when M <= 256 or when 256-token tiles would number at
 * most 64); no workspace. */
int dspark_w8a16_gemm_wide(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb, int M,
                           int N, int K, int epilogue, void* y, int ldy, const void* residual,
                           int ldr, void* copy_f16, int copy_f16_ld, int* status,
                           dspark_stream_t stream);
/* The launch dspark_w8a16_gemm_wide makes for this shape: *bn tokens per tile, *grid CTAs. */
int dspark_w8a16_gemm_wide_plan(int M, int N, int K, int* bn, int* grid);
/* Tokens per tile of dspark_w8a16_gemm_wide, process-wide: 0 (default) picks by M, 128 or 256
 * forces that width (measurements; no reference counterpart). */
int dspark_w8a16_gemm_wide_bn(int bn);

/* -------------------------------------------------------------------------------------
 * K13 — embedding dequant-gather. Replaces mlx QuantizedEmbedding (embed_tokens,
 * src/mlx_dspark/target.py:63; drafter embed src/mlx_dspark/model.py:244-245).
 *   out[m, :] = bf16(scale * q[ids[m], :] + bias) * embed_scale (embed_scale 1 for Qwen3)
 * ids is a device array of M token ids (read on the device, so the call can sit in a
 * CUDA graph whose ids change between replays).
 * ------------------------------------------------------------------------------------- */
int dspark_embed_w8(const int32_t* ids, int M, const uint8_t* wq, const uint32_t* wsb, int V,
                    int H, void* out, int ldo, dspark_stream_t stream);
/* The same gather that also writes the per-128-column-tile row sums of squares of its bf16
 * outputs, sumsq [M, H/128] (the row_sumsq of dspark_gemm_opts), so the first layer's input
 * RMSNorm can run inside the q|k|v GEMM. H % 128 == 0. */
int dspark_embed_w8_sumsq(const int32_t* ids, int M, const uint8_t* wq, const uint32_t* wsb,
                          int V, int H, void* out, int ldo, float* sumsq,
                          dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K6 — RMSNorm over rows, mlx.fast.rms_norm semantics (fp32 math, one bf16 rounding).
 * Replaces the input/post-attention/final norms of the Qwen3 layers and the drafter's
 * hidden_norm / norm (src/mlx_dspark/model.py:247-248,258-262).
 *   y = bf16(x * rsqrt(mean(x^2) + eps) * w). y_bf16 and y_f16 (bf16 value stored as fp16,
 *   the GEMM input format) are both optional.
 * ------------------------------------------------------------------------------------- */
int dspark_rmsnorm(const void* x, int ldx, const void* w, int M, int H, float eps, void* y_bf16,
                   int ldy, void* y_f16, int ldy16, dspark_stream_t stream);

/* paged KV cache layout of one layer.
 * Page p holds `page_size` tokens of every kv head:
 *   bf16 pages: K[Hkv][page_size][head_dim] bf16 then V[Hkv][page_size][head_dim] bf16
 *   8-bit pages: Kq[Hkv][page_size][head_dim] u8, Vq[...] u8, then
 *                Ksb[Hkv][page_size][head_dim/64] u32, Vsb[...] u32 (bf16 scale | bf16 bias<<16)
 * block_table[b * max_pages + i] = physical page of token positions [i*page_size, ...). */
typedef struct dspark_kv_layout {
  void* pool;                 /* this layer's page pool */
  const int32_t* block_table; /* [batch, max_pages] */
  int max_pages;
  int page_size;
  int num_kv_heads;
  int head_dim;
  int kv8;                    /* 0 = bf16 pages, 1 = 8-bit affine group-64 pages */
  int reserved;
  long long page_bytes;       /* bytes per page (the stride between pages) */
} dspark_kv_layout;

long long dspark_kv_page_bytes(int page_size, int num_kv_heads, int head_dim, int kv8);


/* -------------------------------------------------------------------------------------
 * K6+K7+K3 — per-head q/k RMSNorm, non-interleaved RoPE at per-row positions, and the
 * write of the new K/V rows into the paged cache (quantize-on-write for 8-bit pages).
 * Replaces: Qwen3 attention pre-SDPA (mlx-lm qwen3; q_norm/k_norm then rope at
 * cache.offset) with KVCache.update_and_fetch / QuantizedKVCache (target.py:44-46),
 * BatchCache.update_and_fetch (batch_engine.py:132-147), DSparkAttention._kv/update_ctx
 * (model.py:113-128).
 *
 * qkv  : bf16 [B*T, ldqkv]; columns [0, Hq*hd) = q, then Hkv*hd of k, then Hkv*hd of v
 *        (Hq may be 0: then only k and v are present)
 * pos0 : [B] device array; token t of row b sits at position pos0[b] + t, and its K/V go
 *        to that position in the paged cache
 * inv_freq : fp32 [hd/2] device array, theta^(-2i/hd)
 * q_out: bf16 [B*T, Hq*hd] (ignored when Hq == 0)
 * ------------------------------------------------------------------------------------- */
int dspark_qkv_rope_kv_write(const void* qkv, int ldqkv, int B, int T, int Hq, int Hkv, int hd,
                             const void* q_norm_w, const void* k_norm_w, float eps,
                             const float* inv_freq, const int32_t* pos0, void* q_out,
                             const dspark_kv_layout* kv, dspark_stream_t stream);
/* The q|k|v projection and the step above in ONE launch: the W8 GEMM of the fused q|k|v
 * weights (N = (Hq + 2*Hkv)*hd, a multiple of 128) whose epilogue, per finished 128-row tile
 * (one head at hd 128, two at hd 64), stages the tile's bf16 outputs in shared memory and runs
 * the same per-head norm + RoPE + q / K/V writes as dspark_qkv_rope_kv_write. Outputs equal
 * dspark_w8a16_gemm (STORE_BF16) followed by dspark_qkv_rope_kv_write bit for bit; the raw q|k|v
 * row is never stored. M = B*T rows; workspace as dspark_w8a16_gemm; opts as dspark_w8a16_gemm_ex
 * (its input norm is the layer's input RMSNorm; row_sumsq must be NULL). */
int dspark_w8a16_gemm_qkv_rope(const void* x, int ldx, const uint8_t* wq, const uint32_t* wsb,
                               int M, int K, int T, int Hq, int Hkv, int hd, const void* q_norm_w,
                               const void* k_norm_w, float eps, const float* inv_freq,
                               const int32_t* pos0, void* q_out, const dspark_kv_layout* kv,
                               const dspark_gemm_opts* opts, void* workspace,
                               size_t workspace_bytes, int* status, dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K2/K4/K5 — GQA attention of T block queries per row over the paged cache, split-KV.
 * Keys of row b are positions [0, kv_len[b] + T).
 *   causal = 1: query t sees keys j <= kv_len[b] + t   (target verify, mlx-lm mask /
 *               build_batch_mask batch_engine.py:170-178)
 *   causal = 0: every query sees every key              (drafter block attention,
 *               model.py:130-156, dflash_model.py:100-134)
 * q   : bf16 [B*T, Hq*hd]; out: fp16 [B*T, ldo] (bf16-rounded, the o_proj GEMM input)
 * workspace: dspark_attention_workspace_bytes(...) bytes for the split partials.
 * Splits (at most max_splits, at least one page each) are merged in split order by a second
 * launch; with one split the attention launch writes the output directly. `status` (may be
 * NULL) receives DSPARK_ERR_RANGE if an output is past the fp16 range.
 * ------------------------------------------------------------------------------------- */
size_t dspark_attention_workspace_bytes(int B, int T, int Hq, int Hkv, int hd, int max_splits);
int dspark_attention(const void* q, int B, int T, int Hq, const dspark_kv_layout* kv,
                     const int32_t* kv_len, int causal, float scale, void* out, int ldo,
                     int max_splits, void* workspace, size_t workspace_bytes, int* status,
                     dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K8 — fused greedy acceptance. Row-wise argmax of bf16 logits (first index on ties, the
 * mx.argmax rule), accepted-prefix length n, bonus token, and the in-place KV commit /
 * rollback (kv_len[b] += n + 1; the rejected tail is dropped by the length alone).
 * Replaces src/mlx_dspark/generate.py:910-933 and batch_engine.py:573-595.
 *
 * logits   : bf16 [B*T, ld]; verify_ids: [B, T] (column 0 = pending, then the T-1 drafts)
 * argmax   : out [B*T] argmax per row
 * kv_len   : [B] in/out (updated only when commit != 0)
 * pending  : out [B] next pending token (= committed[n])
 * plan     : out [B, T + 2]: {n, count, committed tokens...}; count = n + 1
 * workspace: dspark_accept_workspace_bytes(B*T, V), zero-filled once before first use.
 * ------------------------------------------------------------------------------------- */
size_t dspark_accept_workspace_bytes(int rows, int V);
int dspark_accept_greedy(const void* logits, int ld, int B, int T, int V,
                         const int32_t* verify_ids, int32_t* argmax, int32_t* kv_len,
                         int commit, int32_t* pending, int32_t* plan, void* workspace,
                         size_t workspace_bytes, dspark_stream_t stream);

/* The same greedy acceptance for callers that may not allocate device memory: hosts that
 * hand the library only their input and output buffers, such as a serving process whose
 * device memory pool is fixed at start-up or a binding from another language with no handle
 * on the process's allocator. It has no counterpart in the reference (the reference never
 * manages device memory itself). The kernel's scratch lives in a fixed array inside the
 * library (about 74 KB per GPU that loads the library, held until the process exits), so:
 *   - at most 64 rows (B * T <= 64); larger calls return DSPARK_ERR_UNSUPPORTED;
 *   - every call on a device shares that array: calls that overlap on the GPU (on two
 *     streams at once) race, so order them on one stream;
 *   - the first call on a device looks the array's address up (cudaGetSymbolAddress); make
 *     that first call before any stream capture.
 * It allocates nothing; arguments and results are those of dspark_accept_greedy. */
int dspark_accept_greedy_noalloc(const void* logits, int ld, int B, int T, int V,
                                 const int32_t* verify_ids, int32_t* argmax, int32_t* kv_len,
                                 int commit, int32_t* pending, int32_t* plan,
                                 dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K10 — DSpark Markov head + greedy block sampling: sequential over cap positions,
 *   logits_i = base_i + w2 . w1[prev];  prev = argmax(logits_i)   (first index on ties)
 * Replaces DSparkDrafter.sample_block (src/mlx_dspark/model.py:270-281) and the batched
 * _batched_sample_block (batch_engine.py:414-428).
 * base : bf16 base logits; position i of row b is row (b * rows_per_b + i), i < cap
 * first_prev: [B] (the pending token of each row)
 * w1   : W8 [V, R] Markov embedding, w2: W8 [V, R] (rank R = 256)
 * draft: out [B, cap]; verify_ids (optional): out [B, cap+1] = {first_prev, draft...}
 * workspace: dspark_markov_workspace_bytes(B, V), zero-filled once before first use.
 * ------------------------------------------------------------------------------------- */
size_t dspark_markov_workspace_bytes(int B, int V);
int dspark_markov_sample_block(const void* base, int ld, int rows_per_b, int B, int cap, int V,
                               int R,
                               const uint8_t* w1q, const uint32_t* w1sb, const uint8_t* w2q,
                               const uint32_t* w2sb, const int32_t* first_prev, int32_t* draft,
                               int32_t* verify_ids, void* workspace, size_t workspace_bytes,
                               int* status, dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * K9 — lossless speculative sampling.
 *
 * Distribution of a row: p = truncate(softmax(x)), x = bf16(logits / bf16(T)) (temp_mode 0,
 * the `v_logits / temperature` of generate.py:673,543) or bf16(logits * bf16(1/T))
 * (temp_mode 1, the `logits * inv_t` of model.py:304). Top-k keeps values >= the k-th largest
 * (ties kept); the nucleus keeps values >= the smallest value whose strictly-larger mass is
 * below top_p (src/mlx_dspark/sampling.py:18-44). top_k = 0 and top_p = 1 disable the cuts.
 * Weights are 2^-40 fixed point of a documented exp2 polynomial; every draw is an inverse-CDF
 * draw in vocabulary order from a Philox4x32-10 word, so a CPU restatement reproduces each
 * token exactly.
 * rng: device {seed, offset} pair per group (per request); counter = {offset, row, stream}.
 * ------------------------------------------------------------------------------------- */

/* Draw one token per row from p (sample_probs, sampling.py:47-49; the first token _pick,
 * generate.py:144-146; the DFlash draft, generate.py:541-545).
 * logits: bf16 rows; row r of group g is row (g * rows + r) at stride ld
 * probs (optional): fp32 out, the truncated distribution of each row (the q the accept
 *   test needs), row (g * rows + r) at stride ld_probs
 * tokens: out, row (g * rows + r) at tokens[(g * rows + r) * tok_stride]; tokens2 an
 *   optional second copy. Philox counter row = row_base + r, stream = stream_id. */
int dspark_sample_rows(const void* logits, long long ld, int groups, int rows, int V,
                       float temperature, int temp_mode, double top_p, int top_k,
                       const unsigned long long* rng, int stream_id, int row_base, float* probs,
                       long long ld_probs, int32_t* tokens, int tok_stride, int32_t* tokens2,
                       int tok2_stride, dspark_stream_t stream);

/* Speculative-sampling acceptance (Leviathan / Chen 2023) of B verify blocks; replaces
 * _spec_sample_accept (src/mlx_dspark/generate.py:659-688). Row i < T-1 of block b accepts
 * draft x = verify_ids[b, i+1] iff u < min(1, p_i[x] / max(q_i[x], 1e-9)); the first reject
 * n draws the replacement from norm(max(p_n - q_n, 0)) (uniform over the vocabulary if that is
 * all zero), all accepted draws the bonus from p_{T-1}. Outputs are those of
 * dspark_accept_greedy (plan, pending, kv_len commit) and the call advances rng[b].offset.
 * q_probs: fp32 [B, T-1, ld_q], the distributions the drafts were drawn from (probs of
 *   dspark_sample_rows); q_onehot = 1 takes q_i = one-hot(x_i) instead (lookup drafts,
 *   generate.py:815-824) and q_probs may be NULL.
 * T <= 32, V <= 262144. workspace: dspark_accept_sample_workspace_bytes(B, T), zero-filled
 * once before first use (the call leaves its counters at zero). */
size_t dspark_accept_sample_workspace_bytes(int B, int T);
int dspark_accept_sample(const void* logits, long long ld, int B, int T, int V,
                         const int32_t* verify_ids, const float* q_probs, long long ld_q,
                         int q_onehot, float temperature, int temp_mode, double top_p, int top_k,
                         unsigned long long* rng, int32_t* kv_len, int commit, int32_t* pending,
                         int32_t* plan, void* workspace, size_t workspace_bytes,
                         dspark_stream_t stream);

/* DSpark temperature draft: DSparkDrafter.sample_block_probs (src/mlx_dspark/model.py:283-309).
 * Sequential over cap positions: logits_i = base_i + w2 . w1[prev] (as in K10), then token i
 * drawn from truncate(softmax(logits_i * bf16(1/T))) with Philox row = i, stream 1.
 * q_probs: out fp32 [B, cap, ld_q] (q_i of each row); draft / verify_ids as in K10.
 * workspace: dspark_markov_probs_workspace_bytes(B, V) (the logits row of each step). */
size_t dspark_markov_probs_workspace_bytes(int B, int V);
int dspark_markov_sample_block_probs(const void* base, int ld, int rows_per_b, int B, int cap,
                                     int V, int R, const uint8_t* w1q, const uint32_t* w1sb,
                                     const uint8_t* w2q, const uint32_t* w2sb,
                                     const int32_t* first_prev, int32_t* draft,
                                     int32_t* verify_ids, float temperature, double top_p,
                                     int top_k, const unsigned long long* rng, float* q_probs,
                                     long long ld_q, void* workspace, size_t workspace_bytes,
                                     dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * R8 — OpenAI presence / frequency penalties (_Penalizer, src/mlx_dspark/generate.py:179-228).
 * dspark_apply_penalties subtracts, in place, from row i of each verify block b (bf16 logits
 * [B*T, ld]) the penalty of the completion counts counts[b, V] plus the block's draft prefix
 * verify_ids[b, 1..i]: presence once per token, frequency per occurrence, in MLX's bf16
 * arithmetic (block_penalty / apply, generate.py:202-228). verify_ids may be NULL when T == 1.
 * dspark_penalty_counts_add adds the committed tokens plan[b, 2 .. 2 + plan[b, 1]) to
 * counts[b] (pen.add, generate.py:941-949). T <= 64. */
int dspark_apply_penalties(void* logits, long long ld, int B, int T, int V, const int32_t* counts,
                           const int32_t* verify_ids, double presence, double frequency,
                           dspark_stream_t stream);
int dspark_penalty_counts_add(int32_t* counts, int B, int V, const int32_t* plan, int plan_stride,
                              dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * Length-only commit: len_a[b] += plan[b*plan_stride + 1] (and len_b, if given). Used after
 * the drafter context update so both consumers read the pre-commit length first.
 * Replaces the trims of src/mlx_dspark/generate.py:929-938 (target KV) and the
 * n_cached bookkeeping of :938.
 * ------------------------------------------------------------------------------------- */
int dspark_commit_lengths(const int32_t* plan, int plan_stride, int B, int32_t* len_a,
                          int32_t* len_b, dspark_stream_t stream);

/* -------------------------------------------------------------------------------------
 * Benchmark draft override (BASELINE configs with a Bernoulli(0.7) agree mask): draft slot i
 * of row b becomes ref[b][j] where agree[b][round][i] != 0, else (ref[b][j] + 1) mod V, with
 * j = kv_len[b] - prompt_len[b] + 1 + i; round_ctr[b] is incremented on the device.
 * No reference counterpart (benchmark harness only); writes verify_ids[b, 1 + i].
 * ------------------------------------------------------------------------------------- */
int dspark_draft_override(int B, int cap, int V, const int32_t* ref, int ref_len,
                          const uint8_t* agree, int rounds, int32_t* round_ctr,
                          const int32_t* kv_len, const int32_t* prompt_len, int32_t* verify_ids,
                          dspark_stream_t stream);

/* Row argmax, first index of the maximum (mx.argmax): the greedy draft of a block drafter
 * without a sequential head — DFlash (src/mlx_dspark/generate.py:564) and sample_block without
 * a Markov head (model.py:272-273). Token of row r -> tokens[r * tok_stride] and, if given,
 * tokens2[r * tok2_stride]. */
int dspark_argmax_rows(const void* logits, long long ld, int rows, int V, int32_t* tokens,
                       int tok_stride, int32_t* tokens2, int tok2_stride, float* values,
                       int index_offset, dspark_stream_t stream);

/* Per-token logprobs of committed tokens (_logprobs_for_block, src/mlx_dspark/generate.py:149-176):
 * the raw log-softmax of each row, logp = x - max(x) - log(sum(exp(x - max(x)))) in fp32.
 * Row r's token is ids[(r / T) * ids_ld + r % T] (a plan row's committed tokens: ids = plan + 2,
 * ids_ld = T + 2); logp[r] = its entry, NaN for a token outside [0, V). With top_k > 0 the
 * min(top_k, V) largest entries go to top_ids / top_logp [rows, top_k] in descending order,
 * equal values by smaller index. top_k <= 1024. One CTA per row. */
int dspark_logprobs(const void* logits, long long ld, int rows, int V, const int32_t* ids,
                    int ids_ld, int T, int top_k, float* logp, int32_t* top_ids, float* top_logp,
                    dspark_stream_t stream);

/* DSpark confidence head (ConfidenceHead, src/mlx_dspark/model.py:211-217; confidence_logits
 * :311-320): per row i of hidden [rows, H] (bf16, row pitch ld), logit[i] = bf16(proj_w .
 * [norm(h_i), w1[prev_i]] + proj_b) and conf[i] = bf16(sigmoid(logit[i])), the survival
 * probabilities speculative_generate truncates a draft with (generate.py:875-885).
 * norm_w non-null: the rows are the backbone's pre-norm hidden states and norm(h) =
 * bf16(h * rsqrt(mean(h^2) + eps) * norm_w); null: the rows are already normalised.
 * w1q / w1sb (the packed Markov w1, [V, R] codes and [R/64, V] fp16 scale|bias words) non-null:
 * the features also hold bf16(dequant w1[prev_i]), prev_0 = first_prev[0] and prev_i =
 * prev_rest[i - 1]; proj_w is bf16 [H + R] (R a multiple of 64), else bf16 [H]. proj_b is
 * bf16 [1]. logit may be null. One CTA per row. */
int dspark_confidence(const void* hidden, long long ld, int rows, int H, const void* norm_w,
                      float eps, const uint8_t* w1q, const uint32_t* w1sb, int V, int R,
                      const int32_t* first_prev, const int32_t* prev_rest, const void* proj_w,
                      const void* proj_b, float* logit, float* conf, dspark_stream_t stream);

/* Tensor-parallel pieces (BASELINE C5: Qwen3-32B at TP 2/4/8; NCCL all-reduce after o_proj
 * and down_proj). The reference runs on one device and has no counterpart; they stand in for
 * its single-device o_proj / down_proj residual adds and the lm_head argmax.
 * dspark_residual_add_f32: h = bf16(h + bf16(sum)) — the RESIDUAL_BF16 epilogue applied after
 *   the fp32 partials of a row-split projection were all-reduced.
 * dspark_accept_greedy_sharded: greedy acceptance when each of `shards` ranks holds a vocabulary
 *   slice: values / indices [shards, B*T] are every shard's row maximum and its global index
 *   (dspark_argmax_rows with values and index_offset); the row argmax is the largest value,
 *   ties to the smallest index; outputs as dspark_accept_greedy. T <= 64. */
int dspark_residual_add_f32(void* h, int ldh, const float* sum, int lds, int M, int N,
                            dspark_stream_t stream);
int dspark_accept_greedy_sharded(const float* values, const int32_t* indices, int shards, int B,
                                 int T, const int32_t* verify_ids, int32_t* kv_len, int commit,
                                 int32_t* pending, int32_t* plan, dspark_stream_t stream);

/* drafter block embedding: row b*k + i embeds pending[b] if i == 0 else mask_id
 * (src/mlx_dspark/generate.py:848-849, batch_engine.py:548-549); ids_out optional [B*k] */
int dspark_embed_block_w8(const int32_t* pending, int B, int k, int mask_id, const uint8_t* wq,
                          const uint32_t* wsb, int V, int H, void* out, int ldo, int32_t* ids_out,
                          dspark_stream_t stream);

/* bf16 -> fp16 copy of a [rows, cols] block: the target hidden-state tap written into the
 * fp16 fused-context GEMM input (src/mlx_dspark/target.py:66-69,75) */
int dspark_bf16_to_f16(const void* src, int lds, void* dst, int ldd, int rows, int cols,
                       int* status, dspark_stream_t stream);  /* DSPARK_ERR_RANGE past fp16 */

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* DSPARK_B200_H_ */
