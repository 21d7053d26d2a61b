/*
 * hx_gemm.h — C ABI of the B200 (sm_100a) linear-layer GEMM library.
 *
 * This is the native boundary that replaces the reference's kernel ABIs for
 * the tiled linear-layer matmul (linalg.matmul + its elementwise
 * linalg.generic epilogue):
 *
 *   - the HexKL library call
 *       int hexkl_matmul_f16f16_f32(int64_t n_row, int64_t n_col,
 *                                   int64_t n_inner, float *out,
 *                                   const _Float16 *act, const _Float16 *W)
 *     (qcom_hexagon_backend/bin/runtime/src/HexKLAPI.cpp:15-17,
 *      include/HexKLAPI.h), replaced by hx_matmul_f16f16_f32();
 *   - the MLIR memref-descriptor kernel ABI that the launcher wrappers call
 *     (qcom_hexagon_backend/backend/triton_hexagon_launcher.py:158-168,
 *      torch_mlir_hexagon_launcher.py:68-88), and the `library_call`
 *     escape hatch `_mlir_ciface_<fn>`
 *     (lib/Transforms/ReplaceWithLibraryCallsPass.cpp:85-141),
 *     both replaced by the descriptor call hx_gemm().
 *
 * Conventions (all entry points):
 *   - The caller owns every buffer.  Pointers are device pointers unless the
 *     name says host.  Nothing is allocated per call; the library keeps only
 *     a per-device cache of the SM count and the driver's tensor-map encoder.
 *   - Calls are asynchronous and ordered on the given CUDA stream
 *     (cudaStream_t passed as void*; NULL = legacy default stream).
 *   - Return value: HX_OK (0) or a negative HX_E_* code.  No call aborts or
 *     exits the process.  hx_status_str() names a code.
 *   - Row-major everywhere: A[M,K] (lda), C[M,N] (ldc).  B is either the
 *     nn.Linear weight layout W[N,K] (HX_B_NK, the "matmul_transpose_b" form
 *     the reference folds transpose+matmul into,
 *     lib/Transforms/ScheduleMatmulForHVXPass.cpp:84-93) or B[K,N] (HX_B_KN,
 *     plain linalg.matmul / tl.dot).
 */
#ifndef HX_GEMM_H
#define HX_GEMM_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define HX_OK 0
#define HX_E_INVALID_ARG -1   /* null pointer, negative size, bad enum      */
#define HX_E_UNSUPPORTED -2   /* dtype / layout / epilogue combination       */
#define HX_E_CUDA -3          /* a CUDA runtime or driver call failed        */
#define HX_E_TIMEOUT -4       /* a bounded device wait ran out (see below)   */
#define HX_E_NCCL -5          /* an NCCL call failed                         */
#define HX_E_NO_DEVICE -6     /* no sm_100 device is current                 */
#define HX_E_TOO_LARGE -7     /* size beyond a documented fixed limit        */

/* ---- element types ------------------------------------------------------ */
#define HX_F16 0
#define HX_BF16 1
#define HX_S8 2
#define HX_S32 3
#define HX_F32 4

/* ---- B operand layout --------------------------------------------------- */
#define HX_B_NK 0 /* B stored as W[N,K] row-major (nn.Linear weight)          */
#define HX_B_KN 1 /* B stored as B[K,N] row-major                            */

/* ---- fused epilogues (the linalg.generic ops that follow the matmul) ---- */
#define HX_EPI_NONE 0           /* C = acc                                     */
#define HX_EPI_BIAS 1           /* C = acc + bias[n]                           */
#define HX_EPI_BIAS_GELU_TANH 2 /* C = gelu_tanh(acc + bias[n]); bias optional */
#define HX_EPI_BIAS_RESIDUAL 3  /* C = acc + bias[n] + R[m,n]                  */
#define HX_EPI_RESIDUAL 4       /* C = acc + R[m,n]                            */
#define HX_EPI_SWIGLU 5         /* C = silu(acc_gate) * acc_up; B holds 2N rows:
                                   rows [0,N) gate, rows [N,2N) up (HX_B_NK)   */
#define HX_EPI_DEQUANT_SCALE 6  /* C = acc * scale[n] (+ bias[n] if given)     */
#define HX_EPI_BIAS_SILU 7      /* C = silu(acc + bias[n]); bias optional      */

/* Problem descriptor for hx_gemm().  Zero-initialise and fill what applies. */
typedef struct hx_gemm_desc {
  int64_t M, N, K;         /* C is M x N; for HX_EPI_SWIGLU, B has 2N rows    */
  int32_t a_dtype;         /* HX_F16 | HX_BF16 | HX_S8                        */
  int32_t b_dtype;         /* must equal a_dtype                              */
  int32_t c_dtype;         /* HX_F16 | HX_BF16 | HX_F32 | HX_S32 (S32 only
                              with S8 inputs and HX_EPI_NONE: exact int32)   */
  int32_t b_layout;        /* HX_B_NK | HX_B_KN                               */
  const void *A;
  int64_t lda;             /* elements                                        */
  const void *B;
  int64_t ldb;             /* elements                                        */
  void *C;
  int64_t ldc;             /* elements                                        */
  int32_t epilogue;        /* HX_EPI_*                                        */
  int32_t bias_dtype;      /* dtype of bias[N] (HX_F16 | HX_BF16 | HX_F32)    */
  const void *bias;        /* [N] or NULL                                     */
  const void *residual;    /* [M, N] of c_dtype, or NULL                      */
  int64_t ldr;             /* residual leading dimension, elements            */
  int32_t scale_dtype;     /* dtype of scale[N] (HX_F16 | HX_BF16 | HX_F32)   */
  const void *scale;       /* [N] per-output-channel scale, or NULL           */
  /* Tile override (0 = choose automatically), the analogue of the
     reference's HexagonOptions.tileSizes (backend/hexagon_options.py:75).
     tile_n in {64,96,128,192,256} (96 and 192: B_NK only, 96 not with
     SWIGLU); stages in [2,8]. */
  int32_t tile_n;
  int32_t stages;
  int32_t max_ctas;        /* cap on persistent CTAs (0 = one per SM)         */
  int32_t force_simt;      /* 1 = use the CUDA-core kernel (validation only)  */
  int32_t *error_flag;     /* optional device int32; set non-zero by a kernel
                              whose bounded wait ran out                      */
  uint64_t timeout_cycles; /* bound for each device wait (0 = ~2 s default)   */
  int32_t split_k;         /* CTAs (2..8, one thread-block cluster) sharing a
                              tile's K range, fp32 partials exchanged through
                              an L2 workspace the library owns; 1 = off,
                              0 = automatic                                   */
  int32_t flags;           /* HX_GEMM_* bits below                            */
} hx_gemm_desc;

/* B holds constants (model weights) that no work still running before this
   call in the stream writes: the kernel may fetch its first B tiles before
   waiting for that work (programmatic dependent launch), overlapping the
   previous kernel's tail.  Use only when that holds. */
#define HX_GEMM_B_CONST 1

/* C = epilogue(A . B).  Replaces the linalg.matmul + linalg.generic pair the
   reference compiles through LinalgToLLVMPass
   (lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:188-400) and runs as the
   _mlir_ciface_<fn> entry of the generated .so. */
int hx_gemm(const hx_gemm_desc *d, void *stream);

/* A list of fused GEMMs (a stack of linear layers) as one persistent launch.
   GEMM g may read as A (a_dep[g] >= 0) and/or as its residual (r_dep[g] >= 0)
   the C of an earlier GEMM of the list with the same M; a tile of row block
   m of GEMM g starts as soon as row block m of those producers is complete,
   so consecutive layers overlap instead of running back to back.  f16/bf16,
   W[N,K] layout, 16-byte aligned rows, any epilogue but DEQUANT_SCALE, at
   most 64 GEMMs (HX_E_TOO_LARGE beyond).  `counters` is caller-owned device
   scratch of counters_len int32, at least one per 128-row block of every
   GEMM; this call zeroes them on `stream`.  Output buffers must not alias
   any other GEMM's inputs or outputs of the list.  Replaces the sequence of
   linalg.matmul + linalg.generic ops the reference compiles and runs one by
   one (lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:188-400). */
int hx_gemm_chain(const hx_gemm_desc *descs, const int32_t *a_dep,
                  const int32_t *r_dep, int count, int32_t *counters,
                  int64_t counters_len, int32_t *error_flag, void *stream);

/* HexKL drop-in: out[n_row, n_col] (f32) = act[n_row, n_inner] (f16) .
   W[n_inner, n_col] (f16), fp32 accumulate.  Replaces
   hexkl_matmul_f16f16_f32 (bin/runtime/src/HexKLAPI.cpp:15-17); unlike
   HexKL the accumulator is not rounded to f16 before widening. */
int hx_matmul_f16f16_f32(int64_t n_row, int64_t n_col, int64_t n_inner,
                         float *out, const void *act, const void *W,
                         void *stream);

/* W8A16 skinny-M decode GEMM: y[M,N] (f16) = x[M,K] (f16) . (W[N,K] (s8) *
   scale[N] (f16))^T (+ bias[N] f16 if non-NULL), fp32 accumulate.  The
   reference has no int8 GEMM kernel: it lowers quantised ops to dequantise +
   float matmul (lib/Conversion/LinalgToLLVM/LinalgToLLVMPass.cpp:203-209) and
   reduces unit-M matvec to a dot (lib/Transforms/
   ReduceContractionRankPass.cpp:38-47); this entry replaces that pair. */
int hx_gemv_w8a16(int64_t M, int64_t N, int64_t K, const void *x, int64_t ldx,
                  const int8_t *W, int64_t ldw, const void *scale,
                  const void *bias, void *y, int64_t ldy, void *stream);

/* Flags for hx_gemv_w8a16_ex. */
#define HX_GEMV_WEIGHTS_CONST 1   /* W and scale are constant: nothing still
                                     running before this call in the stream
                                     writes them, so their loads may start
                                     before the previous kernel finishes */
#define HX_GEMV_FORCE_CUDA_CORE 2 /* use the CUDA-core kernel (validation) */

/* hx_gemv_w8a16 with flags (same reference counterpart).  M <= 256 with
   16-byte aligned rows runs on the tensor cores (swap-AB, split-K over a
   thread-block cluster); other shapes on CUDA cores. */
int hx_gemv_w8a16_ex(int64_t M, int64_t N, int64_t K, const void *x,
                     int64_t ldx, const int8_t *W, int64_t ldw,
                     const void *scale, const void *bias, void *y,
                     int64_t ldy, int flags, void *stream);

/* One projection of a grouped W8A16 launch: y[M,N] = x[M,K] . (W[N,K] *
   scale[N])^T (+ bias[N]); all f16 except W (s8).  `dep` names an earlier
   projection of the same launch whose y is this projection's x (the launch
   orders them), or -1.  No y may alias another projection's x or y except
   through such a dependency. */
typedef struct hx_w8a16_proj {
  int64_t N, K;
  const void *x;
  int64_t ldx;
  const int8_t *W;
  int64_t ldw;
  const void *scale;
  const void *bias;
  void *y;
  int64_t ldy;
  int32_t dep;
  int32_t reserved;
} hx_w8a16_proj;

/* Run up to 256 W8A16 projections (a decode step's linears) in one
   persistent launch, M <= 64, K % 16 == 0, 16-byte aligned rows.  Dependent
   projections wait on per-projection completion counters.  Kernel choice
   (every kernel converts int8 -> fp16 exactly and accumulates in fp32):
   M <= 16 with every K a multiple of 64: register-fragment tensor-core MMAs
   fed straight from 128-bit weight loads; else, lists of at most 156
   projections whose K are all multiples of 128: tcgen05 UMMA with the
   converted weights in TMEM; other lists, which must then have M <= 8, run
   on CUDA cores.  `counters` is caller-owned device scratch of `count`
   int32, zeroed by this call (cudaMemsetAsync on the stream); the first
   kernel also uses the last entry, which no projection signals, as its work
   ticket.  Same per-projection arithmetic as hx_gemv_w8a16 (reference:
   dequantise + matmul, LinalgToLLVMPass.cpp:203-209); the grouping itself
   has no reference counterpart. */
int hx_gemv_w8a16_grouped(int64_t M, int count, const hx_w8a16_proj *projs,
                          int32_t *counters, int32_t *error_flag, void *stream);

/* Same as hx_gemv_w8a16_grouped, for callers that cannot allocate device
   memory: no counters argument, and no cudaMalloc/cudaFree or allocating
   library call anywhere in it.  Such callers include serving engines whose
   memory pool owns the whole GPU from start-up, latency-critical decode loops
   where an allocation could synchronise the device, and hosts that reach
   this library through a foreign-function interface and only hand it
   pointers they already own.  The per-projection counters live instead in
   a fixed device array of this library (256 int32 = 1 KB per GPU, kept until
   the process exits), so `count` may be at most 256; larger counts return
   HX_E_TOO_LARGE.  The first call on each device looks up that array's
   device address (with the device current), so make the first call before
   any stream capture.  Each call zeroes the counters on `stream` before its
   launch; all calls share the one array, so calls that can overlap on the
   GPU (different streams, or the same array used from several threads at
   once) race and must be serialised by the caller.  This entry point has no
   counterpart in the reference. */
int hx_gemv_w8a16_grouped_noalloc(int64_t M, int count,
                                  const hx_w8a16_proj *projs,
                                  int32_t *error_flag, void *stream);

/* Column-sharded GEMM followed by an all-gather of the output over NCCL.
   Rank r holds its shard of the weight, B rows [r*Ns, (r+1)*Ns) (HX_B_NK),
   with Ns = d->N, and computes C_r = epilogue(A . B_r^T) into d->C
   ([M, Ns], ldc must equal Ns for the gather).  The gather then fills
   gathered[world][M][Ns] (rank-major, c_dtype) on every rank;
   hx_shards_to_rows() turns that into the row-major logits [M, world*Ns].
   Pass gathered = NULL to keep the output vocab-parallel.  `comm` comes from
   hx_nccl_comm_init.  The reference has no multi-device path; this is the
   N-sharding the B200 build adds. */
int hx_sharded_gemm_allgather(const hx_gemm_desc *d, int rank, int world,
                              void *comm, void *gathered, void *stream);

/* Fused column-sharded GEMM + all-gather over NVLink (no NCCL): the GEMM's
   epilogue stores every output chunk of this rank's shard both into its own
   buffer and, with plain stores through peer pointers, into every other
   rank's, so the gather overlaps the math tile by tile.  gathered[r] is rank
   r's [world][M][N] buffer (N = this shard's width, ldc == N), flags[r] its
   array of `world` int32 (both from hx_peer_alloc, opened on the other ranks
   with hx_peer_open); this rank's shard lands at gathered[r][rank] on every r.
   A bounded flag barrier runs before (peers may be overwritten) and after
   (all peers' shards arrived); `epoch` must count 0, 1, 2, ... across calls
   on one set of buffers, and every rank must make the same calls.  A barrier
   that times out sets *error_flag (41) instead of hanging.  W[N,K] layout,
   K > 0, 16-byte aligned rows; at most 8 ranks.  Reference: none (the
   reference has no multi-device path; this replaces GEMM + NCCL all-gather). */
int hx_sharded_gemm_gather_p2p(const hx_gemm_desc *d, int rank, int world, void *const *gathered,
                               int32_t *const *flags, int32_t epoch, int32_t *error_flag,
                               void *stream);

/* Batched GEMM: `batch` independent products with the descriptor's sizes,
   dtypes, layout and epilogue; item i reads A + i*stride_a, B + i*stride_b
   (and residual + i*stride_r) and writes C + i*stride_c, strides in
   elements.  stride_b = 0 shares one B across the items (bias is always
   shared).  This is linalg.batch_matmul (B[K,N] items, HX_B_KN) and
   batch_matmul_transpose_b (B[N,K] items, HX_B_NK), the two forms
   ScheduleMatmulForHVXPass.cpp:105-167 produces for batched contractions.
   Items whose M is a multiple of 128, with C (and the residual) items back to
   back (stride_c == M*ldc), run as one persistent launch over every item's
   tiles; other shapes run item by item.  SWIGLU is not accepted. */
int hx_gemm_batched(const hx_gemm_desc *d, int64_t batch, int64_t stride_a, int64_t stride_b,
                    int64_t stride_c, int64_t stride_r, void *stream);

/* ---- convolution as an implicit GEMM ----------------------------------- */

/* 2-D convolution, NHWC activations and OHWI filters (channels innermost):
     y[n, oh, ow, o] = epilogue( sum_{kh, kw, c} x[n, oh*sh + kh*dh - ph, ow*sw + kw*dw - pw, c]
                                                 * w[o, kh, kw, c] )
   with zero padding.  As a GEMM: M = N*OH*OW output pixels, N = OC,
   K = KH*KW*C, B = w as W[OC, KH*KW*C].  Reference: MatmulToConvPass.cpp
   (the reverse mapping, matmul -> conv_2d_nhwc_fhwc) and the HMX conv path
   exercised by benchmark_models/micro_bench/test_conv_benchmark.py. */
typedef struct hx_conv2d_desc {
  int64_t N, H, W, C;        /* input [N, H, W, C]                             */
  int64_t OC, KH, KW;        /* filters [OC, KH, KW, C]                        */
  int32_t stride_h, stride_w, pad_h, pad_w, dil_h, dil_w;
  int32_t dtype;             /* HX_F16 or HX_BF16, for x, w and y              */
  const void *x;
  const void *w;
  void *y;                   /* [N, OH, OW, OC], OH = (H + 2ph - dh(KH-1) - 1)/sh + 1 */
  const void *bias;          /* [OC] or NULL                                   */
  int32_t bias_dtype;
  int32_t epilogue;          /* HX_EPI_* except SWIGLU / DEQUANT_SCALE         */
  const void *residual;      /* [N, OH, OW, OC] for the residual epilogues     */
  int32_t *error_flag;       /* optional, as in hx_gemm_desc                   */
} hx_conv2d_desc;

/* Bytes of workspace hx_conv2d needs.  0 for the implicit GEMM (stride 1,
   dilation 1, C a multiple of 64, output rows that tile 128-pixel blocks:
   OW divides 128 or is a multiple of it, 128 / OW <= OH, and N == 1 or OH*OW
   a multiple of 128): each K block is then one filter tap x 64 channels, loaded by a 4-D
   TMA box at the tap-shifted coordinates, whose zero fill is the padding.
   Otherwise M * K elements for an explicit im2col matrix. */
int hx_conv2d_workspace_size(const hx_conv2d_desc *d, int64_t *bytes);
int hx_conv2d(const hx_conv2d_desc *d, void *workspace, int64_t workspace_bytes, void *stream);

/* ---- row kernels either side of the linear layer ---------------------- */

/* Softmax over rows of x[M, N] (dtype HX_F16 / HX_BF16 / HX_F32, row stride
   ldx), written to y (y_dtype, row stride ldy): y = exp(x - max) / sum, or the
   log-softmax x - max - log(sum) when log_softmax != 0.  One pass over x when
   a row fits in shared memory (112 KB: N <= 57344 for 16-bit x), else two.  Reference: the row
   softmax of test/python/triton/test_softmax.py and the online (running max,
   rescaled sum) softmax of test/python/triton/test_online_softmax.py. */
int hx_softmax(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, void *y, int y_dtype,
               int64_t ldy, int log_softmax, void *stream);

/* Vocab-parallel softmax, in three steps, for logits split by column across
   ranks (each rank holds x[M, N_local]):
     hx_softmax_stats    per row of the local shard: stats[m] = {max, sum of
                         exp(x - max)} (float pairs, [M][2]);
     (the caller exchanges the [M][2] stats of all ranks: [world][M][2])
     hx_softmax_combine  the global {max, sum} per row from every rank's pair;
     hx_softmax_apply    the local shard's softmax (or log-softmax) with the
                         global pair.
   The logits themselves never cross GPUs. */
int hx_softmax_stats(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, float *stats,
                     void *stream);
int hx_softmax_combine(const float *stats_all, int world, int64_t M, float *stats, void *stream);
int hx_softmax_apply(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, const float *stats,
                     void *y, int y_dtype, int64_t ldy, int log_softmax, void *stream);

/* Row statistics of a normalisation that the next GEMM folds in:
   kind HX_NORM_LAYER: stats[m] = {mean, 1/sqrt(var + eps)} (biased variance,
   F.layer_norm); HX_NORM_RMS: stats[m] = {0, 1/sqrt(mean(x^2) + eps)}
   (F.rms_norm).  Reference: test/python/triton/test_layer_norm.py,
   test_rms_norm.py. */
#define HX_NORM_LAYER 0
#define HX_NORM_RMS 1
int hx_row_norm_stats(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, int kind, float eps,
                      float *stats, void *stream);

/* GEMM of the un-normalised rows of A with a LayerNorm / RMSNorm folded in:
   with gamma and beta folded into the weight beforehand,
     W'[n,k] = W[n,k] * gamma[k],   col_sum[n] = sum_k W'[n,k],
     bias'[n] = bias[n] + sum_k W[n,k] * beta[k]   (LayerNorm),
   the result equals  epilogue(norm(A) . W^T)  as
     acc * rstd[m] - rstd[m] * mean[m] * col_sum[n]   (RMSNorm: acc * rstd[m])
   followed by the descriptor's epilogue with bias'.  d->B is W'; row_stats
   comes from hx_row_norm_stats on A.  SWIGLU: col_sum has 2N entries (gate,
   then up).  The normalised activation is never written to memory.
   Reference: the norm kernels of test/python/triton/test_layer_norm.py and
   test_rms_norm.py, which run as a separate pass before the matmul. */
int hx_gemm_norm(const hx_gemm_desc *d, int kind, const float *row_stats, const float *col_sum,
                 void *stream);

/* The same result as hx_sharded_gemm_gather_p2p, with the transfer on the
   copy engines instead of the GEMM's epilogue: the GEMM runs in `chunks` row
   chunks (0 = automatic: min(6, M/2048); at most 16) on `stream` with every SM, and as each
   chunk completes it is copied (cudaMemcpyAsync, peer-mapped destination)
   into every peer's buffer, one library-owned stream per peer, overlapping
   the next chunk's GEMM.  Entry and exit are the same bounded flag barriers
   (error 41 on timeout); the call returns with `stream` ordered after the
   exit barrier.  Reference: none (no multi-device path in the reference). */
int hx_sharded_gemm_gather_ce(const hx_gemm_desc *d, int rank, int world, void *const *gathered,
                              int32_t *const *flags, int32_t epoch, int32_t *error_flag, int chunks,
                              void *stream);

/* Device memory other processes' GPUs can map: cudaMalloc'ed and zeroed on the
   current device, exported as a CUDA IPC handle of hx_peer_handle_size()
   bytes.  hx_peer_open maps a peer's handle into this process (peer access
   over NVLink); hx_peer_close / hx_peer_free release them. */
int hx_peer_handle_size(void);
int hx_peer_alloc(int64_t bytes, void **dev_ptr, void *ipc_handle);
int hx_peer_open(const void *ipc_handle, void **peer_ptr);
int hx_peer_close(void *peer_ptr);
int hx_peer_free(void *dev_ptr);

/* dst[M, world*Ns] = concat over r of src[r][M][Ns] along columns
   (elem_bytes per element). */
int hx_shards_to_rows(const void *src, void *dst, int world, int64_t M,
                      int64_t shard_cols, int elem_bytes, void *stream);

/* NCCL communicator plumbing for hx_sharded_gemm_allgather.  The unique id
   is an opaque blob of hx_nccl_unique_id_size() bytes that rank 0 creates
   and the host sends to every rank (e.g. through torch.distributed). */
int hx_nccl_unique_id_size(void);
int hx_nccl_get_unique_id(void *id_out);
int hx_nccl_comm_init(void **comm_out, int world, const void *id, int rank);
int hx_nccl_comm_destroy(void *comm);

/* Scratch bytes a call with this descriptor needs FROM THE CALLER: always 0.
   Split-K plans (explicit split_k, or the planner's automatic choice) use a
   reduction workspace that the library itself allocates with cudaMalloc on
   first use, one per (device, stream), grown on demand and kept until exit;
   a call made during stream capture that would need to grow it runs unsplit
   instead.  Callers that must not allocate set split_k = 1 (or use the
   allocation-free entry points). */
int hx_query_workspace(const hx_gemm_desc *d, int64_t *bytes);

/* Human-readable name of a status code. */
const char *hx_status_str(int status);

/* Last CUDA error text recorded by this thread's failing call, or "". */
const char *hx_last_error(void);

/* Library version, for the Python loader's sanity check. */
int hx_version(void);

#ifdef __cplusplus
}
#endif

#endif /* HX_GEMM_H */
