// hx_gemm.cu — host side of the C ABI declared in include/hx_gemm.h.
//
// Validation, tile selection (the analogue of the reference's
// VTCMTilingOptions::determineTileSizes, lib/Conversion/LinalgToLLVM/
// VTCMTilingOptions.cpp:374-432, re-targeted from a 2 MB VTCM budget to
// 227 KB of shared memory and 512 TMEM columns per SM), TMA descriptor
// encoding and kernel launch.  Every entry returns a status code; nothing
// aborts, and nothing is allocated per call.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "gemm_chain.cuh"
#include "launch.cuh"
#include "gemm_simt.cuh"
#include "gemm_sm100.cuh"
#include "gemv_grouped.cuh"
#include "gemv_grouped_tc.cuh"
#include "gemv_grouped_mma.cuh"
#include "gemv_w8a16.cuh"
#include "w8a16_sm100.cuh"
#include "hx_gemm.h"

#define HX_VERSION 1

namespace hx {
thread_local std::string g_last_error;
namespace {


// ------------------------------------------------------------ device cache
struct DeviceInfo {
  std::atomic<int> sms{0};
  std::atomic<int> major{0};
};
DeviceInfo g_dev[64];

int current_device_info(int *sms, int *major) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return arg_fail("device index out of range");
  int s = g_dev[dev].sms.load(std::memory_order_acquire);
  if (s == 0) {
    int v = 0, mj = 0;
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SMs)");
    e = cudaDeviceGetAttribute(&mj, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(cc)");
    g_dev[dev].major.store(mj, std::memory_order_relaxed);
    g_dev[dev].sms.store(v, std::memory_order_release);
    s = v;
  }
  *sms = s;
  *major = g_dev[dev].major.load(std::memory_order_relaxed);
  return HX_OK;
}

// ------------------------------------------------------------ TMA encode
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  std::call_once(g_encode_once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// 2-D row-major tensor: `inner` contiguous elements per row, `outer` rows.
int make_tmap(CUtensorMap *map, const void *ptr, int dtype, uint64_t inner, uint64_t outer,
              uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer) {
  auto enc = get_encode();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return HX_E_CUDA;
  }
  CUtensorMapDataType dt;
  uint64_t esz;
  switch (dtype) {
    case HX_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; esz = 2; break;
    case HX_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; esz = 2; break;
    case HX_S8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; esz = 1; break;
    default: return unsupported("tensor map dtype");
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * esz};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled failed (code " + std::to_string(int(r)) + ")";
    return HX_E_UNSUPPORTED;
  }
  return HX_OK;
}

// 3-D view of a row-major matrix for multi-block K loads: x = `inner`
// elements of one 128-byte K block, y = row, z = K block (stride 128 bytes).
// Requires K to be a whole number of blocks (no tail inside a block).
int make_tmap3(CUtensorMap *map, const void *ptr, int dtype, uint64_t inner, uint64_t rows,
               uint64_t kblocks, uint64_t row_stride_elems, uint32_t box_rows, uint32_t box_kb) {
  auto enc = get_encode();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return HX_E_CUDA;
  }
  CUtensorMapDataType dt;
  uint64_t esz;
  switch (dtype) {
    case HX_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; esz = 2; break;
    case HX_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; esz = 2; break;
    case HX_S8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; esz = 1; break;
    default: return unsupported("tensor map dtype");
  }
  cuuint64_t dims[3] = {inner, rows, kblocks};
  cuuint64_t strides[2] = {row_stride_elems * esz, inner * esz};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(inner), box_rows, box_kb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string(int(r)) + ")";
    return HX_E_UNSUPPORTED;
  }
  return HX_OK;
}

// 3-D view for batched GEMMs: x = inner (contiguous), y = rows, z = batch
// item; byte strides of a row and of an item; box {box_x, box_y, 1}.
int make_tmap_batched(CUtensorMap *map, const void *ptr, int dtype, uint64_t inner, uint64_t rows,
                      uint64_t items, uint64_t row_stride_bytes, uint64_t item_stride_bytes,
                      uint32_t box_x, uint32_t box_y) {
  auto enc = get_encode();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return HX_E_CUDA;
  }
  CUtensorMapDataType dt;
  switch (dtype) {
    case HX_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case HX_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    case HX_S8: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    default: return unsupported("tensor map dtype");
  }
  cuuint64_t dims[3] = {inner, rows, items};
  cuuint64_t strides[2] = {row_stride_bytes, item_stride_bytes};
  cuuint32_t box[3] = {box_x, box_y, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled (batched) failed (code " + std::to_string(int(r)) + ")";
    return HX_E_UNSUPPORTED;
  }
  return HX_OK;
}

// 4-D view of NHWC activations for the implicit-GEMM convolution:
// {C, W, H, N}, box {64 channels (128 bytes), bw, bh, 1}.
int make_tmap_conv(CUtensorMap *map, const void *ptr, int dtype, uint64_t N, uint64_t H, uint64_t W,
                   uint64_t C, uint32_t box_c, uint32_t bw, uint32_t bh) {
  auto enc = get_encode();
  if (!enc) {
    g_last_error = "cuTensorMapEncodeTiled unavailable";
    return HX_E_CUDA;
  }
  CUtensorMapDataType dt;
  switch (dtype) {
    case HX_F16: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16; break;
    case HX_BF16: dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; break;
    default: return unsupported("convolution dtype");
  }
  const uint64_t ez = 2;
  cuuint64_t dims[4] = {C, W, H, N};
  cuuint64_t strides[3] = {C * ez, W * C * ez, H * W * C * ez};
  cuuint32_t box[4] = {box_c, bw, bh, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, const_cast<void *>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    g_last_error = "cuTensorMapEncodeTiled (conv) failed (code " + std::to_string(int(r)) + ")";
    return HX_E_UNSUPPORTED;
  }
  return HX_OK;
}

int esize(int dtype) {
  switch (dtype) {
    case HX_F16:
    case HX_BF16: return 2;
    case HX_S8: return 1;
    case HX_S32:
    case HX_F32: return 4;
    default: return 0;
  }
}
__host__ __device__ inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }


// ------------------------------------------------------------ launch
// launch_pdl and the tile-GEMM launchers live in launch.cuh; the kernels are
// instantiated per input kind in gemm_kind{0,1,2}.cu (compiled in parallel).
// ------------------------------------------------------------ split-K workspace
// Split-K partials travel through L2 in a device buffer the library owns, one
// per (device, stream) so concurrent streams never share one.  It grows on
// demand outside stream capture; during capture a call that would need a
// larger buffer runs unsplit instead.
struct SplitWorkspace {
  int dev;
  cudaStream_t stream;
  void *ptr;
  size_t bytes;
};
std::mutex g_ws_mu;
std::vector<SplitWorkspace> g_ws;

int split_workspace(size_t need, cudaStream_t s, uint4 **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_ws_mu);
  SplitWorkspace *w = nullptr;
  for (auto &x : g_ws)
    if (x.dev == dev && x.stream == s) w = &x;
  if (w && w->bytes >= need) {
    *out = static_cast<uint4 *>(w->ptr);
    return HX_OK;
  }
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &st);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  if (st != cudaStreamCaptureStatusNone) return kNeedsNoSplit;
  const size_t bytes = std::max<size_t>(need, size_t(16) << 20);
  void *p = nullptr;
  e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return kNeedsNoSplit;
  }
  if (w) {
    // cudaFree waits for work still using the old buffer
    e = cudaFree(w->ptr);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFree(split workspace)");
    w->ptr = p;
    w->bytes = bytes;
  } else {
    g_ws.push_back({dev, s, p, bytes});
  }
  *out = static_cast<uint4 *>(p);
  return HX_OK;
}

int stage_bytes(int bn) { return kBM * kKBytes + bn * kKBytes; }

// Tile plan: width BN (and, only when the caller asks, a split-K factor S).
// Cost model calibrated on B200 measurements of the benchmark shapes: a
// launch costs ~7 us of fixed latency (prologue, first loads, epilogue,
// drain), after which each CTA streams its tiles' K blocks at ~100 GB/s of
// TMA ingest (or the tensor rate, if slower); persistent CTAs overlap the
// fixed part across waves.  Split-K adds ~3.5 us for the exchange of fp32
// partials through L2 and the reduction.
inline bool best_cost_found(double c) { return c < 1e299; }

void plan_tiles(int64_t M, int64_t N, int64_t K, int ez, bool swiglu, bool bmn, int sms, int &bn,
                int &splits, int split_req) {
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  const int64_t k_blocks = (K * ez + kKBytes - 1) / kKBytes;
  const double flop_per_us_sm = 10.9e6 * (ez == 1 ? 2.0 : 1.0);
  // best plan without split-K, and best with it
  double best1 = 1e300, bestS = 1e300;
  int bn1 = bn ? bn : 128, bnS = bn1, sS = 1;
  for (int b : {256, 192, 128, 96, 64}) {
    if (bn && b != bn) continue;
    if (bmn && ez == 1 && b < 128) continue;
    if ((b == 96 || b == 192) && (bmn || (swiglu && b == 96))) continue;
    const int out_w = swiglu ? b / 2 : b;
    const int64_t tiles = m_tiles * ((N + out_w - 1) / out_w);
    for (int sp : {1, 2, 3, 4, 6, 8}) {
      // auto: 1, 2 or 4 CTAs per cluster (clusters of 3, 6 and 8 pack poorly)
      if (split_req == 0 ? (sp == 3 || sp > 4) : sp != split_req) continue;
      if (sp > 1 && (bmn || tiles * sp > sms || sp > k_blocks)) continue;
      const int64_t waves = (tiles * sp + sms - 1) / sms;
      const double kb = static_cast<double>((k_blocks + sp - 1) / sp);
      const double ingest = kb * stage_bytes(b) / 100e3;
      const double mma = kb * (2.0 * kBM * b * (kKBytes / ez)) / flop_per_us_sm;
      const double cost = 7.0 + waves * std::max(ingest, mma) + (sp > 1 ? 3.5 : 0.0);
      double &best = sp > 1 ? bestS : best1;
      if (cost < best * 0.97) {  // prefer the earlier (wider) option on near ties
        best = cost;
        if (sp > 1) {
          bnS = b;
          sS = sp;
        } else {
          bn1 = b;
        }
      }
    }
  }
  // Auto plans split only for a large predicted gain: measured inside CUDA
  // graphs, smaller predicted gains did not hold up.
  const bool take_split = best_cost_found(bestS) &&
                          (split_req > 1 || !best_cost_found(best1) || bestS < 0.85 * best1);
  if (take_split) {
    bn = bnS;
    splits = sS;
  } else if (best_cost_found(best1)) {
    bn = bn1;
    splits = 1;
  } else {  // no feasible plan: let the caller's checks report why
    bn = bn1;
    splits = split_req > 1 ? split_req : 1;
  }
}

int validate(const hx_gemm_desc *d) {
  if (!d) return arg_fail("null descriptor");
  if (d->M < 0 || d->N < 0 || d->K < 0) return arg_fail("negative size");
  if (d->M > INT32_MAX || d->N > INT32_MAX / 2 || d->K > INT32_MAX)
    return unsupported("size beyond int32 range");
  if (d->a_dtype != d->b_dtype) return unsupported("A and B dtypes differ");
  if (d->a_dtype != HX_F16 && d->a_dtype != HX_BF16 && d->a_dtype != HX_S8)
    return unsupported("A/B dtype");
  const bool is_int = d->a_dtype == HX_S8;
  switch (d->c_dtype) {
    case HX_F16:
    case HX_BF16:
    case HX_F32: break;
    case HX_S32:
      if (!is_int || d->epilogue != HX_EPI_NONE)
        return unsupported("int32 output needs int8 inputs and no epilogue");
      break;
    default: return unsupported("C dtype");
  }
  if (d->b_layout != HX_B_NK && d->b_layout != HX_B_KN) return arg_fail("b_layout");
  if (d->flags & ~HX_GEMM_B_CONST) return arg_fail("unknown flags bits");
  if (d->M == 0 || d->N == 0) return HX_OK;
  if (!d->C || (d->K > 0 && (!d->A || !d->B))) return arg_fail("null A/B/C");
  if (d->lda < std::max<int64_t>(d->K, 1)) return arg_fail("lda < K");
  if (d->b_layout == HX_B_NK && d->ldb < std::max<int64_t>(d->K, 1)) return arg_fail("ldb < K");
  if (d->b_layout == HX_B_KN && d->ldb < d->N) return arg_fail("ldb < N");
  if (d->ldc < d->N) return arg_fail("ldc < N");
  switch (d->epilogue) {
    case HX_EPI_NONE: break;
    case HX_EPI_BIAS:
      if (!d->bias) return arg_fail("epilogue needs bias");
      break;
    case HX_EPI_BIAS_GELU_TANH:
    case HX_EPI_BIAS_SILU:
      break;  // bias optional (NULL = no bias)
    case HX_EPI_BIAS_RESIDUAL:
      if (!d->bias || !d->residual) return arg_fail("epilogue needs bias and residual");
      if (d->ldr < d->N) return arg_fail("ldr < N");
      break;
    case HX_EPI_RESIDUAL:
      if (!d->residual) return arg_fail("epilogue needs residual");
      if (d->ldr < d->N) return arg_fail("ldr < N");
      break;
    case HX_EPI_SWIGLU:
      if (d->b_layout != HX_B_NK) return unsupported("SWIGLU needs the W[N,K] layout");
      if (is_int) return unsupported("SWIGLU with int8 inputs");
      break;
    case HX_EPI_DEQUANT_SCALE:
      if (!d->scale) return arg_fail("epilogue needs scale");
      break;
    default: return arg_fail("epilogue");
  }
  if (d->bias && esize(d->bias_dtype) == 0) return arg_fail("bias dtype");
  if (d->bias && d->bias_dtype == HX_S8) return arg_fail("bias dtype");
  if (d->scale && (esize(d->scale_dtype) == 0 || d->scale_dtype == HX_S8))
    return arg_fail("scale dtype");
  if (d->residual && d->residual == d->C && d->ldr != d->ldc)
    return arg_fail("in-place residual needs ldr == ldc");
  return HX_OK;
}

EpiArgs make_epi(const hx_gemm_desc *d) {
  EpiArgs e;
  e.n_peers = 0;
  for (int i = 0; i < 7; ++i) e.peer_C[i] = nullptr;
  e.norm = 0;
  e.row_stats = nullptr;
  e.col_sum = nullptr;
  e.C = d->C;
  e.ldc = d->ldc;
  e.bias = d->bias;
  e.residual = d->residual;
  e.ldr = d->ldr;
  e.scale = d->scale;
  e.c_dtype = d->c_dtype;
  e.bias_dtype = d->bias_dtype;
  e.scale_dtype = d->scale_dtype;
  e.epi = d->epilogue;
  e.M = static_cast<int32_t>(d->M);
  e.N = static_cast<int32_t>(d->N);
  const int cz = esize(d->c_dtype);
  e.c_vec_ok = aligned16(d->C) && ((d->ldc * cz) % 16 == 0);
  e.r_vec_ok = d->residual && aligned16(d->residual) && ((d->ldr * cz) % 16 == 0);
  e.b_vec_ok = d->bias && aligned16(d->bias);
  e.s_vec_ok = d->scale && aligned16(d->scale);
  auto is16 = [](int t) { return t == HX_F16 || t == HX_BF16; };
  const int epi = d->epilogue;
  const bool uses_scale = (epi == HX_EPI_DEQUANT_SCALE);
  const bool uses_bias = d->bias && epi != HX_EPI_NONE && epi != HX_EPI_RESIDUAL && epi != HX_EPI_SWIGLU;
  const bool uses_res = (epi == HX_EPI_BIAS_RESIDUAL || epi == HX_EPI_RESIDUAL);
  e.pre16 = (!uses_scale || (is16(d->scale_dtype) && e.s_vec_ok)) &&
            (!uses_bias || (is16(d->bias_dtype) && e.b_vec_ok)) &&
            (!uses_res || (is16(d->c_dtype) && e.r_vec_ok));
  return e;
}

// A row normalisation folded into the GEMM (hx_gemm_norm).
struct NormSpec {
  int kind;
  const float *row_stats, *col_sum;
};

int run_simt(const hx_gemm_desc *d, cudaStream_t s, const NormSpec *ns = nullptr) {
  SimtParams p;
  p.M = static_cast<int32_t>(d->M);
  p.N = static_cast<int32_t>(d->N);
  p.K = static_cast<int32_t>(d->K);
  p.A = d->A;
  p.lda = d->lda;
  p.B = d->B;
  p.ldb = d->ldb;
  p.ab_dtype = d->a_dtype;
  p.b_kn = d->b_layout == HX_B_KN;
  p.n_half = static_cast<int32_t>(d->N);
  p.epi = make_epi(d);
  if (ns) {
    p.epi.norm = 1 + ns->kind;
    p.epi.row_stats = ns->row_stats;
    p.epi.col_sum = ns->col_sum;
  }
  dim3 grid((p.N + kSimtTile - 1) / kSimtTile, (p.M + kSimtTile - 1) / kSimtTile);
  if (grid.y > 65535) return unsupported("M too large for the CUDA-core kernel");
  const bool sw = d->epilogue == HX_EPI_SWIGLU;
  if (d->a_dtype == HX_S8) {
    hx_gemm_simt_kernel<int, false><<<grid, 256, 0, s>>>(p);
  } else if (sw) {
    hx_gemm_simt_kernel<float, true><<<grid, 256, 0, s>>>(p);
  } else {
    hx_gemm_simt_kernel<float, false><<<grid, 256, 0, s>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemm_simt_kernel launch");
  return HX_OK;
}

// Other GPUs' copies of C for the fused all-gather (hx_sharded_gemm_gather_p2p).
struct PeerTargets {
  int n;
  void *C[7];
};

// Batch items of hx_gemm_batched: count and element strides between items.
struct BatchSpec {
  int64_t count, sa, sb, sc, sr;
};
constexpr int kNeedsLoop = 2;  // internal: the batch is not one launch; run item by item

// The implicit-GEMM convolution's geometry (hx_conv2d): output dims OH x OW,
// box of bw x bh input pixels per 128-row tile.
struct ConvSpec {
  int64_t N, H, W, C, OH, OW, KH, KW;
  int pad_h, pad_w, bw, bh;
};

int gemm_impl(const hx_gemm_desc *d, cudaStream_t s, const PeerTargets *peers = nullptr,
              const BatchSpec *bt = nullptr, const NormSpec *ns = nullptr, const ConvSpec *cv = nullptr) {
  int rc = validate(d);
  if (rc != HX_OK) return rc;
  if (d->M == 0 || d->N == 0) return HX_OK;
  int sms = 0, major = 0;
  rc = current_device_info(&sms, &major);
  if (rc != HX_OK) return rc;
  if (major != 10) {
    g_last_error = "current device is not sm_100";
    return HX_E_NO_DEVICE;
  }
  const int ez = esize(d->a_dtype);
  const bool swiglu = d->epilogue == HX_EPI_SWIGLU;
  const bool bmn = d->b_layout == HX_B_KN;
  const bool tma_ok = !d->force_simt && d->K > 0 && aligned16(d->A) && aligned16(d->B) &&
                      (d->lda * ez) % 16 == 0 && (d->ldb * ez) % 16 == 0;
  // One launch over every batch item when each item's rows are whole tiles
  // and C (and the residual) are items of rows back to back.
  const bool batched = bt != nullptr && bt->count > 1;
  if (cv && !tma_ok) return unsupported("implicit convolution needs 16-byte aligned operands");
  if (batched) {
    const bool one_launch = tma_ok && !swiglu && peers == nullptr && d->M % kBM == 0 &&
                            bt->sc == d->M * d->ldc && (!d->residual || bt->sr == d->M * d->ldr) &&
                            (bt->sa * ez) % 16 == 0 && (bt->sb * ez) % 16 == 0 && d->split_k <= 1 &&
                            bt->sa >= d->M * d->lda && bt->sb >= (bmn ? d->K : d->N) * d->ldb &&
                            bt->count * d->M <= INT32_MAX && bt->count <= 65535;
    if (!one_launch) return kNeedsLoop;
  }
  if (!tma_ok) return run_simt(d, s, ns);

  if (d->split_k < 0 || d->split_k > 8) return arg_fail("split_k must be 0..8");
  int bn = d->tile_n;
  int splits = d->split_k > 0 ? d->split_k : 1;
  if (bmn) splits = 1;  // split-K is built for the W[N,K] path
  if (bn == 0 || d->split_k == 0) {
    plan_tiles(batched ? d->M * bt->count : d->M, d->N, d->K, ez, swiglu, bmn, sms, bn, splits,
               batched ? 1 : d->split_k);
  }
  if (batched || cv) splits = 1;
  if (bn != 64 && bn != 96 && bn != 128 && bn != 192 && bn != 256)
    return arg_fail("tile_n must be 64, 96, 128, 192 or 256");
  if (bmn && ez == 1 && bn < 128) return unsupported("tile_n 64 with int8 B[K,N]");
  if (bn == 96 && swiglu) return unsupported("tile_n 96 with SWIGLU");
  if ((bn == 96 || bn == 192) && bmn) return unsupported("tile_n 96 / 192 with B[K,N]");
  // Several 128-byte K blocks per TMA instruction when K is whole blocks:
  // the per-instruction cost of TMA, not bytes, limits small boxes.
  const bool use3d = !batched && !cv && !bmn && (d->K * ez) % kKBytes == 0;
  // CTA pairs (256 x 256 tiles, cta_group::2) for GEMMs with at least a wave
  // of pair tiles: each SM then ingests 1/3 fewer bytes per flop.
  bool pair = false;
  {
    const int64_t pair_tiles = ((d->M + 2 * kBM - 1) / (2 * kBM)) * ((d->N + (swiglu ? 127 : 255)) / (swiglu ? 128 : 256));
    pair = use3d && splits == 1 && d->tile_n == 0 && d->stages == 0 && d->max_ctas == 0 &&
           pair_tiles >= sms / 2;
    if (const char *env = std::getenv("HX_GEMM_PAIR")) pair = pair || (use3d && std::atoi(env) > 0 && splits == 1);
    if (const char *env = std::getenv("HX_GEMM_PAIR")) if (std::atoi(env) == 0) pair = false;
    if (pair) bn = 256;
  }
  // Narrow tiles gain most (their boxes are smallest); wide tiles keep depth.
  int kbs = !use3d ? 1 : (bn == 64 ? 4 : 2);
  if (const char *env = std::getenv("HX_GEMM_KBS"))  // tuning switch
    if (use3d) kbs = std::max(1, std::min(4, std::atoi(env)));
  int stages = d->stages;
  const int per_stage = pair ? kBM * kKBytes + (bn / 2) * kKBytes : stage_bytes(bn);
  auto fit = [&](int kb) {
    return std::min(8, (kMaxDynSmem - 1024 - kBarBytes - kStageOutBytes) / (kb * per_stage));
  };
  // an explicit stage count takes precedence: fewer K blocks per load until it fits
  while (kbs > 1 && fit(kbs) < std::max(2, stages)) kbs >>= 1;
  const int max_stages = fit(kbs);
  if (stages == 0) stages = max_stages;
  if (stages < 2 || stages > max_stages) return arg_fail("stages out of range for tile_n");

  const int kind = d->a_dtype == HX_F16 ? 0 : (d->a_dtype == HX_BF16 ? 1 : 2);
  const int bk = kKBytes / ez;
  const int out_w = swiglu ? bn / 2 : bn;

  CUtensorMap ta, tb;
  if (cv) {
    rc = make_tmap_conv(&ta, d->A, d->a_dtype, cv->N, cv->H, cv->W, cv->C, bk, cv->bw, cv->bh);
    if (rc != HX_OK) return rc;
    rc = make_tmap(&tb, d->B, d->b_dtype, d->K, d->N, d->ldb, bk, bn);
    if (rc != HX_OK) return rc;
  } else if (batched) {
    rc = make_tmap_batched(&ta, d->A, d->a_dtype, d->K, d->M, bt->count, d->lda * ez, bt->sa * ez, bk, kBM);
    if (rc != HX_OK) return rc;
    if (bmn)
      rc = make_tmap_batched(&tb, d->B, d->b_dtype, d->N, d->K, bt->count, d->ldb * ez, bt->sb * ez,
                             kKBytes / ez, bk);
    else
      rc = make_tmap_batched(&tb, d->B, d->b_dtype, d->K, d->N, bt->count, d->ldb * ez, bt->sb * ez, bk, bn);
    if (rc != HX_OK) return rc;
  } else if (use3d) {
    const uint64_t kblocks = static_cast<uint64_t>(d->K) / bk;
    rc = make_tmap3(&ta, d->A, d->a_dtype, bk, d->M, kblocks, d->lda, kBM, kbs);
    if (rc != HX_OK) return rc;
    const uint64_t rows = swiglu ? 2 * d->N : d->N;
    rc = make_tmap3(&tb, d->B, d->b_dtype, bk, rows, kblocks, d->ldb, (swiglu || pair) ? bn / 2 : bn, kbs);
    if (rc != HX_OK) return rc;
  } else {
  rc = make_tmap(&ta, d->A, d->a_dtype, d->K, d->M, d->lda, bk, kBM);
  if (rc != HX_OK) return rc;
  if (bmn) {
    rc = make_tmap(&tb, d->B, d->b_dtype, d->N, d->K, d->ldb, kKBytes / ez, bk);
  } else {
    const uint64_t rows = swiglu ? 2 * d->N : d->N;
    rc = make_tmap(&tb, d->B, d->b_dtype, d->K, rows, d->ldb, bk, swiglu ? bn / 2 : bn);
  }
  if (rc != HX_OK) return rc;
  }

  GemmParams p;
  p.M = static_cast<int32_t>(d->M);
  p.K = static_cast<int32_t>(d->K);
  p.m_tiles = static_cast<int32_t>((d->M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM));
  p.n_tiles = static_cast<int32_t>((d->N + out_w - 1) / out_w);
  p.k_blocks = static_cast<int32_t>((d->K + bk - 1) / bk);
  p.n_half = static_cast<int32_t>(d->N);
  // Grouped raster: 16 row blocks per group, so a group's A panel stays in L2
  // while it sweeps every column block and each B tile is fetched once per
  // group.  Larger groups, which would fetch B once in all, measured slower
  // on the LM head: with 64 row blocks (a 67 MB A panel) the streamed C
  // writes evict A from L2 and DRAM reads rose from 0.89 to 3.3 GB a launch.
  {
    int64_t gm = 16;
    if (const char *env = std::getenv("HX_GEMM_GROUP_M"))  // tuning switch
      gm = std::max(1, std::atoi(env));
    p.group_m = static_cast<int32_t>(std::min<int64_t>(gm, p.m_tiles));
  }
  const int64_t item_tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  const int64_t total = item_tiles * (batched ? bt->count : 1);
  if (total > INT32_MAX) return unsupported("too many tiles");
  p.batch = batched ? static_cast<int32_t>(bt->count) : 1;
  p.batch_tiles = static_cast<int32_t>(item_tiles);
  p.batch_rows = static_cast<int32_t>(d->M);
  p.conv = cv ? 1 : 0;
  p.conv_H = cv ? static_cast<int32_t>(cv->OH) : 0;
  p.conv_W = cv ? static_cast<int32_t>(cv->OW) : 0;
  p.conv_KW = cv ? static_cast<int32_t>(cv->KW) : 0;
  p.conv_cpb = cv ? static_cast<int32_t>(cv->C / bk) : 0;
  p.conv_pad_h = cv ? cv->pad_h : 0;
  p.conv_pad_w = cv ? cv->pad_w : 0;
  p.total_tiles = static_cast<int32_t>(total);
  p.stages = stages;
  p.kbs = kbs;
  p.stage_blocks = (p.k_blocks + kbs - 1) / kbs;
  p.use3d = use3d ? 1 : 0;
  p.splits = splits;
  p.timeout = d->timeout_cycles ? d->timeout_cycles : kDefaultTimeout;
  p.err_flag = d->error_flag;
  p.epi = make_epi(d);
  if (batched) p.epi.M = static_cast<int32_t>(d->M * bt->count);  // flattened rows of C
  if (ns) {
    p.epi.norm = 1 + ns->kind;
    p.epi.row_stats = ns->row_stats;
    p.epi.col_sum = ns->col_sum;
  }
  if (peers) {
    p.epi.n_peers = peers->n;
    for (int j = 0; j < peers->n; ++j) p.epi.peer_C[j] = peers->C[j];
  }

  if (splits > 1 && (total * splits > sms || splits > p.stage_blocks)) {
    if (d->split_k > 1) return unsupported("split_k: tiles x split_k exceeds the SMs or the K blocks");
    splits = p.splits = 1;
  }
  p.ws = nullptr;
  p.red_smem = 0;
  p.b_const = (d->flags & HX_GEMM_B_CONST) ? 1 : 0;
  if (splits > 1) {
    const size_t need = static_cast<size_t>(total) * splits * bn * kBM * 4;
    rc = split_workspace(need, s, &p.ws);
    if (rc == kNeedsNoSplit) {
      if (d->split_k > 1) return unsupported("split_k: no workspace (stream capture or device memory)");
      splits = p.splits = 1;
    } else if (rc != HX_OK) {
      return rc;
    }
  }
  int ctas = sms;
  if (d->max_ctas > 0) ctas = std::min(ctas, static_cast<int>(d->max_ctas));
  int grid = splits > 1 ? static_cast<int>(total * splits)
                        : static_cast<int>(std::min<int64_t>(total, ctas));
  auto dispatch = [&]() {
    switch (kind) {
      case 0: return dispatch_kind<0>(bn, bmn, swiglu, ta, tb, p, grid, s);
      case 1: return dispatch_kind<1>(bn, bmn, swiglu, ta, tb, p, grid, s);
      default: return dispatch_kind<2>(bn, bmn, swiglu, ta, tb, p, grid, s);
    }
  };
  if (pair) {
    const int pairs = static_cast<int>(std::min<int64_t>(total, sms / 2));
    switch (kind) {
      case 0: return dispatch_pair_kind<0>(bn, swiglu, ta, tb, p, 2 * pairs, s);
      case 1: return dispatch_pair_kind<1>(bn, swiglu, ta, tb, p, 2 * pairs, s);
      default: return dispatch_pair_kind<2>(bn, swiglu, ta, tb, p, 2 * pairs, s);
    }
  }
  int r = dispatch();
  if (r == kNeedsNoSplit) {  // clusters would not all fit at once: run unsplit
    if (d->split_k > 1) return unsupported("split_k clusters do not all fit on the GPU at once");
    p.splits = 1;
    grid = static_cast<int>(std::min<int64_t>(total, ctas));
    r = dispatch();
  }
  return r;
}

// ------------------------------------------------------------ W8A16
// Tensor-core W8A16 (swap-AB, cluster split-K).  Returns HX_E_UNSUPPORTED
// when the shape is outside what the kernel takes, so the caller can use
// the CUDA-core kernels instead.
template <int MPAD>
int launch_w8a16_tc(const CUtensorMap &tw, const CUtensorMap &tx, const W8A16Params &p, int grid,
                    cudaStream_t s) {
  auto kern = hx_w8a16_tc_kernel<MPAD>;
  const int smem = W8Cfg<MPAD>::smem_bytes(p.stages);
  static SmemAttrOnce attr_once;
  {
    cudaError_t e = ensure_max_smem(kern, attr_once);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(w8a16)");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kW8Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tw, tx, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_w8a16_tc_kernel launch");
  return HX_OK;
}

int w8a16_tc(int64_t M, int64_t N, int64_t K, const void *x, int64_t ldx, const int8_t *W,
             int64_t ldw, const void *scale, const void *bias, void *y, int64_t ldy, int flags,
             cudaStream_t s) {
  if (M > 256 || K == 0 || ldw % 16 != 0 || ldx % 8 != 0 || !aligned16(x) || !aligned16(W))
    return HX_E_UNSUPPORTED;
  int sms = 0, major = 0;
  int rc = current_device_info(&sms, &major);
  if (rc != HX_OK) return rc;
  if (major != 10) {
    g_last_error = "current device is not sm_100";
    return HX_E_NO_DEVICE;
  }
  const int mpad = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256)));
  CUtensorMap tw, tx;
  rc = make_tmap(&tw, W, HX_S8, K, N, ldw, kW8KBlock, 128);
  if (rc != HX_OK) return rc;
  rc = make_tmap(&tx, x, HX_F16, K, M, ldx, 64, mpad);
  if (rc != HX_OK) return rc;
  W8A16Params p;
  p.M = static_cast<int32_t>(M);
  p.N = static_cast<int32_t>(N);
  p.K = static_cast<int32_t>(K);
  p.k_blocks = static_cast<int32_t>((K + kW8KBlock - 1) / kW8KBlock);
  const int64_t n_tiles = (N + 127) / 128;
  // Cluster size: enough CTAs to cover the SMs in one wave, at most 4 (so
  // clusters place easily next to a previous kernel's CTAs).
  int splits = static_cast<int>(std::min<int64_t>(4, std::max<int64_t>(1, sms / n_tiles)));
  if (const char *env = std::getenv("HX_W8A16_SPLITS")) splits = std::atoi(env);  // tuning override
  splits = std::max(1, std::min(std::min(splits, 8), p.k_blocks));
  if (n_tiles * splits > INT32_MAX) return unsupported("size");
  p.splits = splits;
  const int stage_bytes = 128 * 128 * 3 + 2 * mpad * 128;
  // Two stages keep a CTA near 100 KB so two fit on an SM (a decode GEMM and
  // the next one, launched early, side by side).
  p.stages = 2;
  if (const char *env = std::getenv("HX_W8A16_STAGES")) p.stages = std::atoi(env);  // tuning override
  p.stages = std::max(2, std::min(p.stages, (kMaxDynSmem - 1280) / stage_bytes));
  p.weights_const = (flags & HX_GEMV_WEIGHTS_CONST) ? 1 : 0;
  p.scale = static_cast<const __half *>(scale);
  p.bias = static_cast<const __half *>(bias);
  p.y = static_cast<__half *>(y);
  p.ldy = ldy;
  p.timeout = kDefaultTimeout;
  p.err_flag = nullptr;
  const int grid = static_cast<int>(n_tiles * splits);
  switch (mpad) {
    case 16: return launch_w8a16_tc<16>(tw, tx, p, grid, s);
    case 32: return launch_w8a16_tc<32>(tw, tx, p, grid, s);
    case 64: return launch_w8a16_tc<64>(tw, tx, p, grid, s);
    case 128: return launch_w8a16_tc<128>(tw, tx, p, grid, s);
    default: return launch_w8a16_tc<256>(tw, tx, p, grid, s);
  }
}

int gemv_impl(int64_t M, int64_t N, int64_t K, const void *x, int64_t ldx, const int8_t *W,
              int64_t ldw, const void *scale, const void *bias, void *y, int64_t ldy, int flags,
              cudaStream_t s) {
  if (M < 0 || N < 0 || K < 0) return arg_fail("negative size");
  if (M == 0 || N == 0) return HX_OK;
  if (!x || !W || !scale || !y) return arg_fail("null pointer");
  if (ldx < K || ldw < K || ldy < N) return arg_fail("leading dimension too small");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return unsupported("size");
  GemvParams p;
  p.M = static_cast<int32_t>(M);
  p.N = static_cast<int32_t>(N);
  p.K = static_cast<int32_t>(K);
  p.x = static_cast<const __half *>(x);
  p.ldx = ldx;
  p.W = W;
  p.ldw = ldw;
  p.scale = static_cast<const __half *>(scale);
  p.bias = static_cast<const __half *>(bias);
  p.y = static_cast<__half *>(y);
  p.ldy = ldy;
  const bool vec_ok = K > 0 && K % 16 == 0 && ldw % 16 == 0 && ldx % 8 == 0 && aligned16(x) &&
                      aligned16(W);
  if (vec_ok && M <= 8 && !(flags & HX_GEMV_FORCE_CUDA_CORE)) {
    // Streaming CUDA-core kernel: R rows x K int8 per CTA, up to 48 KB.
    int R = K <= 1536 ? 32 : (K <= 3072 ? 16 : 8);
    if (static_cast<int64_t>(R) * K <= 48 * 1024) {
      GemvStreamParams sp;
      sp.g = p;
      sp.rows_per_cta = R;
      sp.weights_const = (flags & HX_GEMV_WEIGHTS_CONST) ? 1 : 0;
      sp.timeout = kDefaultTimeout;
      const size_t smem = static_cast<size_t>(R) * K + 16;
      const int64_t blocks = (N + R - 1) / R;
      auto launch = [&](auto kern) -> cudaError_t {
        cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kMaxDynSmem);
        if (r != cudaSuccess) return r;
        r = launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(256), smem, s, sp);
        return r == cudaSuccess ? cudaGetLastError() : r;
      };
      cudaError_t e;
      if (M <= 1) e = launch(hx_gemv_w8a16_stream_kernel<1>);
      else if (M <= 2) e = launch(hx_gemv_w8a16_stream_kernel<2>);
      else if (M <= 4) e = launch(hx_gemv_w8a16_stream_kernel<4>);
      else e = launch(hx_gemv_w8a16_stream_kernel<8>);
      if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_stream_kernel");
      return HX_OK;
    }
  }
  if (!(flags & HX_GEMV_FORCE_CUDA_CORE)) {
    const int rc = w8a16_tc(M, N, K, x, ldx, W, ldw, scale, bias, y, ldy, flags, s);
    if (rc != HX_E_UNSUPPORTED) return rc;
    g_last_error.clear();
  }
  const bool vec = K > 0 && K % 16 == 0 && ldw % 16 == 0 && ldx % 8 == 0 && aligned16(x) &&
                   aligned16(W);
  cudaError_t e;
  if (vec) {
    int mc = M <= 1 ? 1 : (M <= 2 ? 2 : (M <= 4 ? 4 : 8));
    while (mc > 1 && static_cast<int64_t>(mc) * K * 2 > kMaxDynSmem) mc >>= 1;
    const int64_t smem = static_cast<int64_t>(mc) * K * 2;
    if (smem <= kMaxDynSmem) {
      constexpr int ROWS = 2;
      const int64_t blocks = (N + 4 * ROWS - 1) / (4 * ROWS);
      auto launch = [&](auto kern) -> cudaError_t {
        cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kMaxDynSmem);
        if (r != cudaSuccess) return r;
        r = launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(128), static_cast<size_t>(smem), s, p);
        return r == cudaSuccess ? cudaGetLastError() : r;
      };
      switch (mc) {
        case 1: e = launch(hx_gemv_w8a16_kernel<ROWS, 1>); break;
        case 2: e = launch(hx_gemv_w8a16_kernel<ROWS, 2>); break;
        case 4: e = launch(hx_gemv_w8a16_kernel<ROWS, 4>); break;
        default: e = launch(hx_gemv_w8a16_kernel<ROWS, 8>); break;
      }
      if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_kernel");
      return HX_OK;
    }
  }
  const int64_t warps = M * N;
  const int64_t blocks = (warps * 32 + 127) / 128;
  if (blocks > INT32_MAX) return unsupported("size");
  hx_gemv_w8a16_scalar_kernel<<<static_cast<unsigned>(blocks), 128, 0, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_scalar_kernel");
  return HX_OK;
}

// ------------------------------------------------------------ GEMM chain
static_assert(sizeof(ChainParams) < 32000, "chain parameter block must fit the launch limit");

int gemm_chain_impl(const hx_gemm_desc *descs, const int32_t *a_dep, const int32_t *r_dep,
                    int count, int32_t *counters, int64_t counters_len, int32_t *error_flag,
                    cudaStream_t s) {
  if (count < 0) return arg_fail("negative count");
  if (count == 0) return HX_OK;
  if (count > kChainMax) {
    g_last_error = "hx_gemm_chain takes at most 64 GEMMs per call";
    return HX_E_TOO_LARGE;
  }
  if (!descs || !a_dep || !r_dep || !counters) return arg_fail("null argument");
  int sms = 0, major = 0;
  int rc = current_device_info(&sms, &major);
  if (rc != HX_OK) return rc;
  if (major != 10) {
    g_last_error = "current device is not sm_100";
    return HX_E_NO_DEVICE;
  }
  constexpr int BN = 128;
  constexpr int KBS = 2;  // K blocks per TMA instruction: 3 stages of 64 KB
  static ChainParams p;  // ~26 KB, passed by value at launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  int64_t tiles = 0, ctrs = 0;
  for (int g = 0; g < count; ++g) {
    const hx_gemm_desc *d = &descs[g];
    rc = validate(d);
    if (rc != HX_OK) return rc;
    if (d->M == 0 || d->N == 0 || d->K == 0) return unsupported("empty GEMM in a chain");
    if (d->a_dtype != HX_F16 && d->a_dtype != HX_BF16) return unsupported("chain takes f16/bf16");
    if (d->b_layout != HX_B_NK) return unsupported("chain takes the W[N,K] layout");
    if (d->epilogue == HX_EPI_DEQUANT_SCALE) return unsupported("chain epilogue");
    if (!aligned16(d->A) || !aligned16(d->B) || (d->lda * 2) % 16 || (d->ldb * 2) % 16)
      return unsupported("chain operands need 16-byte aligned rows");
    if (d->K % 64) return unsupported("chain GEMMs need K a multiple of 64 (whole 128-byte K blocks)");
    for (const int32_t dep : {a_dep[g], r_dep[g]}) {
      if (dep < -1 || dep >= g) return arg_fail("dependencies must name earlier GEMMs");
      if (dep >= 0 && descs[dep].M != d->M) return arg_fail("a dependency must have the same M");
    }
    if (r_dep[g] >= 0 && !d->residual) return arg_fail("r_dep without a residual");
    const bool sw = d->epilogue == HX_EPI_SWIGLU;
    ChainGemm &c = p.g[g];
    c.m_tiles = static_cast<int32_t>((d->M + kBM - 1) / kBM);
    const int out_w = sw ? BN / 2 : BN;
    c.n_tiles = static_cast<int32_t>((d->N + out_w - 1) / out_w);
    c.k_blocks = static_cast<int32_t>((d->K + 63) / 64);
    c.n_half = static_cast<int32_t>(d->N);
    c.swiglu = sw ? 1 : 0;
    c.a_dep = a_dep[g];
    c.r_dep = r_dep[g];
    c.tile_begin = static_cast<int32_t>(tiles);
    c.ctr_begin = static_cast<int32_t>(ctrs);
    c.idesc = make_idesc(d->a_dtype == HX_F16 ? 0 : 1, false, kBM, BN);
    c.idesc_half = make_idesc(d->a_dtype == HX_F16 ? 0 : 1, false, kBM, BN / 2);
    c.epi = make_epi(d);
    const uint64_t kblocks = static_cast<uint64_t>(d->K) / 64;
    rc = make_tmap3(&p.tma[g], d->A, d->a_dtype, 64, d->M, kblocks, d->lda, kBM, KBS);
    if (rc != HX_OK) return rc;
    rc = make_tmap3(&p.tmb[g], d->B, d->b_dtype, 64, sw ? 2 * d->N : d->N, kblocks, d->ldb,
                    sw ? BN / 2 : BN, KBS);
    if (rc != HX_OK) return rc;
    tiles += static_cast<int64_t>(c.m_tiles) * c.n_tiles;
    ctrs += c.m_tiles;
    if (tiles > INT32_MAX) return unsupported("too many tiles");
  }
  if (counters_len < ctrs) {
    g_last_error = "counters buffer too small: needs one int32 per 128-row block of every GEMM";
    return HX_E_INVALID_ARG;
  }
  p.count = count;
  p.total_tiles = static_cast<int32_t>(tiles);
  const int fixed = 1024 + kBarBytes + kStageOutBytes;
  p.stages = std::min(8, (kMaxDynSmem - fixed) / (KBS * stage_bytes(BN)));
  p.counters = counters;
  p.err_flag = error_flag;
  p.timeout = kDefaultTimeout;
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int32_t) * ctrs, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(chain counters)");
  auto kern = hx_gemm_chain_kernel<BN, KBS>;
  const int smem = p.stages * KBS * stage_bytes(BN) + fixed;
  static SmemAttrOnce attr_once;
  e = ensure_max_smem(kern, attr_once);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(chain)");
  const int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
  e = launch_pdl(kern, dim3(grid), dim3(kThreads), static_cast<size_t>(smem), s, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemm_chain_kernel launch");
  return HX_OK;
}

// ------------------------------------------------------------ grouped W8A16
// Tensor-core grouped launch (gemv_grouped_tc.cuh) when every projection
// fits it: M <= 64, at most kGtMaxProj projections, K % 128 == 0, 16-byte
// aligned rows.  Returns kNeedsNoSplit (internal) when it does not apply.
int gemv_grouped_tc_impl(int64_t M, int count, const hx_w8a16_proj *projs, int32_t *counters,
                         int32_t *error_flag, cudaStream_t s, int sms) {
  if (M > kGtMaxM || count > kGtMaxProj) return kNeedsNoSplit;
  if (const char *env = std::getenv("HX_GROUPED_CUDA_CORE"))
    if (std::atoi(env) > 0) return kNeedsNoSplit;
  for (int g = 0; g < count; ++g) {
    const hx_w8a16_proj &q = projs[g];
    if (q.K % 128 || q.ldw % 16 || q.ldx % 8 || !aligned16(q.x) || !aligned16(q.W)) return kNeedsNoSplit;
  }
  int kbs = 4;  // K blocks per weight TMA load
  if (const char *env = std::getenv("HX_GT_KBS")) kbs = std::atoi(env);
  if (kbs != 1 && kbs != 2) kbs = 4;
  static GtParams p;  // ~30 KB: built on the host, passed by value at launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  p.G = count;
  p.M = static_cast<int32_t>(M);
  p.counters = counters;
  p.err_flag = error_flag;
  p.timeout = kDefaultTimeout;
  int64_t items = 0;
  for (int g = 0; g < count; ++g) {
    const hx_w8a16_proj &q = projs[g];
    int rc = make_tmap3(&p.tmW[g], q.W, HX_S8, 128, static_cast<uint64_t>(q.N),
                        static_cast<uint64_t>(q.K / 128), static_cast<uint64_t>(q.ldw), 128, kbs);
    if (rc != HX_OK) return rc;
    GtDesc &d = p.d[g];
    d.x = static_cast<const __half *>(q.x);
    d.scale = static_cast<const __half *>(q.scale);
    d.bias = static_cast<const __half *>(q.bias);
    d.y = static_cast<__half *>(q.y);
    d.N = static_cast<int32_t>(q.N);
    d.K = static_cast<int32_t>(q.K);
    d.ldx = static_cast<int32_t>(q.ldx);
    d.ldy = static_cast<int32_t>(q.ldy);
    d.dep = q.dep;
    d.item_begin = static_cast<int32_t>(items);
    d.kblocks = static_cast<int32_t>(q.K / 128);
    d.signal = 0;
    if (q.dep >= 0) p.d[q.dep].signal = 1;
    items += (q.N + 127) / 128;
    if (items > INT32_MAX) return unsupported("too many items");
  }
  p.total_items = static_cast<int32_t>(items);
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int32_t) * count, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
  const int grid = static_cast<int>(std::min<int64_t>(items, sms));
  auto launch = [&](auto kern, int smem, SmemAttrOnce &once) -> cudaError_t {
    cudaError_t r = ensure_max_smem(kern, once, smem);
    if (r != cudaSuccess) return r;
    return launch_pdl(kern, dim3(grid), dim3(kGtThreads), smem, s, p);
  };
  int nacc = M <= 16 ? 4 : (M <= 32 ? 2 : 1);
  if (const char *env = std::getenv("HX_GT_NACC")) nacc = std::atoi(env);
  static SmemAttrOnce conf[3][3][3];
  const int kv = kbs == 1 ? 0 : (kbs == 2 ? 1 : 2);
  const int av = nacc == 1 ? 0 : (nacc == 2 ? 1 : 2);
#define HX_GT_LAUNCH(MP, KB, NAC)                                                                 \
  launch(hx_gemv_w8a16_grouped_tc_kernel<MP, KB, NAC>, GtCfg<MP, KB, NAC>::kSmemBytes,            \
         conf[MP == 16 ? 0 : (MP == 32 ? 1 : 2)][kv][av])
#define HX_GT_LAUNCH_K(MP, NAC) \
  (kbs == 1 ? HX_GT_LAUNCH(MP, 1, NAC) : (kbs == 2 ? HX_GT_LAUNCH(MP, 2, NAC) : HX_GT_LAUNCH(MP, 4, NAC)))
#define HX_GT_LAUNCH_A(MP) \
  (nacc == 1 ? HX_GT_LAUNCH_K(MP, 1) : (nacc == 2 ? HX_GT_LAUNCH_K(MP, 2) : HX_GT_LAUNCH_K(MP, 4)))
  if (M <= 16) e = HX_GT_LAUNCH_A(16);
  else if (M <= 32) e = HX_GT_LAUNCH_A(32);
  else e = nacc == 1 ? HX_GT_LAUNCH_K(64, 1) : HX_GT_LAUNCH_K(64, 2);
#undef HX_GT_LAUNCH_A
#undef HX_GT_LAUNCH_K
#undef HX_GT_LAUNCH
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_grouped_tc_kernel");
  return HX_OK;
}

// Register-fragment MMA grouped launch (gemv_grouped_mma.cuh) for M <= 16
// when every projection has K % 64 == 0 and 16-byte aligned rows.  Returns
// kNeedsNoSplit (internal) when it does not apply.
int gemv_grouped_mma_impl(int64_t M, int count, const hx_w8a16_proj *projs, int32_t *counters,
                          int32_t *error_flag, cudaStream_t s, int sms) {
  // Wider batches: measured 1.0-1.9 TB/s here against 2.3-2.8 on tcgen05.
  if (M > 16) return kNeedsNoSplit;
  if (const char *env = std::getenv("HX_GROUPED_CUDA_CORE"))
    if (std::atoi(env) > 0) return kNeedsNoSplit;
  if (const char *env = std::getenv("HX_GROUPED_PATH"))  // tuning switch: "tc" or "cc" skip this kernel
    if (std::strcmp(env, "mma") != 0) return kNeedsNoSplit;
  const int rows = 32;
  // two 16-byte pieces of a row per lane (128-byte row segments per lane
  // quad) when every K allows it, else one
  int pieces = 2;
  for (int g = 0; g < count; ++g) {
    const hx_w8a16_proj &q = projs[g];
    if (q.K % 64 || q.ldw % 16 || q.ldx % 8 || !aligned16(q.x) || !aligned16(q.W)) return kNeedsNoSplit;
    if (q.K % 128) pieces = 1;
  }
  if (const char *env = std::getenv("HX_GM_P"))  // tuning switch
    if (std::atoi(env) == 1) pieces = 1;
  static GroupParams p;  // built on the host, passed by value at launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  p.G = count;
  p.M = static_cast<int32_t>(M);
  p.counters = counters;
  p.err_flag = error_flag;
  p.timeout = kDefaultTimeout;
  int64_t items = 0;
  for (int g = 0; g < count; ++g) {
    const hx_w8a16_proj &q = projs[g];
    GroupDesc &d = p.d[g];
    d.W = q.W;
    d.scale = static_cast<const __half *>(q.scale);
    d.bias = static_cast<const __half *>(q.bias);
    d.x = static_cast<const __half *>(q.x);
    d.y = static_cast<__half *>(q.y);
    d.N = static_cast<int32_t>(q.N);
    d.K = static_cast<int32_t>(q.K);
    d.ldw = static_cast<int32_t>(q.ldw);
    d.ldx = static_cast<int32_t>(q.ldx);
    d.ldy = static_cast<int32_t>(q.ldy);
    d.dep = q.dep;
    d.item_begin = static_cast<int32_t>(items);
    d.rows = rows;
    d.signal = 0;
    d.x_in_slot = 0;
    if (q.dep >= 0) p.d[q.dep].signal = 1;
    items += (q.N + rows - 1) / rows;
    if (items > INT32_MAX) return unsupported("too many items");
  }
  p.total_items = static_cast<int32_t>(items);
  // counters[count - 1] doubles as the work ticket (no projection signals it)
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int32_t) * count, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
  auto launch = [&](auto kern) -> cudaError_t {
    // every CTA must be resident at once (dependent items spin on counters)
    int per_sm = 0;
    cudaError_t r = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kGmWarps * 32, 0);
    if (r != cudaSuccess) return r;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>(static_cast<int64_t>(per_sm) * sms, (items + kGmWarps - 1) / kGmWarps)));
    r = launch_pdl(kern, dim3(grid), dim3(kGmWarps * 32), 0, s, p);
    return r == cudaSuccess ? cudaGetLastError() : r;
  };
#define HX_GM_LAUNCH(P_)                                        \
  (M <= 8 ? launch(hx_gemv_w8a16_grouped_mma_kernel<1, 2, P_>) \
          : launch(hx_gemv_w8a16_grouped_mma_kernel<2, 2, P_>))
  e = pieces == 2 ? HX_GM_LAUNCH(2) : HX_GM_LAUNCH(1);
#undef HX_GM_LAUNCH
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_grouped_mma_kernel");
  return HX_OK;
}

int gemv_grouped_impl(int64_t M, int count, const hx_w8a16_proj *projs, int32_t *counters,
                      int32_t *error_flag, cudaStream_t s) {
  if (M < 0 || count < 0) return arg_fail("negative size");
  if (count == 0 || M == 0) return HX_OK;
  if (count > kGroupMax) return unsupported("more projections than one grouped launch takes (256)");
  if (M > kGtMaxM) return unsupported("grouped W8A16 takes M <= 64");
  if (!projs || !counters) return arg_fail("null projections or counters");
  int sms = 0, major = 0;
  int rc = current_device_info(&sms, &major);
  if (rc != HX_OK) return rc;
  if (major != 10) {
    g_last_error = "current device is not sm_100";
    return HX_E_NO_DEVICE;
  }
  for (int g = 0; g < count; ++g) {  // validate before choosing a kernel
    const hx_w8a16_proj &q = projs[g];
    if (q.N <= 0 || q.K <= 0 || !q.x || !q.W || !q.scale || !q.y) return arg_fail("bad projection");
    if (q.ldx < q.K || q.ldw < q.K || q.ldy < q.N) return arg_fail("leading dimension too small");
    if (q.N > INT32_MAX || q.K > INT32_MAX || q.ldx > INT32_MAX || q.ldw > INT32_MAX || q.ldy > INT32_MAX)
      return unsupported("size");
    if (q.dep >= g || q.dep < -1) return arg_fail("dep must name an earlier projection or be -1");
  }
  rc = gemv_grouped_mma_impl(M, count, projs, counters, error_flag, s, sms);
  if (rc != kNeedsNoSplit) return rc;
  rc = gemv_grouped_tc_impl(M, count, projs, counters, error_flag, s, sms);
  if (rc != kNeedsNoSplit) return rc;
  if (M > 8) return unsupported("grouped W8A16 on CUDA cores takes M <= 8");
  static GroupParams p;  // 18 KB: built on the host, passed by value at launch
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  p.G = count;
  p.M = static_cast<int32_t>(M);
  p.counters = counters;
  p.err_flag = error_flag;
  p.timeout = kDefaultTimeout;
  int64_t items = 0;
  for (int g = 0; g < count; ++g) {
    const hx_w8a16_proj &q = projs[g];
    if (q.N <= 0 || q.K <= 0 || !q.x || !q.W || !q.scale || !q.y) return arg_fail("bad projection");
    if (q.ldx < q.K || q.ldw < q.K || q.ldy < q.N) return arg_fail("leading dimension too small");
    if (q.N > INT32_MAX || q.K > INT32_MAX || q.ldx > INT32_MAX || q.ldw > INT32_MAX || q.ldy > INT32_MAX)
      return unsupported("size");
    if (q.dep >= g || q.dep < -1) return arg_fail("dep must name an earlier projection or be -1");
    if (q.K % 16 || q.ldw % 16 || q.ldx % 8 || !aligned16(q.x) || !aligned16(q.W))
      return unsupported("grouped W8A16 needs K % 16 == 0 and 16-byte aligned rows");
    int R = M <= 2 ? 16 : 8;  // rows per item; 8 compute warps take R / 8 each
    while (R > 8 && static_cast<int64_t>(R) * q.K > kGroupSlotBytes) R >>= 1;
    if (static_cast<int64_t>(R) * q.K > kGroupSlotBytes) return unsupported("K too large for a slot");
    GroupDesc &d = p.d[g];
    d.W = q.W;
    d.scale = static_cast<const __half *>(q.scale);
    d.bias = static_cast<const __half *>(q.bias);
    d.x = static_cast<const __half *>(q.x);
    d.y = static_cast<__half *>(q.y);
    d.N = static_cast<int32_t>(q.N);
    d.K = static_cast<int32_t>(q.K);
    d.ldw = static_cast<int32_t>(q.ldw);
    d.ldx = static_cast<int32_t>(q.ldx);
    d.ldy = static_cast<int32_t>(q.ldy);
    d.dep = q.dep;
    d.item_begin = static_cast<int32_t>(items);
    d.rows = R;
    d.signal = 0;
    d.x_in_slot = ((static_cast<int64_t>(R) * q.K + 15) / 16) * 16 + M * q.K * 2 <= kGroupSlotBytes &&
                  (q.ldx * 2) % 16 == 0;
    if (q.dep >= 0) p.d[q.dep].signal = 1;
    items += (q.N + R - 1) / R;
    if (items > INT32_MAX) return unsupported("too many items");
  }
  p.total_items = static_cast<int32_t>(items);
  cudaError_t e = cudaMemsetAsync(counters, 0, sizeof(int32_t) * count, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(counters)");
  const int grid = static_cast<int>(std::min<int64_t>(items, 2 * sms));  // two CTAs per SM
  const size_t smem =
      kGroupSlots * kGroupSlotBytes + 16 * kGroupSlots + 64;
  auto launch = [&](auto kern) -> cudaError_t {
    // dynamic + static shared memory must stay within the 227 KB per block
    cudaError_t r = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (r != cudaSuccess) return r;
    r = launch_pdl(kern, dim3(grid), dim3(kGroupThreads + 32), smem, s, p);
    return r == cudaSuccess ? cudaGetLastError() : r;
  };
  if (M <= 1) e = launch(hx_gemv_w8a16_grouped_kernel<1, 2>);
  else if (M <= 2) e = launch(hx_gemv_w8a16_grouped_kernel<2, 2>);
  else if (M <= 4) e = launch(hx_gemv_w8a16_grouped_kernel<4, 1>);
  else e = launch(hx_gemv_w8a16_grouped_kernel<8, 1>);
  if (e != cudaSuccess) return cuda_fail(e, "hx_gemv_w8a16_grouped_kernel");
  return HX_OK;
}

// ------------------------------------------------------------ shard reorder
// src[world][M][Ns] (rank-major all-gather result) -> dst[M][world*Ns].
__global__ void shards_to_rows_kernel(const uint8_t *__restrict__ src, uint8_t *__restrict__ dst,
                                      int world, int64_t M, int64_t row_bytes) {
  // one 16-byte (or 1-byte tail) chunk per thread, row-major over dst
  const int64_t dst_row = row_bytes * world;
  const int64_t chunks_per_row = (row_bytes + 15) / 16;
  const int64_t total = M * world * chunks_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = i % chunks_per_row;
    const int64_t rm = i / chunks_per_row;
    const int64_t r = rm % world, m = rm / world;
    const uint8_t *sp = src + (r * M + m) * row_bytes + c * 16;
    uint8_t *dp = dst + m * dst_row + r * row_bytes + c * 16;
    const int64_t rem = row_bytes - c * 16;
    const int64_t n = rem < 16 ? rem : 16;
    if (n == 16 && aligned16(sp) && aligned16(dp)) {
      *reinterpret_cast<uint4 *>(dp) = *reinterpret_cast<const uint4 *>(sp);
    } else {
      for (int64_t b = 0; b < n; ++b) dp[b] = sp[b];
    }
  }
}

}  // namespace
}  // namespace hx

// NCCL's ABI, restated for the dlopen'd symbols (nccl.h 2.x).
typedef struct {
  char internal[128];
} hx_nccl_unique_id_t;
typedef int (*hx_nccl_get_unique_id_fn)(hx_nccl_unique_id_t *);
typedef int (*hx_nccl_comm_init_rank_fn)(void **, int, hx_nccl_unique_id_t, int);
typedef int (*hx_nccl_all_gather_fn)(const void *, void *, size_t, int /*ncclDataType_t*/,
                                     void * /*comm*/, cudaStream_t);
typedef int (*hx_nccl_comm_destroy_fn)(void *);
typedef const char *(*hx_nccl_error_string_fn)(int);

namespace {
struct NcclSyms {
  hx_nccl_get_unique_id_fn get_unique_id = nullptr;
  hx_nccl_comm_init_rank_fn comm_init_rank = nullptr;
  hx_nccl_all_gather_fn all_gather = nullptr;
  hx_nccl_comm_destroy_fn comm_destroy = nullptr;
  hx_nccl_error_string_fn error_string = nullptr;
};
NcclSyms g_nccl;
std::once_flag g_nccl_once;

bool load_nccl() {
  std::call_once(g_nccl_once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    g_nccl.get_unique_id = reinterpret_cast<hx_nccl_get_unique_id_fn>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank =
        reinterpret_cast<hx_nccl_comm_init_rank_fn>(dlsym(h, "ncclCommInitRank"));
    g_nccl.all_gather = reinterpret_cast<hx_nccl_all_gather_fn>(dlsym(h, "ncclAllGather"));
    g_nccl.comm_destroy = reinterpret_cast<hx_nccl_comm_destroy_fn>(dlsym(h, "ncclCommDestroy"));
    g_nccl.error_string = reinterpret_cast<hx_nccl_error_string_fn>(dlsym(h, "ncclGetErrorString"));
  });
  return g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_gather &&
         g_nccl.comm_destroy;
}
int nccl_fail(int r, const char *where) {
  hx::g_last_error = std::string(where) + ": " +
                     (g_nccl.error_string ? g_nccl.error_string(r) : std::to_string(r));
  return HX_E_NCCL;
}
}  // namespace

// ------------------------------------------------------------ convolution
namespace hx {
namespace {
// Explicit im2col for convolutions the implicit GEMM does not take:
// col[pixel][(kh * KW + kw) * C + c] = x[n][ih][iw][c], zero outside the image.
// VEC elements (16 bytes or 2) per thread.
template <int VEC>
__global__ void im2col_kernel(const uint16_t *x, uint16_t *col, int64_t N, int64_t H, int64_t W, int64_t C,
                              int64_t OH, int64_t OW, int64_t KH, int64_t KW, int sh, int sw, int ph, int pw,
                              int dh, int dw) {
  const int64_t cv = C / VEC;
  const int64_t total = N * OH * OW * KH * KW * cv;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int64_t c = (r % cv) * VEC;
    r /= cv;
    const int64_t kw = r % KW;
    r /= KW;
    const int64_t kh = r % KH;
    const int64_t pix = r / KH;
    const int64_t ow = pix % OW, oh = (pix / OW) % OH, n = pix / (OW * OH);
    const int64_t ih = oh * sh + kh * dh - ph, iw = ow * sw + kw * dw - pw;
    uint16_t *dst = col + pix * (KH * KW * C) + (kh * KW + kw) * C + c;
    const bool in = ih >= 0 && ih < H && iw >= 0 && iw < W;
    if constexpr (VEC == 8) {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (in) v = *reinterpret_cast<const uint4 *>(x + ((n * H + ih) * W + iw) * C + c);
      *reinterpret_cast<uint4 *>(dst) = v;
    } else {
      dst[0] = in ? x[((n * H + ih) * W + iw) * C + c] : uint16_t(0);
    }
  }
}

struct ConvGeom {
  int64_t OH, OW, M, K;
  bool implicit;
  int bw, bh;
};

int conv_geom(const hx_conv2d_desc *d, ConvGeom *g) {
  if (!d) return arg_fail("null descriptor");
  if (d->N < 0 || d->H <= 0 || d->W <= 0 || d->C <= 0 || d->OC <= 0 || d->KH <= 0 || d->KW <= 0)
    return arg_fail("convolution sizes");
  if (d->stride_h <= 0 || d->stride_w <= 0 || d->dil_h <= 0 || d->dil_w <= 0 || d->pad_h < 0 || d->pad_w < 0)
    return arg_fail("convolution stride / dilation / padding");
  if (d->dtype != HX_F16 && d->dtype != HX_BF16) return unsupported("convolution takes f16 or bf16");
  if (d->epilogue == HX_EPI_SWIGLU || d->epilogue == HX_EPI_DEQUANT_SCALE)
    return unsupported("convolution epilogue");
  g->OH = (d->H + 2 * d->pad_h - int64_t(d->dil_h) * (d->KH - 1) - 1) / d->stride_h + 1;
  g->OW = (d->W + 2 * d->pad_w - int64_t(d->dil_w) * (d->KW - 1) - 1) / d->stride_w + 1;
  if (g->OH <= 0 || g->OW <= 0) return arg_fail("convolution output is empty");
  g->M = d->N * g->OH * g->OW;
  g->K = d->KH * d->KW * d->C;
  if (g->M > INT32_MAX || g->K > INT32_MAX || d->OC > INT32_MAX / 2) return unsupported("size beyond int32 range");
  const bool rows_tile = (g->OW <= kBM && kBM % g->OW == 0) || g->OW % kBM == 0;
  g->implicit = d->stride_h == 1 && d->stride_w == 1 && d->dil_h == 1 && d->dil_w == 1 && d->C % 64 == 0 &&
                rows_tile && (d->N == 1 || (g->OH * g->OW) % kBM == 0) && aligned16(d->x) && aligned16(d->w) &&
                d->W <= INT32_MAX && d->H <= INT32_MAX;
  g->bw = static_cast<int>(std::min<int64_t>(g->OW, kBM));
  g->bh = kBM / g->bw;
  // every box lies within the image's rows: a tile never needs rows past OH
  // (images smaller than one 128-pixel tile take the im2col path)
  if (g->bh > g->OH) g->implicit = false;
  return HX_OK;
}

hx_gemm_desc conv_gemm_desc(const hx_conv2d_desc *d, const ConvGeom &g, const void *a) {
  hx_gemm_desc q;
  std::memset(&q, 0, sizeof(q));
  q.M = g.M;
  q.N = d->OC;
  q.K = g.K;
  q.a_dtype = q.b_dtype = q.c_dtype = d->dtype;
  q.b_layout = HX_B_NK;
  q.A = a;
  q.lda = g.K;
  q.B = d->w;
  q.ldb = g.K;
  q.C = d->y;
  q.ldc = d->OC;
  q.epilogue = d->epilogue;
  q.bias = d->bias;
  q.bias_dtype = d->bias_dtype;
  q.residual = d->residual;
  q.ldr = d->OC;
  q.error_flag = d->error_flag;
  q.split_k = 1;
  return q;
}
}  // namespace
}  // namespace hx

// ============================================================ C ABI
// ------------------------------------------------------------ fused all-gather over NVLink
namespace hx {
namespace {
struct PeerBarrierArgs {
  int32_t *flags[8];  // flags[r]: rank r's flag array (world int32), in its GPU memory
  int32_t rank, world, value;
  uint64_t timeout;
  int32_t *err_flag;
};

// One warp: lane p != rank publishes `value` into peer p's slot for this rank
// (release, system scope), then waits (acquire, bounded) until peer p has
// published at least `value` into this rank's array.  On timeout the error
// word is set and the kernel returns: nothing hangs.
__global__ void peer_barrier_kernel(const __grid_constant__ PeerBarrierArgs a) {
  const int p = threadIdx.x;
  if (p >= a.world || p == a.rank) return;
  int32_t *remote = a.flags[p] + a.rank;
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(remote), "r"(a.value) : "memory");
  const int32_t *mine = a.flags[a.rank] + p;
  const uint64_t t0 = clock64();
  for (;;) {
    int32_t v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (v >= a.value) break;
    if (static_cast<uint64_t>(clock64() - t0) > a.timeout) {
      if (a.err_flag) atomicExch(a.err_flag, 41);
      break;
    }
    __nanosleep(256);
  }
}

int peer_barrier(int32_t *const *flags, int rank, int world, int32_t value, int32_t *err_flag,
                 cudaStream_t s) {
  PeerBarrierArgs a;
  for (int i = 0; i < 8; ++i) a.flags[i] = i < world ? flags[i] : nullptr;
  a.rank = rank;
  a.world = world;
  a.value = value;
  a.timeout = kDefaultTimeout;
  a.err_flag = err_flag;
  peer_barrier_kernel<<<1, 32, 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "peer_barrier_kernel");
  return HX_OK;
}
}  // namespace
}  // namespace hx

extern "C" {

int hx_version(void) { return HX_VERSION; }

const char *hx_status_str(int status) {
  switch (status) {
    case HX_OK: return "HX_OK";
    case HX_E_INVALID_ARG: return "HX_E_INVALID_ARG";
    case HX_E_UNSUPPORTED: return "HX_E_UNSUPPORTED";
    case HX_E_CUDA: return "HX_E_CUDA";
    case HX_E_TIMEOUT: return "HX_E_TIMEOUT";
    case HX_E_NCCL: return "HX_E_NCCL";
    case HX_E_NO_DEVICE: return "HX_E_NO_DEVICE";
    case HX_E_TOO_LARGE: return "HX_E_TOO_LARGE";
    default: return "HX_E_UNKNOWN";
  }
}

const char *hx_last_error(void) { return hx::g_last_error.c_str(); }

int hx_gemm(const hx_gemm_desc *d, void *stream) {
  hx::g_last_error.clear();
  return hx::gemm_impl(d, static_cast<cudaStream_t>(stream));
}

int hx_gemm_batched(const hx_gemm_desc *d, int64_t batch, int64_t stride_a, int64_t stride_b,
                    int64_t stride_c, int64_t stride_r, void *stream) {
  hx::g_last_error.clear();
  if (!d || batch < 0 || stride_a < 0 || stride_b < 0 || stride_c < 0 || stride_r < 0)
    return HX_E_INVALID_ARG;
  if (batch == 0) return HX_OK;
  if (d->epilogue == HX_EPI_SWIGLU) {
    hx::g_last_error = "batched GEMM takes no SWIGLU epilogue";
    return HX_E_UNSUPPORTED;
  }
  if (stride_c > 0 && stride_c < d->M * d->ldc && batch > 1) {
    hx::g_last_error = "batch items of C overlap (stride_c < M * ldc)";
    return HX_E_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = hx::kNeedsLoop;
  if (stride_b == 0) {
    // One shared B: with A, C and residual items back to back this is one
    // GEMM over batch * M rows.
    if (stride_a == d->M * d->lda && stride_c == d->M * d->ldc &&
        (!d->residual || stride_r == d->M * d->ldr) && batch * d->M <= INT32_MAX) {
      hx_gemm_desc dm = *d;
      dm.M = batch * d->M;
      return hx::gemm_impl(&dm, s);
    }
  } else {
    const hx::BatchSpec bt{batch, stride_a, stride_b, stride_c, stride_r};
    rc = hx::gemm_impl(d, s, nullptr, &bt);
  }
  if (rc != hx::kNeedsLoop) return rc;
  // Item by item: items whose rows are not whole tiles, or whose C rows are
  // not back to back, or operands TMA cannot address as one 3-D view.
  const int ez = hx::esize(d->a_dtype), cz = hx::esize(d->c_dtype);
  for (int64_t i = 0; i < batch; ++i) {
    hx_gemm_desc di = *d;
    di.A = static_cast<const uint8_t *>(d->A) + i * stride_a * ez;
    di.B = static_cast<const uint8_t *>(d->B) + i * stride_b * ez;
    di.C = static_cast<uint8_t *>(d->C) + i * stride_c * cz;
    if (d->residual) di.residual = static_cast<const uint8_t *>(d->residual) + i * stride_r * cz;
    rc = hx::gemm_impl(&di, s);
    if (rc != HX_OK) return rc;
  }
  return HX_OK;
}

int hx_conv2d_workspace_size(const hx_conv2d_desc *d, int64_t *bytes) {
  hx::g_last_error.clear();
  if (!bytes) return HX_E_INVALID_ARG;
  hx::ConvGeom g;
  const int rc = hx::conv_geom(d, &g);
  if (rc != HX_OK) return rc;
  *bytes = g.implicit ? 0 : (g.M * g.K * 2 + 15) / 16 * 16;
  return HX_OK;
}

int hx_conv2d(const hx_conv2d_desc *d, void *workspace, int64_t workspace_bytes, void *stream) {
  hx::g_last_error.clear();
  hx::ConvGeom g;
  int rc = hx::conv_geom(d, &g);
  if (rc != HX_OK) return rc;
  if (g.M == 0) return HX_OK;
  if (!d->x || !d->w || !d->y) return HX_E_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (g.implicit) {
    hx_gemm_desc q = hx::conv_gemm_desc(d, g, d->x);
    const hx::ConvSpec cv{d->N, d->H, d->W, d->C, g.OH, g.OW, d->KH, d->KW, d->pad_h, d->pad_w, g.bw, g.bh};
    return hx::gemm_impl(&q, s, nullptr, nullptr, nullptr, &cv);
  }
  const int64_t need = (g.M * g.K * 2 + 15) / 16 * 16;
  if (!workspace || workspace_bytes < need) {
    hx::g_last_error = "hx_conv2d needs hx_conv2d_workspace_size() bytes of workspace for this shape";
    return HX_E_INVALID_ARG;
  }
  if (!hx::aligned16(workspace)) return HX_E_INVALID_ARG;
  const bool v8 = d->C % 8 == 0 && hx::aligned16(d->x);
  const int64_t items = g.M * d->KH * d->KW * (v8 ? d->C / 8 : d->C);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((items + 255) / 256, 148 * 16));
  auto x = static_cast<const uint16_t *>(d->x);
  auto col = static_cast<uint16_t *>(workspace);
  if (v8)
    hx::im2col_kernel<8><<<blocks, 256, 0, s>>>(x, col, d->N, d->H, d->W, d->C, g.OH, g.OW, d->KH, d->KW,
                                                d->stride_h, d->stride_w, d->pad_h, d->pad_w, d->dil_h, d->dil_w);
  else
    hx::im2col_kernel<1><<<blocks, 256, 0, s>>>(x, col, d->N, d->H, d->W, d->C, g.OH, g.OW, d->KH, d->KW,
                                                d->stride_h, d->stride_w, d->pad_h, d->pad_w, d->dil_h, d->dil_w);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return hx::cuda_fail(e, "im2col_kernel");
  hx_gemm_desc q = hx::conv_gemm_desc(d, g, workspace);
  return hx::gemm_impl(&q, s);
}

int hx_gemm_norm(const hx_gemm_desc *d, int kind, const float *row_stats, const float *col_sum,
                 void *stream) {
  hx::g_last_error.clear();
  if (!d) return HX_E_INVALID_ARG;
  if (kind != HX_NORM_LAYER && kind != HX_NORM_RMS) return HX_E_INVALID_ARG;
  if (d->M > 0 && d->N > 0 && (!row_stats || (kind == HX_NORM_LAYER && !col_sum))) return HX_E_INVALID_ARG;
  if (d->a_dtype != HX_F16 && d->a_dtype != HX_BF16) {
    hx::g_last_error = "a folded normalisation needs f16 / bf16 inputs";
    return HX_E_UNSUPPORTED;
  }
  if (d->epilogue == HX_EPI_DEQUANT_SCALE) return HX_E_UNSUPPORTED;
  const hx::NormSpec ns{kind, row_stats, col_sum};
  return hx::gemm_impl(d, static_cast<cudaStream_t>(stream), nullptr, nullptr, &ns);
}

int hx_matmul_f16f16_f32(int64_t n_row, int64_t n_col, int64_t n_inner, float *out,
                         const void *act, const void *W, void *stream) {
  hx_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.M = n_row;
  d.N = n_col;
  d.K = n_inner;
  d.a_dtype = d.b_dtype = HX_F16;
  d.c_dtype = HX_F32;
  d.b_layout = HX_B_KN;
  d.A = act;
  d.lda = n_inner;
  d.B = W;
  d.ldb = n_col;
  d.C = out;
  d.ldc = n_col;
  d.epilogue = HX_EPI_NONE;
  return hx_gemm(&d, stream);
}

int hx_gemv_w8a16(int64_t M, int64_t N, int64_t K, const void *x, int64_t ldx, const int8_t *W,
                  int64_t ldw, const void *scale, const void *bias, void *y, int64_t ldy,
                  void *stream) {
  hx::g_last_error.clear();
  return hx::gemv_impl(M, N, K, x, ldx, W, ldw, scale, bias, y, ldy, 0,
                       static_cast<cudaStream_t>(stream));
}

int hx_gemv_w8a16_ex(int64_t M, int64_t N, int64_t K, const void *x, int64_t ldx,
                     const int8_t *W, int64_t ldw, const void *scale, const void *bias, void *y,
                     int64_t ldy, int flags, void *stream) {
  hx::g_last_error.clear();
  if (flags & ~(HX_GEMV_WEIGHTS_CONST | HX_GEMV_FORCE_CUDA_CORE)) return HX_E_INVALID_ARG;
  return hx::gemv_impl(M, N, K, x, ldx, W, ldw, scale, bias, y, ldy, flags,
                       static_cast<cudaStream_t>(stream));
}

int hx_gemm_chain(const hx_gemm_desc *descs, const int32_t *a_dep, const int32_t *r_dep, int count,
                  int32_t *counters, int64_t counters_len, int32_t *error_flag, void *stream) {
  hx::g_last_error.clear();
  return hx::gemm_chain_impl(descs, a_dep, r_dep, count, counters, counters_len, error_flag,
                             static_cast<cudaStream_t>(stream));
}

int hx_gemv_w8a16_grouped(int64_t M, int count, const hx_w8a16_proj *projs, int32_t *counters,
                          int32_t *error_flag, void *stream) {
  hx::g_last_error.clear();
  return hx::gemv_grouped_impl(M, count, projs, counters, error_flag,
                               static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ------------------------------------------------------------ allocation-free grouped W8A16
// Completion counters for hx_gemv_w8a16_grouped_noalloc, one int32 per
// projection, in a fixed device array that every GPU loading this library
// holds until the process exits (1 KB).  In host code `g_noalloc_counters`
// names a host-side stand-in, not device memory: its device address is
// looked up per device with cudaGetSymbolAddress below.
#define HX_NOALLOC_MAX_PROJS 256
static __device__ __align__(256) int32_t g_noalloc_counters[HX_NOALLOC_MAX_PROJS];

namespace hx {
namespace {
std::mutex g_noalloc_mu;
int32_t *g_noalloc_ptr[64] = {};  // device address of the array, per device

// Set-up, once per device, with that device current.
int noalloc_counters(int32_t **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return arg_fail("device index out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_counters);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_counters)");
    g_noalloc_ptr[dev] = static_cast<int32_t *>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return HX_OK;
}
}  // namespace
}  // namespace hx

extern "C" {

int hx_gemv_w8a16_grouped_noalloc(int64_t M, int count, const hx_w8a16_proj *projs,
                                  int32_t *error_flag, void *stream) {
  hx::g_last_error.clear();
  if (count > HX_NOALLOC_MAX_PROJS) {
    hx::g_last_error = "hx_gemv_w8a16_grouped_noalloc takes at most 256 projections";
    return HX_E_TOO_LARGE;
  }
  int32_t *counters = nullptr;
  const int rc = hx::noalloc_counters(&counters);
  if (rc != HX_OK) return rc;
  // gemv_grouped_impl zeroes the counters with cudaMemsetAsync on `stream`
  // before the launch; it allocates nothing.
  return hx::gemv_grouped_impl(M, count, projs, counters, error_flag,
                               static_cast<cudaStream_t>(stream));
}

int hx_query_workspace(const hx_gemm_desc *d, int64_t *bytes) {
  if (!d || !bytes) return HX_E_INVALID_ARG;
  *bytes = 0;
  return HX_OK;
}

int hx_nccl_unique_id_size(void) { return static_cast<int>(sizeof(hx_nccl_unique_id_t)); }

int hx_nccl_get_unique_id(void *id_out) {
  if (!id_out) return HX_E_INVALID_ARG;
  if (!load_nccl()) {
    hx::g_last_error = "libnccl.so.2 not loadable";
    return HX_E_NCCL;
  }
  hx_nccl_unique_id_t id;
  int r = g_nccl.get_unique_id(&id);
  if (r != 0) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id_out, &id, sizeof(id));
  return HX_OK;
}

int hx_nccl_comm_init(void **comm_out, int world, const void *id, int rank) {
  if (!comm_out || !id || world < 1 || rank < 0 || rank >= world) return HX_E_INVALID_ARG;
  if (!load_nccl()) {
    hx::g_last_error = "libnccl.so.2 not loadable";
    return HX_E_NCCL;
  }
  hx_nccl_unique_id_t uid;
  std::memcpy(&uid, id, sizeof(uid));
  int r = g_nccl.comm_init_rank(comm_out, world, uid, rank);
  if (r != 0) return nccl_fail(r, "ncclCommInitRank");
  return HX_OK;
}

int hx_nccl_comm_destroy(void *comm) {
  if (!comm) return HX_E_INVALID_ARG;
  if (!load_nccl()) return HX_E_NCCL;
  int r = g_nccl.comm_destroy(comm);
  if (r != 0) return nccl_fail(r, "ncclCommDestroy");
  return HX_OK;
}

int hx_peer_alloc(int64_t bytes, void **dev_ptr, void *ipc_handle) {
  if (bytes <= 0 || !dev_ptr || !ipc_handle) return HX_E_INVALID_ARG;
  hx::g_last_error.clear();
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return hx::cuda_fail(e, "cudaIpcGetMemHandle");
  }
  *dev_ptr = p;
  return HX_OK;
}

int hx_peer_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int hx_peer_open(const void *ipc_handle, void **peer_ptr) {
  if (!ipc_handle || !peer_ptr) return HX_E_INVALID_ARG;
  hx::g_last_error.clear();
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaIpcOpenMemHandle");
  return HX_OK;
}

int hx_peer_close(void *peer_ptr) {
  if (!peer_ptr) return HX_E_INVALID_ARG;
  cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaIpcCloseMemHandle");
  return HX_OK;
}

int hx_peer_free(void *dev_ptr) {
  if (!dev_ptr) return HX_E_INVALID_ARG;
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaFree(peer buffer)");
  return HX_OK;
}

int hx_sharded_gemm_gather_p2p(const hx_gemm_desc *d, int rank, int world, void *const *gathered,
                               int32_t *const *flags, int32_t epoch, int32_t *error_flag,
                               void *stream) {
  hx::g_last_error.clear();
  if (!d || !gathered || !flags || world < 1 || world > 8 || rank < 0 || rank >= world || epoch < 0 ||
      epoch > (INT32_MAX - 2) / 2)
    return HX_E_INVALID_ARG;
  for (int r = 0; r < world; ++r)
    if (!gathered[r] || !flags[r]) return HX_E_INVALID_ARG;
  if (d->ldc != d->N) {
    hx::g_last_error = "gather needs a contiguous shard (ldc == N)";
    return HX_E_INVALID_ARG;
  }
  const int ez = hx::esize(d->a_dtype), cz = hx::esize(d->c_dtype);
  if (d->K == 0 || d->force_simt || d->b_layout != HX_B_NK || !hx::aligned16(d->A) || !hx::aligned16(d->B) ||
      (d->lda * ez) % 16 || (d->ldb * ez) % 16 || (d->N * cz) % 16 ||
      reinterpret_cast<uintptr_t>(gathered[rank]) % 16) {
    hx::g_last_error = "fused gather needs the tensor-core path: W[N,K], K > 0, 16-byte aligned rows";
    return HX_E_UNSUPPORTED;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Entry: every peer reached this call (its earlier readers of its buffer
  // are stream-ordered before it), so its buffer may be overwritten.
  int rc = hx::peer_barrier(flags, rank, world, 2 * epoch + 1, error_flag, s);
  if (rc != HX_OK) return rc;
  // This rank's shard lands at gathered[r][rank] on every rank r.
  const size_t off = static_cast<size_t>(rank) * d->M * d->N * cz;
  hx_gemm_desc dd = *d;
  dd.C = static_cast<uint8_t *>(gathered[rank]) + off;
  dd.split_k = 1;
  if (!dd.error_flag) dd.error_flag = error_flag;
  hx::PeerTargets peers;
  peers.n = 0;
  for (int r = 0; r < world; ++r)
    if (r != rank) peers.C[peers.n++] = static_cast<uint8_t *>(gathered[r]) + off;
  rc = hx::gemm_impl(&dd, s, &peers);
  if (rc != HX_OK) return rc;
  // Exit: every peer's stores into this rank's buffer are complete.
  return hx::peer_barrier(flags, rank, world, 2 * epoch + 2, error_flag, s);
}

// Per-device streams and events of the copy-engine gather: one stream per
// peer slot (copies to different peers run on different DMA engines at once)
// and a pool of events for the chunk hand-offs.  Created on first use, kept
// until exit.
namespace hx {
namespace {
constexpr int kCeMaxChunks = 16;
struct CeResources {
  bool ready = false;
  cudaStream_t peer_stream[7];
  cudaEvent_t chunk_done[kCeMaxChunks];
  cudaEvent_t entry_done, peer_done[7];
};
CeResources g_ce[kMaxDevices];
std::mutex g_ce_mu;

int ce_resources(CeResources **out) {
  const int dev = current_device_ordinal();
  if (dev < 0) return arg_fail("device index out of range");
  std::lock_guard<std::mutex> lock(g_ce_mu);
  CeResources &r = g_ce[dev];
  if (!r.ready) {
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 7 && e == cudaSuccess; ++i)
      e = cudaStreamCreateWithFlags(&r.peer_stream[i], cudaStreamNonBlocking);
    for (int i = 0; i < kCeMaxChunks && e == cudaSuccess; ++i)
      e = cudaEventCreateWithFlags(&r.chunk_done[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r.entry_done, cudaEventDisableTiming);
    for (int i = 0; i < 7 && e == cudaSuccess; ++i)
      e = cudaEventCreateWithFlags(&r.peer_done[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "copy-engine gather set-up");
    r.ready = true;
  }
  *out = &r;
  return HX_OK;
}
}  // namespace
}  // namespace hx

int hx_sharded_gemm_gather_ce(const hx_gemm_desc *d, int rank, int world, void *const *gathered,
                              int32_t *const *flags, int32_t epoch, int32_t *error_flag, int chunks,
                              void *stream) {
  hx::g_last_error.clear();
  if (!d || !gathered || !flags || world < 1 || world > 8 || rank < 0 || rank >= world || epoch < 0 ||
      epoch > (INT32_MAX - 2) / 2 || chunks < 0 || chunks > hx::kCeMaxChunks)
    return HX_E_INVALID_ARG;
  for (int r = 0; r < world; ++r)
    if (!gathered[r] || !flags[r]) return HX_E_INVALID_ARG;
  if (d->ldc != d->N) {
    hx::g_last_error = "gather needs a contiguous shard (ldc == N)";
    return HX_E_INVALID_ARG;
  }
  const int cz = hx::esize(d->c_dtype), az = hx::esize(d->a_dtype);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t slot = static_cast<size_t>(rank) * d->M * d->N * cz;
  hx_gemm_desc dd = *d;
  dd.C = static_cast<uint8_t *>(gathered[rank]) + slot;
  if (world == 1) return hx::gemm_impl(&dd, s);
  hx::CeResources *R = nullptr;
  int rc = hx::ce_resources(&R);
  if (rc != HX_OK) return rc;
  // Row chunks: whole 256-row pair tiles.  Automatic: up to 6, measured best
  // at the 16384-row LM head on 2 GPUs (fewer leave a long last copy, more
  // add per-chunk GEMM tails).
  if (chunks == 0) chunks = static_cast<int>(std::min<int64_t>(6, std::max<int64_t>(1, d->M / 2048)));
  int64_t rows = (d->M + chunks - 1) / chunks;
  rows = std::max<int64_t>(256, (rows + 255) / 256 * 256);
  chunks = static_cast<int>((d->M + rows - 1) / rows);
  cudaError_t e;
  // Entry barrier on the first peer stream, concurrent with the first GEMM
  // chunk (which writes only this rank's own buffer): every peer has reached
  // this call, so its buffer may be overwritten.
  e = cudaEventRecord(R->chunk_done[0], s);  // peer streams start after the caller's prior work
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaEventRecord");
  e = cudaStreamWaitEvent(R->peer_stream[0], R->chunk_done[0], 0);
  if (e != cudaSuccess) return hx::cuda_fail(e, "cudaStreamWaitEvent");
  rc = hx::peer_barrier(flags, rank, world, 2 * epoch + 1, error_flag, R->peer_stream[0]);
  if (rc != HX_OK) return rc;
  if ((e = cudaEventRecord(R->entry_done, R->peer_stream[0])) != cudaSuccess)
    return hx::cuda_fail(e, "cudaEventRecord");
  const int npeer = world - 1;
  for (int i = 1; i < npeer; ++i)
    if ((e = cudaStreamWaitEvent(R->peer_stream[i], R->entry_done, 0)) != cudaSuccess)
      return hx::cuda_fail(e, "cudaStreamWaitEvent");
  for (int c = 0; c < chunks; ++c) {
    const int64_t r0 = c * rows, nr = std::min<int64_t>(rows, d->M - r0);
    hx_gemm_desc cd = dd;
    cd.M = nr;
    cd.A = static_cast<const uint8_t *>(d->A) + static_cast<size_t>(r0) * d->lda * az;
    cd.C = static_cast<uint8_t *>(dd.C) + static_cast<size_t>(r0) * d->N * cz;
    if (cd.residual)
      cd.residual = static_cast<const uint8_t *>(d->residual) + static_cast<size_t>(r0) * d->ldr * cz;
    rc = hx::gemm_impl(&cd, s);
    if (rc != HX_OK) return rc;
    if ((e = cudaEventRecord(R->chunk_done[c], s)) != cudaSuccess) return hx::cuda_fail(e, "cudaEventRecord");
    const size_t bytes = static_cast<size_t>(nr) * d->N * cz;
    for (int i = 0, r = 0; r < world; ++r) {
      if (r == rank) continue;
      cudaStream_t ps = R->peer_stream[i++];
      if ((e = cudaStreamWaitEvent(ps, R->chunk_done[c], 0)) != cudaSuccess)
        return hx::cuda_fail(e, "cudaStreamWaitEvent");
      e = cudaMemcpyAsync(static_cast<uint8_t *>(gathered[r]) + slot + static_cast<size_t>(r0) * d->N * cz,
                          cd.C, bytes, cudaMemcpyDeviceToDevice, ps);
      if (e != cudaSuccess) return hx::cuda_fail(e, "cudaMemcpyAsync(peer chunk)");
    }
  }
  // Exit: after every copy of this rank has landed, publish and wait for the
  // peers' copies into this rank's buffer (bounded).
  for (int i = 1; i < npeer; ++i) {
    if ((e = cudaEventRecord(R->peer_done[i], R->peer_stream[i])) != cudaSuccess)
      return hx::cuda_fail(e, "cudaEventRecord");
    if ((e = cudaStreamWaitEvent(R->peer_stream[0], R->peer_done[i], 0)) != cudaSuccess)
      return hx::cuda_fail(e, "cudaStreamWaitEvent");
  }
  rc = hx::peer_barrier(flags, rank, world, 2 * epoch + 2, error_flag, R->peer_stream[0]);
  if (rc != HX_OK) return rc;
  if ((e = cudaEventRecord(R->peer_done[0], R->peer_stream[0])) != cudaSuccess)
    return hx::cuda_fail(e, "cudaEventRecord");
  if ((e = cudaStreamWaitEvent(s, R->peer_done[0], 0)) != cudaSuccess)
    return hx::cuda_fail(e, "cudaStreamWaitEvent");
  return HX_OK;
}

int hx_sharded_gemm_allgather(const hx_gemm_desc *d, int rank, int world, void *comm,
                              void *gathered, void *stream) {
  if (!d || world < 1 || rank < 0 || rank >= world) return HX_E_INVALID_ARG;
  int rc = hx_gemm(d, stream);
  if (rc != HX_OK || gathered == nullptr) return rc;
  if (d->ldc != d->N) {
    hx::g_last_error = "gather needs a contiguous shard (ldc == N)";
    return HX_E_INVALID_ARG;
  }
  if (!comm) return HX_E_INVALID_ARG;
  if (!load_nccl()) return HX_E_NCCL;
  const size_t bytes = static_cast<size_t>(d->M) * d->N * hx::esize(d->c_dtype);
  // ncclInt8 == 0: gather raw bytes.
  int r = g_nccl.all_gather(d->C, gathered, bytes, 0, comm, static_cast<cudaStream_t>(stream));
  if (r != 0) return nccl_fail(r, "ncclAllGather");
  return HX_OK;
}

int hx_shards_to_rows(const void *src, void *dst, int world, int64_t M, int64_t shard_cols,
                      int elem_bytes, void *stream) {
  if (!src || !dst || world < 1 || M < 0 || shard_cols < 0 || elem_bytes <= 0)
    return HX_E_INVALID_ARG;
  const int64_t row_bytes = shard_cols * elem_bytes;
  const int64_t total = M * world * ((row_bytes + 15) / 16);
  if (total == 0) return HX_OK;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 16);
  hx::shards_to_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                              static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), world, M, row_bytes);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return hx::cuda_fail(e, "shards_to_rows_kernel");
  return HX_OK;
}

}  // extern "C"

