// launch.cuh — host-side launch helpers shared by the library's translation
// units: error reporting, programmatic-dependent launch, and the tile-GEMM
// launchers whose kernels are instantiated per input kind in gemm_kind*.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <string>
#include <utility>

#include "gemm_sm100.cuh"
#include "hx_gemm.h"

namespace hx {

extern thread_local std::string g_last_error;

inline int cuda_fail(cudaError_t e, const char *where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return HX_E_CUDA;
}
inline int arg_fail(const char *why) {
  g_last_error = why;
  return HX_E_INVALID_ARG;
}
inline int unsupported(const char *why) {
  g_last_error = why;
  return HX_E_UNSUPPORTED;
}

constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in limit per block on sm_100
constexpr int kNeedsNoSplit = 1;     // internal: split-K clusters would not all be resident
constexpr uint64_t kDefaultTimeout = 4000000000ull;  // ~2 s at 2 GHz

// cudaFuncSetAttribute acts on the current device only, so a process that
// drives several GPUs must set a kernel's dynamic shared-memory limit once per
// device.  One SmemAttrOnce per kernel instantiation records, as a bit per
// device ordinal, where the attribute has been set.
struct SmemAttrOnce {
  std::atomic<uint64_t> mask{0};
};
constexpr int kMaxDevices = 64;

template <typename K>
cudaError_t ensure_max_smem(K kern, SmemAttrOnce &once, int bytes = kMaxDynSmem) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = (dev >= 0 && dev < kMaxDevices) ? (1ull << dev) : 0;
  if (bit && (once.mask.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) once.mask.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

inline int current_device_ordinal() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

// Launch with programmatic stream serialization (PDL): the kernel may begin
// while its predecessor finishes; it calls griddepcontrol.wait before its
// first global-memory access, so ordering is unchanged.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}


// Tile-GEMM launch for input kind KIND (0 f16, 1 bf16, 2 int8): picks the
// kernel instantiation for (tile_n, B layout, SwiGLU) or the CTA-pair kernel.
template <int KIND>
int dispatch_kind(int bn, bool bmn, bool sw, const CUtensorMap &ta, const CUtensorMap &tb,
                  const GemmParams &p, int grid, cudaStream_t s);
template <int KIND>
int dispatch_pair_kind(int bn, bool sw, const CUtensorMap &ta, const CUtensorMap &tb,
                       const GemmParams &p, int grid, cudaStream_t s);

}  // namespace hx
