// Test infrastructure only (the checker, never the product): a C entry point
// around the reference's own CPU matmul check, compiled from the reference
// source where it lies.
//
// test/python/mlir/hexkl_linalg_matmul/wrapper.cpp:46-66 holds `check()`,
// the plain C++ fp32-accumulated matmul the reference's HexKL test uses as
// its golden (`acc += (float)inAct[row * K + entry] * inW[entry * M + col]`,
// |out - acc| <= 1e-2 per element).  The rest of that file needs the Hexagon
// SDK and HexKL, so oracle/Makefile copies only that function's lines, at
// build time and into oracle/_ref/ (git-ignored), and this harness supplies
// what they name: the sizes and tolerance of the same file (lines 29-32) and
// a silent FARF.
#include <cstdint>

#define restrict __restrict__
#define FARF(level, ...) ((void)0)
#define MAX_DIFF 1e-2
constexpr uint32_t N = 1024;
constexpr uint32_t K = 64;
constexpr uint32_t M = 512;

#include "check_extract.inc"

// act: [N, K] fp16 bits, w: [K, M] fp16 bits, out: [N, M] fp32.
// Returns 1 when every element is within MAX_DIFF of the reference's sum.
extern "C" int hx_ref_check(const float *out, const uint16_t *act, const uint16_t *w) {
  return check(const_cast<float *>(out), reinterpret_cast<const _Float16 *>(act),
               reinterpret_cast<const _Float16 *>(w))
             ? 1
             : 0;
}

extern "C" int hx_ref_check_sizes(uint32_t *n, uint32_t *k, uint32_t *m) {
  *n = N;
  *k = K;
  *m = M;
  return 0;
}
