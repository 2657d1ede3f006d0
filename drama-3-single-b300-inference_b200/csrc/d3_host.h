// Host-side helpers shared by the C-ABI translation units: error reporting,
// argument checks and TMA tensor-map encoding through the driver entry point.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "d3moe.h"  // include/ of the repository root (passed with -I)

namespace d3 {

// Records a printf-style message as this thread's last error and returns `code`.
int set_error(int code, const char* fmt, ...);

// Checks the launch that was just enqueued.
int check_launch(const char* what);

// Encodes a 2-D tiled tensor map over a row-major [rows, cols] tensor of
// `elem_bytes`-byte elements with row pitch `pitch_bytes`, a box of
// [box_rows, box_cols] and 128-byte swizzle. Returns D3_OK or an error.
int encode_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows);

// Number of SMs of the current device (cached per device).
int sm_count();

// Whether kernels are launched with programmatic stream serialisation (PDL):
// on unless D3MOE_PDL=0 in the environment (read once).
bool pdl_enabled();

// Launches kern<<<grid, block, smem, s>>>(args...) through cudaLaunchKernelEx
// with programmatic stream serialisation, so its launch and prologue overlap
// the tail of the previous kernel in the stream; every kernel of this library
// calls pdl_wait() before touching memory earlier kernels wrote. Errors are
// left for check_launch() like a <<<>>> launch.
template <typename... KArgs, typename... Args>
void launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                   Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace d3

#define D3_REQUIRE(cond, ...)                                  \
  do {                                                         \
    if (!(cond)) return ::d3::set_error(D3_EINVAL, __VA_ARGS__); \
  } while (0)
