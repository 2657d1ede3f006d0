// Error string, launch checks, SM count and tensor-map encoding for the C ABI.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "d3_host.h"

namespace d3 {

namespace {
thread_local std::string g_last_error;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}
}  // namespace

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(D3_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return D3_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("D3MOE_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

int encode_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t cols,
                   uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto fn = get_encode_fn();
  if (!fn) return set_error(D3_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned(base, 16)) return set_error(D3_EINVAL, "TMA base address must be 16-byte aligned");
  if (pitch_bytes % 16) return set_error(D3_EINVAL, "TMA row pitch must be a multiple of 16 bytes");
  CUtensorMapDataType dt;
  switch (elem_bytes) {
    case 1: dt = CU_TENSOR_MAP_DATA_TYPE_UINT8; break;
    case 2: dt = CU_TENSOR_MAP_DATA_TYPE_UINT16; break;
    case 4: dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32; break;
    default: return set_error(D3_EINVAL, "unsupported TMA element size %d", elem_bytes);
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(D3_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return D3_OK;
}

}  // namespace d3

extern "C" int d3_version(void) { return 1; }

extern "C" const char* d3_last_error_string(void) { return d3::g_last_error.c_str(); }
