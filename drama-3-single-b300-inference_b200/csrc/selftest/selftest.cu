// Test-only library (libd3moe_selftest.so), kept out of the product library:
// a self-test of the failure path every waiting kernel of libd3moe.so shares.
// One thread waits, through the bounded mbar_wait of d3_common.cuh, on an
// mbarrier that nothing arrives on. The wait gives up at its limit
// (kWaitLimitNs) and the kernel records D3_STATUS_WAIT_TIMEOUT in the caller's
// status word, as a kernel whose producer never delivered would. Nothing
// faults and the context stays usable.
#include "../d3_common.cuh"
#include "d3moe_selftest.h"

namespace d3 {

namespace {

__global__ void wait_timeout_probe_kernel(int32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_mbar_init();
  // phase 0 of a fresh barrier completes only when one thread arrives; none does
  if (!mbar_wait(&bar, 0)) atomicExch(status, kDevWaitTimeout);
}

}  // namespace

}  // namespace d3

extern "C" int d3_wait_timeout_probe(int32_t* status, d3_stream_t stream) {
  if (status == nullptr) return D3_EINVAL;
  d3::wait_timeout_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(status);
  return cudaGetLastError() == cudaSuccess ? D3_OK : D3_ECUDA;
}
