// Shared device helpers for the d3moe sm_100a kernels.
//
// Everything here is hand-written inline PTX or plain CUDA: mbarrier rings with
// bounded waits, 2-D TMA tile loads into the issuing CTA's own shared memory,
// ldmatrix / mma.sync fragments, and the number formats of the FP8 MoE path
// (E4M3 activations and weights, BF16 tensors, FP32 block scales).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "d3_internal.h"

namespace d3 {

// Status codes a kernel writes into its caller-provided status word.
enum DeviceStatus : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,  // an mbarrier or dependency wait gave up (bounded spin)
  kDevBadRow = 2,       // a row map named a row outside its tensor (row 0 was used)
};

// Row gather (RowGather, d3_internal.h): a keep value outside [0, x_rows)
// records kDevBadRow in the status word and reads row 0 instead, so no access
// leaves the tensor.

__device__ __forceinline__ int64_t gather_row(const RowGather& g, int64_t t) {
  if (g.keep == nullptr) return t;
  const int64_t r = __ldg(g.keep + t);
  if (r >= 0 && r < g.x_rows) return r;
  if (g.status) atomicExch(g.status, kDevBadRow);
  return 0;
}

__device__ __forceinline__ bool padding_row(const PaddingRoute& p, int64_t t) {
  if (p.slots == nullptr) return false;
  const int64_t slot = p.slots_i64 ? __ldg(static_cast<const int64_t*>(p.slots) + t)
                                   : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(p.slots) + t));
  return slot >= p.padding_start;
}

// Upper bound of any device-side wait, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch. Every kernel of this library calls pdl_wait()
// before it reads anything a preceding kernel wrote: when it was launched
// with programmatic stream serialisation it may have started while that
// kernel was still running, and the wait returns once the predecessor has
// completed and its writes are visible (a no-op otherwise). pdl_trigger()
// lets the next kernel of the stream begin launching early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Entry of the library's short kernels: allow the next kernel of the stream
// to start launching right away, then wait for the previous one. The next
// kernel is released only once every CTA of this grid has executed the
// trigger (so all of them are resident and none can be starved of an SM by
// it), and its own pdl_wait() still waits for this whole grid to complete,
// so only launch latency and prologue overlap, never data.
__device__ __forceinline__ void pdl_enter() {
  pdl_trigger();
  pdl_wait();
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false when
// the wait ran past kWaitLimitNs; the caller records the failure and unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// -------------------------------------------------------------------- TMA --
// 2-D tiled bulk tensor load into this CTA's shared memory, completion counted
// on an mbarrier in bytes. Coordinates are {inner (bytes/elements), row}.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t c0,
                                            int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Same as tma_load_2d with an L2 eviction-priority hint (evict_first for
// weights that are streamed exactly once per call).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map,
                                                 int32_t c0, int32_t c1, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned)
// from this CTA's shared memory to global memory, tracked in the calling
// thread's bulk-async group state.
__device__ __forceinline__ void bulk_store_s2g(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(ssrc)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Until every group this thread committed has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Until every group this thread committed has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 4-byte asynchronous global->shared copy (LDGSTS), completion tracked by an
// mbarrier through cp_async_arrive_noinc.
__device__ __forceinline__ void cp_async_4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

// 16-byte asynchronous global->shared copy that bypasses L1, tracked by
// commit/wait groups.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Wait until at most N committed groups of this thread are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Arrive on `bar` once every cp.async issued so far by this thread has landed.
// The arrival is not added to the pending count (.noinc): the barrier's
// expected count must include it.
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile written by TMA
// with CU_TENSOR_MAP_SWIZZLE_128B (rows of 128 bytes, 1024-byte aligned base).
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ------------------------------------------------------- ldmatrix / mma.sync --
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

// D = A(16x32 e4m3, row) * B(32x8 e4m3, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_e4m3_16832(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]),
        "f"(c[2]), "f"(c[3]));
}

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1,
                                              const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// Two E4M3 bytes (low byte first) -> f16x2, exact (E4M3 is a subset of f16).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// fp32 -> E4M3 byte, round-to-nearest-even, saturating to +-448.
__device__ __forceinline__ uint8_t f32_to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// bf16_round on the integer pipes (round-to-nearest-even on the bit pattern;
// finite inputs, overflow rounds to infinity like the conversion does). Keeps
// the conversion unit free for the exponentials of the SiLU.
__device__ __forceinline__ float bf16_round_alu(float v) {
  uint32_t u = __float_as_uint(v);
  u += 0x7fffu + ((u >> 16) & 1u);
  return __uint_as_float(u & 0xffff0000u);
}

// acc = fma(hi(x), hi(w), fma(lo(x), lo(w), acc)) for bf16x2 words x, w: the
// mixed-precision FMA takes bf16 operands directly (their products are exact
// in fp32), so no bf16 -> fp32 unpacking is needed.
__device__ __forceinline__ float fma_bf16x2_seq(uint32_t x, uint32_t w, float acc) {
  asm("{\n\t.reg .b16 xl, xh, wl, wh;\n\t"
      "mov.b32 {xl, xh}, %1;\n\t"
      "mov.b32 {wl, wh}, %2;\n\t"
      "fma.rn.f32.bf16 %0, xl, wl, %0;\n\t"
      "fma.rn.f32.bf16 %0, xh, wh, %0;\n\t}"
      : "+f"(acc)
      : "r"(x), "r"(w));
  return acc;
}

// (a0, a1) += (x0, x1) * s as one packed fp32x2 FMA (two IEEE fp32 FMAs).
__device__ __forceinline__ void ffma2(float& a0, float& a1, float x0, float x1, float s) {
  asm("{\n\t.reg .b64 d, x, s2, c;\n\t"
      "mov.b64 x, {%2, %3};\n\t"
      "mov.b64 s2, {%4, %4};\n\t"
      "mov.b64 c, {%0, %1};\n\t"
      "fma.rn.f32x2 d, x, s2, c;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(x0), "f"(x1), "f"(s));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Named barrier among `nthreads` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Gated projection input (src/drama3/fused_projection.py:22-29): with a gate,
// x becomes bf16(x * a) where a = bf16(silu(g)) (mode 1, GATE_SWIGLU) or
// bf16(sigmoid(g)) (mode 2, GATE_SIGMOID), sigmoid(g) = 1 / (1 + exp(-g)) in
// fp32.
__device__ __forceinline__ float gate_activation(float g, int mode) {
  const float sg = 1.0f / (1.0f + expf(-g));
  return bf16_round(mode == 1 ? g * sg : sg);
}

// Activation FP8 quantiser for one 128-element group: scale = max(amax,1e-10)/448
// (IEEE division), element = clamp(x/scale, -448, 448) rounded to E4M3.
__device__ __forceinline__ float act_scale_from_amax(float amax) {
  return __fdiv_rn(fmaxf(amax, 1e-10f), 448.0f);
}
__device__ __forceinline__ uint8_t act_quant(float x, float scale) {
  float q = __fdiv_rn(x, scale);
  q = fminf(fmaxf(q, -448.0f), 448.0f);
  return f32_to_e4m3(q);
}

// x / scale rounded to nearest, from rs = RN(1/scale) with one correction
// step (Markstein, IBM J. Res. Dev. 34(1), 1990): q0 = RN(x*rs), the remainder
// r = x - q0*scale is exact in one FMA, and RN(q0 + r*rs) is the correctly
// rounded quotient for the normal range the activation quantiser works in
// (|x/scale| <= 448). A zero remainder means q0 is already exact; keeping it
// also keeps the sign of a zero quotient (x = -0 gives -0, like the division).
// Costs 3 operations per element instead of a division.
__device__ __forceinline__ float div_by_scale(float x, float scale, float rs) {
  const float q0 = x * rs;
  const float r = fmaf(-q0, scale, x);
  return r == 0.0f ? q0 : fmaf(r, rs, q0);
}

// Two floats -> two E4M3 bytes (lo in the low byte), round-to-nearest-even,
// saturating to +-448.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// act_quant with rs = __frcp_rn(scale) computed once per group: the same
// bytes (x / scale is correctly rounded by div_by_scale).
__device__ __forceinline__ float act_quant_value(float x, float scale, float rs) {
  return fminf(fmaxf(div_by_scale(x, scale, rs), -448.0f), 448.0f);
}
__device__ __forceinline__ uint32_t act_quant4(float x0, float x1, float x2, float x3, float scale,
                                               float rs) {
  return static_cast<uint32_t>(f32x2_to_e4m3x2(act_quant_value(x0, scale, rs),
                                               act_quant_value(x1, scale, rs))) |
         (static_cast<uint32_t>(f32x2_to_e4m3x2(act_quant_value(x2, scale, rs),
                                                act_quant_value(x3, scale, rs)))
          << 16);
}

// Exact split of a bf16 activation group for the FP8 tensor cores: with s
// chosen so that the group's max magnitude lies in [2^7, 2^8) after scaling
// by 2^s, x * 2^s = hi + lo / 16 with hi = e4m3(x * 2^s) and
// lo = e4m3((x * 2^s - hi) * 16), exact for |x * 2^s| >= 2^-6 (error below
// 2^-21 of the group max otherwise). shift_for_amax returns s.
__device__ __forceinline__ int shift_for_amax(float amax) {
  int e = 8;
  if (amax > 0.f && isfinite(amax)) frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
  return 8 - e;
}
// Four scaled values -> their hi and lo E4M3 bytes (little-endian order).
__device__ __forceinline__ void split_e4m3x4(const float (&xs)[4], uint32_t& hi, uint32_t& lo) {
  const uint16_t h01 = f32x2_to_e4m3x2(xs[0], xs[1]), h23 = f32x2_to_e4m3x2(xs[2], xs[3]);
  const uint32_t hh01 = e4m3x2_to_f16x2(h01), hh23 = e4m3x2_to_f16x2(h23);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hh01));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&hh23));
  hi = static_cast<uint32_t>(h01) | (static_cast<uint32_t>(h23) << 16);
  lo = static_cast<uint32_t>(f32x2_to_e4m3x2((xs[0] - a.x) * 16.0f, (xs[1] - a.y) * 16.0f)) |
       (static_cast<uint32_t>(f32x2_to_e4m3x2((xs[2] - b.x) * 16.0f, (xs[3] - b.y) * 16.0f)) << 16);
}

}  // namespace d3
