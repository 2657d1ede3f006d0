// Router projection on the tensor cores for prefill-sized batches:
//   logits[t, r] = bf16( sum_h x[t,h] * W[r,h]  + bias[r] )
// with x bf16 [T, H] and W bf16 [R, H] (the E router rows + the shared-expert
// gate row). The reference computes this projection with a bf16 GEMM as well
// (F.linear, src/drama3/model.py:496-504), so the fp32 summation order inside
// the tensor core is as unspecified there as here.
//
// One CTA per 128-token x NT-row tile (NT <= 256, a multiple of 16; the rows
// are split into enough tiles that the grid covers the SMs): warp 0
// streams 64-wide K blocks of x and W through a 4-stage TMA ring (128-byte
// swizzled, K-major), warp 1 issues tcgen05.mma kind::f16 (bf16 x bf16 ->
// fp32, M=128, N=NT, K=16) into one TMEM accumulator, and all four warps read
// the accumulator back (warp w owns TMEM lanes 32w..32w+31 = tokens) and store
// bf16 logits. Every wait is bounded (mbar_wait); on a timeout the CTA sets the
// status word, drains its own copies and returns without storing.
#pragma once

#include "d3_common.cuh"
#include "tcgen05.cuh"

namespace d3 {

constexpr int kRtcStages = 4;
constexpr int kRtcThreads = 128;
constexpr int kRtcMaxN = 256;
constexpr int kRtcTokens = 128;

struct RouterTcArgs {
  const float* bias;  // [nbias] added before the bf16 rounding (nullable)
  int nbias;
  int R, T, KB;       // rows of W, tokens, 64-wide K blocks
  int nt;             // rows of W per tile (multiple of 16, <= 256)
  int tmem_cols;      // TMEM columns allocated (power of two >= max(32, nt))
  __nv_bfloat16* out;
  int64_t out_stride;
  int32_t* status;    // nullable
};

// Shared memory of one CTA for a tile of nt rows.
struct RtcSmem {
  static constexpr uint32_t kA = kRtcTokens * 128;  // x K block: 128 rows x 128 bytes
  __host__ __device__ static uint32_t stage(int nt) { return kA + static_cast<uint32_t>(nt) * 128; }
  __host__ __device__ static uint32_t bar_off(int nt) { return kRtcStages * stage(nt); }
  // full[S], empty[S], done
  static constexpr int kNumBars = 2 * kRtcStages + 1;
  __host__ __device__ static uint32_t tmem_off(int nt) { return bar_off(nt) + kNumBars * 8; }
  __host__ __device__ static uint32_t abort_off(int nt) { return tmem_off(nt) + 16; }
  __host__ __device__ static size_t bytes(int nt) { return 1024 + static_cast<size_t>(abort_off(nt)) + 16; }
};

// Instruction descriptor for kind::f16 with bf16 A and B, both K-major, fp32
// accumulation: D format F32 (1) in bits [4,6), A and B format BF16 (1) in
// [7,10) and [10,13), N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool rtc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                         int32_t* status) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  if (status) atomicExch(status, kDevWaitTimeout);
  return false;
}

__global__ void __launch_bounds__(kRtcThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const RouterTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int nt = args.nt;
  const uint32_t stage_bytes = RtcSmem::stage(nt);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + RtcSmem::bar_off(nt));
  uint64_t* empty = full + kRtcStages;
  uint64_t* done = empty + kRtcStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + RtcSmem::tmem_off(nt));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + RtcSmem::abort_off(nt));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kRtcTokens;
  const int r0 = blockIdx.y * nt;
  const int KB = args.KB;
  const int pre = min(KB, kRtcStages);
  int armed[kRtcStages];
#pragma unroll
  for (int s = 0; s < kRtcStages; ++s) armed[s] = -1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRtcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    // router weights of the first stages right away: constants, no dependency
    prefetch_tensormap(&tm_w);
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], stage_bytes);
      armed[kb] = 0;
      tma_load_2d(smem + kb * stage_bytes + RtcSmem::kA, &tm_w, kb * 64, r0, &full[kb]);
    }
  }
  if (warp == 1) {
    tc::tmem_alloc(tslot, static_cast<uint32_t>(args.tmem_cols));
    tc::tmem_relinquish();
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA --
    if (lane == 0) {
      prefetch_tensormap(&tm_x);
      pdl_wait();  // x belongs to an earlier kernel
      for (int kb = 0; kb < pre; ++kb) tma_load_2d(smem + kb * stage_bytes, &tm_x, kb * 64, t0, &full[kb]);
      for (int kb = pre; kb < KB; ++kb) {
        const int s = kb % kRtcStages;
        const uint32_t ph = (kb / kRtcStages) & 1;
        if (!rtc_wait(&empty[s], ph ^ 1, abort_flag, args.status)) break;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        armed[s] = static_cast<int>(ph);
        uint8_t* st = smem + s * stage_bytes;
        tma_load_2d(st + RtcSmem::kA, &tm_w, kb * 64, r0, &full[s]);
        tma_load_2d(st, &tm_x, kb * 64, t0, &full[s]);
      }
      pdl_trigger();
      // no copy may still be writing shared memory when the CTA moves on
      for (int s = 0; s < kRtcStages; ++s)
        if (armed[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(armed[s]));
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA --
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_f32(kRtcTokens, nt);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kRtcStages;
        if (!rtc_wait(&full[s], (kb / kRtcStages) & 1, abort_flag, args.status)) break;
        tc::fence_after_thread_sync();
        const uint32_t a0 = smem_u32(smem + s * stage_bytes);
        const uint32_t b0 = a0 + RtcSmem::kA;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)  // K = 16 bf16 = 32 bytes per MMA
          mma_bf16(tmem, tc::smem_desc_sw128(a0 + ks * 32), tc::smem_desc_sw128(b0 + ks * 32), idesc,
                   (kb | ks) != 0 ? 1u : 0u);
        tc::mma_commit(&empty[s]);
      }
      tc::mma_commit(done);  // every MMA issued so far has completed once `done` flips
    }
    __syncwarp();
  }

  // ------------------------------------------------------------ epilogue --
  const bool ok = rtc_wait(done, 0, abort_flag, args.status);
  tc::fence_after_thread_sync();
  pdl_wait();  // the logits may still be read by an earlier kernel
  const int row = 32 * warp + lane;  // TMEM lane = token of the tile
  const int t = t0 + row;
  if (ok && !*abort_flag) {
    for (int c0 = 0; c0 < nt; c0 += 16) {
      float v[16];
      tc::tmem_ld_32x32b_x16(tc::tmem_addr(tmem, 32 * warp, c0), v);
      tc::tmem_ld_wait();
      if (t < args.T) {
        __nv_bfloat16* o = args.out + static_cast<int64_t>(t) * args.out_stride;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int r = r0 + c0 + i;
          if (r < args.R && c0 + i < nt)
            o[r] = __float2bfloat16_rn(v[i] + ((args.bias && r < args.nbias) ? __ldg(args.bias + r) : 0.f));
        }
      }
    }
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_thread_sync();
    tc::tmem_dealloc(tmem, static_cast<uint32_t>(args.tmem_cols));
  }
}

}  // namespace d3
