// Weight-only FP8 GEMV / small GEMM on tcgen05: y bf16 [T,N] = x bf16 [T,K] .
// dequant(Wq e4m3 [N,K], S f32 [N/128, K/128])^T, fp32 accumulation.
//
// The reference's dense FP8 projection (experimental_fp8._gemv) multiplies
// bf16 activations by block-dequantised FP8 weights. Here the weights stay in
// E4M3 for the MMA (no widening: the tensor core reads the bytes TMA put in
// shared memory) and the activations are split beforehand, exactly, into two
// E4M3 terms per 1x128 group (dense_split_kernel: x * 2^s = hi + lo / 16,
// exact for every element within 2^13 of its group's maximum, error below
// 2^-21 of that maximum otherwise). One tcgen05.mma kind::f8f6f4 with
// N = 2*TP computes W.hi^T and W.lo^T side by side into one TMEM slot. The
// 128x128 weight block scale is uniform over one 128-wide K block of a
// 128-row tile, so each K block has its own TMEM slot, folded into registers
// as acc += (D_hi + D_lo / 16) * S[tile][kb] * 2^-s[t][kb].
//
// Widening the weights to bf16 in shared memory instead (kind::f16) was
// built and measured first: the e4m3 -> bf16 pass costs 700-1200 cycles per
// 16 KB K block per SM (integer/FMA and shared-memory bound), which kept that
// kernel at about 10 us for 4096x2048; splitting the activations moves the
// only conversion to 1/32 of the bytes.
//
// One CTA per (128-row tile, K range, 64-token group); the K ranges of a tile
// form one thread-block cluster (1, 2, 4 or 8 CTAs), whose CTAs add their fp32
// partials through distributed shared memory in a fixed rank order
// (deterministic, no global scratch, no atomics).
//
// Warp roles (10 warps):
//   warp 0     TMA: per K block the e4m3 weight tile [128 rows x 128 B] and the
//              hi and lo activation tiles [TP rows x 128 B] into a 5-stage
//              ring. Weight loads do not depend on earlier kernels, so the
//              first stages are issued right after the barriers are
//              initialised, before the TMEM allocation and the
//              programmatic-dependent-launch wait; activation loads after it.
//   warp 1     MMA issue (one thread): 4 MMAs (M=128, N=2*TP, K=32) per K
//              block into TMEM slot kb % 4; commits hand the slot to the
//              promoters and the ring stage back to the loader.
//   warps 2-9  promoters: fold TMEM slot kb into fp32 registers (warp w reads
//              the 32 lanes of quadrant w % 4 and half of the TP tokens: one
//              weight row per thread).
// Epilogue: partials [TP][128] fp32 in shared memory (reusing the ring). CTA
// rank r owns tokens [r*TP/split, (r+1)*TP/split): every CTA pushes each
// peer's token rows into that peer's receive buffer with one bulk copy
// (shared::cta -> shared::cluster, completion counted in bytes on the
// receiver's mbarrier), and the owner adds the split partials of its rows in
// rank order and stores bf16. Two split cluster barriers (arrive early, wait
// late) order the receivers' barrier set-up before any push and keep every
// CTA, and so every push source and target, alive until all owners have
// received; the arrivals come long before the waits, so the waits cost
// nothing in the common case. Every thread of every CTA reaches both
// barriers, also after a timed-out wait.
#pragma once

#include "d3_common.cuh"
#include "tcgen05.cuh"

namespace d3 {

constexpr int kDtStages = 5;
constexpr int kDtSlots = 4;
constexpr int kDtPromoterWarps = 8;
constexpr int kDtThreads = 64 + 32 * kDtPromoterWarps;
constexpr int kDtMaxSplit = 8;    // 1, 2, 4 or 8
constexpr int kDtTokens = 64;     // tokens per CTA (grid.y walks 64-token groups)
constexpr int kDtMaxKbPerCta = 32;

struct DenseTcArgs {
  const float* wscale;   // [tiles, KB]
  const float* xscale;   // [T, KB] = 2^-s of each activation group
  __nv_bfloat16* y;      // [T, y_ld]
  int64_t y_ld;
  int T, N, KB;
  int split;             // K ranges per tile (= cluster size along grid.x)
  int kb_per_split;      // <= kDtMaxKbPerCta
  int vec_store;         // y rows allow 8-byte stores (y_ld % 4 == 0, y 8-byte aligned)
  int32_t* status;
};

template <int TP>
struct DtSmem {
  static constexpr int kW = 128 * 128;      // e4m3 weight K block
  static constexpr int kX = 2 * TP * 128;   // e4m3 hi rows then lo rows of one K block
  static constexpr int kStage = kW + kX;
  static constexpr int kRing = kDtStages * kStage;
  static constexpr int kRecvOff = kRing;    // [split][TP/split][128] fp32 from peers
  static constexpr int kRecv = TP * 128 * 4;
  static constexpr int kXscOff = kRecvOff + kRecv;  // [TP][kDtMaxKbPerCta] f32
  static constexpr int kBarOff = kXscOff + TP * kDtMaxKbPerCta * 4;
  // full[S], empty[S], dfull[SL], dempty[SL], drain, recv
  static constexpr int kNumBars = 2 * kDtStages + 2 * kDtSlots + 2;
  static constexpr int kTmemOff = kBarOff + kNumBars * 8;
  static constexpr int kAbortOff = kTmemOff + 16;
  static constexpr int kEnd = kAbortOff + 16;
  static constexpr size_t bytes() { return 1024 + static_cast<size_t>(kEnd); }
  static constexpr uint32_t kTmemCols = kDtSlots * 2 * TP < 32 ? 32 : kDtSlots * 2 * TP;
  static_assert(TP * 128 * 4 <= kRing, "partials must fit in the ring");
  static_assert(kDtSlots * 2 * TP <= 512, "TMEM slots");
};
static_assert(DtSmem<64>::bytes() <= 227 * 1024, "dense tcgen05 GEMV shared memory");

// 32 lanes x N columns of fp32 from TMEM (N = 8, 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&r)[N]) {
  if constexpr (N == 32) {
    tc::tmem_ld_32x32b_x32(taddr, r);
  } else if constexpr (N == 16) {
    tc::tmem_ld_32x32b_x16(taddr, r);
  } else {
    static_assert(N == 8, "8, 16 or 32 columns");
    uint32_t u[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
          "=r"(u[7])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = __uint_as_float(u[i]);
  }
}

// Relaxed arrival: no release ordering of this thread's earlier memory
// operations (with .release the arrive waited for the weight TMA loads thread 0
// had just issued, over a microsecond). The barriers' visibility comes from
// fence.mbarrier_init.release.cluster, and the pushes complete through the
// receivers' mbarriers, so the cluster barriers only order lifetimes.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}

// Bulk copy of `bytes` (multiple of 16) from this CTA's shared memory to a
// peer's shared memory (addresses from cluster_map), completion counted in
// bytes on the peer's mbarrier.
__device__ __forceinline__ void bulk_push_dsmem(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                                uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ bool dt_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int32_t* status) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  if (status) atomicExch(status, kDevWaitTimeout);
  return false;
}

template <int TP>
__global__ void __launch_bounds__(kDtThreads, 1)
    dense_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_hi,
                    const __grid_constant__ CUtensorMap tm_lo, const DenseTcArgs args) {
  using L = DtSmem<TP>;
  constexpr int HALF = TP / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + kDtStages;
  uint64_t* dfull = empty + kDtStages;
  uint64_t* dempty = dfull + kDtSlots;
  uint64_t* drain = dempty + kDtSlots;
  uint64_t* recv = drain + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::kTmemOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOff);
  float* xsc = reinterpret_cast<float*>(smem + L::kXscOff);  // [TP][kDtMaxKbPerCta]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = args.split;
  const int tile = blockIdx.x / split;
  const int crank = blockIdx.x - tile * split;  // rank in the cluster (1-D clusters along x)
  const int kb0 = crank * args.kb_per_split;
  const int nkb = max(0, min(args.kb_per_split, args.KB - kb0));
  const int t0 = blockIdx.y * kDtTokens;
  const int rows_per_rank = TP / split;                 // token rows each rank owns
  const uint32_t slice_bytes = rows_per_rank * 128 * 4;  // one rank's rows of a partial
  const int pre = min(nkb, kDtStages);
  int armed[kDtStages];
#pragma unroll
  for (int s = 0; s < kDtStages; ++s) armed[s] = -1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < kDtSlots; ++s) {
      mbar_init(&dfull[s], 1);
      mbar_init(&dempty[s], kDtPromoterWarps);
    }
    mbar_init(drain, 1);
    mbar_init(recv, 1);
    *abort_flag = 0;
    fence_mbar_init();
    // the bytes every peer will push (armed before this CTA arrives on the
    // cluster barrier the pushers wait for)
    if (split > 1) mbar_arrive_expect_tx(recv, (split - 1) * slice_bytes);
    // weights of the first stages right away: constants, no dependency
    prefetch_tensormap(&tm_w);
    const uint64_t pol_w = l2_policy_evict_first();
    for (int kb = 0; kb < pre; ++kb) {
      mbar_arrive_expect_tx(&full[kb], L::kStage);
      armed[kb] = 0;
      tma_load_2d_hint(smem + kb * L::kStage, &tm_w, (kb0 + kb) * 128, tile * 128, &full[kb], pol_w);
    }
  }
  if (warp == 1) {
    tc::tmem_alloc(tslot, L::kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  if (split > 1) cluster_arrive();  // this CTA's receive barrier is set up
  tc::fence_after_thread_sync();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA --
    if (lane == 0) {
      prefetch_tensormap(&tm_hi);
      prefetch_tensormap(&tm_lo);
      const uint64_t pol_w = l2_policy_evict_first();
      pdl_wait();  // the activation split belongs to an earlier kernel
      for (int kb = 0; kb < pre; ++kb) {
        uint8_t* xs = smem + kb * L::kStage + L::kW;
        tma_load_2d(xs, &tm_hi, (kb0 + kb) * 128, t0, &full[kb]);
        tma_load_2d(xs + TP * 128, &tm_lo, (kb0 + kb) * 128, t0, &full[kb]);
      }
      for (int kb = pre; kb < nkb; ++kb) {
        const int s = kb % kDtStages;
        const uint32_t ph = (kb / kDtStages) & 1;
        if (!dt_wait(&empty[s], ph ^ 1, abort_flag, args.status)) break;
        mbar_arrive_expect_tx(&full[s], L::kStage);
        armed[s] = static_cast<int>(ph);
        uint8_t* st = smem + s * L::kStage;
        tma_load_2d_hint(st, &tm_w, (kb0 + kb) * 128, tile * 128, &full[s], pol_w);
        tma_load_2d(st + L::kW, &tm_hi, (kb0 + kb) * 128, t0, &full[s]);
        tma_load_2d(st + L::kW + TP * 128, &tm_lo, (kb0 + kb) * 128, t0, &full[s]);
      }
      pdl_trigger();
      // no copy may still be writing shared memory when the CTA moves on
      for (int s = 0; s < kDtStages; ++s)
        if (armed[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(armed[s]));
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA --
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_e4m3_f32(128, 2 * TP);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % kDtStages, slot = kb % kDtSlots;
        ok = dt_wait(&full[s], (kb / kDtStages) & 1, abort_flag, args.status) &&
             dt_wait(&dempty[slot], ((kb / kDtSlots) & 1) ^ 1, abort_flag, args.status);
        if (!ok) break;
        tc::fence_after_thread_sync();
        const uint32_t w0 = smem_u32(smem + s * L::kStage);
        const uint32_t x0 = w0 + L::kW;
        const uint32_t d = tmem + slot * 2 * TP;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          tc::mma_f8f6f4(d, tc::smem_desc_sw128(w0 + ks * 32), tc::smem_desc_sw128(x0 + ks * 32), idesc,
                         ks != 0 ? 1u : 0u);
        tc::mma_commit(&dfull[slot]);
        tc::mma_commit(&empty[s]);
      }
      // every MMA issued so far has completed once `drain` flips (bounded)
      tc::mma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
  }

  // ----------------------------------------------------------- promoters --
  float acc[HALF];
#pragma unroll
  for (int i = 0; i < HALF; ++i) acc[i] = 0.f;
  const bool promoter = warp >= 2;
  const int quad = warp & 3, half = (warp - 2) >> 2;
  const int row = 32 * quad + lane;  // weight row of the tile (TMEM lane)
  if (promoter) {
    // the activation group scales of this CTA's tokens and K blocks
    pdl_wait();
    for (int i = threadIdx.x - 64; i < TP * nkb; i += 32 * kDtPromoterWarps) {
      const int t = i / nkb, j = i - t * nkb;
      xsc[t * kDtMaxKbPerCta + j] =
          t0 + t < args.T ? __ldg(args.xscale + static_cast<int64_t>(t0 + t) * args.KB + kb0 + j) : 0.f;
    }
    named_bar_sync(1, 32 * kDtPromoterWarps);
    const float* ws = args.wscale + static_cast<int64_t>(tile) * args.KB + kb0;
    for (int j = 0; j < nkb; ++j) {
      const int slot = j % kDtSlots;
      if (!dt_wait(&dfull[slot], (j / kDtSlots) & 1, abort_flag, args.status)) break;
      tc::fence_after_thread_sync();
      float vh[HALF], vl[HALF];
      const uint32_t col = slot * 2 * TP + half * HALF;
      tmem_ld_cols<HALF>(tc::tmem_addr(tmem, 32 * quad, col), vh);
      tmem_ld_cols<HALF>(tc::tmem_addr(tmem, 32 * quad, col + TP), vl);
      tc::tmem_ld_wait();
      const float sw = __ldg(ws + j);
#pragma unroll
      for (int i = 0; i < HALF; ++i) {
        const float f = sw * xsc[(half * HALF + i) * kDtMaxKbPerCta + j];
        acc[i] = fmaf(vh[i], f, acc[i]);
        acc[i] = fmaf(vl[i], f * 0.0625f, acc[i]);
      }
      tc::fence_before_thread_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[slot]);
    }
  }

  // ----------------------------------------------------------- epilogue --
  // all MMAs drained (the MMA thread waited) and all TMEM loads done; the
  // ring is free for the partials
  tc::fence_before_thread_sync();
  __syncthreads();
  if (warp == 1) {  // TMEM is no longer needed: free it for the next kernel
    tc::fence_after_thread_sync();
    tc::tmem_dealloc(tmem, L::kTmemCols);
  }
  float* part = reinterpret_cast<float*>(smem);  // [TP][128]
  if (promoter) {
#pragma unroll
    for (int i = 0; i < HALF; ++i) part[(half * HALF + i) * 128 + row] = acc[i];
    fence_proxy_async_smem();  // the partials are read by bulk copies
  }
  __syncthreads();
  const float* rbuf = reinterpret_cast<const float*>(smem + L::kRecvOff);  // [split][rows][128]
  if (split > 1) {
    cluster_wait();  // every peer's receive barrier is set up
    // push every peer its token rows of this CTA's partial
    if (threadIdx.x == 0) {
      const uint32_t rdst = smem_u32(smem + L::kRecvOff) + crank * slice_bytes;
      for (int r = 0; r < split; ++r) {
        if (r == crank) continue;
        bulk_push_dsmem(cluster_map(rdst, r), part + r * rows_per_rank * 128, slice_bytes,
                        cluster_map(smem_u32(recv), r));
      }
    }
    if (promoter) dt_wait(recv, 0, abort_flag, args.status);  // the peers' rows have landed
    __syncthreads();
    cluster_arrive();  // this CTA has received everything pushed to it
  }
  pdl_wait();  // y may be read by earlier kernels
  if (promoter && !*abort_flag) {
    const int wt = threadIdx.x - 64;
    const int own0 = crank * rows_per_rank;  // first token row this rank owns
    for (int g = wt; g < rows_per_rank * 32; g += 32 * kDtPromoterWarps) {
      const int tr = g >> 5, c4 = (g & 31) * 4;  // row within the slice, first column
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < split; ++r) {  // rank order
        const float4 v = r == crank
                             ? *reinterpret_cast<const float4*>(part + (own0 + tr) * 128 + c4)
                             : *reinterpret_cast<const float4*>(rbuf + (r * rows_per_rank + tr) * 128 + c4);
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      const int t = t0 + own0 + tr, n = tile * 128 + c4;
      if (t < args.T && n < args.N) {
        __nv_bfloat16* yr = args.y + static_cast<int64_t>(t) * args.y_ld + n;
        if (args.vec_store && n + 3 < args.N) {
          uint2 pk;
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk.x) : "f"(sum.y), "f"(sum.x));
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk.y) : "f"(sum.w), "f"(sum.z));
          *reinterpret_cast<uint2*>(yr) = pk;
        } else {
          const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (n + q < args.N) yr[q] = __float2bfloat16_rn(sv[q]);
        }
      }
    }
  }
  // no CTA leaves while a peer may still push into it or read its partials
  if (split > 1) cluster_wait();
}

}  // namespace d3
