// Prefill grouped GEMM on tcgen05 (tensor cores with TMEM accumulators).
//
// At prefill every expert sees hundreds to thousands of tokens, so the
// expert GEMMs are tensor-bound and belong on tcgen05. One persistent CTA per
// SM walks a static round-robin list of 128 x 256 output tiles:
//   gate_up: rows = 128 tokens of one expert, cols = 128 gate + 128 up rows of
//            W13 (the same i range), K = H;
//   down:    rows = 128 tokens (requantised activations), cols = 256 rows of
//            W2, K = I.
// Warp roles (10 warps): warp 0 issues TMA loads of A [128 x 128 B] and B
// [256 x 128 B] per 128-wide K block into a 4-stage ring; warp 1 owns TMEM
// (512 columns = two 256-column accumulators) and issues 4 MMAs
// (M=128, N=256, K=32, kind::f8f6f4, E4M3 x E4M3 -> fp32) per K block into one
// accumulator; warps 2..9 are two epilogue warpgroups that, per K block, read
// that block's partial product from TMEM and fold it into fp32 registers with
// act_scale[row][kb] * weight_scale[col block][kb] (the 128x128 block-scale
// promotion: the scales are arbitrary fp32, so they cannot ride in the MMA),
// while the MMA of the next K block fills the other accumulator.
// The tile epilogue is the same arithmetic as the decode engine: gate_up
// rounds gate and up to bf16, a = bf16(silu(gate)) * up, requantises a per
// 128-group to E4M3; down stores fp32 rows for the fixed-order combine.
#pragma once

#include "d3_common.cuh"
#include "tcgen05.cuh"

namespace d3 {

enum TcKind { TC_GATE_UP = 0, TC_DOWN = 1 };

struct TcArgs {
  const int32_t* counts;  // [E] tokens per routed expert
  const int32_t* starts;  // [E] first activation row of each expert
  int E;
  int has_shared;         // group 0 is the shared expert when set
  int shared_row0;
  int shared_count;
  int ntiles;             // 256-column tiles per group (gate_up: I/128, down: H/256)
  int KB;                 // K / 128
  int rows_per_expert;    // weight rows per routed expert (2I or H)
  int second_box;         // row offset of the second 128-row B box (gate_up: I, down: 128)
  int nt_stride;          // weight rows per n tile (gate_up: 128, down: 256)
  int act_rows;           // rows of the activation buffer (for scale loads)
  const float* wscale;    // routed weight scales [E, rows/128, KB]
  const float* wscale_sh; // shared weight scales [rows/128, KB]
  const float* act_scale; // [act_rows, KB]
  uint8_t* out_q;         // gate_up: a e4m3 [rows, I]
  float* out_qs;          // gate_up: sa f32 [rows, I/128]
  int I;
  float* out_rows;        // down: f32 [rows, out_ld]
  int out_ld;
  int32_t* status;
};

constexpr int kTcStages = 4;
constexpr int kTcThreads = 320;
constexpr int kTcABytes = 128 * 128;
constexpr int kTcBBytes = 256 * 128;
constexpr int kTcStageBytes = kTcABytes + kTcBBytes;
constexpr int kTcMaxGroups = 1025;

struct TcSmem {
  static constexpr int kRing = kTcStages * kTcStageBytes;
  static constexpr int kBars = kRing;                                   // full[S], empty[S], tfull[2], tempty[2]
  static constexpr int kTmemSlot = kBars + (2 * kTcStages + 4) * 8;
  static constexpr int kAbort = kTmemSlot + 16;
  static constexpr int kAmax = kAbort + 16;                             // [2][128] f32
  static constexpr int kPrefix = kAmax + 2 * 128 * 4;                   // [groups + 1] int
  static constexpr size_t bytes() { return 1024 + kPrefix + (kTcMaxGroups + 1) * 4; }
};

struct TcTile {
  int group, mt, nt;
  int row0;     // first activation row of the tile
  int mvalid;   // rows of the tile that belong to the group
  int wrow;     // first B row (first box)
  int shared;
};

// tile index -> (group, m tile, n tile) by binary search over the prefix of
// tiles per group.
__device__ __forceinline__ TcTile tc_tile(const TcArgs& a, const int* prefix, int ngroups, int i) {
  int lo = 0, hi = ngroups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= i) lo = mid; else hi = mid - 1;
  }
  TcTile t;
  t.group = lo;
  const int local = i - prefix[lo];
  t.mt = local / a.ntiles;
  t.nt = local - t.mt * a.ntiles;
  int gstart, gcount, e;
  if (a.has_shared && lo == 0) {
    t.shared = 1;
    e = 0;
    gstart = a.shared_row0;
    gcount = a.shared_count;
  } else {
    t.shared = 0;
    e = lo - a.has_shared;
    gstart = a.starts[e];
    gcount = a.counts[e];
  }
  t.row0 = gstart + 128 * t.mt;
  t.mvalid = min(128, gcount - 128 * t.mt);
  t.wrow = e * a.rows_per_expert + t.nt * a.nt_stride;
  return t;
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                        int32_t* status) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  if (status) atomicExch(status, kDevWaitTimeout);
  return false;
}

template <int KIND>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_grouped_kernel(const __grid_constant__ CUtensorMap tm_act,
                      const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_w_sh, const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + TcSmem::kBars);
  uint64_t* empty = full + kTcStages;
  uint64_t* tfull = empty + kTcStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + TcSmem::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + TcSmem::kAbort);
  float* amax_x = reinterpret_cast<float*>(smem + TcSmem::kAmax);
  int* prefix = reinterpret_cast<int*>(smem + TcSmem::kPrefix);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = args.E + args.has_shared;

  // tiles per group and their exclusive prefix (serial in one warp: <= 1025 groups)
  if (warp == 0) {
    int running = 0;
    for (int base = 0; base < ngroups; base += 32) {
      const int g = base + lane;
      int nt = 0;
      if (g < ngroups) {
        const int cnt = (args.has_shared && g == 0) ? args.shared_count
                                                    : args.counts[g - args.has_shared];
        nt = ((cnt + 127) / 128) * args.ntiles;
      }
      int incl = nt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (g < ngroups) prefix[g] = running + incl - nt;
      running += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) prefix[ngroups] = running;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();
  const uint32_t tbase = *tslot;
  const int total_tiles = prefix[ngroups];

  if (warp == 0) {
    // -------------------------------------------------------------- TMA --
    if (lane == 0) {
      prefetch_tensormap(&tm_act);
      prefetch_tensormap(&tm_w);
      if (args.has_shared) prefetch_tensormap(&tm_w_sh);
      uint32_t it = 0;
      int last_parity[kTcStages];
#pragma unroll
      for (int s = 0; s < kTcStages; ++s) last_parity[s] = -1;
      bool ok = true;
      for (int i = blockIdx.x; i < total_tiles && ok; i += gridDim.x) {
        const TcTile t = tc_tile(args, prefix, ngroups, i);
        const CUtensorMap* wmap = t.shared ? &tm_w_sh : &tm_w;
        for (int kb = 0; kb < args.KB; ++kb, ++it) {
          const int s = it % kTcStages;
          const uint32_t ph = (it / kTcStages) & 1;
          if (!tc_wait(&empty[s], ph ^ 1, abort_flag, args.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kTcStageBytes;
          mbar_arrive_expect_tx(&full[s], kTcStageBytes);
          last_parity[s] = static_cast<int>(ph);
          tma_load_2d(st, &tm_act, kb * 128, t.row0, &full[s]);
          tma_load_2d(st + kTcABytes, wmap, kb * 128, t.wrow, &full[s]);
          tma_load_2d(st + kTcABytes + 16384, wmap, kb * 128, t.wrow + args.second_box, &full[s]);
        }
      }
      for (int s = 0; s < kTcStages; ++s)
        if (last_parity[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_parity[s]));
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA --
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_e4m3_f32(128, 256);
      uint32_t it = 0, kbc = 0;
      int last_tfull[2] = {-1, -1};
      bool ok = true;
      for (int i = blockIdx.x; i < total_tiles && ok; i += gridDim.x) {
        for (int kb = 0; kb < args.KB; ++kb, ++it, ++kbc) {
          const int s = it % kTcStages;
          const uint32_t b = kbc & 1;
          if (!tc_wait(&full[s], (it / kTcStages) & 1, abort_flag, args.status) ||
              !tc_wait(&tempty[b], ((kbc >> 1) & 1) ^ 1, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc::fence_after_thread_sync();
          const uint32_t a0 = smem_u32(smem + s * kTcStageBytes);
          const uint32_t b0 = a0 + kTcABytes;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_f8f6f4(tbase + b * 256, tc::smem_desc_sw128(a0 + ks * 32),
                           tc::smem_desc_sw128(b0 + ks * 32), idesc, ks > 0 ? 1u : 0u);
          tc::mma_commit(&empty[s]);
          tc::mma_commit(&tfull[b]);
          last_tfull[b] = static_cast<int>((kbc >> 1) & 1);
        }
      }
      // TMEM is freed below: make sure no MMA of this thread is still running
      for (int b = 0; b < 2; ++b)
        if (last_tfull[b] >= 0) mbar_wait(&tfull[b], static_cast<uint32_t>(last_tfull[b]));
    }
  } else {
    // --------------------------------------------------------- epilogue --
    const int ew = warp - 2;           // 0..7
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int wg = ew >> 2;            // column half
    const int row = quad * 32 + lane;  // tile row of this thread
    uint32_t kbc = 0;
    for (int i = blockIdx.x; i < total_tiles; i += gridDim.x) {
      const TcTile t = tc_tile(args, prefix, ngroups, i);
      const float* wscale = t.shared ? args.wscale_sh : args.wscale;
      const int grow = t.row0 + row;
      const bool row_ok = grow < args.act_rows;
      // weight-scale rows of this thread's columns
      int sb0, sb1;
      if (KIND == TC_GATE_UP) {
        sb0 = (t.wrow + 0) / 128;                       // gate block
        sb1 = (t.wrow + args.second_box) / 128;         // up block
      } else {
        sb0 = (t.wrow + 128 * wg) / 128;                // this half's block
        sb1 = sb0;
      }
      float acc0[64], acc1[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc0[j] = acc1[j] = 0.f;
      for (int kb = 0; kb < args.KB; ++kb, ++kbc) {
        const uint32_t b = kbc & 1;
        const float sa = row_ok ? args.act_scale[static_cast<int64_t>(grow) * args.KB + kb] : 0.f;
        const float f0 = sa * wscale[sb0 * args.KB + kb];
        const float f1 = sa * wscale[sb1 * args.KB + kb];
        tc_wait(&tfull[b], (kbc >> 1) & 1, abort_flag, args.status);
        __syncwarp();  // the TMEM loads below are warp-collective
        tc::fence_after_thread_sync();
        const uint32_t tl = tbase + b * 256 + (static_cast<uint32_t>(quad * 32) << 16);
        // columns of this thread: gate_up -> [64wg, 64wg+64) and [128+64wg, ...);
        // down -> [128wg, 128wg+128) split as two runs of 64
        const uint32_t c0 = KIND == TC_GATE_UP ? 64 * wg : 128 * wg;
        const uint32_t c1 = KIND == TC_GATE_UP ? 128 + 64 * wg : 128 * wg + 64;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          float r0[16], r1[16];
          tc::tmem_ld_32x32b_x16(tl + c0 + 16 * ch, r0);
          tc::tmem_ld_32x32b_x16(tl + c1 + 16 * ch, r1);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            acc0[16 * ch + j] = fmaf(r0[j], f0, acc0[16 * ch + j]);
            acc1[16 * ch + j] = fmaf(r1[j], f1, acc1[16 * ch + j]);
          }
        }
        tc::fence_before_thread_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
      }
      // ------------------------------------------------------ tile epilogue --
      const bool store = row < t.mvalid;
      if constexpr (KIND == TC_GATE_UP) {
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const float gv = bf16_round(acc0[j]);
          const float uv = bf16_round(acc1[j]);
          const float sg = bf16_round(gv * (1.0f / (1.0f + expf(-gv))));
          acc0[j] = sg * uv;
          amax = fmaxf(amax, fabsf(acc0[j]));
        }
        amax_x[wg * 128 + row] = amax;
        named_bar_sync(1, 256);
        const float sc = act_scale_from_amax(fmaxf(amax_x[row], amax_x[128 + row]));
        if (store) {
          uint8_t* q = args.out_q + static_cast<int64_t>(grow) * args.I + t.nt * 128 + 64 * wg;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t w4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              uint32_t word = 0;
#pragma unroll
              for (int b8 = 0; b8 < 4; ++b8)
                word |= static_cast<uint32_t>(act_quant(acc0[16 * v + 4 * u + b8], sc)) << (8 * b8);
              w4[u] = word;
            }
            reinterpret_cast<uint4*>(q)[v] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          if (wg == 0) args.out_qs[static_cast<int64_t>(grow) * (args.I / 128) + t.nt] = sc;
        }
        named_bar_sync(1, 256);  // amax_x is reused by the next tile
      } else {
        if (store) {
          float* o = args.out_rows + static_cast<int64_t>(grow) * args.out_ld + t.nt * 256 + 128 * wg;
#pragma unroll
          for (int v = 0; v < 16; ++v)
            reinterpret_cast<float4*>(o)[v] =
                make_float4(acc0[4 * v], acc0[4 * v + 1], acc0[4 * v + 2], acc0[4 * v + 3]);
#pragma unroll
          for (int v = 0; v < 16; ++v)
            reinterpret_cast<float4*>(o + 64)[v] =
                make_float4(acc1[4 * v], acc1[4 * v + 1], acc1[4 * v + 2], acc1[4 * v + 3]);
        }
      }
    }
  }
  tc::fence_before_thread_sync();
  __syncthreads();
  tc::fence_after_thread_sync();
  if (warp == 1) {
    __syncwarp();
    tc::tmem_dealloc(tbase, 512);
  }
}

}  // namespace d3
