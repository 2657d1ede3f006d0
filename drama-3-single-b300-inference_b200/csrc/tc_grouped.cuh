// Prefill grouped GEMM on tcgen05 (tensor cores with TMEM accumulators).
//
// At prefill every expert sees hundreds to thousands of tokens, so the
// expert GEMMs are tensor-bound and belong on tcgen05. One persistent CTA per
// SM walks a static round-robin list of 128 x 256 output tiles:
//   gate_up: rows = 128 tokens of one expert, cols = 128 gate + 128 up rows of
//            W13 (the same i range), K = H;
//   down:    rows = 128 tokens (requantised activations), cols = 256 rows of
//            W2, K = I.
// Warp roles (12 warps, three warpgroups):
//   warp 0      TMA: A [128 x 128 B] and B [256 x 128 B] per 128-wide K block
//               into a 3-stage ring;
//   warp 1      owns TMEM (512 columns = two 256-column accumulators) and
//               issues 4 MMAs (M=128, N=256, K=32, kind::f8f6f4, E4M3 x E4M3
//               -> fp32) per K block into one accumulator;
//   warps 2-3   gate_up only: activation warps (see below);
//   warps 4-11  promotion: per K block they read that block's partial product
//               from TMEM and fold it into fp32 registers with
//               act_scale[row][kb] * weight_scale[col block][kb] (the 128x128
//               block-scale promotion: the scales are arbitrary fp32, so they
//               cannot ride in the MMA), while the MMA of the next K block fills
//               the other accumulator.
// Warpgroup 0 runs on 40 registers a thread and the promotion warpgroups on
// 232 (setmaxnreg), which lets a promotion thread hold its 128 accumulators
// plus 64 freshly loaded TMEM columns.
// Tile epilogues:
//   gate_up  the promotion warps compute a = bf16(silu(bf16(gate))) * bf16(up)
//            and its per-row amax in registers and hand a over in shared memory
//            ([128 rows][128] fp32, 64 KB); the two activation warps (a row per
//            thread) turn it into the row's 1x128 E4M3 scale and bytes and store
//            them, while the promotion warps already work on the next tile;
//   down     the promotion warps round the rows to bf16 (half the bytes of
//            fp32 to store here and to read in the combine), put each row in
//            shared memory and hand it to the bulk-copy engine, which stores it
//            for the fixed-order combine while the warps go on to the next tile.
#pragma once

#include "d3_common.cuh"
#include "tcgen05.cuh"

namespace d3 {

// TC_UP_GATE is gate_up over w13 rows stored [up | gate] (the gate half
// starts I rows into each expert); TC_GATE_UP reads [gate | up].
enum TcKind { TC_GATE_UP = 0, TC_DOWN = 1, TC_UP_GATE = 2 };

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
  int second_box;         // offset of the second B box from the first (gate_up: up - gate,
                          // +I or -I; down: 128)
  int nt_stride;          // weight rows per n tile (gate_up: 128, down: 256)
  int act_rows;           // rows of the activation buffer (for scale loads)
  const float* wscale;    // routed weight scales [E, rows/128, KB]
  const float* wscale_sh; // shared weight scales [rows/128, KB]
  const float* act_scale; // [act_rows, KB]
  uint8_t* out_q;         // gate_up: a e4m3 [rows, I]
  float* out_qs;          // gate_up: sa f32 [rows, I/128]
  int I;
  float* out_rows;        // down: bf16 [rows, out_ld] (stored through this pointer)
  int out_ld;
  int32_t* status;
};

constexpr int kTcThreads = 384;
constexpr int kTcRegsLow = 40, kTcRegsHigh = 232;  // 128*40 + 256*232 = 384*168
constexpr int kTcLaunchRegs = 168;
static_assert(128 * kTcRegsLow + 256 * kTcRegsHigh <= kTcThreads * kTcLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kTcABytes = 128 * 128;
constexpr int kTcBBytes = 256 * 128;
constexpr int kTcStageBytes = kTcABytes + kTcBBytes;
constexpr int kTcMaxGroups = 1025;
// down: staging row of one thread (128 bf16 columns + 16 bytes of padding,
// which keeps the rows' 16-byte vector stores free of bank conflicts)
constexpr int kTcDownStageRow = 272;

template <int KIND>
struct TcSmem {
  static constexpr int kStages = 3;
  static constexpr int kRing = kStages * kTcStageBytes;
  // full[S], empty[S], tfull[2], tempty[2], hfull, hempty
  static constexpr int kBars = kRing;
  static constexpr int kTmemSlot = kBars + (2 * kStages + 6) * 8;
  static constexpr int kAbort = kTmemSlot + 16;
  static constexpr int kPrefix = kAbort + 16;  // [groups + 1] int
  // gate_up: handoff tile [128 rows][32 chunks of 4 fp32] + row amax [2][128]
  // down:    staging tiles [8 warps][32 rows][4 chunks of 4 floats]
  static constexpr int kAux = (kPrefix + (kTcMaxGroups + 1) * 4 + 1023) / 1024 * 1024;
  static constexpr int kAuxBytes = KIND != TC_DOWN ? 128 * 128 * 4 + 2 * 128 * 4 : 8 * 32 * kTcDownStageRow;
  static constexpr size_t bytes() { return 1024 + kAux + kAuxBytes; }
};
static_assert(TcSmem<TC_GATE_UP>::bytes() <= 227 * 1024, "gate_up shared memory");
static_assert(TcSmem<TC_DOWN>::bytes() <= 227 * 1024, "down shared memory");

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

// TC_UP_GATE tiles start their first (gate) box I rows into the expert.
template <int KIND>
__device__ __forceinline__ TcTile tc_tile_k(const TcArgs& a, const int* prefix, int ngroups, int i) {
  TcTile t = tc_tile(a, prefix, ngroups, i);
  if constexpr (KIND == TC_UP_GATE) t.wrow += a.I;
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

// Two floats rounded to bf16 in one conversion: returns the bf16x2 word
// (lo in the low half) and writes the rounded values back.
__device__ __forceinline__ uint32_t bf16x2_round(float& lo, float& hi) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(hi), "f"(lo));
  lo = __uint_as_float(p << 16);
  hi = __uint_as_float(p & 0xffff0000u);
  return p;
}

template <int KIND>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_grouped_kernel(const __grid_constant__ CUtensorMap tm_act,
                      const __grid_constant__ CUtensorMap tm_w,
                      const __grid_constant__ CUtensorMap tm_w_sh, const TcArgs args) {
  using L = TcSmem<KIND>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* hfull = tempty + 2;
  uint64_t* hempty = hfull + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlot);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbort);
  int* prefix = reinterpret_cast<int*>(smem + L::kPrefix);
  uint8_t* aux = smem + L::kAux;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = args.E + args.has_shared;

  pdl_wait();  // counts, activations and outputs belong to earlier kernels
  // tiles per group and their exclusive prefix (serial in one warp: <= 1025
  // groups). The counts of 8 x 32 groups are loaded together before the scan
  // consumes them (one L2 round trip per 256 groups instead of per 32).
  if (warp == 0) {
    constexpr int kPass = 8;
    int running = 0;
    for (int b0 = 0; b0 < ngroups; b0 += 32 * kPass) {
      int cnt[kPass];
#pragma unroll
      for (int j = 0; j < kPass; ++j) {
        const int g = b0 + 32 * j + lane;
        cnt[j] = g >= ngroups ? 0
                 : (args.has_shared && g == 0) ? args.shared_count
                                               : args.counts[g - args.has_shared];
      }
#pragma unroll
      for (int j = 0; j < kPass; ++j) {
        const int g = b0 + 32 * j + lane;
        const int nt = g < ngroups ? ((cnt[j] + 127) / 128) * args.ntiles : 0;
        int incl = nt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int n = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += n;
        }
        if (g < ngroups) prefix[g] = running + incl - nt;
        running += __shfl_sync(0xffffffffu, incl, 31);
      }
    }
    if (lane == 0) prefix[ngroups] = running;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(hfull, 8);   // promotion warps
    mbar_init(hempty, 2);  // activation warps
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

  if (warp < 4) {
    tc::setmaxnreg_dec<kTcRegsLow>();
    if (warp == 0) {
      if (lane == 0) {
        // ---------------------------------------------------------- TMA --
        prefetch_tensormap(&tm_act);
        prefetch_tensormap(&tm_w);
        if (args.has_shared) prefetch_tensormap(&tm_w_sh);
        uint32_t it = 0;
        int last_parity[S];
#pragma unroll
        for (int s = 0; s < S; ++s) last_parity[s] = -1;
        bool ok = true;
        for (int i = blockIdx.x; i < total_tiles && ok; i += gridDim.x) {
          const TcTile t = tc_tile_k<KIND>(args, prefix, ngroups, i);
          const CUtensorMap* wmap = t.shared ? &tm_w_sh : &tm_w;
          for (int kb = 0; kb < args.KB; ++kb, ++it) {
            const int s = it % S;
            const uint32_t ph = (it / S) & 1;
            if (!tc_wait(&empty[s], ph ^ 1, abort_flag, args.status)) {
              ok = false;
              break;
            }
            uint8_t* st = smem + s * kTcStageBytes;
            mbar_arrive_expect_tx(&full[s], kTcStageBytes);
#pragma unroll
            for (int q = 0; q < S; ++q)
              if (q == s) last_parity[q] = static_cast<int>(ph);
            tma_load_2d(st, &tm_act, kb * 128, t.row0, &full[s]);
            tma_load_2d(st + kTcABytes, wmap, kb * 128, t.wrow, &full[s]);
            tma_load_2d(st + kTcABytes + 16384, wmap, kb * 128, t.wrow + args.second_box, &full[s]);
          }
        }
        pdl_trigger();  // every load of this CTA is issued
#pragma unroll
        for (int s = 0; s < S; ++s)
          if (last_parity[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_parity[s]));
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ---------------------------------------------------------- MMA --
        const uint32_t idesc = tc::idesc_e4m3_f32(128, 256);
        uint32_t it = 0, kbc = 0;
        int last_tfull[2] = {-1, -1};
        bool ok = true;
        for (int i = blockIdx.x; i < total_tiles && ok; i += gridDim.x) {
          for (int kb = 0; kb < args.KB; ++kb, ++it, ++kbc) {
            const int s = it % S;
            const uint32_t b = kbc & 1;
            if (!tc_wait(&full[s], (it / S) & 1, abort_flag, args.status) ||
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
            if (b == 0) last_tfull[0] = static_cast<int>((kbc >> 1) & 1);
            else last_tfull[1] = static_cast<int>((kbc >> 1) & 1);
          }
        }
        // TMEM is freed below: make sure no MMA of this thread is still running
        if (last_tfull[0] >= 0) mbar_wait(&tfull[0], static_cast<uint32_t>(last_tfull[0]));
        if (last_tfull[1] >= 0) mbar_wait(&tfull[1], static_cast<uint32_t>(last_tfull[1]));
      }
    } else if constexpr (KIND != TC_DOWN) {
      // ------------------------------------------------------- activation --
      // Thread t (0..63) of the two activation warps owns rows t and t + 64 of
      // each handed-over tile: scale = max(row amax halves) / 448, then the
      // row's 128 values are quantised and stored (128 contiguous bytes).
      const int at = threadIdx.x - 64;
      const uint4* hbuf = reinterpret_cast<const uint4*>(aux);
      const float* hamax = reinterpret_cast<const float*>(aux + 128 * 128 * 4);
      uint32_t n = 0;
      for (int i = blockIdx.x; i < total_tiles; i += gridDim.x, ++n) {
        const TcTile t = tc_tile_k<KIND>(args, prefix, ngroups, i);
        tc_wait(hfull, n & 1, abort_flag, args.status);
        __syncwarp();
#pragma unroll 1
        for (int rr = 0; rr < 2; ++rr) {
          const int r = at + 64 * rr;
          if (r < t.mvalid) {
            const uint4* hrow = hbuf + r * 32;
            const int sw = r & 7;
            const float sc = act_scale_from_amax(fmaxf(hamax[r], hamax[128 + r]));
            const float rs = __frcp_rn(sc);
            const int64_t grow = t.row0 + r;
            uint4* q = reinterpret_cast<uint4*>(args.out_q + grow * args.I + t.nt * 128);
#pragma unroll 2
            for (int c8 = 0; c8 < 8; ++c8) {
              uint32_t word[4];
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const uint4 v = hrow[(4 * c8 + c) ^ sw];
                word[c] = act_quant4(__uint_as_float(v.x), __uint_as_float(v.y),
                                     __uint_as_float(v.z), __uint_as_float(v.w), sc, rs);
              }
              q[c8] = make_uint4(word[0], word[1], word[2], word[3]);
            }
            args.out_qs[grow * (args.I / 128) + t.nt] = sc;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(hempty);
      }
    }
  } else {
    // ---------------------------------------------------------- promotion --
    tc::setmaxnreg_inc<kTcRegsHigh>();
    const int ew = warp - 4;           // 0..7
    const int quad = warp & 3;         // TMEM lane quadrant this warp may access
    const int wg = ew >> 2;            // column half
    const int row = quad * 32 + lane;  // tile row of this thread
    const int KB = args.KB;
    // columns of this thread: gate_up -> [64wg, 64wg+64) gate and [128+64wg, ...) up;
    // down -> [128wg, 128wg+128) as two runs of 64
    const uint32_t c0 = KIND != TC_DOWN ? 64 * wg : 128 * wg;
    const uint32_t c1 = KIND != TC_DOWN ? 128 + 64 * wg : 128 * wg + 64;
    // scale of (row, kb) and the two weight blocks of this thread's columns
    auto load_scales = [&](const TcTile& t, int kb, float& sa, float& w0, float& w1) {
      const float* wscale = t.shared ? args.wscale_sh : args.wscale;
      const int sb0 = KIND != TC_DOWN ? t.wrow / 128 : (t.wrow + 128 * wg) / 128;
      const int sb1 = KIND != TC_DOWN ? (t.wrow + args.second_box) / 128 : sb0;
      const int grow = t.row0 + row;
      sa = grow < args.act_rows ? __ldg(args.act_scale + static_cast<int64_t>(grow) * KB + kb) : 0.f;
      w0 = __ldg(wscale + sb0 * KB + kb);
      w1 = __ldg(wscale + sb1 * KB + kb);
    };
    uint32_t kbc = 0, n = 0;
    int i = blockIdx.x;
    TcTile t{};
    float p_sa = 0.f, p_w0 = 0.f, p_w1 = 0.f;
    if (i < total_tiles) {
      t = tc_tile_k<KIND>(args, prefix, ngroups, i);
      load_scales(t, 0, p_sa, p_w0, p_w1);
    }
    for (; i < total_tiles; i += gridDim.x, ++n) {
      const int inext = i + gridDim.x;
      TcTile tn{};
      if (inext < total_tiles) tn = tc_tile_k<KIND>(args, prefix, ngroups, inext);
      float acc0[64], acc1[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc0[j] = acc1[j] = 0.f;
      for (int kb = 0; kb < KB; ++kb, ++kbc) {
        const uint32_t b = kbc & 1;
        const float f0 = p_sa * p_w0, f1 = p_sa * p_w1;
        // scales of the next K block (or the next tile's first) load under this one
        if (kb + 1 < KB) load_scales(t, kb + 1, p_sa, p_w0, p_w1);
        else if (inext < total_tiles) load_scales(tn, 0, p_sa, p_w0, p_w1);
        tc_wait(&tfull[b], (kbc >> 1) & 1, abort_flag, args.status);
        __syncwarp();  // the TMEM loads below are warp-collective
        tc::fence_after_thread_sync();
        const uint32_t tl = tbase + b * 256 + (static_cast<uint32_t>(quad * 32) << 16);
        // two 32-column halves of both runs, each half's two loads waited for
        // once (two TMEM round trips per K block)
        float qa[32], qb[32];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          tc::tmem_ld_32x32b_x32(tl + c0 + 32 * h, qa);
          tc::tmem_ld_32x32b_x32(tl + c1 + 32 * h, qb);
          tc::tmem_ld_wait_regs(qa, qb);
          if (h == 1) {
            // the last half is in registers: the accumulator is free for the
            // MMA of K block kbc + 2 while that half is folded in
            tc::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            ffma2(acc0[32 * h + j], acc0[32 * h + j + 1], qa[j], qa[j + 1], f0);
            ffma2(acc1[32 * h + j], acc1[32 * h + j + 1], qb[j], qb[j + 1], f1);
          }
        }
      }
      // ------------------------------------------------------ tile epilogue --
      if constexpr (KIND != TC_DOWN) {
        // a = bf16(silu(g)) * u with g, u the bf16-rounded gate and up and
        // silu(g) = g / (1 + exp(-g)) on the fast exponential and divide; a goes
        // to the activation warps as fp32 (16-byte chunk c of row r at chunk
        // c ^ (r & 7): conflict-free by row and by chunk) with this half's amax
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 64; j += 2) {
          bf16x2_round(acc0[j], acc1[j]);
          bf16x2_round(acc0[j + 1], acc1[j + 1]);
          float s0 = __fdividef(acc0[j], 1.0f + __expf(-acc0[j]));
          float s1 = __fdividef(acc0[j + 1], 1.0f + __expf(-acc0[j + 1]));
          bf16x2_round(s0, s1);
          acc0[j] = s0 * acc1[j];
          acc0[j + 1] = s1 * acc1[j + 1];
          amax = fmaxf(amax, fmaxf(fabsf(acc0[j]), fabsf(acc0[j + 1])));
        }
        tc_wait(hempty, (n & 1) ^ 1, abort_flag, args.status);
        __syncwarp();
        uint4* hbuf = reinterpret_cast<uint4*>(aux);
#pragma unroll
        for (int c = 0; c < 16; ++c)
          hbuf[row * 32 + ((16 * wg + c) ^ (row & 7))] =
              make_uint4(__float_as_uint(acc0[4 * c]), __float_as_uint(acc0[4 * c + 1]),
                         __float_as_uint(acc0[4 * c + 2]), __float_as_uint(acc0[4 * c + 3]));
        reinterpret_cast<float*>(aux + 128 * 128 * 4)[wg * 128 + row] = amax;
        __syncwarp();
        if (lane == 0) mbar_arrive(hfull);
      } else {
        // bf16 rows (the tcgen05 path rounds its per-expert down rows to bf16
        // before the fixed-order combine). Thread = tile row: its 128 columns
        // (acc0 then acc1) go to its own 256-byte row of the staging area and
        // from there to global memory by one bulk copy, which runs while the
        // warp goes on to the next tile. A row is rewritten only after its
        // previous copy has read it (long done by then: a tile's K loop lies
        // between). Rows past the group's end are neither staged nor stored.
        uint8_t* srow = aux + (ew * 32 + lane) * kTcDownStageRow;
        bulk_wait_read_all();
        if (row < t.mvalid) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float* src = c < 8 ? acc0 + 8 * c : acc1 + 8 * (c - 8);
            uint32_t p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const __nv_bfloat162 v = __floats2bfloat162_rn(src[2 * i], src[2 * i + 1]);
              p[i] = *reinterpret_cast<const uint32_t*>(&v);
            }
            *reinterpret_cast<uint4*>(srow + 16 * c) = make_uint4(p[0], p[1], p[2], p[3]);
          }
          fence_proxy_async_smem();
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.out_rows) +
                               static_cast<int64_t>(t.row0 + row) * args.out_ld + t.nt * 256 + 128 * wg;
          bulk_store_s2g(dst, srow, 256);
          bulk_commit();
        }
      }
      t = tn;
    }
    // the staged rows must stay in place until their copies are done
    if constexpr (KIND == TC_DOWN) bulk_wait_all();
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
