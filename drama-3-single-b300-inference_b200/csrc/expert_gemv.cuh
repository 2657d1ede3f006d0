// Weight-streaming FP8 engine of the decode path (1..64 tokens per expert).
//
// The weights are the only large operand at decode, so every weight byte must
// cross HBM once, at full bandwidth. Design:
//   * persistent CTAs, one per SM, walk a static round-robin list of work items
//     (expert, 128-row weight tile); the list is built on the device from the
//     routing counts, so one launch shape serves every routing (graph-safe);
//   * one producer warp streams [128 rows x 128 bytes] weight tiles (K-major,
//     the checkpoint layout, 128B-swizzled) and the matching activation rows by
//     TMA into a STAGES-deep mbarrier ring that runs across item boundaries;
//   * eight consumer warps each own 16 weight rows and run mma.sync
//     m16n8k32 e4m3 (weights as A, tokens as B in chunks of 8) per 128-wide K
//     block, then fold that block's partial sums into fp32 registers with
//     weight_scale[n/128][k/128] * act_scale[token][k/128] (the 128x128
//     block-scale promotion, done in registers at no memory cost). The inner
//     loop is instantiated per token-chunk count (1, 2, 4, 8) and chosen per
//     item, so a stage costs work proportional to the expert's real tokens;
//   * epilogues: gate_up -> bf16(gate), bf16(up), a = bf16(silu(gate))*up,
//     FP8 requant per 128-group across the 8 warps (EPI_GATE_UP);
//     down -> fp32 rows for the fixed-order combine (EPI_DOWN);
//     dense weight-only GEMV -> bf16 (EPI_DENSE; activations f16, see below).
// Tensor-core work at <= 64 tokens is <= 16 flop per weight byte, far below the
// B200 ridge, so mma.sync's throughput is not a limit here; what matters is
// bytes in flight per SM (STAGES x 16-32 KB) and no pipeline drain between
// items.
//
// EPI_DENSE computes x_bf16 . dequant(W)^T exactly (weight-only FP8): W bytes
// are widened to f16 in registers (exact), x is pre-scaled per 128-group by a
// power of two into f16 (exact), and mma.sync m16n8k16 f16 accumulates in
// fp32; the power of two is removed in the promotion step.
#pragma once

#include "d3_common.cuh"

namespace d3 {

enum EpilogueKind { EPI_GATE_UP = 0, EPI_DOWN = 1, EPI_DENSE = 2 };

constexpr int kEngineConsumerWarps = 8;
constexpr int kEngineConsumerThreads = kEngineConsumerWarps * 32;
constexpr int kEngineThreads = kEngineConsumerThreads + 32;
constexpr int kTokensPerGroup = 64;

struct EngineArgs {
  // Work list. Routed experts come from `active[0..*n_active)` (or 0..num_groups
  // when active == nullptr); a shared expert, when present, is item group 0.
  const int32_t* counts;    // [E] tokens per expert (nullptr: dense, count = dense_count)
  const int32_t* starts;    // [E] first activation row of each expert
  const int32_t* active;    // [E] active expert ids, ascending
  const int32_t* n_active;  // [1]
  int num_groups;           // routed groups when active == nullptr
  int shared_groups;        // work groups of the shared expert (0: none)
  int shared_chunk;         // tokens per shared-expert work group
  int shared_row0;          // first activation row of the shared expert
  int shared_count;         // its token count
  int dense_count;          // token count in dense mode
  int tiles;                // 128-row weight tiles per group
  int KB;                   // K / 128
  int rows_per_expert;      // weight rows per routed expert in the map (2I or H)
  int up_offset;            // EPI_GATE_UP: row offset of the up half (= I)
  const float* wscale;      // routed weight scales [E, rows/128, KB]
  const float* wscale_sh;   // shared weight scales [rows/128, KB]
  const float* act_scale;   // [rows, KB]: fp8 act scales, or 2^-s for EPI_DENSE
  // outputs
  uint8_t* out_q;           // EPI_GATE_UP: a e4m3 [rows, I]
  float* out_qs;            // EPI_GATE_UP: sa f32 [rows, I/128]
  float* out_rows;          // EPI_DOWN: d f32 [rows, out_ld]
  __nv_bfloat16* out_bf16;  // EPI_DENSE: y bf16 [T, out_ld]
  int out_ld;               // row stride of the output (elements)
  int out_cols;             // EPI_GATE_UP: I; EPI_DENSE: N (columns >= N not stored)
  int32_t* status;          // D3_STATUS_* (may be null)
};

struct WorkItem {
  int wrow;     // first weight row of the tile (gate half for EPI_GATE_UP)
  int wrow_up;  // first up-half weight row (EPI_GATE_UP)
  int tile;     // tile index within the group
  int row0;     // first activation row
  int m;        // tokens
  int shared;   // uses the shared-expert tensor map / scales
};

__device__ __forceinline__ WorkItem engine_item(const EngineArgs& a, int i) {
  WorkItem w;
  const int gi = i / a.tiles;
  w.tile = i - gi * a.tiles;
  int e;
  if (gi < a.shared_groups) {
    // the shared expert's tokens are split into groups spread over CTAs
    w.shared = 1;
    e = 0;
    w.row0 = a.shared_row0 + gi * a.shared_chunk;
    w.m = min(a.shared_chunk, a.shared_count - gi * a.shared_chunk);
  } else {
    w.shared = 0;
    const int ri = gi - a.shared_groups;
    e = a.active ? a.active[ri] : ri;
    w.row0 = a.starts ? a.starts[e] : 0;
    w.m = a.counts ? a.counts[e] : a.dense_count;
  }
  w.wrow = e * a.rows_per_expert + w.tile * 128;
  w.wrow_up = w.wrow + a.up_offset;
  return w;
}

template <int EPI, bool ACT_F16, int STAGES>
struct EngineSmem {
  static constexpr int kWBytes = (EPI == EPI_GATE_UP ? 2 : 1) * 128 * 128;
  static constexpr int kActBytes = (ACT_F16 ? 2 : 1) * kTokensPerGroup * 128;
  static constexpr int kStageBytes = kWBytes + kActBytes;
  static constexpr int kRingBytes = STAGES * kStageBytes;
  // after the ring: full[STAGES], empty[STAGES], abort flag, amax[8][64],
  // weight-scale slab [2][KB], activation-scale slab [64][KB]
  static constexpr int kBarOffset = kRingBytes;
  static constexpr int kAbortOffset = kBarOffset + 2 * STAGES * 8;
  static constexpr int kAmaxOffset = kAbortOffset + 16;
  static constexpr int kWsOffset = kAmaxOffset + kEngineConsumerWarps * kTokensPerGroup * 4;
  __host__ __device__ static int slab_offset(int KB) { return kWsOffset + 2 * KB * 4; }
  static size_t bytes(int KB) {
    return 1024 + static_cast<size_t>(slab_offset(KB)) + static_cast<size_t>(kTokensPerGroup) * KB * 4;
  }
};

// Waits that give up early once the CTA has aborted (another wait timed out).
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  *abort_flag = 1;
  if (status) atomicExch(status, kDevWaitTimeout);
  return false;
}

struct ConsumerCtx {
  uint8_t* smem;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  float* amax_sm;  // [8][64]
  float* wsl;      // [2][KB] weight scales of the current item (gate, up)
  float* slab;     // [64][KB] activation scales of the current group
  int warp, lane;
};

// All K blocks of one token group (mg <= 8*NC tokens) of one work item, then
// its epilogue. `it` is the ring position, shared with the producer's order.
template <int EPI, bool ACT_F16, int STAGES, int NC>
__device__ __forceinline__ void consume_group(const EngineArgs& args, const ConsumerCtx& cx,
                                              const WorkItem& w, int g0, int mg, uint32_t& it) {
  using L = EngineSmem<EPI, ACT_F16, STAGES>;
  constexpr int NACC = (EPI == EPI_GATE_UP) ? 2 : 1;
  const int warp = cx.warp, lane = cx.lane;
  const int g = lane >> 2, tq = lane & 3;
  const int KB = args.KB;
  const float zero4[4] = {0.f, 0.f, 0.f, 0.f};

  float acc[NACC][NC][4];
#pragma unroll
  for (int h = 0; h < NACC; ++h)
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[h][c][j] = 0.f;

  // per-lane smem offsets that do not change across stages
  const uint32_t ar = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
  const uint32_t a_hi = lane >> 4;
  const uint32_t br = lane & 7, b_hi = (lane >> 3) & 1;

  for (int kb = 0; kb < KB; ++kb, ++it) {
    const int s = it % STAGES;
    const uint32_t ph = (it / STAGES) & 1;
    ring_wait(&cx.full[s], ph, cx.abort_flag, args.status);
    const uint32_t wsm = smem_u32(cx.smem + s * L::kStageBytes);
    const uint32_t asm_ = wsm + L::kWBytes;
    float tmp[NACC][NC][4];
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t a[NACC][4];
#pragma unroll
      for (int h = 0; h < NACC; ++h)
        ldmatrix_x4(wsm + h * 16384 + swz128(ar, 2 * ks + a_hi), a[h][0], a[h][1], a[h][2], a[h][3]);
      if constexpr (!ACT_F16) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          uint32_t b0, b1;
          ldmatrix_x2(asm_ + swz128(c * 8 + br, 2 * ks + b_hi), b0, b1);
#pragma unroll
          for (int h = 0; h < NACC; ++h) {
            if (ks == 0)
              mma_e4m3_16832(tmp[h][c], a[h], b0, b1, zero4);
            else
              mma_e4m3_16832(tmp[h][c], a[h], b0, b1, tmp[h][c]);
          }
        }
      } else {
        // widen the fp8 A fragment to two f16 k16 fragments
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = e4m3x2_to_f16x2(static_cast<uint16_t>(a[0][j] & 0xffffu));
          hi[j] = e4m3x2_to_f16x2(static_cast<uint16_t>(a[0][j] >> 16));
        }
        const uint32_t half_base = asm_ + (ks >> 1) * 8192;
        const uint32_t ch = 4 * (ks & 1) + (tq >> 1);
        const uint32_t off = (tq & 1) * 8;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint32_t row = c * 8 + g;
          uint32_t b0, b1, b2, b3;
          asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                       : "=r"(b0), "=r"(b1)
                       : "r"(half_base + swz128(row, ch) + off));
          asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                       : "=r"(b2), "=r"(b3)
                       : "r"(half_base + swz128(row, ch + 2) + off));
          if (ks == 0)
            mma_f16_16816(tmp[0][c], lo[0], lo[1], hi[0], hi[1], b0, b1, zero4);
          else
            mma_f16_16816(tmp[0][c], lo[0], lo[1], hi[0], hi[1], b0, b1, tmp[0][c]);
          mma_f16_16816(tmp[0][c], lo[2], lo[3], hi[2], hi[3], b2, b3, tmp[0][c]);
        }
      }
    }
    // release the stage as soon as its shared memory has been read
    __syncwarp();
    if (lane == 0) mbar_arrive(&cx.empty[s]);
    // block-scale promotion
    const float ws_g = cx.wsl[kb];
    const float ws_u = (EPI == EPI_GATE_UP) ? cx.wsl[KB + kb] : 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int t0 = c * 8 + 2 * tq;
      const float f0 = cx.slab[t0 * KB + kb], f1 = cx.slab[(t0 + 1) * KB + kb];
#pragma unroll
      for (int h = 0; h < NACC; ++h) {
        const float ws = h ? ws_u : ws_g;
        const float p0 = ws * f0, p1 = ws * f1;
        acc[h][c][0] = fmaf(tmp[h][c][0], p0, acc[h][c][0]);
        acc[h][c][1] = fmaf(tmp[h][c][1], p1, acc[h][c][1]);
        acc[h][c][2] = fmaf(tmp[h][c][2], p0, acc[h][c][2]);
        acc[h][c][3] = fmaf(tmp[h][c][3], p1, acc[h][c][3]);
      }
    }
  }

  // -------------------------------------------------------------- epilogue --
  const int out_row0 = w.row0 + g0;
  const int col0 = w.tile * 128 + 16 * warp + g;  // rows g and g+8 of this warp
  if constexpr (EPI == EPI_GATE_UP) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gv = bf16_round(acc[0][c][j]);
        const float uv = bf16_round(acc[1][c][j]);
        const float sg = bf16_round(gv * (1.0f / (1.0f + expf(-gv))));
        acc[0][c][j] = sg * uv;
      }
      float m0 = fmaxf(fabsf(acc[0][c][0]), fabsf(acc[0][c][2]));
      float m1 = fmaxf(fabsf(acc[0][c][1]), fabsf(acc[0][c][3]));
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
      }
      if (g == 0) {
        cx.amax_sm[warp * kTokensPerGroup + c * 8 + 2 * tq] = m0;
        cx.amax_sm[warp * kTokensPerGroup + c * 8 + 2 * tq + 1] = m1;
      }
    }
    named_bar_sync(1, kEngineConsumerThreads);
    const int I = args.out_cols;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = c * 8 + 2 * tq + u;
        if (t < mg) {
          float am = 0.f;
#pragma unroll
          for (int w2 = 0; w2 < kEngineConsumerWarps; ++w2)
            am = fmaxf(am, cx.amax_sm[w2 * kTokensPerGroup + t]);
          const float sc = act_scale_from_amax(am);
          uint8_t* qrow = args.out_q + static_cast<int64_t>(out_row0 + t) * I;
          qrow[col0] = act_quant(acc[0][c][u], sc);
          qrow[col0 + 8] = act_quant(acc[0][c][u + 2], sc);
          if (warp == 0 && g == 0)
            args.out_qs[static_cast<int64_t>(out_row0 + t) * (I / 128) + w.tile] = sc;
        }
      }
    }
  } else if constexpr (EPI == EPI_DOWN) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = c * 8 + 2 * tq + u;
        if (t < mg) {
          float* orow = args.out_rows + static_cast<int64_t>(out_row0 + t) * args.out_ld;
          orow[col0] = acc[0][c][u];
          orow[col0 + 8] = acc[0][c][u + 2];
        }
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = c * 8 + 2 * tq + u;
        if (t < mg) {
          __nv_bfloat16* orow = args.out_bf16 + static_cast<int64_t>(out_row0 + t) * args.out_ld;
          if (col0 < args.out_cols) orow[col0] = __float2bfloat16_rn(acc[0][c][u]);
          if (col0 + 8 < args.out_cols) orow[col0 + 8] = __float2bfloat16_rn(acc[0][c][u + 2]);
        }
      }
    }
  }
}

// MAXNC: largest token-chunk count (8 tokens each) any item of this launch can
// need, i.e. ceil(min(max tokens per expert, 64) / 8) rounded up to 1, 2, 4, 8.
template <int EPI, bool ACT_F16, int STAGES, int MAXNC>
__global__ void __launch_bounds__(kEngineThreads, 1)
    expert_gemv_kernel(const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_w_sh,
                       const __grid_constant__ CUtensorMap tm_act, const EngineArgs args) {
  using L = EngineSmem<EPI, ACT_F16, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOffset);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = args.KB;
  const int n_groups = (args.active ? *args.n_active : args.num_groups) + args.shared_groups;
  const int n_items = n_groups * args.tiles;
  constexpr int kGroup = MAXNC * 8 < kTokensPerGroup ? MAXNC * 8 : kTokensPerGroup;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kEngineConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kEngineConsumerWarps) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      prefetch_tensormap(&tm_w);
      prefetch_tensormap(&tm_act);
      if (args.shared_groups) prefetch_tensormap(&tm_w_sh);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_a = l2_policy_evict_last();
      uint32_t it = 0;
      int last_parity[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
      for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
        const WorkItem w = engine_item(args, i);
        const CUtensorMap* wmap = w.shared ? &tm_w_sh : &tm_w;
        for (int g0 = 0; g0 < w.m; g0 += kGroup) {
          const int mg = min(kGroup, w.m - g0);
          const int nbox = (mg + 15) / 16;
          const uint32_t bytes = L::kWBytes + nbox * (ACT_F16 ? 4096 : 2048);
          for (int kb = 0; kb < KB; ++kb, ++it) {
            const int s = it % STAGES;
            const uint32_t ph = (it / STAGES) & 1;
            if (!ring_wait(&empty[s], ph ^ 1, abort_flag, args.status)) goto producer_done;
            uint8_t* st = smem + s * L::kStageBytes;
            mbar_arrive_expect_tx(&full[s], bytes);
            last_parity[s] = static_cast<int>(ph);
            tma_load_2d_hint(st, wmap, kb * 128, w.wrow, &full[s], pol_w);
            if (EPI == EPI_GATE_UP)
              tma_load_2d_hint(st + 128 * 128, wmap, kb * 128, w.wrow_up, &full[s], pol_w);
            uint8_t* act = st + L::kWBytes;
            for (int b = 0; b < nbox; ++b) {
              const int row = w.row0 + g0 + 16 * b;
              tma_load_2d_hint(act + b * 2048, &tm_act, kb * 128, row, &full[s], pol_a);
              if (ACT_F16)
                tma_load_2d_hint(act + 8192 + b * 2048, &tm_act, kb * 128 + 64, row, &full[s],
                                 pol_a);
            }
          }
        }
      }
    producer_done:
      // Never leave the CTA while a bulk copy may still be writing its ring.
      for (int s = 0; s < STAGES; ++s)
        if (last_parity[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_parity[s]));
    }
    return;
  }

  // -------------------------------------------------------------- consumers --
  ConsumerCtx cx;
  cx.smem = smem;
  cx.full = full;
  cx.empty = empty;
  cx.abort_flag = abort_flag;
  cx.amax_sm = reinterpret_cast<float*>(smem + L::kAmaxOffset);
  cx.wsl = reinterpret_cast<float*>(smem + L::kWsOffset);
  cx.slab = reinterpret_cast<float*>(smem + L::slab_offset(KB));
  cx.warp = warp;
  cx.lane = lane;
  const int ctid = threadIdx.x;  // 0..255
  uint32_t it = 0;

  for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
    const WorkItem w = engine_item(args, i);
    const float* wscale = w.shared ? args.wscale_sh : args.wscale;
    for (int g0 = 0; g0 < w.m; g0 += kGroup) {
      const int mg = min(kGroup, w.m - g0);
      // stage this group's scales in shared memory: weights [2][KB], acts [mg][KB]
      named_bar_sync(1, kEngineConsumerThreads);
      {
        const float* src = args.act_scale + static_cast<int64_t>(w.row0 + g0) * KB;
        for (int idx = ctid; idx < mg * KB; idx += kEngineConsumerThreads) cx.slab[idx] = src[idx];
        for (int idx = ctid; idx < KB; idx += kEngineConsumerThreads) {
          cx.wsl[idx] = wscale[(w.wrow / 128) * KB + idx];
          if (EPI == EPI_GATE_UP) cx.wsl[KB + idx] = wscale[(w.wrow_up / 128) * KB + idx];
        }
      }
      named_bar_sync(1, kEngineConsumerThreads);
      const int nc = (mg + 7) / 8;
      if (MAXNC == 1 || nc <= 1)
        consume_group<EPI, ACT_F16, STAGES, 1>(args, cx, w, g0, mg, it);
      else if (MAXNC == 2 || nc <= 2)
        consume_group<EPI, ACT_F16, STAGES, (MAXNC >= 2 ? 2 : 1)>(args, cx, w, g0, mg, it);
      else if (MAXNC == 4 || nc <= 4)
        consume_group<EPI, ACT_F16, STAGES, (MAXNC >= 4 ? 4 : 1)>(args, cx, w, g0, mg, it);
      else
        consume_group<EPI, ACT_F16, STAGES, (MAXNC >= 8 ? 8 : 1)>(args, cx, w, g0, mg, it);
    }
  }
}

}  // namespace d3
