// Weight-streaming FP8 engine of the decode path (1..64 tokens per expert).
//
// The weights are the only large operand at decode, so every weight byte must
// cross HBM once, at full bandwidth. Design:
//   * persistent CTAs, one per SM, walk a static round-robin list of work items
//     (expert, 128-row weight tile[, K split]); the list is built on the device
//     from the routing counts, so one launch shape serves every routing
//     (graph-safe). The routing metadata is copied to shared memory once;
//   * one producer warp streams [128 rows x 128 bytes] weight tiles (K-major,
//     the checkpoint layout, 128B-swizzled) and the matching activation rows by
//     TMA into a STAGES-deep mbarrier ring that runs across item boundaries.
//     Per token group it also stages a slab (group header + weight and
//     activation scales) with cp.async into one of two buffers, so the
//     consumers never wait on global memory for metadata;
//   * eight consumer warps each own 16 weight rows and run mma.sync
//     m16n8k32 e4m3 (weights as A, tokens as B in chunks of 8) per 128-wide K
//     block, then fold that block's partial sums into fp32 registers with
//     weight_scale[n/128][k/128] * act_scale[token][k/128] (the 128x128
//     block-scale promotion, done in registers at no memory cost). The inner
//     loop is instantiated per token-chunk count (1, 2, 4, 8) and chosen per
//     group, so a stage costs work proportional to the expert's real tokens;
//   * epilogues: gate_up -> bf16(gate), bf16(up), a = bf16(silu(gate))*up,
//     FP8 requant per 128-group across the 8 warps (EPI_GATE_UP);
//     down -> fp32 rows for the fixed-order combine (EPI_DOWN);
//     dense weight-only GEMV -> bf16, optionally split along K with a
//     deterministic last-CTA reduction (EPI_DENSE; activations f16, below).
// Tensor-core work at <= 64 tokens is <= 16 flop per weight byte, far below the
// B200 ridge, so mma.sync's throughput is not a limit here; what matters is
// bytes in flight per SM and no pipeline drain between items.
//
// EPI_DENSE computes x_bf16 . dequant(W)^T exactly (weight-only FP8): W bytes
// are widened to f16 in registers (exact), x is pre-scaled per 128-group by a
// power of two into f16 (exact) and stored in a k order that makes the
// B-fragment loads bank-conflict free (dense_act_position), and mma.sync
// m16n8k16 f16 accumulates in fp32; the power of two is removed in the
// promotion step.
#pragma once

#include "d3_common.cuh"

namespace d3 {

// EPI_DOWN2: down over pairs of 128-row weight tiles (256 output columns per
// work item, two accumulator sets like gate/up), so an item streams twice the
// weight bytes of EPI_DOWN for the same per-item overhead.
enum EpilogueKind { EPI_GATE_UP = 0, EPI_DOWN = 1, EPI_DENSE = 2, EPI_DOWN2 = 3 };

// Two 128-row weight boxes (and two accumulator sets) per stage.
template <int EPI>
constexpr bool kTwoBoxes = EPI == EPI_GATE_UP || EPI == EPI_DOWN2;

constexpr int kEngineConsumerWarps = 8;
constexpr int kEngineConsumerThreads = kEngineConsumerWarps * 32;
constexpr int kEngineThreads = kEngineConsumerThreads + 32;
constexpr int kTokensPerGroup = 64;
constexpr int kEngineMaxExperts = 1024;

// Position (in f16 elements, within one 128-element K block) at which the
// dense activation prep stores element k. Element k = 16c + 4q + j (c: 16-wide
// fp8 chunk of the A fragment, q: lane quad index tq, j: 0..3) goes to
// 64*(c/4) + 8*((c%4) + 4*(q/2)) + 4*(q%2) + j, so that the 16 lanes of one
// 64-bit shared-load phase read 16 distinct bank pairs after the 128B swizzle.
__host__ __device__ __forceinline__ int dense_act_position(int k) {
  const int c = k >> 4, q = (k >> 2) & 3, j = k & 3;
  return 64 * (c >> 2) + 8 * ((c & 3) + 4 * (q >> 1)) + 4 * (q & 1) + j;
}

struct EngineArgs {
  // Work list. Routed experts come from `active[0..*n_active)` (or 0..num_groups
  // when active == nullptr); shared-expert groups come first.
  const int32_t* counts;    // [E] tokens per expert (nullptr: dense, count = dense_count)
  const int32_t* starts;    // [E] first activation row of each expert
  const int32_t* active;    // [E] active expert ids, ascending
  const int32_t* n_active;  // [1]
  int num_experts;          // E (size of counts/starts/active)
  int num_groups;           // routed groups when active == nullptr
  int shared_groups;        // work groups of the shared expert (0: none)
  int shared_chunk;         // tokens per shared-expert work group
  int shared_row0;          // first activation row of the shared expert
  int shared_count;         // its token count
  int dense_count;          // token count in dense mode
  int tiles;                // 128-row weight tiles per group
  int KB;                   // K / 128
  int rows_per_expert;      // weight rows per routed expert in the map (2I or H)
  int first_off;            // row offset of the gate half (EPI_GATE_UP: 0 or I)
  int up_offset;            // EPI_GATE_UP: up-half rows relative to the gate half (+I or -I)
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
  // EPI_DENSE split-K: each 128-row tile is cut into `ksplit` K ranges of
  // kb_per_split blocks handled by different CTAs; fp32 partials
  // [ksplit][dense_count][tiles*128] are summed in split order by the CTA that
  // finishes a (tile, token group) last (tile_counters zeroed before launch).
  int ksplit;
  int kb_per_split;
  float* partials;
  int32_t* tile_counters;   // [tiles * token groups]
  // Dynamic schedule: after its first item (blockIdx.x) a CTA takes the next
  // item index from gridDim.x + atomicAdd(work_counter, 1), so CTAs that drew
  // light items take more of them (zeroed before launch; nullptr: static
  // round-robin i += gridDim.x).
  int32_t* work_counter;
};

struct WorkItem {
  int wrow;     // first weight row of the tile (gate half for EPI_GATE_UP)
  int wrow_up;  // first up-half weight row (EPI_GATE_UP)
  int tile;     // tile index within the group
  int row0;     // first activation row
  int m;        // tokens
  int shared;   // uses the shared-expert tensor map / scales
  int split;    // K split index (EPI_DENSE)
  int kb0;      // first K block of this item
  int nkb;      // K blocks of this item
};

// The per-group record the producer hands to the consumers in the slab.
struct GroupHeader {
  int wrow, wrow_up, tile, row0, g0, mg, shared, split, kb0, nkb, done, pad[5];
};
static_assert(sizeof(GroupHeader) == 64, "slab header is 16 words");

template <int EPI>
__device__ __forceinline__ WorkItem engine_item(const EngineArgs& a, const int* sm_active,
                                                const int* sm_counts, const int* sm_starts,
                                                int i) {
  WorkItem w;
  const int q = i / a.ksplit;
  w.split = i - q * a.ksplit;
  w.kb0 = w.split * a.kb_per_split;
  w.nkb = min(a.kb_per_split, a.KB - w.kb0);
  const int gi = q / a.tiles;
  w.tile = q - gi * a.tiles;
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
    e = a.active ? sm_active[ri] : ri;
    w.row0 = a.starts ? sm_starts[e] : 0;
    w.m = a.counts ? sm_counts[e] : a.dense_count;
  }
  // EPI_DOWN2 tiles are 256 rows: rows [256 tile, +128) and [+128, +256)
  w.wrow = e * a.rows_per_expert + w.tile * (EPI == EPI_DOWN2 ? 256 : 128) + a.first_off;
  w.wrow_up = w.wrow + (EPI == EPI_DOWN2 ? 128 : a.up_offset);
  return w;
}

// ACT_ROWS: activation rows per stage = tokens per group rounded up to 16.
template <int EPI, bool ACT_F16, int STAGES, int ACT_ROWS>
struct EngineSmem {
  static constexpr int kWBytes = (kTwoBoxes<EPI> ? 2 : 1) * 128 * 128;
  static constexpr int kActHalf = ACT_ROWS * 128;  // one 128-byte column block of act rows
  static constexpr int kActBytes = (ACT_F16 ? 2 : 1) * kActHalf;
  static constexpr int kStageBytes = kWBytes + kActBytes;
  static constexpr int kRingBytes = STAGES * kStageBytes;
  // after the ring: full[STAGES], empty[STAGES], slab_full[2], slab_empty[2],
  // abort flag, amax[8][64], metadata (active, counts, starts: 3 x E ints),
  // then two slabs, each a GroupHeader, weight scales [2][KB] and activation
  // scales [ACT_ROWS][KB]
  static constexpr int kBarOffset = kRingBytes;
  static constexpr int kAbortOffset = kBarOffset + (2 * STAGES + 4) * 8;
  static constexpr int kAmaxOffset = kAbortOffset + 16;
  static constexpr int kMetaOffset = kAmaxOffset + kEngineConsumerWarps * kTokensPerGroup * 4;
  __host__ __device__ static int slab_offset(int E) { return kMetaOffset + 3 * E * 4; }
  __host__ __device__ static int slab_floats(int KB) { return 16 + 2 * KB + ACT_ROWS * KB; }
  static size_t bytes(int KB, int E) {
    return 1024 + static_cast<size_t>(slab_offset(E)) + 2 * static_cast<size_t>(slab_floats(KB)) * 4;
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
  const float* wsl;   // [2][KB] weight scales of the current group (gate, up)
  const float* slab;  // [ACT_ROWS][KB] activation scales of the current group
  int warp, lane;
};

// All K blocks of one token group (mg <= 8*NC tokens) of one work item, then
// its epilogue. `it` is the ring position, shared with the producer's order.
template <int EPI, bool ACT_F16, int STAGES, int ACT_ROWS, int NC>
__device__ __forceinline__ void consume_group(const EngineArgs& args, const ConsumerCtx& cx,
                                              const GroupHeader& w, uint32_t& it) {
  using L = EngineSmem<EPI, ACT_F16, STAGES, ACT_ROWS>;
  constexpr int NACC = kTwoBoxes<EPI> ? 2 : 1;
  const int warp = cx.warp, lane = cx.lane;
  const int g = lane >> 2, tq = lane & 3;
  const int KB = args.KB;
  const int mg = w.mg;
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

  for (int kb = w.kb0; kb < w.kb0 + w.nkb; ++kb, ++it) {
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
        // widen the fp8 A fragment (chunks 2ks, 2ks+1) to two f16 k16 fragments
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          lo[j] = e4m3x2_to_f16x2(static_cast<uint16_t>(a[0][j] & 0xffffu));
          hi[j] = e4m3x2_to_f16x2(static_cast<uint16_t>(a[0][j] >> 16));
        }
        // B for fp8 chunk c: f16 k = 16c + 4tq .. +3 at dense_act_position
        const int c1 = 2 * ks, c2 = 2 * ks + 1;
        const uint32_t base1 = asm_ + (c1 >> 2) * L::kActHalf;
        const uint32_t base2 = asm_ + (c2 >> 2) * L::kActHalf;
        const uint32_t ch1 = (c1 & 3) + 4 * (tq >> 1), ch2 = (c2 & 3) + 4 * (tq >> 1);
        const uint32_t off = (tq & 1) * 8;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint32_t row = c * 8 + g;
          uint32_t b0, b1, b2, b3;
          asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                       : "=r"(b0), "=r"(b1)
                       : "r"(base1 + swz128(row, ch1) + off));
          asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];"
                       : "=r"(b2), "=r"(b3)
                       : "r"(base2 + swz128(row, ch2) + off));
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
    const float ws_u = kTwoBoxes<EPI> ? cx.wsl[KB + kb] : 0.f;
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
  const int out_row0 = w.row0 + w.g0;
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
          const float rs = __frcp_rn(sc);
          uint8_t* qrow = args.out_q + static_cast<int64_t>(out_row0 + t) * I;
          qrow[col0] = f32_to_e4m3(act_quant_value(acc[0][c][u], sc, rs));
          qrow[col0 + 8] = f32_to_e4m3(act_quant_value(acc[0][c][u + 2], sc, rs));
          if (warp == 0 && g == 0)
            args.out_qs[static_cast<int64_t>(out_row0 + t) * (I / 128) + w.tile] = sc;
        }
      }
    }
    named_bar_sync(1, kEngineConsumerThreads);  // amax_sm is reused by the next group
  } else if constexpr (EPI == EPI_DOWN || EPI == EPI_DOWN2) {
    // EPI_DOWN2: the item's columns start at 256 * tile; set h adds 128
    const int cbase = EPI == EPI_DOWN2 ? w.tile * 256 + 16 * warp + g : col0;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = c * 8 + 2 * tq + u;
        if (t < mg) {
          float* orow = args.out_rows + static_cast<int64_t>(out_row0 + t) * args.out_ld;
#pragma unroll
          for (int h = 0; h < NACC; ++h) {
            orow[cbase + 128 * h] = acc[h][c][u];
            orow[cbase + 128 * h + 8] = acc[h][c][u + 2];
          }
        }
      }
    }
  } else if (args.ksplit == 1) {
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
  } else {
    // split-K: publish this split's fp32 partial, then the last CTA to finish
    // the (tile, token group) sums all splits in split order and stores bf16.
    const int T = args.dense_count;
    const int ldp = args.tiles * 128;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = c * 8 + 2 * tq + u;
        if (t < mg) {
          float* prow = args.partials + (static_cast<int64_t>(w.split) * T + out_row0 + t) * ldp;
          prow[col0] = acc[0][c][u];
          prow[col0 + 8] = acc[0][c][u + 2];
        }
      }
    }
    __threadfence();
    named_bar_sync(1, kEngineConsumerThreads);
    int* last = reinterpret_cast<int*>(cx.amax_sm);
    if (warp == 0 && lane == 0) {
      const int ngroups = (T + kTokensPerGroup - 1) / kTokensPerGroup;
      const int slot = w.tile * ngroups + w.g0 / kTokensPerGroup;
      *last = atomicAdd(&args.tile_counters[slot], 1) == args.ksplit - 1;
    }
    named_bar_sync(1, kEngineConsumerThreads);
    if (*last) {
      __threadfence();
      // thread -> 4 consecutive columns of one token; the split loads of a
      // pass are issued before any is summed (the sum order stays split order)
      const int ctid = warp * 32 + lane;
      for (int idx = ctid; idx < mg * 32; idx += kEngineConsumerThreads) {
        const int t = idx >> 5, col = w.tile * 128 + (idx & 31) * 4;
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < args.ksplit; s0 += 4) {
          float4 v[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (s0 + q < args.ksplit)
              v[q] = __ldcg(reinterpret_cast<const float4*>(
                  args.partials + (static_cast<int64_t>(s0 + q) * T + out_row0 + t) * ldp + col));
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (s0 + q < args.ksplit) {
              sum.x += v[q].x;
              sum.y += v[q].y;
              sum.z += v[q].z;
              sum.w += v[q].w;
            }
        }
        __nv_bfloat16* yrow = args.out_bf16 + static_cast<int64_t>(out_row0 + t) * args.out_ld;
        const float sv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (col + q < args.out_cols) yrow[col + q] = __float2bfloat16_rn(sv[q]);
      }
    }
    named_bar_sync(1, kEngineConsumerThreads);
  }
}

// MAXNC: largest token-chunk count (8 tokens each) any group of this launch
// can need: 1, 2, 4 or 8 (groups hold min(8*MAXNC, 64) tokens).
template <int EPI, bool ACT_F16, int STAGES, int MAXNC>
__global__ void __launch_bounds__(kEngineThreads, 1)
    expert_gemv_kernel(const __grid_constant__ CUtensorMap tm_w,
                       const __grid_constant__ CUtensorMap tm_w_sh,
                       const __grid_constant__ CUtensorMap tm_act, const EngineArgs args) {
  constexpr int kGroup = MAXNC * 8 < kTokensPerGroup ? MAXNC * 8 : kTokensPerGroup;
  constexpr int kActRows = kGroup < 16 ? 16 : kGroup;
  using L = EngineSmem<EPI, ACT_F16, STAGES, kActRows>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* slab_full = empty + STAGES;
  uint64_t* slab_empty = slab_full + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOffset);
  int* sm_active = reinterpret_cast<int*>(smem + L::kMetaOffset);
  int* sm_counts = sm_active + args.num_experts;
  int* sm_starts = sm_counts + args.num_experts;
  float* slabs = reinterpret_cast<float*>(smem + L::slab_offset(args.num_experts));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = args.KB;
  const int slab_n = L::slab_floats(KB);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kEngineConsumerWarps);
    }
    for (int b = 0; b < 2; ++b) {
      // 32 cp.async completion arrivals + the producer leader's header arrival
      mbar_init(&slab_full[b], 33);
      mbar_init(&slab_empty[b], kEngineConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // routing metadata, activations and outputs belong to earlier kernels

  if (warp == kEngineConsumerWarps) {
    // ------------------------------------------------------------ producer --
    const bool leader = lane == 0;
    // routing metadata into shared memory: up to 8 experts a lane per pass,
    // every load of a pass issued before any is stored (storing each value as
    // it arrived serialised one L2 round trip per expert group: 4-6 us before
    // the first weight load at E = 128-256)
    const int n_routed = args.active ? *args.n_active : args.num_groups;
    if (args.counts) {
      constexpr int kPass = 8;
      for (int e0 = 0; e0 < args.num_experts; e0 += 32 * kPass) {
        int c[kPass], st[kPass], ac[kPass];
#pragma unroll
        for (int j = 0; j < kPass; ++j) {
          const int e = e0 + 32 * j + lane;
          const bool in = e < args.num_experts;
          c[j] = in ? args.counts[e] : 0;
          st[j] = in ? args.starts[e] : 0;
          ac[j] = (in && args.active) ? args.active[e] : 0;
        }
#pragma unroll
        for (int j = 0; j < kPass; ++j) {
          const int e = e0 + 32 * j + lane;
          if (e < args.num_experts) {
            sm_counts[e] = c[j];
            sm_starts[e] = st[j];
            if (args.active) sm_active[e] = ac[j];
          }
        }
      }
      __syncwarp();
    }
    const int n_items = (n_routed + args.shared_groups) * args.tiles * args.ksplit;
    uint64_t pol_w = 0, pol_a = 0;
    if (leader) {
      prefetch_tensormap(&tm_w);
      prefetch_tensormap(&tm_act);
      if (args.shared_groups) prefetch_tensormap(&tm_w_sh);
      pol_w = l2_policy_evict_first();
      pol_a = l2_policy_evict_last();
    }
    uint32_t it = 0, gc = 0;
    int last_parity[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
    bool ok = true;
    for (int i = blockIdx.x; ok;) {
      const bool have = i < n_items;
      // claim the next item now; the atomic's latency hides behind this item
      int next = i + gridDim.x;
      if (have && args.work_counter && leader) next = gridDim.x + atomicAdd(args.work_counter, 1);
      WorkItem w{};
      if (have) w = engine_item<EPI>(args, sm_active, sm_counts, sm_starts, i);
      const CUtensorMap* wmap = w.shared ? &tm_w_sh : &tm_w;
      const float* wscale = w.shared ? args.wscale_sh : args.wscale;
      // one slab per token group; one final slab marks the end of the work
      const int ngroups = have ? (w.m + kGroup - 1) / kGroup : 1;
      for (int gq = 0; gq < ngroups && ok; ++gq, ++gc) {
        const int g0 = gq * kGroup;
        const int mg = have ? min(kGroup, w.m - g0) : 0;
        const int sb = gc & 1;
        const uint32_t sph = (gc >> 1) & 1;
        if (leader) ok = ring_wait(&slab_empty[sb], sph ^ 1, abort_flag, args.status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        float* slab = slabs + sb * slab_n;
        if (have) {
          for (int idx = lane; idx < KB; idx += 32) {
            cp_async_4(slab + 16 + idx, wscale + (w.wrow / 128) * KB + idx);
            if (kTwoBoxes<EPI>)
              cp_async_4(slab + 16 + KB + idx, wscale + (w.wrow_up / 128) * KB + idx);
          }
          const float* src = args.act_scale + static_cast<int64_t>(w.row0 + g0) * KB;
          for (int idx = lane; idx < mg * KB; idx += 32) cp_async_4(slab + 16 + 2 * KB + idx, src + idx);
        }
        cp_async_arrive_noinc(&slab_full[sb]);
        if (leader) {
          GroupHeader* hdr = reinterpret_cast<GroupHeader*>(slab);
          hdr->wrow = w.wrow;
          hdr->wrow_up = w.wrow_up;
          hdr->tile = w.tile;
          hdr->row0 = w.row0;
          hdr->g0 = g0;
          hdr->mg = mg;
          hdr->shared = w.shared;
          hdr->split = w.split;
          hdr->kb0 = w.kb0;
          hdr->nkb = w.nkb;
          hdr->done = have ? 0 : 1;
          mbar_arrive(&slab_full[sb]);
          if (have) {
            const int nbox = (mg + 15) / 16;
            const uint32_t bytes = L::kWBytes + nbox * (ACT_F16 ? 4096 : 2048);
            for (int kb = w.kb0; kb < w.kb0 + w.nkb; ++kb, ++it) {
              const int s = it % STAGES;
              const uint32_t ph = (it / STAGES) & 1;
              if (!ring_wait(&empty[s], ph ^ 1, abort_flag, args.status)) {
                ok = false;
                break;
              }
              uint8_t* st = smem + s * L::kStageBytes;
              mbar_arrive_expect_tx(&full[s], bytes);
              last_parity[s] = static_cast<int>(ph);
              tma_load_2d_hint(st, wmap, kb * 128, w.wrow, &full[s], pol_w);
              if (kTwoBoxes<EPI>)
                tma_load_2d_hint(st + 128 * 128, wmap, kb * 128, w.wrow_up, &full[s], pol_w);
              uint8_t* act = st + L::kWBytes;
              for (int b = 0; b < nbox; ++b) {
                const int row = w.row0 + g0 + 16 * b;
                tma_load_2d_hint(act + b * 2048, &tm_act, kb * 128, row, &full[s], pol_a);
                if (ACT_F16)
                  tma_load_2d_hint(act + L::kActHalf + b * 2048, &tm_act, kb * 128 + 64, row,
                                   &full[s], pol_a);
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (!have) break;
      i = args.work_counter ? __shfl_sync(0xffffffffu, next, 0) : next;
    }
    pdl_trigger();  // every load of this CTA is issued: the next kernel may start launching
    // Never leave the CTA while a copy may still be writing its shared memory.
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (leader)
      for (int s = 0; s < STAGES; ++s)
        if (last_parity[s] >= 0) mbar_wait(&full[s], static_cast<uint32_t>(last_parity[s]));
    return;
  }

  // -------------------------------------------------------------- consumers --
  ConsumerCtx cx;
  cx.smem = smem;
  cx.full = full;
  cx.empty = empty;
  cx.abort_flag = abort_flag;
  cx.amax_sm = reinterpret_cast<float*>(smem + L::kAmaxOffset);
  cx.warp = warp;
  cx.lane = lane;
  uint32_t it = 0;
  for (uint32_t gc = 0;; ++gc) {
    const int sb = gc & 1;
    if (!ring_wait(&slab_full[sb], (gc >> 1) & 1, abort_flag, args.status)) break;
    const float* slab = slabs + sb * slab_n;
    const GroupHeader w = *reinterpret_cast<const GroupHeader*>(slab);
    if (w.done) break;
    cx.wsl = slab + 16;
    cx.slab = slab + 16 + 2 * KB;
    const int nc = (w.mg + 7) / 8;
    if (MAXNC == 1 || nc <= 1)
      consume_group<EPI, ACT_F16, STAGES, kActRows, 1>(args, cx, w, it);
    else if (MAXNC == 2 || nc <= 2)
      consume_group<EPI, ACT_F16, STAGES, kActRows, (MAXNC >= 2 ? 2 : 1)>(args, cx, w, it);
    else if (MAXNC == 4 || nc <= 4)
      consume_group<EPI, ACT_F16, STAGES, kActRows, (MAXNC >= 4 ? 4 : 1)>(args, cx, w, it);
    else
      consume_group<EPI, ACT_F16, STAGES, kActRows, (MAXNC >= 8 ? 8 : 1)>(args, cx, w, it);
    __syncwarp();
    if (lane == 0) mbar_arrive(&slab_empty[sb]);
  }
}

}  // namespace d3
