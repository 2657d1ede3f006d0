// C ABI of the expert pipeline: d3_moe_experts, d3_moe_layer, d3_fp8_gemv.
//
// Pipeline for T tokens, top-k, E experts (P = T*k pairs, R = P + T rows when
// a shared expert runs):
//   1. permute       ids -> counts, starts, inverse rows, active list
//   2. quant_scatter x -> e4m3 rows in expert order (+ T shared rows), scales
//   3. gate_up       engine EPI_GATE_UP (decode) or tcgen05 grouped GEMM
//                    (prefill): a e4m3 [R, I], sa [R, I/128]
//   4. down          engine EPI_DOWN or tcgen05 grouped GEMM: d f32 [R, H]
//   5. combine       routed/shared/out bf16 [T, H] in fixed rank order, or the
//                    combine fused with the residual update and RMSNorm
// All buffers live in the caller's workspace; nothing is allocated here.
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "d3_host.h"
#include "d3_internal.h"
#include "dense_tc.cuh"
#include "expert_gemv.cuh"
#include "tc_grouped.cuh"

namespace d3 {

namespace {

thread_local void* const* g_stage_events = nullptr;

inline void stage_mark(int i, cudaStream_t s) {
  if (g_stage_events) cudaEventRecord(static_cast<cudaEvent_t>(g_stage_events[i]), s);
}

struct Carve {
  uint8_t* base;
  size_t off = 0;
  template <typename T>
  T* take(size_t count) {
    off = align_up(off, 256);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

struct MoeBuffers {
  int32_t* status;
  int32_t* counts;
  int32_t* starts;
  int32_t* total;
  int32_t* active;
  int32_t* n_active;
  int32_t* inv;
  int32_t* permute_scratch;
  int32_t* work;  // engine work counters: [0] gate_up, [1] down
  uint8_t* xq;
  float* sx;
  uint8_t* a;
  float* sa;
  float* d;
  __nv_bfloat16* logits;  // layer only: [T, E+1]
  int64_t* ids;           // layer only
  __nv_bfloat16* weights; // layer only
  size_t bytes;
};

MoeBuffers carve_moe(void* ws, int T, int k, int E, int I, int H, int has_shared, int layer) {
  Carve c{static_cast<uint8_t*>(ws)};
  const int64_t P = static_cast<int64_t>(T) * k;
  const int64_t R = P + (has_shared ? T : 0);
  MoeBuffers b;
  b.status = c.take<int32_t>(4);
  b.counts = c.take<int32_t>(E);
  b.starts = c.take<int32_t>(E);
  b.total = c.take<int32_t>(1);
  b.active = c.take<int32_t>(E);
  b.n_active = c.take<int32_t>(1);
  b.inv = c.take<int32_t>(P > 0 ? P : 1);
  b.permute_scratch = c.take<int32_t>(permute_scratch_ints(E));
  b.work = c.take<int32_t>(2);
  b.xq = c.take<uint8_t>(R * H);
  b.sx = c.take<float>(R * (H / 128));
  b.a = c.take<uint8_t>(R * I);
  b.sa = c.take<float>(R * (I / 128));
  b.d = c.take<float>(R * H);
  if (layer) {
    b.logits = c.take<__nv_bfloat16>(static_cast<size_t>(T) * (E + 1));
    b.ids = c.take<int64_t>(P);
    b.weights = c.take<__nv_bfloat16>(P);
  } else {
    b.logits = nullptr;
    b.ids = nullptr;
    b.weights = nullptr;
  }
  b.bytes = c.off + 256;
  return b;
}

int nch_for(int max_tokens) {
  const int m = max_tokens < kTokensPerGroup ? max_tokens : kTokensPerGroup;
  if (m <= 8) return 1;
  if (m <= 16) return 2;
  if (m <= 32) return 4;
  return 8;
}

template <int EPI, bool ACT_F16, int NCH, int STAGES>
int launch_engine_inst(const CUtensorMap& tw, const CUtensorMap& twsh, const CUtensorMap& ta,
                       const EngineArgs& args, int grid, cudaStream_t s) {
  auto kern = expert_gemv_kernel<EPI, ACT_F16, STAGES, NCH>;
  constexpr int kGroup = NCH * 8 < kTokensPerGroup ? NCH * 8 : kTokensPerGroup;
  constexpr int kActRows = kGroup < 16 ? 16 : kGroup;
  const size_t smem = EngineSmem<EPI, ACT_F16, STAGES, kActRows>::bytes(args.KB, args.num_experts);
  if (smem > 227 * 1024)
    return set_error(D3_EUNSUPPORTED, "engine: %zu bytes of shared memory needed (K=%d too large)",
                     smem, args.KB * 128);
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || configured[dev] < static_cast<int>(smem)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return set_error(D3_ECUDA, "engine: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) configured[dev] = static_cast<int>(smem);
  }
  launch_kernel(kern, dim3(grid), dim3(kEngineThreads), smem, s, tw, twsh, ta, args);
  return check_launch("expert engine");
}

template <int EPI, bool ACT_F16, int STAGES>
int launch_engine(int nch, const CUtensorMap& tw, const CUtensorMap& twsh, const CUtensorMap& ta,
                  const EngineArgs& args, int grid, cudaStream_t s) {
  // gate_up and paired-tile down hold two accumulator sets
  constexpr int kMax = kTwoBoxes<EPI> ? 4 : 8;
  switch (nch) {
    case 1: return launch_engine_inst<EPI, ACT_F16, 1, STAGES>(tw, twsh, ta, args, grid, s);
    case 2: return launch_engine_inst<EPI, ACT_F16, 2, STAGES>(tw, twsh, ta, args, grid, s);
    case 4: return launch_engine_inst<EPI, ACT_F16, 4, STAGES>(tw, twsh, ta, args, grid, s);
    default: return launch_engine_inst<EPI, ACT_F16, kMax, STAGES>(tw, twsh, ta, args, grid, s);
  }
}

// Ring depths: the deepest ring that fits 227 KB of shared memory with E <= 1024
// experts of routing metadata (gate_up: 36 KB stages, down: 24 KB, dense: 32 KB).
constexpr int kStagesGateUp = 5;
constexpr int kStagesDown = 8;
constexpr int kStagesDense = 6;

// Token count from which the expert GEMMs run on tcgen05 (128-token tiles)
// instead of the streaming engine. D3MOE_PREFILL_MIN_T overrides it.
int default_prefill_min_tokens() {
  static const int v = [] {
    const char* e = std::getenv("D3MOE_PREFILL_MIN_T");
    const int t = e ? std::atoi(e) : 0;
    return t > 0 ? t : 1024;
  }();
  return v;
}

std::atomic<int> g_prefill_min_tokens{0};

int prefill_min_tokens() {
  const int t = g_prefill_min_tokens.load(std::memory_order_relaxed);
  return t > 0 ? t : default_prefill_min_tokens();
}

template <int KIND>
int launch_tc(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& twsh,
              const TcArgs& args, int grid, cudaStream_t s) {
  auto kern = tc_grouped_kernel<KIND>;
  const size_t smem = TcSmem<KIND>::bytes();
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    // The warpgroup register split (setmaxnreg) is sized for exactly
    // kTcLaunchRegs registers per thread at launch; any other allocation would
    // make the increase wait forever, so refuse to launch instead.
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess || fa.numRegs != kTcLaunchRegs)
      return set_error(D3_ECUDA, "tc grouped GEMM: built with %d registers per thread, expected %d",
                       fa.numRegs, kTcLaunchRegs);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return set_error(D3_ECUDA, "tc grouped GEMM: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  launch_kernel(kern, dim3(grid), dim3(kTcThreads), smem, s, ta, tw, twsh, args);
  return check_launch("tc grouped GEMM");
}

// Upper bound of the 128 x 256 tiles of one grouped GEMM (every group's rows
// rounded up to 128), used to size the grid before the counts are known.
int tc_grid(int R, int groups, int ntiles, int sms) {
  const int64_t mt = (static_cast<int64_t>(R) + 127) / 128 + groups;
  const int64_t tiles = mt * ntiles;
  return static_cast<int>(tiles < sms ? tiles : sms);
}

// Row layout of w13 within an expert: [gate | up] (D3_GATE_UP, the checkpoint
// order) or [up | gate] (D3_UP_GATE, FlashInfer's SwiGLU order).
int gate_first_row(const d3_experts_t* e) { return e->gate_up_order == D3_UP_GATE ? e->I : 0; }
int up_minus_gate(const d3_experts_t* e) { return e->gate_up_order == D3_UP_GATE ? -e->I : e->I; }

int check_experts(const d3_experts_t* e, const char* what) {
  D3_REQUIRE(e != nullptr, "%s: expert weights missing", what);
  D3_REQUIRE(e->w13 && e->s13 && e->w2 && e->s2, "%s: null weight pointer", what);
  D3_REQUIRE(e->E > 0 && e->I > 0 && e->H > 0, "%s: bad expert shape", what);
  D3_REQUIRE(e->I % 128 == 0 && e->H % 128 == 0, "%s: H=%d and I=%d must be multiples of 128", what, e->H, e->I);
  D3_REQUIRE(aligned(e->w13, 16) && aligned(e->w2, 16), "%s: weights must be 16-byte aligned", what);
  D3_REQUIRE(e->gate_up_order == D3_GATE_UP || e->gate_up_order == D3_UP_GATE,
             "%s: gate_up_order must be D3_GATE_UP or D3_UP_GATE", what);
  return D3_OK;
}

// Residual update and RMSNorm fused into the combine (the layer exit).
struct AddNorm {
  void* residual = nullptr;         // bf16 [T (or T_out), H], updated in place
  const void* weight = nullptr;     // bf16 [H]
  float eps = 0.f;
  const int64_t* inverse = nullptr; // [T_out]: residual row t takes MoE row inverse[t]
  int T_out = 0;
  int32_t* status = nullptr;        // receives kDevBadRow for an inverse value outside [0, T)
};

// Step 5: the fixed-order combine, or (with an AddNorm) the combine fused with
// the residual update and RMSNorm of the layer exit.
// rows_bf16: the expert rows in b.d are bf16 (written by the tcgen05 down
// kernel) rather than fp32 (the decode engine).
int finish_layer(const MoeBuffers& b, int H, const void* weights, int T, int k, int has_shared,
                 const void* gate, int64_t gate_stride, void* routed_out, void* shared_out,
                 void* out, const AddNorm& an, cudaStream_t s, bool rows_bf16 = false) {
  if (an.residual)
    return launch_combine_rows_add_norm(b.d, H, b.inv, weights, T, k, gate, gate_stride,
                                        an.residual, an.weight, an.eps, out, s, an.inverse,
                                        an.T_out, an.status, rows_bf16);
  launch_combine_rows(b.d, H, b.inv, weights, T, k, has_shared, gate, gate_stride, routed_out,
                      shared_out, out, s, rows_bf16);
  return check_launch("combine_rows");
}

// Already-quantised input of d3_moe_experts_fp8 (replaces the bf16 x).
struct PreQuant {
  const uint8_t* q = nullptr;
  int64_t q_stride = 0;
  const float* scales = nullptr;
  int transposed = 0;
};

// Whether the bucketing of a call runs fused into the activation
// quantisation (one CTA per token, every CTA counting over all pairs).
bool fused_permute(int T, int k, int E) {
  return static_cast<int64_t>(T) * k < kFusedPermuteMaxPairs && E <= kFusedPermuteMaxExperts;
}

// Whether the expert GEMMs of a T-token call run on tcgen05 (prefill) or on
// the decode engine. Both stages of a call take this decision the same way,
// so the threshold must not change between them.
bool use_tc(int T, int H) { return T >= prefill_min_tokens() && H % 256 == 0; }

TcArgs tc_common(const MoeBuffers& b, int E, int I, int T, int P, int R, int has_shared,
                 int32_t* status) {
  TcArgs a{};
  a.counts = b.counts;
  a.starts = b.starts;
  a.E = E;
  a.has_shared = has_shared;
  a.shared_row0 = P;
  a.shared_count = T;
  a.act_rows = R;
  a.I = I;
  a.status = status;
  return a;
}

// Steps 1-3 on an already carved workspace: the bucketing (unless done),
// x into expert order as e4m3 (or pre-quantised rows copied there), and
// gate_up + SiLU*mul + FP8 requant into b.a / b.sa.
int experts_up(const void* x, int64_t x_stride, const int64_t* ids, int T, int k,
               const d3_experts_t* ex, const d3_experts_t* sh, const MoeBuffers& b,
               int32_t* status, cudaStream_t s, bool permuted, const RowGather& rg,
               const PreQuant& pq) {
  const int E = ex->E, I = ex->I, H = ex->H;
  const int P = T * k;
  const int has_shared = sh ? 1 : 0;
  const int R = P + (has_shared ? T : 0);
  int rc = D3_OK;
  if (!permuted && !pq.q && fused_permute(T, k, E)) {
    // decode sizes: bucketing and activation quantisation in one kernel
    launch_permute_quant(x, x_stride, T, H, k, ids, E, has_shared, b.xq, b.sx, b.counts, b.starts,
                         b.total, b.inv, b.active, b.n_active, s, b.work, 2, rg);
    if ((rc = check_launch("permute_quant"))) return rc;
  } else {
    if (!permuted) {
      // the pipeline reads counts, starts, the inverse map and the active list;
      // the reference's sorted-pair and per-tile expert buffers are not written
      rc = launch_permute(ids, T, k, E, 1, b.counts, b.starts, b.total, nullptr, nullptr, P,
                          b.inv, b.active, b.n_active, s, b.permute_scratch);
      if (rc) return rc;
    }
    if (pq.q)
      launch_prequant_scatter(pq.q, pq.q_stride, pq.scales, pq.transposed, T, H, k, b.inv, b.xq,
                              b.sx, s, b.work, 2);
    else
      launch_quant_scatter(x, x_stride, T, H, k, b.inv, P, has_shared, b.xq, b.sx, s, b.work, 2, rg);
    if ((rc = check_launch("quant_scatter"))) return rc;
  }

  const int sms = sm_count();
  stage_mark(1, s);
  if (use_tc(T, H)) {
    // ---- prefill: tcgen05
    TcArgs a = tc_common(b, E, I, T, P, R, has_shared, status);
    {
      CUtensorMap tw, twsh, ta;
      if ((rc = encode_tmap_2d(&tw, ex->w13, 1, H, static_cast<uint64_t>(E) * 2 * I, H, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&twsh, has_shared ? sh->w13 : ex->w13, 1, H,
                               static_cast<uint64_t>(2) * I, H, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&ta, b.xq, 1, H, R, H, 128, 128))) return rc;
      a.ntiles = I / 128;
      a.KB = H / 128;
      a.rows_per_expert = 2 * I;
      a.second_box = up_minus_gate(ex);  // the gate half's offset is I (TC_UP_GATE)
      a.nt_stride = 128;
      a.wscale = ex->s13;
      a.wscale_sh = has_shared ? sh->s13 : ex->s13;
      a.act_scale = b.sx;
      a.out_q = b.a;
      a.out_qs = b.sa;
      rc = ex->gate_up_order == D3_UP_GATE
               ? launch_tc<TC_UP_GATE>(ta, tw, twsh, a, tc_grid(R, E + has_shared, a.ntiles, sms), s)
               : launch_tc<TC_GATE_UP>(ta, tw, twsh, a, tc_grid(R, E + has_shared, a.ntiles, sms), s);
      if (rc) return rc;
    }
  } else {
    // ---- gate_up
    {
      CUtensorMap tw, twsh, ta;
      if ((rc = encode_tmap_2d(&tw, ex->w13, 1, H, static_cast<uint64_t>(E) * 2 * I, H, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&twsh, has_shared ? sh->w13 : ex->w13, 1, H,
                               static_cast<uint64_t>(2) * I, H, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&ta, b.xq, 1, H, R, H, 128, 16))) return rc;
      EngineArgs a{};
      a.counts = b.counts;
      a.starts = b.starts;
      a.active = b.active;
      a.n_active = b.n_active;
      a.num_experts = E;
      // gate_up keeps two accumulator sets (gate, up): at most 4 token chunks
      // (32 tokens) per group fit the 168 registers a 9-warp CTA gets
      const int nch = nch_for(T) < 4 ? nch_for(T) : 4;
      a.shared_chunk = nch * 8;
      a.shared_groups = has_shared ? (T + a.shared_chunk - 1) / a.shared_chunk : 0;
      a.shared_row0 = P;
      a.shared_count = T;
      a.tiles = I / 128;
      a.KB = H / 128;
      a.ksplit = 1;
      a.kb_per_split = a.KB;
      a.rows_per_expert = 2 * I;
      a.first_off = gate_first_row(ex);
      a.up_offset = up_minus_gate(ex);
      a.wscale = ex->s13;
      a.wscale_sh = has_shared ? sh->s13 : ex->s13;
      a.act_scale = b.sx;
      a.out_q = b.a;
      a.out_qs = b.sa;
      a.out_cols = I;
      a.status = status;
      a.work_counter = b.work;
      const int max_items = (E + a.shared_groups) * (I / 128);
      const int grid = max_items < sms ? max_items : sms;
      rc = launch_engine<EPI_GATE_UP, false, kStagesGateUp>(nch, tw, twsh, ta, a, grid, s);
      if (rc) return rc;
    }
  }
  stage_mark(2, s);
  return D3_OK;
}

// Steps 4-5: down into b.d and the fixed-order combine, or the combine fused
// with the layer exit.
int experts_down(const void* weights, int T, int k, const d3_experts_t* ex,
                 const d3_experts_t* sh, const void* gate, int64_t gate_stride, void* routed_out,
                 void* shared_out, void* out, const MoeBuffers& b, int32_t* status,
                 cudaStream_t s, const AddNorm& an) {
  const int E = ex->E, I = ex->I, H = ex->H;
  const int P = T * k;
  const int has_shared = sh ? 1 : 0;
  const int R = P + (has_shared ? T : 0);
  const int sms = sm_count();
  const bool tc = use_tc(T, H);
  int rc = D3_OK;
  if (tc) {
    // ---- prefill: tcgen05, bf16 rows
    TcArgs a = tc_common(b, E, I, T, P, R, has_shared, status);
    {
      CUtensorMap tw, twsh, ta;
      if ((rc = encode_tmap_2d(&tw, ex->w2, 1, I, static_cast<uint64_t>(E) * H, I, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&twsh, has_shared ? sh->w2 : ex->w2, 1, I, H, I, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&ta, b.a, 1, I, R, I, 128, 128))) return rc;
      a.ntiles = H / 256;
      a.KB = I / 128;
      a.rows_per_expert = H;
      a.second_box = 128;
      a.nt_stride = 256;
      a.wscale = ex->s2;
      a.wscale_sh = has_shared ? sh->s2 : ex->s2;
      a.act_scale = b.sa;
      a.out_q = nullptr;
      a.out_qs = nullptr;
      a.out_rows = b.d;
      a.out_ld = H;
      rc = launch_tc<TC_DOWN>(ta, tw, twsh, a, tc_grid(R, E + has_shared, a.ntiles, sms), s);
      if (rc) return rc;
    }
  } else {
    // ---- down
    {
      CUtensorMap tw, twsh, ta;
      if ((rc = encode_tmap_2d(&tw, ex->w2, 1, I, static_cast<uint64_t>(E) * H, I, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&twsh, has_shared ? sh->w2 : ex->w2, 1, I, H, I, 128, 128))) return rc;
      if ((rc = encode_tmap_2d(&ta, b.a, 1, I, R, I, 128, 16))) return rc;
      EngineArgs a{};
      a.counts = b.counts;
      a.starts = b.starts;
      a.active = b.active;
      a.n_active = b.n_active;
      a.num_experts = E;
      // pairs of 128-row tiles per item when H allows (two accumulator sets:
      // at most 4 token chunks per group, like gate_up)
      const bool pair = H % 256 == 0;
      const int nch = pair ? (nch_for(T) < 4 ? nch_for(T) : 4) : nch_for(T);
      a.shared_chunk = nch * 8;
      a.shared_groups = has_shared ? (T + a.shared_chunk - 1) / a.shared_chunk : 0;
      a.shared_row0 = P;
      a.shared_count = T;
      a.tiles = pair ? H / 256 : H / 128;
      a.KB = I / 128;
      a.ksplit = 1;
      a.kb_per_split = a.KB;
      a.rows_per_expert = H;
      a.wscale = ex->s2;
      a.wscale_sh = has_shared ? sh->s2 : ex->s2;
      a.act_scale = b.sa;
      a.out_rows = b.d;
      a.out_ld = H;
      a.status = status;
      a.work_counter = b.work + 1;
      const int max_items = (E + a.shared_groups) * a.tiles;
      const int grid = max_items < sms ? max_items : sms;
      rc = pair ? launch_engine<EPI_DOWN2, false, kStagesGateUp>(nch, tw, twsh, ta, a, grid, s)
                : launch_engine<EPI_DOWN, false, kStagesDown>(nch, tw, twsh, ta, a, grid, s);
      if (rc) return rc;
    }
  }
  stage_mark(3, s);
  rc = finish_layer(b, H, weights, T, k, has_shared, gate, gate_stride, routed_out, shared_out, out,
                    an, s, tc);
  stage_mark(4, s);
  return rc;
}

// Steps 1-5: ids/weights are device tensors [T,k]; gate (nullable) feeds the
// shared-expert combine.
int run_experts(const void* x, int64_t x_stride, const int64_t* ids, const void* weights, int T,
                int k, const d3_experts_t* ex, const d3_experts_t* sh, const void* gate,
                int64_t gate_stride, void* routed_out, void* shared_out, void* out,
                const MoeBuffers& b, int32_t* status, cudaStream_t s, bool permuted,
                const AddNorm& an = AddNorm{}, const RowGather& rg = RowGather{},
                const PreQuant& pq = PreQuant{}) {
  int rc = experts_up(x, x_stride, ids, T, k, ex, sh, b, status, s, permuted, rg, pq);
  if (rc) return rc;
  return experts_down(weights, T, k, ex, sh, gate, gate_stride, routed_out, shared_out, out, b,
                      status, s, an);
}

}  // namespace

}  // namespace d3

using namespace d3;

extern "C" int d3_set_stage_events(void* const* events, int n) {
  D3_REQUIRE(events == nullptr || n >= 5, "set_stage_events: need at least 5 events");
  g_stage_events = events;
  return D3_OK;
}

extern "C" int d3_set_prefill_min_tokens(int t) {
  const int prev = prefill_min_tokens();
  g_prefill_min_tokens.store(t > 0 ? t : 0, std::memory_order_relaxed);
  return prev;
}

extern "C" int d3_moe_workspace_size(int T, int k, int E, int I, int H, int has_shared,
                                     size_t* bytes) {
  D3_REQUIRE(bytes != nullptr, "moe_workspace_size: null output");
  D3_REQUIRE(T >= 0 && k > 0 && E > 0 && I > 0 && H > 0, "moe_workspace_size: bad shape");
  *bytes = carve_moe(nullptr, T, k, E, I, H, has_shared, 1).bytes;
  return D3_OK;
}

static int check_common(const void* x, int64_t x_stride, int T, int k, const d3_experts_t* ex,
                        const d3_experts_t* sh, void* ws, size_t ws_bytes, const char* what) {
  int rc = check_experts(ex, what);
  if (rc) return rc;
  if (sh) {
    if ((rc = check_experts(sh, what))) return rc;
    D3_REQUIRE(sh->E == 1 && sh->I == ex->I && sh->H == ex->H,
               "%s: the shared expert must have E=1 and the routed I/H", what);
    D3_REQUIRE(sh->gate_up_order == ex->gate_up_order,
               "%s: routed and shared experts must use the same gate_up_order", what);
  }
  D3_REQUIRE(T >= 0 && k > 0 && k <= 32 && k <= ex->E, "%s: bad top-k %d", what, k);
  D3_REQUIRE(ex->E <= 1024, "%s: E=%d above 1024", what, ex->E);
  D3_REQUIRE(ex->H <= 4096, "%s: H=%d above 4096", what, ex->H);
  D3_REQUIRE(static_cast<int64_t>(T) * k < (1 << 24), "%s: too many pairs", what);
  D3_REQUIRE(x_stride >= ex->H && x_stride % 8 == 0, "%s: x row stride must be >= H and a multiple of 8", what);
  D3_REQUIRE(aligned(x, 16), "%s: x must be 16-byte aligned", what);
  D3_REQUIRE(ws != nullptr && aligned(ws, 256), "%s: workspace must be 256-byte aligned", what);
  size_t need = carve_moe(nullptr, T, k, ex->E, ex->I, ex->H, sh != nullptr, 1).bytes;
  if (ws_bytes < need)
    return set_error(D3_EWORKSPACE, "%s: workspace %zu bytes < %zu", what, ws_bytes, need);
  return D3_OK;
}

extern "C" int d3_moe_experts(const void* x, int64_t x_stride, const int64_t* ids,
                              const void* weights, int T, int k, const d3_experts_t* experts,
                              const d3_experts_t* shared, void* routed_out, void* shared_out,
                              void* workspace, size_t workspace_bytes, int32_t* status,
                              d3_stream_t stream) {
  int rc = check_common(x, x_stride, T, k, experts, shared, workspace, workspace_bytes,
                        "moe_experts");
  if (rc) return rc;
  D3_REQUIRE(ids && weights && routed_out, "moe_experts: null ids, weights or output");
  D3_REQUIRE(aligned(routed_out, 16) && (!shared_out || aligned(shared_out, 16)), "moe_experts: outputs must be 16-byte aligned");
  if (T == 0) return D3_OK;
  auto b = carve_moe(workspace, T, k, experts->E, experts->I, experts->H, shared != nullptr, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  stage_mark(0, s);
  return run_experts(x, x_stride, ids, weights, T, k, experts, shared, nullptr, 0, routed_out,
                     shared_out, nullptr, b, status ? status : b.status, s, false);
}

namespace {
// Host-side record of the workspaces d3_moe_gate_up_silu filled, with the
// call's shape, so that d3_moe_down_combine refuses a workspace whose bucketing
// and activations it would otherwise read unchecked (garbage counts or rows
// would send its kernels' stores anywhere). The record costs no device work
// and no synchronisation; it does not see device-side reuse of the workspace
// by other calls between the two stages, which the caller must avoid.
struct StageRecord {
  const void* ws;
  int T, k, E, I, H, has_shared;
  bool operator==(const StageRecord& o) const {
    return ws == o.ws && T == o.T && k == o.k && E == o.E && I == o.I && H == o.H &&
           has_shared == o.has_shared;
  }
};
constexpr size_t kMaxStageRecords = 64;
std::mutex g_stage_mutex;
StageRecord g_stage_records[kMaxStageRecords];
size_t g_stage_count = 0, g_stage_next = 0;

void stage_record(const StageRecord& r) {
  std::lock_guard<std::mutex> lock(g_stage_mutex);
  for (size_t i = 0; i < g_stage_count; ++i)
    if (g_stage_records[i].ws == r.ws) {
      g_stage_records[i] = r;
      return;
    }
  g_stage_records[g_stage_next] = r;  // oldest record replaced once the table is full
  g_stage_next = (g_stage_next + 1) % kMaxStageRecords;
  if (g_stage_count < kMaxStageRecords) ++g_stage_count;
}

bool stage_recorded(const StageRecord& r) {
  std::lock_guard<std::mutex> lock(g_stage_mutex);
  for (size_t i = 0; i < g_stage_count; ++i)
    if (g_stage_records[i] == r) return true;
  return false;
}

// A down_combine that ran consumes its record: the next one needs a fresh
// gate_up_silu into the workspace.
void stage_forget(const StageRecord& r) {
  std::lock_guard<std::mutex> lock(g_stage_mutex);
  for (size_t i = 0; i < g_stage_count; ++i)
    if (g_stage_records[i] == r) g_stage_records[i].ws = nullptr;
}
}  // namespace

extern "C" int d3_moe_gate_up_silu(const void* x, int64_t x_stride, const int64_t* ids, int T,
                                   int k, const d3_experts_t* experts, const d3_experts_t* shared,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   d3_stream_t stream) {
  int rc = check_common(x, x_stride, T, k, experts, shared, workspace, workspace_bytes,
                        "moe_gate_up_silu");
  if (rc) return rc;
  D3_REQUIRE(ids != nullptr, "moe_gate_up_silu: null ids");
  if (T == 0) return D3_OK;
  auto b = carve_moe(workspace, T, k, experts->E, experts->I, experts->H, shared != nullptr, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  stage_mark(0, s);
  rc = experts_up(x, x_stride, ids, T, k, experts, shared, b, status ? status : b.status, s, false,
                  RowGather{}, PreQuant{});
  if (rc == D3_OK)
    stage_record({workspace, T, k, experts->E, experts->I, experts->H, shared != nullptr});
  return rc;
}

extern "C" int d3_moe_down_combine(const void* weights, int T, int k, const d3_experts_t* experts,
                                   const d3_experts_t* shared, void* routed_out, void* shared_out,
                                   void* workspace, size_t workspace_bytes, int32_t* status,
                                   d3_stream_t stream) {
  D3_REQUIRE(experts != nullptr, "moe_down_combine: expert weights missing");
  // no input rows here: the checks of the shared entry point run with x absent
  int rc = check_common(nullptr, experts->H, T, k, experts, shared, workspace, workspace_bytes,
                        "moe_down_combine");
  if (rc) return rc;
  D3_REQUIRE(weights && routed_out, "moe_down_combine: null weights or output");
  D3_REQUIRE(T == 0 || stage_recorded({workspace, T, k, experts->E, experts->I, experts->H,
                                       shared != nullptr}),
             "moe_down_combine: the workspace was not filled by d3_moe_gate_up_silu with T=%d, "
             "k=%d, E=%d, I=%d, H=%d and %s shared expert", T, k, experts->E, experts->I,
             experts->H, shared ? "a" : "no");
  D3_REQUIRE(aligned(routed_out, 16) && (!shared_out || aligned(shared_out, 16)),
             "moe_down_combine: outputs must be 16-byte aligned");
  if (T == 0) return D3_OK;
  auto b = carve_moe(workspace, T, k, experts->E, experts->I, experts->H, shared != nullptr, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = experts_down(weights, T, k, experts, shared, nullptr, 0, routed_out, shared_out, nullptr, b,
                    status ? status : b.status, s, AddNorm{});
  if (rc == D3_OK)
    stage_forget({workspace, T, k, experts->E, experts->I, experts->H, shared != nullptr});
  return rc;
}

extern "C" int d3_moe_experts_fp8(const uint8_t* q, int64_t q_stride, const float* q_scales,
                                  int scales_transposed, const int64_t* ids, const void* weights,
                                  int T, int k, const d3_experts_t* experts, void* routed_out,
                                  void* workspace, size_t workspace_bytes, int32_t* status,
                                  d3_stream_t stream) {
  int rc = check_common(q, q_stride, T, k, experts, nullptr, workspace, workspace_bytes,
                        "moe_experts_fp8");
  if (rc) return rc;
  D3_REQUIRE(q_stride % 16 == 0, "moe_experts_fp8: q row stride must be a multiple of 16 bytes");
  D3_REQUIRE(q_scales && ids && weights && routed_out && aligned(routed_out, 16),
             "moe_experts_fp8: null or misaligned scales / ids / weights / output");
  if (T == 0) return D3_OK;
  auto b = carve_moe(workspace, T, k, experts->E, experts->I, experts->H, 0, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  PreQuant pq;
  pq.q = q;
  pq.q_stride = q_stride;
  pq.scales = q_scales;
  pq.transposed = scales_transposed ? 1 : 0;
  stage_mark(0, s);
  return run_experts(nullptr, 0, ids, weights, T, k, experts, nullptr, nullptr, 0, routed_out,
                     nullptr, nullptr, b, status ? status : b.status, s, false, AddNorm{},
                     RowGather{}, pq);
}

static int moe_layer_impl(const void* x, int64_t x_stride, const void* router_w,
                          const float* router_bias, int T, int k, const d3_experts_t* experts,
                          const d3_experts_t* shared, void* out, int64_t* ids_out,
                          void* weights_out, void* workspace, size_t workspace_bytes,
                          int32_t* status, d3_stream_t stream, const AddNorm& an_in,
                          const d3_rows_t* rows = nullptr) {
  int rc = check_common(x, x_stride, T, k, experts, shared, workspace, workspace_bytes,
                        "moe_layer");
  if (rc) return rc;
  D3_REQUIRE(shared != nullptr, "moe_layer: the layer needs its shared expert");
  D3_REQUIRE(router_w && out && aligned(router_w, 16) && aligned(out, 16), "moe_layer: null or misaligned router weight / output");
  D3_REQUIRE(experts->H <= 3072, "moe_layer: H=%d above the 3072 the router kernel stages", experts->H);
  if (T == 0) return D3_OK;
  const int E = experts->E, H = experts->H;
  auto b = carve_moe(workspace, T, k, E, experts->I, H, 1, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int64_t* ids = ids_out ? ids_out : b.ids;
  void* wts = weights_out ? weights_out : static_cast<void*>(b.weights);
  int32_t* st = status ? status : b.status;
  RowGather rg;
  PaddingRoute pr;
  AddNorm an = an_in;
  if (rows) {
    rg.keep = rows->keep;
    rg.x_rows = rows->x_rows;
    rg.status = st;
    pr.slots = rows->row_slots;
    pr.slots_i64 = rows->row_slots_int64;
    pr.padding_start = rows->padding_start;
    an.inverse = rows->inverse;
    an.T_out = rows->T_out;
    an.status = st;
  }
  stage_mark(0, s);
  // b.d (expert rows, written only by the down step) holds the kept rows
  // for the tensor-core router when a keep map is given
  launch_router_logits(x, x_stride, router_w, router_bias, E, E + 1, H, T, b.logits, E + 1, s, rg, st, b.d);
  if ((rc = check_launch("router_logits"))) return rc;
  const int P = T * k;
  const bool fused = fused_permute(T, k, E);
  if (fused) {
    // the bucketing runs inside the quantisation kernel of run_experts
    launch_route_topk(b.logits, D3_DTYPE_BF16, E + 1, T, E, k, nullptr, ids, wts, D3_DTYPE_BF16, s, pr);
    if ((rc = check_launch("route_topk"))) return rc;
  } else {
    rc = launch_route_permute(b.logits, D3_DTYPE_BF16, E + 1, T, E, k, nullptr, ids, wts,
                              D3_DTYPE_BF16, 1, b.counts, b.starts, b.total, nullptr, nullptr, P,
                              b.inv, b.active, b.n_active, s, b.permute_scratch, pr);
    if (rc) return rc;
  }
  return run_experts(x, x_stride, ids, wts, T, k, experts, shared, b.logits + E, E + 1, nullptr,
                     nullptr, out, b, st, s, !fused, an, rg);
}

extern "C" int d3_moe_layer(const void* x, int64_t x_stride, const void* router_w,
                            const float* router_bias, int T, int k, const d3_experts_t* experts,
                            const d3_experts_t* shared, void* out, int64_t* ids_out,
                            void* weights_out, void* workspace, size_t workspace_bytes,
                            int32_t* status, d3_stream_t stream) {
  return moe_layer_impl(x, x_stride, router_w, router_bias, T, k, experts, shared, out, ids_out,
                        weights_out, workspace, workspace_bytes, status, stream, AddNorm{});
}

extern "C" int d3_moe_layer_add_norm(const void* x, int64_t x_stride, const void* router_w,
                                     const float* router_bias, int T, int k,
                                     const d3_experts_t* experts, const d3_experts_t* shared,
                                     void* residual, const void* norm_weight, float eps, void* out,
                                     int64_t* ids_out, void* weights_out, void* workspace,
                                     size_t workspace_bytes, int32_t* status, d3_stream_t stream) {
  D3_REQUIRE(residual && norm_weight && aligned(residual, 16) && aligned(norm_weight, 16),
             "moe_layer_add_norm: null or misaligned residual / norm weight");
  D3_REQUIRE(experts && experts->H % 8 == 0 && experts->H <= 8192,
             "moe_layer_add_norm: H must be a multiple of 8 up to 8192");
  AddNorm an;
  an.residual = residual;
  an.weight = norm_weight;
  an.eps = eps;
  return moe_layer_impl(x, x_stride, router_w, router_bias, T, k, experts, shared, out, ids_out,
                        weights_out, workspace, workspace_bytes, status, stream, an);
}

extern "C" int d3_moe_layer_rows(const void* x, int64_t x_stride, const void* router_w,
                                 const float* router_bias, int T, int k,
                                 const d3_experts_t* experts, const d3_experts_t* shared,
                                 const d3_rows_t* rows, void* residual, const void* norm_weight,
                                 float eps, void* out, int64_t* ids_out, void* weights_out,
                                 void* workspace, size_t workspace_bytes, int32_t* status,
                                 d3_stream_t stream) {
  if (rows) {
    D3_REQUIRE(rows->keep == nullptr || rows->x_rows > 0,
               "moe_layer_rows: keep needs the row count of x (x_rows > 0)");
    D3_REQUIRE(rows->inverse == nullptr || (residual != nullptr && rows->T_out >= 0),
               "moe_layer_rows: an inverse map needs the fused exit (residual) and T_out >= 0");
    D3_REQUIRE(rows->row_slots == nullptr || rows->padding_start > 0,
               "moe_layer_rows: padding_start must be a positive reserved-slot boundary");
  }
  AddNorm an;
  if (residual) {
    D3_REQUIRE(norm_weight && aligned(residual, 16) && aligned(norm_weight, 16),
               "moe_layer_rows: null or misaligned residual / norm weight");
    D3_REQUIRE(experts && experts->H % 8 == 0 && experts->H <= 8192,
               "moe_layer_rows: H must be a multiple of 8 up to 8192");
    an.residual = residual;
    an.weight = norm_weight;
    an.eps = eps;
  }
  return moe_layer_impl(x, x_stride, router_w, router_bias, T, k, experts, shared, out, ids_out,
                        weights_out, workspace, workspace_bytes, status, stream, an, rows);
}

namespace {
// Workspace of d3_fp8_gemv / d3_fp8_gated_gemv: a status word and the
// activations split into two E4M3 terms (hi, lo [T, K]) with their group
// scales [T, K/128].
struct DenseBuffers {
  int32_t* status;
  uint8_t* hi;
  uint8_t* lo;
  float* sc;
  size_t bytes;
};

DenseBuffers carve_dense(void* ws, int T, int K) {
  Carve c{static_cast<uint8_t*>(ws)};
  DenseBuffers b;
  b.status = c.take<int32_t>(4);
  b.hi = c.take<uint8_t>(static_cast<size_t>(T) * K);
  b.lo = c.take<uint8_t>(static_cast<size_t>(T) * K);
  b.sc = c.take<float>(static_cast<size_t>(T) * (K / 128));
  b.bytes = c.off + 256;
  return b;
}

// Most clusters of `split` CTAs of the TP instance that can be resident at
// once (cached per device).
template <int TP>
int dense_max_clusters(int dev, int split) {
  static int cache[64][kDtMaxSplit + 1] = {};
  if (dev >= 0 && dev < 64 && cache[dev][split]) return cache[dev][split];
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(split, 1, 1);
  cfg.blockDim = dim3(kDtThreads);
  cfg.dynamicSmemBytes = DtSmem<TP>::bytes();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, dense_tc_kernel<TP>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = 1;
  }
  if (dev >= 0 && dev < 64) cache[dev][split] = n;
  return n;
}

template <int TP>
int launch_dense_tc(const CUtensorMap& tw, const CUtensorMap& thi, const CUtensorMap& tlo, DenseTcArgs a,
                    int tiles, int groups, cudaStream_t s) {
  auto kern = dense_tc_kernel<TP>;
  const size_t smem = DtSmem<TP>::bytes();
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return set_error(D3_ECUDA, "dense GEMV: cannot reserve %zu bytes of shared memory", smem);
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  // K ranges per tile (a power of two up to 8): enough CTAs for about one
  // wave of SMs, in clusters that can all be resident at once, and at most
  // kDtMaxKbPerCta K blocks per CTA
  const int clusters = tiles * groups;
  const int cap = sm_count() / clusters;
  int need = 1;  // smallest split that keeps a CTA's K range within the limit
  while (need * kDtMaxKbPerCta < a.KB) need *= 2;
  if (need > kDtMaxSplit)
    return set_error(D3_EUNSUPPORTED, "dense GEMV: K=%d above %d", a.KB * 128,
                     kDtMaxSplit * kDtMaxKbPerCta * 128);
  int split = need;
  while (split * 2 <= cap && split * 2 <= kDtMaxSplit && split * 2 <= a.KB) split *= 2;
  while (split > need && dense_max_clusters<TP>(dev, split) < clusters) split /= 2;
  a.split = split;
  a.kb_per_split = (a.KB + split - 1) / split;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles * split, groups);
  cfg.blockDim = dim3(kDtThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  int na = 1;
  if (split > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = split;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaLaunchKernelEx(&cfg, kern, tw, thi, tlo, a);
  return check_launch("dense tcgen05 GEMV");
}
}  // namespace

extern "C" int d3_fp8_gemv_workspace_size(int T, int N, int K, size_t* bytes) {
  D3_REQUIRE(bytes != nullptr && T >= 0 && N > 0 && K > 0 && K % 128 == 0,
             "fp8_gemv_workspace_size: bad arguments T=%d N=%d K=%d", T, N, K);
  *bytes = carve_dense(nullptr, T, K).bytes;
  return D3_OK;
}

static int fp8_gemv_impl(const void* x, int64_t x_stride, const void* gate, int64_t gate_stride,
                         int mode, const uint8_t* wq, const float* s, int T, int N, int K, void* y,
                         int64_t y_stride, void* workspace, size_t workspace_bytes, int32_t* status,
                         d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && N > 0 && K > 0 && K % 128 == 0, "fp8_gemv: bad shape T=%d N=%d K=%d", T, N, K);
  D3_REQUIRE(x_stride >= K && x_stride % 8 == 0, "fp8_gemv: x row stride must be >= K and a multiple of 8");
  D3_REQUIRE(y_stride >= N, "fp8_gemv: y row stride must be >= N");
  D3_REQUIRE(x && wq && s && y && aligned(x, 16) && aligned(wq, 16), "fp8_gemv: null or misaligned pointer");
  D3_REQUIRE(workspace && aligned(workspace, 256), "fp8_gemv: workspace must be 256-byte aligned");
  const DenseBuffers need = carve_dense(nullptr, T, K);
  if (workspace_bytes < need.bytes)
    return set_error(D3_EWORKSPACE, "fp8_gemv: workspace %zu bytes < %zu", workspace_bytes, need.bytes);
  if (T == 0) return D3_OK;
  const DenseBuffers b = carve_dense(workspace, T, K);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // activations (gated first, for d3_fp8_gated_gemv) split into hi + lo / 16
  launch_dense_split(x, x_stride, T, K, gate, gate_stride, mode, b.hi, b.lo, b.sc, st);
  int rc = check_launch("dense_split");
  if (rc) return rc;
  const int tiles = (N + 127) / 128;
  const int groups = (T + kDtTokens - 1) / kDtTokens;
  const int TP = T > 32 ? 64 : (T > 16 ? 32 : 16);
  CUtensorMap tw, thi, tlo;
  if ((rc = encode_tmap_2d(&tw, wq, 1, K, N, K, 128, 128))) return rc;
  if ((rc = encode_tmap_2d(&thi, b.hi, 1, K, T, K, 128, TP))) return rc;
  if ((rc = encode_tmap_2d(&tlo, b.lo, 1, K, T, K, 128, TP))) return rc;
  DenseTcArgs a{};
  a.wscale = s;
  a.xscale = b.sc;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.y_ld = y_stride;
  a.T = T;
  a.N = N;
  a.KB = K / 128;
  a.vec_store = (y_stride % 4 == 0 && aligned(y, 8)) ? 1 : 0;
  a.status = status ? status : b.status;
  switch (TP) {
    case 16: return launch_dense_tc<16>(tw, thi, tlo, a, tiles, groups, st);
    case 32: return launch_dense_tc<32>(tw, thi, tlo, a, tiles, groups, st);
    default: return launch_dense_tc<64>(tw, thi, tlo, a, tiles, groups, st);
  }
}

extern "C" int d3_fp8_gemv(const void* x, int64_t x_stride, const uint8_t* wq, const float* s,
                           int T, int N, int K, void* y, int64_t y_stride, void* workspace,
                           size_t workspace_bytes, int32_t* status, d3_stream_t stream) {
  return fp8_gemv_impl(x, x_stride, nullptr, 0, GATE_NONE, wq, s, T, N, K, y, y_stride, workspace,
                       workspace_bytes, status, stream);
}

extern "C" int d3_fp8_gated_gemv(const void* x, int64_t x_stride, const void* gate,
                                 int64_t gate_stride, int mode, const uint8_t* wq, const float* s,
                                 int T, int N, int K, void* y, int64_t y_stride, void* workspace,
                                 size_t workspace_bytes, int32_t* status, d3_stream_t stream) {
  D3_REQUIRE(mode == D3_GATE_SWIGLU || mode == D3_GATE_SIGMOID,
             "fp8_gated_gemv: mode must be D3_GATE_SWIGLU or D3_GATE_SIGMOID");
  D3_REQUIRE(gate && aligned(gate, 16) && gate_stride >= K && gate_stride % 8 == 0,
             "fp8_gated_gemv: null or misaligned gate, or gate row stride < K / not a multiple of 8");
  return fp8_gemv_impl(x, x_stride, gate, gate_stride, mode == D3_GATE_SWIGLU ? GATE_SWIGLU : GATE_SIGMOID,
                       wq, s, T, N, K, y, y_stride, workspace, workspace_bytes, status, stream);
}

// --------------------------------------------------------------------------
// Weight-only FP8 GEMV for callers that cannot allocate device memory.
//
// d3_fp8_gemv needs a caller-provided workspace (the f16 copy of x, its
// per-group scales and the split-K partial sums). Some callers have no way to
// provide one: a host runtime that gives a plugin only its input and output
// buffers and a stream, and does not let it grow device memory while a request
// is in flight, because an allocation there can synchronise the device or fail
// under memory pressure. This variant keeps that scratch in a fixed array in
// the library's own device memory instead. Each GPU that loads the library
// holds the array (D3_GEMV_NOALLOC_SCRATCH_BYTES) until the process exits.
// Its address is looked up once per device (cudaGetSymbolAddress, with that
// device current) on the first call; that first call should therefore come
// before any stream capture. All calls share the array: the split-K counters
// are cleared at the start of each call, and two calls whose work overlaps on
// the GPU (different streams, or different host threads) race on it.
namespace {
constexpr int kNoAllocSplit = 4;
constexpr size_t kNoAllocXhBytes =
    static_cast<size_t>(D3_GEMV_NOALLOC_MAX_T) * D3_GEMV_NOALLOC_MAX_K * 2;
constexpr size_t kNoAllocInvBytes =
    static_cast<size_t>(D3_GEMV_NOALLOC_MAX_T) * (D3_GEMV_NOALLOC_MAX_K / 128) * 4;
constexpr size_t kNoAllocPartialBytes = static_cast<size_t>(kNoAllocSplit) *
                                        D3_GEMV_NOALLOC_MAX_T * D3_GEMV_NOALLOC_MAX_N * 4;
constexpr size_t kNoAllocCounterBytes = (D3_GEMV_NOALLOC_MAX_N / 128) * 4;
// layout: [status 256][xh][inv][partials][counters], each 256-byte aligned
constexpr size_t kNoAllocXhOff = 256;
constexpr size_t kNoAllocInvOff = kNoAllocXhOff + kNoAllocXhBytes;
constexpr size_t kNoAllocPartOff = kNoAllocInvOff + ((kNoAllocInvBytes + 255) / 256) * 256;
constexpr size_t kNoAllocCntOff = kNoAllocPartOff + kNoAllocPartialBytes;
static_assert(kNoAllocCntOff + kNoAllocCounterBytes <= D3_GEMV_NOALLOC_SCRATCH_BYTES,
              "scratch array too small for the stated limits");

static __device__ __align__(256) uint8_t g_gemv_noalloc_scratch[D3_GEMV_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mutex;
void* g_noalloc_addr[64] = {nullptr};

int noalloc_scratch(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(D3_ECUDA, "fp8_gemv_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(D3_ECUDA, "fp8_gemv_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    g_noalloc_addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_noalloc_addr[dev]);
  return D3_OK;
}
}  // namespace

extern "C" int d3_fp8_gemv_noalloc(const void* x, int64_t x_stride, const uint8_t* wq,
                                   const float* s, int T, int N, int K, void* y,
                                   int64_t y_stride, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && N > 0 && K > 0 && K % 128 == 0, "fp8_gemv_noalloc: bad shape T=%d N=%d K=%d", T, N, K);
  D3_REQUIRE(T <= D3_GEMV_NOALLOC_MAX_T && N <= D3_GEMV_NOALLOC_MAX_N && K <= D3_GEMV_NOALLOC_MAX_K,
             "fp8_gemv_noalloc: T=%d N=%d K=%d exceeds the fixed scratch limits T<=%d N<=%d K<=%d; "
             "use d3_fp8_gemv with a workspace", T, N, K, D3_GEMV_NOALLOC_MAX_T,
             D3_GEMV_NOALLOC_MAX_N, D3_GEMV_NOALLOC_MAX_K);
  D3_REQUIRE(x_stride >= K && x_stride % 8 == 0, "fp8_gemv_noalloc: x row stride must be >= K and a multiple of 8");
  D3_REQUIRE(y_stride >= N, "fp8_gemv_noalloc: y row stride must be >= N");
  D3_REQUIRE(x && wq && s && y && aligned(x, 16) && aligned(wq, 16), "fp8_gemv_noalloc: null or misaligned pointer");
  uint8_t* base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  if (T == 0) return D3_OK;
  int32_t* status = reinterpret_cast<int32_t*>(base);
  __half* xh = reinterpret_cast<__half*>(base + kNoAllocXhOff);
  float* inv = reinterpret_cast<float*>(base + kNoAllocInvOff);
  float* partials = reinterpret_cast<float*>(base + kNoAllocPartOff);
  int32_t* counters = reinterpret_cast<int32_t*>(base + kNoAllocCntOff);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int tiles = (N + 127) / 128, KB = K / 128;
  int split = sm_count() / tiles;
  split = split < 1 ? 1 : (split > kNoAllocSplit ? kNoAllocSplit : split);
  split = split > KB ? KB : split;
  const int kbps = (KB + split - 1) / split;
  split = (KB + kbps - 1) / kbps;
  // the split-K counters left by the previous call are cleared by the
  // activation prep kernel (the status word only records timeouts)
  launch_dense_act_prep(x, x_stride, T, K, xh, inv, st, counters,
                        static_cast<int>(kNoAllocCounterBytes / sizeof(int32_t)));
  if ((rc = check_launch("dense_act_prep"))) return rc;
  CUtensorMap tw, ta;
  if ((rc = encode_tmap_2d(&tw, wq, 1, K, N, K, 128, 128))) return rc;
  if ((rc = encode_tmap_2d(&ta, xh, 2, K, T, static_cast<uint64_t>(K) * 2, 64, 16))) return rc;
  EngineArgs a{};
  a.num_groups = 1;
  a.dense_count = T;
  a.tiles = tiles;
  a.KB = KB;
  a.ksplit = split;
  a.kb_per_split = kbps;
  a.partials = partials;
  a.tile_counters = counters;
  a.wscale = s;
  a.wscale_sh = s;
  a.act_scale = inv;
  a.out_bf16 = static_cast<__nv_bfloat16*>(y);
  a.out_ld = static_cast<int>(y_stride);
  a.out_cols = N;
  a.status = status;
  const int items = tiles * split;
  const int sms = sm_count();
  const int grid = items < sms ? items : sms;
  return launch_engine<EPI_DENSE, true, kStagesDense>(nch_for(T), tw, tw, ta, a, grid, st);
}

// The bounded waits of d3_fp8_gemv_noalloc record a timeout in the first word
// of the fixed array, and nothing else reads that word. This copies it to the
// caller (stream-ordered) and clears it, so a timeout is reported once.
extern "C" int d3_fp8_gemv_noalloc_status(int32_t* status_out, d3_stream_t stream) {
  D3_REQUIRE(status_out != nullptr, "fp8_gemv_noalloc_status: null output");
  uint8_t* base = nullptr;
  int rc = noalloc_scratch(&base);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(status_out, base, sizeof(int32_t), cudaMemcpyDefault, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(base, 0, sizeof(int32_t), st);
  if (e != cudaSuccess)
    return set_error(D3_ECUDA, "fp8_gemv_noalloc_status: %s", cudaGetErrorString(e));
  return D3_OK;
}
