// Launchers shared between translation units (not part of the public C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace d3 {

// Row maps of a mixed decode + packed-prefill layer call
// (src/drama3/mixed_model.py:193-246). MoE row t reads x row keep[t]
// (keep == nullptr: row t); keep values must lie in [0, x_rows).
struct RowGather {
  const int64_t* keep = nullptr;
  int64_t x_rows = 0;
  int32_t* status = nullptr;
};

// Reserved padding rows (src/drama3/moe_input.py:32-36): a row whose slot
// (int32 or int64) is at or above padding_start routes with row 0's logits.
// slots == nullptr: no such rows.
struct PaddingRoute {
  const void* slots = nullptr;
  int slots_i64 = 0;
  int64_t padding_start = 0;
};


// Activation quantisation into expert order: token t is quantised once (1x128
// groups, e4m3 + f32 scale) and written to rows inv_rows[t*k + j] (negative =
// skipped) and, with with_shared, to row P + t. Rows not named are untouched.
// The first CTA also zeroes zero[0..nzero) (the engines' work counters).
void launch_quant_scatter(const void* x, int64_t x_stride, int T, int H, int k,
                          const int32_t* inv_rows, int P, int with_shared, uint8_t* xq, float* sx,
                          cudaStream_t s, int32_t* zero = nullptr, int nzero = 0,
                          const RowGather& rg = RowGather{});

// The bucketing (block_m = 1: counts, starts, total, inverse rows, active list)
// fused with launch_quant_scatter, one CTA per token, for fewer than
// kFusedPermuteMaxPairs pairs and E <= kFusedPermuteMaxExperts. Same outputs
// as launch_permute followed by launch_quant_scatter.
constexpr int kFusedPermuteMaxPairs = 2048;
constexpr int kFusedPermuteMaxExperts = 1024;
void launch_permute_quant(const void* x, int64_t x_stride, int T, int H, int k, const int64_t* ids,
                          int E, int with_shared, uint8_t* xq, float* sx, int32_t* counts,
                          int32_t* starts, int32_t* total, int32_t* inv_rows, int32_t* active,
                          int32_t* n_active, cudaStream_t s, int32_t* zero = nullptr, int nzero = 0,
                          const RowGather& rg = RowGather{});

// Already-quantised activations (q e4m3 [T,H], scales [H/128,T] when
// transposed, else [T,H/128]) copied into expert order like
// launch_quant_scatter (routed rows only).
void launch_prequant_scatter(const uint8_t* q, int64_t q_stride, const float* qs, int transposed,
                             int T, int H, int k, const int32_t* inv_rows, uint8_t* xq, float* sx,
                             cudaStream_t s, int32_t* zero, int nzero);

// Weight-only GEMV activation prep: x bf16 [T,K] -> f16 [T,K] scaled by a
// power of two per 1x128 group (exact), inv f32 [T,K/128] = the inverse factor.
// The first CTA also zeroes zero[0..nzero) (split-K tile counters, status).
// With a gate (bf16 [T,K], row stride gate_stride) x is first replaced by
// bf16(x * bf16(act(gate))), act = silu (GATE_SWIGLU) or sigmoid (GATE_SIGMOID).
enum GateMode { GATE_NONE = 0, GATE_SWIGLU = 1, GATE_SIGMOID = 2 };
void launch_dense_act_prep(const void* x, int64_t x_stride, int T, int K, __half* xh, float* inv,
                           cudaStream_t s, int32_t* zero = nullptr, int nzero = 0,
                           const void* gate = nullptr, int64_t gate_stride = 0,
                           int mode = GATE_NONE);

// Activations of the tcgen05 dense GEMV split into two E4M3 terms per 1x128
// group: x * 2^s = hi + lo / 16 (exact for every element within 2^13 of the
// group maximum), hi / lo e4m3 [T,K] (row stride K), sc f32 [T,K/128] = 2^-s.
// With a gate (GATE_SWIGLU / GATE_SIGMOID) x is first bf16(x * act(gate)).
void launch_dense_split(const void* x, int64_t x_stride, int T, int K, const void* gate,
                        int64_t gate_stride, int mode, uint8_t* hi, uint8_t* lo, float* sc,
                        cudaStream_t s);

// Final combine of the expert rows (see d3_moe_experts / d3_moe_layer).
//   routed[t] = bf16(sum_r w[t,r] * d[inv_rows[t*k+r]])
//   shared[t] = bf16(d[P+t])                                   (when with_shared)
//   out[t]    = routed + bf16(shared * bf16(sigmoid(gate[t]))) (when gate != null)
// rows_bf16: d holds bf16 rows (the tcgen05 path) instead of fp32.
void launch_combine_rows(const float* d, int H, const int32_t* inv_rows, const void* weights,
                         int T, int k, int with_shared, const void* gate, int64_t gate_stride,
                         void* routed_out, void* shared_out, void* out, cudaStream_t s,
                         bool rows_bf16 = false);

// Fused layer exit: routed/shared rows combined as in
// d3_combine_experts_add_norm, residual updated in place, out = RMSNorm. With
// `inverse` (int64 [T_out]) residual row t takes MoE row inverse[t].
int launch_combine_rows_add_norm(const float* d, int W, const int32_t* inv_rows,
                                 const void* weights, int T, int k, const void* gate,
                                 int64_t gate_stride, void* residual, const void* norm_w, float eps,
                                 void* out, cudaStream_t s, const int64_t* inverse = nullptr,
                                 int T_out = 0, int32_t* status = nullptr, bool rows_bf16 = false);

// Router projection. Below 256 tokens CUDA-core kernels with one fixed fp32
// summation order (the oracle's); from 256 tokens a tcgen05 bf16 GEMM (fp32
// accumulation in the tensor core's own order, like the reference's F.linear).
// Rows named by a keep map are first copied into `gather_scratch` (bf16
// [T, H], nullable: without it they stay on the CUDA-core kernels), so a
// gathered call and a call on the materialised rows give the same logits.
// `status` (nullable) receives a bounded-wait timeout or a bad keep row.
void launch_router_logits(const void* x, int64_t x_stride, const void* w, const float* bias,
                          int nbias, int R, int H, int T, void* logits, int64_t logits_stride,
                          cudaStream_t s, const RowGather& rg = RowGather{},
                          int32_t* status = nullptr, void* gather_scratch = nullptr);

void launch_route_topk(const void* logits, int logits_dtype, int64_t stride, int T, int E, int k,
                       const float* bias, int64_t* ids, void* weights, int weights_dtype,
                       cudaStream_t s, const PaddingRoute& pr = PaddingRoute{});

// route_topk followed by permute (two launches).
int launch_route_permute(const void* logits, int logits_dtype, int64_t stride, int T, int E,
                         int k, const float* bias, int64_t* ids, void* weights, int weights_dtype,
                         int block_m, int32_t* counts, int32_t* starts, int32_t* total,
                         int32_t* sorted_ids, int32_t* expert_ids, int64_t max_rows,
                         int32_t* inv_rows, int32_t* active, int32_t* n_active, cudaStream_t s,
                         int32_t* scratch = nullptr, const PaddingRoute& pr = PaddingRoute{});

// Stable token->expert bucketing. With `scratch` (permute_scratch_ints(E)
// ints) and T*k >= 8192 pairs it runs as three multi-CTA kernels; otherwise as
// one 1024-thread CTA. Both give identical outputs.
int launch_permute(const int64_t* ids, int T, int k, int E, int block_m, int32_t* counts,
                   int32_t* starts, int32_t* total, int32_t* sorted_ids, int32_t* expert_ids,
                   int64_t max_rows, int32_t* inv_rows, int32_t* active, int32_t* n_active,
                   cudaStream_t s, int32_t* scratch = nullptr);
size_t permute_scratch_ints(int E);

}  // namespace d3
