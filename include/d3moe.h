/*
 * d3moe.h — C ABI of the B200 (sm_100a) FP8 mixture-of-experts hot path.
 *
 * Every entry point is stream-ordered (it only enqueues work on `stream`),
 * performs no device or pinned allocation and never synchronises the device.
 * That makes every call capturable into a CUDA graph, the way the reference
 * runtime captures its decode step (reference: src/drama3/engine.py:84-92).
 * Process-wide state is small and named: a per-thread error string, the
 * prefill token threshold (d3_set_prefill_min_tokens), the host-side record
 * of workspaces d3_moe_gate_up_silu filled, per-device kernel attributes set
 * on first use, the fixed scratch of d3_fp8_gemv_noalloc, and the per-thread
 * profiling hook d3_set_stage_events (off unless a caller sets it).
 *
 * Return value: D3_OK (0) or a negative D3_E* code. Argument errors are found
 * on the host before anything is launched; d3_last_error_string() explains the
 * last failure of the calling thread.
 *
 * Tensors are raw device pointers, row-major, with explicit row strides in
 * elements where the reference accepts strided inputs. Number formats:
 *   bf16 — IEEE bfloat16 (uint16 storage)
 *   e4m3 — OCP FP8 E4M3 "fn" (uint8 storage, max 448, no infinities)
 *   f32  — IEEE binary32
 * Expert weights keep the reference checkpoint layout (src/drama3/kernels.py:
 * 298-299, 313-318; src/drama3/model.py:195-198):
 *   w13 e4m3 [E, 2I, H], rows [gate(0:I) | up(I:2I)];  s13 f32 [E, 2I/128, H/128]
 *   w2  e4m3 [E, H, I];                                  s2  f32 [E, H/128, I/128]
 * H and I must be multiples of 128.
 */
#ifndef D3MOE_H_
#define D3MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* d3_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define D3_API __attribute__((visibility("default")))
#else
#define D3_API
#endif

#define D3_OK 0
#define D3_EINVAL (-1)       /* bad shape, stride, alignment or pointer */
#define D3_ECUDA (-2)        /* a CUDA runtime / driver call failed */
#define D3_EWORKSPACE (-3)   /* workspace smaller than the *_workspace_size answer */
#define D3_EUNSUPPORTED (-4) /* a size beyond what this build supports */

/* dtype tags used where the reference accepts more than one */
#define D3_DTYPE_BF16 0
#define D3_DTYPE_F32 1

/* Device status word values written by kernels that wait on barriers. */
#define D3_STATUS_OK 0
#define D3_STATUS_WAIT_TIMEOUT 1
#define D3_STATUS_BAD_ROW 2 /* a row map named a row outside its tensor; row 0 was read instead */

D3_API int d3_version(void);
D3_API const char* d3_last_error_string(void);

/* ------------------------------------------------------------- (a3) quant --
 * Activation FP8 quantisation per 1x128 group: scale = max(amax,1e-10)/448,
 * q = e4m3(clamp(x/scale, -448, 448)) with IEEE division and round-to-nearest-
 * even. x bf16 [T,H] (row stride x_stride >= H, multiple of 8).
 * scales_transposed = 0: scales f32 [T, H/128] (Fish quantize_groups layout,
 *   used by src/drama3/kernels.py:297 and model.py:554);
 * scales_transposed = 1: scales f32 [H/128, T] (FlashInfer layout written by
 *   src/drama3/moe_input.py:28-30).
 * Replaces Fish `quantize_groups(quant_kernel, x, H)` (kernels.py:332). */
D3_API int d3_quant_act_fp8(const void* x, int64_t x_stride, int T, int H, uint8_t* q, float* scales,
                     int scales_transposed, d3_stream_t stream);

/* Fused activation quant + router-logit conversion.
 * Replaces prepare_moe_input (src/drama3/moe_input.py:40-79; kernel :8-37).
 * q e4m3 [T,H]; scales_t f32 [H/128, T]; logits f32 [T,E] from router bf16
 * [T,E] (stride router_stride). row_slots (int32 or int64 [T], may be NULL)
 * with padding_start > 0: rows whose slot >= padding_start take row 0's
 * logits (moe_input.py:32-36). */
D3_API int d3_prepare_moe_input(const void* x, int64_t x_stride, const void* router,
                         int64_t router_stride, int T, int H, int E, const void* row_slots,
                         int row_slots_int64, int64_t padding_start, uint8_t* q, float* scales_t,
                         float* logits, d3_stream_t stream);

/* --------------------------------------------------- (a1) router projection --
 * logits bf16 [T, R] = bf16(x bf16 [T,H] . W bf16 [R,H]^T + bias[r]) with
 * fp32 accumulation; bias f32 [nbias] (nullable) is added to the first nbias
 * columns before the rounding. Replaces linear(x, layer.gate.weight) / the
 * packed router slice (src/drama3/model.py:496-504, kernels.py:274-287).
 * R = E (+1 for the shared-expert gate row). Below 256 tokens the sum runs
 * in one fixed fp32 order (restated by oracle.moe_oracle.router_logits); from
 * 256 tokens, with H a multiple of 64, it is a tcgen05 bf16 GEMM whose fp32
 * accumulation order is the tensor core's own (as in the reference's bf16
 * F.linear), deterministic from call to call. d3_moe_layer and its variants
 * use the same kernels, so this call reproduces a layer's logits bit for bit
 * at the same T. */
D3_API int d3_router_logits(const void* x, int64_t x_stride, const void* w, const float* bias,
                            int nbias, int R, int H, int T, void* logits, int64_t logits_stride,
                            d3_stream_t stream);


/* ------------------------------------------------------------ (a2) route --
 * fp32 softmax over E logits, top-k by (logit, lower index first), weights
 * renormalised over the k picks. logits bf16 or f32 [T,E] with row stride;
 * bias f32 [E] (may be NULL) is added to the fp32 logits first.
 * ids int64 [T,k] (descending probability); weights [T,k] in weights_dtype.
 * Replaces route / route_kernel (src/drama3/kernels.py:360-383) and the torch
 * prefill routing (src/drama3/model.py:526-528). E <= 1024, k <= 32. */
D3_API int d3_route_topk(const void* logits, int logits_dtype, int64_t stride, int T, int E, int k,
                  const float* bias, int64_t* ids, void* weights, int weights_dtype,
                  d3_stream_t stream);

/* d3_route_topk with reserved padding rows: with row_slots (int32, or int64
 * when row_slots_int64 = 1) and padding_start > 0, a row whose slot is >=
 * padding_start routes with row 0's logits; its ids and weights still go to
 * its own row (src/drama3/moe_input.py:32-36, model.py:546-553). */
D3_API int d3_route_topk_rows(const void* logits, int logits_dtype, int64_t stride, int T, int E,
                              int k, const float* bias, const void* row_slots, int row_slots_int64,
                              int64_t padding_start, int64_t* ids, void* weights, int weights_dtype,
                              d3_stream_t stream);

/* ---------------------------------------------------------- (a4) permute --
 * Token->expert bucketing with the reference's device layout
 * (src/drama3/kernels.py:658-699, buffers :711-731). Pairs p = t*k + r.
 * counts[E]; starts[E] (each expert's segment padded to block_m); total[1];
 * sorted_ids[max_rows]: pair ids ascending within each expert, padding slots
 * hold the sentinel P = T*k, slots at and after `total` are also set to P;
 * expert_ids[max_rows/block_m]: owning expert per block_m tile, -1 after total.
 * Optional outputs (NULL to skip): inv_rows[P] = slot of each pair;
 * active[E] = experts with count > 0 in ascending order, n_active[1].
 * max_rows must be >= cdiv(P + min(P,E)*(block_m-1), block_m)*block_m. */
D3_API int d3_moe_permute(const int64_t* ids, int T, int k, int E, int block_m, int32_t* counts,
                   int32_t* starts, int32_t* total, int32_t* sorted_ids, int32_t* expert_ids,
                   int64_t max_rows, int32_t* inv_rows, int32_t* active, int32_t* n_active,
                   d3_stream_t stream);

/* Same outputs as d3_moe_permute, computed by three multi-CTA kernels (per-chunk
 * histogram, one-CTA scan, per-chunk stable scatter) when T*k >= 8192; the
 * caller provides d3_moe_permute_scratch_size(E) bytes of device scratch.
 * Prefill sizes: the reference's multi-program expert_counts / offsets /
 * scatter kernels (src/drama3/kernels.py:658-699) split the same way. */
D3_API int d3_moe_permute_scratch_size(int E, size_t* bytes);
D3_API int d3_moe_permute_chunked(const int64_t* ids, int T, int k, int E, int block_m,
                           int32_t* counts, int32_t* starts, int32_t* total, int32_t* sorted_ids,
                           int32_t* expert_ids, int64_t max_rows, int32_t* inv_rows,
                           int32_t* active, int32_t* n_active, int32_t* scratch,
                           size_t scratch_bytes, d3_stream_t stream);

/* ----------------------------------------------------- (a6) SiLU * mul --
 * out bf16 [rows, W] = bf16(bf16(silu(gate)) * up), gate = in[:, :W],
 * up = in[:, W:2W]. Replaces silu_mul (src/drama3/kernels.py:386-402). */
D3_API int d3_silu_mul(const void* in, int64_t in_stride, int rows, int W, void* out,
                d3_stream_t stream);

/* SiLU*mul fused with FP8 requantisation per 1x128 group:
 * a = bf16(silu(gate)) * up (fp32), q e4m3 [rows,W], scales f32 [rows,W/128].
 * Replaces Fish quantize_groups(silu_mul_quant_kernel, gate_up, W)
 * (src/drama3/kernels.py:344, :748). */
D3_API int d3_silu_mul_quant(const void* in, int64_t in_stride, int rows, int W, uint8_t* q,
                      float* scales, d3_stream_t stream);

/* -------------------------------------------------------- (a9) combine --
 * out bf16 [T,H] = routed + bf16(shared * bf16(sigmoid(gate))), gate bf16
 * [T,1] with row stride gate_stride. Replaces combine_experts
 * (src/drama3/kernels.py:427-445). */
D3_API int d3_combine_experts(const void* routed, const void* shared, const void* gate,
                       int64_t gate_stride, int T, int H, void* out, d3_stream_t stream);

/* ------------------------------------------ (f1) residual + RMSNorm exit --
 * residual bf16 [T,W] (updated in place) <- bf16(x + residual) in fp32;
 * out bf16 [T,W] = bf16(residual * rsqrt(mean(residual^2) + eps) * (1 + weight)),
 * weight bf16 [W]. W a multiple of 8, at most 8192.
 * Replaces add_norm (src/drama3/kernels.py:405-423). */
D3_API int d3_add_norm(const void* x, void* residual, const void* weight, float eps, int T, int W,
                void* out, d3_stream_t stream);

/* Same exit with the expert combine in front of it:
 *   combined = fma.rn.bf16(shared, bf16(sigmoid(gate)), routed)   (one rounding)
 *   residual <- bf16(combined + residual), out = RMSNorm as above.
 * With inverse (int32 [T], may be NULL) the routed/shared/gate rows of row t
 * are taken from row inverse[t]. Replaces combine_experts_add_norm and
 * combine_experts_add_norm_inverse (src/drama3/kernels.py:448-556). */
D3_API int d3_combine_experts_add_norm(const void* routed, const void* shared, const void* gate,
                                int64_t gate_stride, const int32_t* inverse, int T, int W,
                                void* residual, const void* weight, float eps, void* out,
                                d3_stream_t stream);

/* ------------------------------------------------ (a10) dense FP8 GEMV --
 * 128x128 block weight quantisation: scale = max(amax,1e-8)/448 per block,
 * q = e4m3(w/scale). w bf16 [N,K] (K multiple of 128); q e4m3 [Npad,K],
 * scales f32 [Npad/128, K/128], Npad = cdiv(N,128)*128 (padding rows are 0).
 * Replaces experimental_fp8._quantize / register (experimental_fp8.py:10-53). */
D3_API int d3_fp8_quantize_weight(const void* w, int N, int K, uint8_t* q, float* scales,
                           d3_stream_t stream);

/* y bf16 [T,N] = x bf16 [T,K] . dequant(Wq,S)^T with fp32 accumulation and
 * bf16 activations (weight-only FP8, the arithmetic of experimental_fp8._gemv,
 * experimental_fp8.py:21-29, for every T). Wq e4m3 [>=N, K], S f32
 * [cdiv(N,128), K/128]. Needs workspace of d3_fp8_gemv_workspace_size bytes.
 * Small N is split along K over several CTAs; the fp32 partial sums are added
 * in a fixed split order, so results are deterministic.
 * status (device int32, may be NULL) receives D3_STATUS_*. */
D3_API int d3_fp8_gemv_workspace_size(int T, int N, int K, size_t* bytes);
D3_API int d3_fp8_gemv(const void* x, int64_t x_stride, const uint8_t* wq, const float* s, int T, int N,
                int K, void* y, int64_t y_stride, void* workspace, size_t workspace_bytes,
                int32_t* status, d3_stream_t stream);

/* Gated projection (replaces gated_gemv, src/drama3/fused_projection.py:9-60,
 * with FP8 weights): x is first replaced by bf16(x * a), a = bf16(silu(gate))
 * (D3_GATE_SWIGLU) or bf16(sigmoid(gate)) (D3_GATE_SIGMOID), gate bf16 [T,K]
 * with row stride gate_stride; then y = d3_fp8_gemv of that. Any T (the
 * reference takes one row). Workspace: d3_fp8_gemv_workspace_size. */
#define D3_GATE_SWIGLU 1
#define D3_GATE_SIGMOID 2
D3_API int d3_fp8_gated_gemv(const void* x, int64_t x_stride, const void* gate, int64_t gate_stride,
                             int mode, const uint8_t* wq, const float* s, int T, int N, int K, void* y,
                             int64_t y_stride, void* workspace, size_t workspace_bytes,
                             int32_t* status, d3_stream_t stream);

/* The same weight-only FP8 GEMV for callers that cannot allocate device
 * memory, and so cannot pass a workspace: for example a host runtime that
 * hands a plugin only its inputs, outputs and a stream and does not let it
 * allocate while a request runs. No counterpart in the reference.
 * Scratch lives in a fixed array inside the library (D3_GEMV_NOALLOC_SCRATCH_BYTES
 * on every GPU that loads it, held until the process exits). Limits: T <= 64,
 * N <= 4096, K <= 4096; larger sizes return D3_EINVAL. Nothing is allocated.
 * The first call on a device looks up the array's device address (once per
 * device), so make that first call before any stream capture. All calls share
 * the array: calls whose GPU work overlaps (other streams or host threads)
 * race on it and must be serialised by the caller. The device address is
 * kept for the life of the process: after cudaDeviceReset (or any other end
 * of the device's primary context) the entry point must not be called again. */
#define D3_GEMV_NOALLOC_MAX_T 64
#define D3_GEMV_NOALLOC_MAX_N 4096
#define D3_GEMV_NOALLOC_MAX_K 4096
#define D3_GEMV_NOALLOC_SCRATCH_BYTES (5u << 20) /* 5 MiB */
D3_API int d3_fp8_gemv_noalloc(const void* x, int64_t x_stride, const uint8_t* wq, const float* s,
                               int T, int N, int K, void* y, int64_t y_stride,
                               d3_stream_t stream);

/* Status of the calls above. d3_fp8_gemv_noalloc has no status argument: its
 * bounded waits record D3_STATUS_WAIT_TIMEOUT in a word inside the fixed
 * array, where it stays until read. This call enqueues on `stream` a copy of
 * that word for the current device into *status_out (device memory, or host
 * memory the GPU can address: read it after the stream has synchronised) and
 * then clears the word. A result other than D3_STATUS_OK means that some
 * call since the previous read gave up a wait, and its y is not valid.
 * Allocates nothing. */
D3_API int d3_fp8_gemv_noalloc_status(int32_t* status_out, d3_stream_t stream);

/* --------------------------------------------- (a5-a8) routed experts --
 * Expert weights of one MoE layer (reference container: experts.w13_weight,
 * w13_scale_inv, w2_weight, w2_scale_inv; src/drama3/kernels.py:336-350).
 * A shared expert is described with E = 1. */
typedef struct d3_experts {
  const uint8_t* w13;
  const float* s13;
  const uint8_t* w2;
  const float* s2;
  int E;
  int I;
  int H;
  int gate_up_order; /* D3_GATE_UP (0): w13 rows [gate | up], the checkpoint order;
                        D3_UP_GATE (1): [up | gate], FlashInfer's SwiGLU order
                        (src/drama3/model.py:196-201); s13 row blocks follow w13 */
} d3_experts_t;

#define D3_GATE_UP 0
#define D3_UP_GATE 1

/* Workspace for d3_moe_experts / d3_moe_layer at T tokens, top-k. */
D3_API int d3_moe_workspace_size(int T, int k, int E, int I, int H, int has_shared, size_t* bytes);

/* Routed (and optionally shared) expert computation for given routing:
 *   routed[t] = bf16( sum_r w[t,r] * down_e(silu_mul_quant(gate_up_e(q(x_t)))) )
 * in fixed rank order r = 0..k-1 with fp32 accumulation.
 * ids int64 [T,k], weights bf16 [T,k]. routed_out bf16 [T,H].
 * If `shared` is not NULL the shared expert runs in the same launches and
 * shared_out bf16 [T,H] receives bf16(down_shared(...)).
 * Replaces small_batch_moe (src/drama3/kernels.py:325-357), native_moe
 * (kernels.py:702-779) and the routed/shared parts of moe_parts
 * (src/drama3/model.py:490-541). */
D3_API int d3_moe_experts(const void* x, int64_t x_stride, const int64_t* ids, const void* weights,
                   int T, int k, const d3_experts_t* experts, const d3_experts_t* shared,
                   void* routed_out, void* shared_out, void* workspace, size_t workspace_bytes,
                   int32_t* status, d3_stream_t stream);

/* The two stages of d3_moe_experts as separate calls, for callers that
 * schedule other work between the expert GEMMs (the reference's decode path
 * runs expert_up_kernel, then the down kernel: src/drama3/kernels.py:290-322,
 * 344-350; FlashInfer's FC1 / FC2 split in trtllm_fp8_block_scale_moe).
 * d3_moe_gate_up_silu buckets the pairs, quantises x into expert order and
 * runs gate_up + SiLU*mul + FP8 requant; the activations stay in `workspace`.
 * d3_moe_down_combine then runs the down GEMM and the fixed-order combine
 * from that workspace and writes routed_out (and shared_out with a shared
 * expert). Both calls take the same T, k, experts, shared and workspace, on
 * the same stream, with the prefill threshold unchanged in between; the pair
 * gives d3_moe_experts' outputs bit for bit. d3_moe_down_combine returns
 * D3_EINVAL for a workspace that d3_moe_gate_up_silu has not filled with the
 * same T, k, expert shapes and shared expert (a host-side record, no device
 * work). The record is best-effort: it is keyed on the workspace address and
 * the shapes, so a different allocation that lands at the same address with
 * the same shapes passes it; each successful d3_moe_down_combine consumes the
 * record, so one d3_moe_gate_up_silu call permits one d3_moe_down_combine.
 * Other use of the workspace between the two calls is the caller's to avoid. */
D3_API int d3_moe_gate_up_silu(const void* x, int64_t x_stride, const int64_t* ids, int T, int k,
                               const d3_experts_t* experts, const d3_experts_t* shared,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               d3_stream_t stream);
D3_API int d3_moe_down_combine(const void* weights, int T, int k, const d3_experts_t* experts,
                               const d3_experts_t* shared, void* routed_out, void* shared_out,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               d3_stream_t stream);

/* Routed experts over already-quantised activations, the calling convention
 * of FlashInfer's trtllm_fp8_block_scale_moe (src/drama3/model.py:544-580):
 * q e4m3 [T,H] (row stride q_stride bytes, a multiple of 16), q_scales f32
 * [H/128, T] (scales_transposed = 1, the layout prepare_moe_input writes) or
 * [T, H/128]. ids int64 [T,k] (ids outside [0,E) contribute nothing), weights
 * bf16 [T,k]; routed_out bf16 [T,H] as d3_moe_experts. experts may use either
 * gate_up_order. Workspace: d3_moe_workspace_size(T, k, E, I, H, 0). */
D3_API int d3_moe_experts_fp8(const uint8_t* q, int64_t q_stride, const float* q_scales,
                              int scales_transposed, const int64_t* ids, const void* weights, int T,
                              int k, const d3_experts_t* experts, void* routed_out, void* workspace,
                              size_t workspace_bytes, int32_t* status, d3_stream_t stream);

/* One whole MoE layer: router projection over [E+1, H] bf16 (rows 0..E-1 the
 * router, row E the shared-expert gate; src/drama3/model.py:236-245), top-k
 * routing with optional per-expert bias, routed + shared experts, and
 *   out = routed + bf16(shared * bf16(sigmoid(gate)))
 * Replaces DramaModel.moe (src/drama3/model.py:485-488). Optional debug
 * outputs (NULL to skip): ids int64 [T,k], weights bf16 [T,k]. */
D3_API int d3_moe_layer(const void* x, int64_t x_stride, const void* router_w, const float* router_bias,
                 int T, int k, const d3_experts_t* experts, const d3_experts_t* shared, void* out,
                 int64_t* ids_out, void* weights_out, void* workspace, size_t workspace_bytes,
                 int32_t* status, d3_stream_t stream);

/* d3_moe_layer with the layer exit fused into its final kernel: the combine
 * of d3_combine_experts_add_norm (bf16 fma of shared and gate onto routed),
 * residual bf16 [T,H] updated in place, out = RMSNorm(residual) * (1 + norm_weight).
 * The routed/shared bf16 tensors of moe_parts + combine_experts_add_norm
 * (src/drama3/model.py:506-517, kernels.py:448-499) never reach HBM. */
D3_API int d3_moe_layer_add_norm(const void* x, int64_t x_stride, const void* router_w,
                          const float* router_bias, int T, int k, const d3_experts_t* experts,
                          const d3_experts_t* shared, void* residual, const void* norm_weight,
                          float eps, void* out, int64_t* ids_out, void* weights_out,
                          void* workspace, size_t workspace_bytes, int32_t* status,
                          d3_stream_t stream);

/* Row maps of the mixed decode + packed-prefill MoE call (decode rows first,
 * then packed prompt rows and their padding; src/drama3/mixed_model.py:193-246):
 *   keep        int64 [T]: MoE row t reads x row keep[t] (NULL: row t); x has
 *               x_rows rows. Replaces normalized.index_select(0, keep).
 *   inverse     int64 [T_out]: residual/output row t takes MoE row inverse[t]
 *               (NULL: row t, T_out = T). Replaces the inverse gather of
 *               combine_experts_add_norm_inverse (src/drama3/kernels.py:502-556);
 *               needs the fused exit (residual != NULL).
 *   row_slots   int32 or int64 [T] (row_slots_int64 = 1 for int64), with
 *               padding_start > 0: MoE rows whose slot >= padding_start route
 *               with row 0's logits (src/drama3/moe_input.py:32-36).
 * A keep or inverse value outside its tensor sets D3_STATUS_BAD_ROW in the
 * status word and reads row 0 in its place. */
typedef struct d3_rows {
  const int64_t* keep;
  int64_t x_rows;
  const int64_t* inverse;
  int T_out;
  const void* row_slots;
  int row_slots_int64;
  int64_t padding_start;
} d3_rows_t;

/* d3_moe_layer (residual == NULL: out bf16 [T,H]) or d3_moe_layer_add_norm
 * (residual, out bf16 [T_out,H]) over the row maps `rows` (may be NULL). The
 * workspace is sized for the T MoE rows. */
D3_API int d3_moe_layer_rows(const void* x, int64_t x_stride, const void* router_w,
                             const float* router_bias, int T, int k, const d3_experts_t* experts,
                             const d3_experts_t* shared, const d3_rows_t* rows, void* residual,
                             const void* norm_weight, float eps, void* out, int64_t* ids_out,
                             void* weights_out, void* workspace, size_t workspace_bytes,
                             int32_t* status, d3_stream_t stream);

/* ---------------------------------------------- (e) expert parallelism --
 * The reference runs on one GPU and has no expert parallelism; these entry
 * points are the device-side steps of the EP layer in d3moe/ep.py (dispatch
 * and combine over NCCL all-to-all). Experts are owned contiguously: rank
 * r holds experts [r*experts_per_rank, (r+1)*experts_per_rank).
 *
 * d3_ep_plan_rows: one dispatch row per (token, owning rank). Rank d needs
 * token t when it owns at least one of t's k experts (ids outside
 * [0, experts_per_rank*ranks) are ignored). Rows are ordered by destination
 * rank, then token: send_counts int32 [ranks] = rows for each rank, and
 * slot int32 [T, ranks] = the row's index in the send buffer, -1 where d needs
 * no row of t. The same slot map, flattened, is the inv_rows argument of
 * d3_combine_pairs (k = ranks, weight 1) once the partial rows are back in
 * the send order. ranks <= 32. */
D3_API int d3_ep_plan_rows(const int64_t* ids, int T, int k, int experts_per_rank, int ranks,
                           int32_t* send_counts, int32_t* slot, d3_stream_t stream);

/* Fixed-capacity dispatch (no host-visible counts): for each rank d and token
 * t, meta_ids int64 [ranks, T, k] = ids[t][j] - d*experts_per_rank where rank d
 * owns that expert, else -1; meta_w bf16 [ranks, T, k] = the routing weight
 * there, else 0. */
D3_API int d3_ep_dispatch_meta(const int64_t* ids, const void* weights, int T, int k,
                               int experts_per_rank, int ranks, int64_t* meta_ids, void* meta_w,
                               d3_stream_t stream);

/* Packed FP8 dispatch (one buffer, one all_to_all): each token is quantised
 * once (1x128 E4M3 groups, the bytes and scales the expert pipeline's own
 * quantiser produces) and each of its rows holds q e4m3 (H bytes), the H/128
 * group scales (f32), the k owner-local ids of d3_ep_dispatch_meta (int64, -1
 * elsewhere) and its k bf16 weights, zero padded to d3_ep_row_bytes_fp8(H, k)
 * bytes (a multiple of 16). With slot == NULL, send is [ranks][T] rows (fixed
 * capacity: every token to every rank); with the slot map of d3_ep_plan_rows,
 * token t's row for rank d is row slot[t*ranks + d] and no row is written
 * where that is -1. d3_ep_unpack_fp8 copies the scales [rows, H/128], ids
 * [rows, k] and weights [rows, k] of `rows` received rows out; the e4m3 bytes
 * are read in place (row stride row_bytes), e.g. by d3_moe_experts_fp8 with
 * scales_transposed = 0. H a multiple of 128; send and recv 16-byte aligned
 * (D3_EINVAL otherwise). */
D3_API int d3_ep_row_bytes_fp8(int H, int k, int* bytes);
D3_API int d3_ep_pack_fp8(const void* x, int64_t x_stride, const int64_t* ids, const void* weights,
                          int T, int k, int H, int experts_per_rank, int ranks, const int32_t* slot,
                          uint8_t* send, d3_stream_t stream);
D3_API int d3_ep_unpack_fp8(const uint8_t* recv, int rows, int k, int H, float* scales,
                            int64_t* ids, void* weights, d3_stream_t stream);

/* out bf16 [T,H] = bf16(sum_r w[t,r] * rows[inv[t*k+r]]) + bf16(shared * bf16(sigmoid(gate)))
 * with rows bf16 [*, H] (expert outputs returned to the token's rank), the
 * sum in fp32 in r order; an inv entry < 0 is skipped; shared and gate may
 * be NULL. */
D3_API int d3_combine_pairs(const void* rows, const int32_t* inv_rows, const void* weights,
                            int T, int k, int H, const void* shared, const void* gate,
                            int64_t gate_stride, void* out, d3_stream_t stream);

/* Profiling hook, off by default: while set, d3_moe_experts / d3_moe_layer
 * calls made by the calling thread (the setting is per host thread) record
 * events[i] (cudaEvent_t handles, n >= 5) on their stream at stage
 * boundaries: 0 call start, 1 before the gate_up engine, 2 after gate_up,
 * 3 after the down engine, 4 call end. NULL clears it. A caller that never
 * sets it sees no effect. No counterpart in the reference (its scripts time
 * whole calls with CUDA events, src/drama3/profiling.py:11-102). */
D3_API int d3_set_stage_events(void* const* events, int n);

/* Token count T from which d3_moe_experts / d3_moe_layer run both expert GEMMs
 * on the tcgen05 grouped kernel (128-token x 256-column tiles, TMEM
 * accumulators) instead of the weight-streaming decode engine; H must be a
 * multiple of 256 for that path. Default 1024, or D3MOE_PREFILL_MIN_T from the
 * environment at first use. t <= 0 restores the default. Returns the previous
 * value. Process-wide. The reference switches kernels by token count the
 * same way (src/drama3/model.py:522-540: small_batch_moe up to
 * small_moe_max_batch tokens, native_moe with tuned tiles from 1024). */
D3_API int d3_set_prefill_min_tokens(int t);

#ifdef __cplusplus
}
#endif

#endif /* D3MOE_H_ */
