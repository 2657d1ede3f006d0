// Bandwidth-bound row kernels of the MoE path: activation FP8 quantisation
// (plain, fused with router-logit conversion, and gathered into expert order),
// SiLU*mul (+ requant), routed/shared combine, 128x128 weight quantisation and
// the f16 activation prep of the weight-only dense GEMV.
//
// Layout rule for the quantisers: one warp owns two 128-element groups of one
// row (warps = rows x ceil(groups/2), so every load is issued at once); a
// half-warp owns one group, each lane 8 consecutive elements (16-byte loads),
// so the group amax is a 4-step shuffle inside the half-warp.
#include "d3_common.cuh"
#include "d3_host.h"
#include "d3_internal.h"

namespace d3 {

namespace {

constexpr int kRowWarps = 8;  // rows per 256-thread CTA

__device__ __forceinline__ void unpack_bf16x8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint2 quant8(const float (&f)[8], float scale) {
  const float rs = __frcp_rn(scale);
  return make_uint2(act_quant4(f[0], f[1], f[2], f[3], scale, rs),
                    act_quant4(f[4], f[5], f[6], f[7], scale, rs));
}

__device__ __forceinline__ float half_warp_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Quantise groups 2*gp and 2*gp+1 of one bf16 row (warp-cooperative). The
// scale of group g goes to s[g * s_step].
__device__ __forceinline__ void quant_pair(const __nv_bfloat16* x, int G, int gp, uint8_t* q,
                                           float* s, int64_t s_step) {
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int g = 2 * gp + half;
  const bool valid = g < G;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + g * 128 + hl * 8));
  float f[8];
  unpack_bf16x8(v, f);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
  amax = half_warp_max(amax);
  const float scale = act_scale_from_amax(amax);
  if (valid) {
    *reinterpret_cast<uint2*>(q + g * 128 + hl * 8) = quant8(f, scale);
    if (hl == 0) s[g * s_step] = scale;
  }
}

// Global warp index -> (row, group pair).
struct RowPair {
  int row, gp;
};
__device__ __forceinline__ RowPair row_pair(int G) {
  const int gw = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  const int GP = (G + 1) / 2;
  return {gw / GP, gw % GP};
}

__global__ void quant_act_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T,
                                 int H, uint8_t* __restrict__ q, float* __restrict__ scales,
                                 int transposed) {
  pdl_enter();
  const int G = H / 128;
  const RowPair rp = row_pair(G);
  if (rp.row >= T) return;
  float* s = transposed ? scales + rp.row : scales + static_cast<int64_t>(rp.row) * G;
  quant_pair(x + rp.row * x_stride, G, rp.gp, q + static_cast<int64_t>(rp.row) * H, s,
             transposed ? T : 1);
}

__global__ void prepare_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                               const __nv_bfloat16* __restrict__ router, int64_t router_stride,
                               int T, int H, int E, const void* row_slots, int slots64,
                               int64_t padding_start, uint8_t* __restrict__ q,
                               float* __restrict__ scales_t, float* __restrict__ logits) {
  pdl_enter();
  const int G = H / 128;
  const RowPair rp = row_pair(G);
  const int row = rp.row;
  if (row >= T) return;
  quant_pair(x + row * x_stride, G, rp.gp, q + static_cast<int64_t>(row) * H, scales_t + row, T);
  if (rp.gp != 0) return;
  int router_row = row;
  if (padding_start > 0 && row_slots) {
    const int64_t slot = slots64 ? static_cast<const int64_t*>(row_slots)[row]
                                 : static_cast<const int32_t*>(row_slots)[row];
    if (slot >= padding_start) router_row = 0;
  }
  const __nv_bfloat16* r = router + router_row * router_stride;
  for (int e = threadIdx.x & 31; e < E; e += 32)
    logits[static_cast<int64_t>(row) * E + e] = __bfloat162float(r[e]);
}

// One warp per (token, pair of 128-groups): the two groups of x[t] are read
// and quantised once, then written to each row the token occupies in expert
// order (inv_rows[t*k + j], j < k; skipped when negative) and, with
// with_shared, to the shared-expert row P + t. Same bytes as quantising each
// expert-ordered row, with the quantisation done once per token instead of
// once per (token, expert) pair.
__global__ void quant_scatter_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T,
                                     int H, int k, const int32_t* __restrict__ inv_rows, int P,
                                     int with_shared, uint8_t* __restrict__ xq,
                                     float* __restrict__ sx, int32_t* __restrict__ zero, int nzero,
                                     RowGather rg) {
  pdl_enter();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  const int G = H / 128;
  const RowPair rp = row_pair(G);
  const int t = rp.row;
  if (t >= T) return;
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int g = 2 * rp.gp + half;
  const bool valid = g < G;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + gather_row(rg, t) * x_stride + g * 128 + hl * 8));
  float f[8];
  unpack_bf16x8(v, f);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  amax = half_warp_max(amax);
  const float scale = act_scale_from_amax(amax);
  const uint2 qb = quant8(f, scale);
  if (!valid) return;
  const int ndest = k + (with_shared ? 1 : 0);
  for (int j = 0; j < ndest; ++j) {
    const int d = j < k ? __ldg(inv_rows + static_cast<int64_t>(t) * k + j) : P + t;
    if (d < 0) continue;
    *reinterpret_cast<uint2*>(xq + static_cast<int64_t>(d) * H + g * 128 + hl * 8) = qb;
    if (hl == 0) sx[static_cast<int64_t>(d) * G + g] = scale;
  }
}

// Bucketing and activation quantisation in one kernel, for calls of fewer
// than kFusedPermuteMaxPairs pairs (the decode sizes). CTA t owns token t:
//   * the expert-ordered row of each of its pairs p = t*k + j is the pair's
//     position in the stable counting sort of all pairs by expert, i.e. the
//     number of valid pairs q with (ids[q], q) < (ids[p], p); one warp counts
//     it for one pair by scanning all P ids (ids outside [0, E) are skipped
//     and get row -1). This is the row the one-CTA permute kernel assigns.
//   * the token's row is quantised once (1x128 E4M3) and written to those
//     rows and, with a shared expert, to row P + t, as quant_scatter_kernel.
// CTA 0 also writes the per-expert counts and starts, the total, the active
// expert list and its length (the outputs of the permute kernel with
// block_m = 1) and zeroes `zero` (the engines' work counters).
__global__ void __launch_bounds__(256)
    permute_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T, int H, int k,
                         const int64_t* __restrict__ ids, int E, int with_shared,
                         uint8_t* __restrict__ xq, float* __restrict__ sx,
                         int32_t* __restrict__ counts, int32_t* __restrict__ starts,
                         int32_t* __restrict__ total, int32_t* __restrict__ inv_rows,
                         int32_t* __restrict__ active, int32_t* __restrict__ n_active,
                         int32_t* __restrict__ zero, int nzero, RowGather rg) {
  pdl_enter();
  __shared__ int slot[32];
  __shared__ int hist[kFusedPermuteMaxExperts];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = T * k;
  // this thread's first activation chunk, loaded while the pairs are counted
  const int G = H / 128;
  const int half = lane >> 4, hl = lane & 15;
  const int64_t src = gather_row(rg, t);
  uint4 v0 = make_uint4(0, 0, 0, 0);
  if (warp < (G + 1) / 2 && 2 * warp + half < G)
    v0 = __ldg(reinterpret_cast<const uint4*>(x + src * x_stride + (2 * warp + half) * 128 + hl * 8));
  for (int j = warp; j < k; j += 8) {
    const int p = t * k + j;
    const int64_t e = __ldg(ids + p);
    const bool ok = e >= 0 && e < E;
    int c = 0;
    if (ok)
#pragma unroll 8
      for (int q = lane; q < P; q += 32) {
        const int64_t f = __ldg(ids + q);
        c += (f >= 0 && f < E && (f < e || (f == e && q < p))) ? 1 : 0;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) {
      slot[j] = ok ? c : -1;
      inv_rows[p] = ok ? c : -1;
    }
  }
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    for (int q = threadIdx.x; q < P; q += blockDim.x) {
      const int64_t f = __ldg(ids + q);
      if (f >= 0 && f < E) atomicAdd(&hist[f], 1);
    }
    __syncthreads();
    if (warp == 0) {
      int run = 0, nact = 0;
      for (int base = 0; base < E; base += 32) {
        const int e = base + lane;
        const int c = e < E ? hist[e] : 0;
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const unsigned act = __ballot_sync(0xffffffffu, c > 0);
        if (e < E) {
          counts[e] = c;
          starts[e] = run + incl - c;
          if (c > 0) active[nact + __popc(act & ((1u << lane) - 1u))] = e;
        }
        run += __shfl_sync(0xffffffffu, incl, 31);
        nact += __popc(act);
      }
      if (lane == 0) {
        total[0] = run;
        n_active[0] = nact;
      }
    }
  }
  __syncthreads();
  for (int gp = warp; gp < (G + 1) / 2; gp += 8) {
    const int g = 2 * gp + half;
    const bool valid = g < G;
    uint4 v = v0;
    if (gp != warp) {
      v = make_uint4(0, 0, 0, 0);
      if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + src * x_stride + g * 128 + hl * 8));
    }
    float f[8];
    unpack_bf16x8(v, f);
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
    amax = half_warp_max(amax);
    const float scale = act_scale_from_amax(amax);
    const uint2 qb = quant8(f, scale);
    if (!valid) continue;
    const int ndest = k + (with_shared ? 1 : 0);
    for (int j = 0; j < ndest; ++j) {
      const int d = j < k ? slot[j] : P + t;
      if (d < 0) continue;
      *reinterpret_cast<uint2*>(xq + static_cast<int64_t>(d) * H + g * 128 + hl * 8) = qb;
      if (hl == 0) sx[static_cast<int64_t>(d) * G + g] = scale;
    }
  }
}

// Already-quantised activations into expert order (the FlashInfer calling
// convention): q e4m3 [T, H] rows are copied unchanged to rows inv_rows[t*k + j]
// (negative = skipped) and their group scales, read from [H/128, T]
// (transposed) or [T, H/128], to sx [rows, H/128]. One thread per 16 bytes.
__global__ void prequant_scatter_kernel(const uint8_t* __restrict__ q, int64_t q_stride,
                                        const float* __restrict__ qs, int transposed, int T, int H,
                                        int k, const int32_t* __restrict__ inv_rows,
                                        uint8_t* __restrict__ xq, float* __restrict__ sx,
                                        int32_t* __restrict__ zero, int nzero) {
  pdl_enter();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  const int chunks = H / 16, G = H / 128;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(T) * chunks) return;
  const int t = static_cast<int>(idx / chunks), c = static_cast<int>(idx - static_cast<int64_t>(t) * chunks);
  const uint4 v = __ldg(reinterpret_cast<const uint4*>(q + static_cast<int64_t>(t) * q_stride) + c);
  const bool scale_lane = (c & 7) == 0;
  const int g = c >> 3;
  float sc = 0.f;
  if (scale_lane) sc = __ldg(qs + (transposed ? static_cast<int64_t>(g) * T + t : static_cast<int64_t>(t) * G + g));
  for (int j = 0; j < k; ++j) {
    const int d = __ldg(inv_rows + static_cast<int64_t>(t) * k + j);
    if (d < 0) continue;
    reinterpret_cast<uint4*>(xq + static_cast<int64_t>(d) * H)[c] = v;
    if (scale_lane) sx[static_cast<int64_t>(d) * G + g] = sc;
  }
}

// Exact bf16 -> f16 transfer: each 128-group is multiplied by 2^s with s chosen
// so that the group amax lands in [2^14, 2^15); the GEMV multiplies by 2^-s.
// Within each 128-element block, element k is stored at dense_act_position(k)
// (expert_gemv.cuh).

__global__ void dense_act_prep_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T,
                                      int K, __half* __restrict__ xh, float* __restrict__ inv,
                                      int32_t* __restrict__ zero, int nzero,
                                      const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                      int mode) {
  pdl_enter();
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  const int G = K / 128;
  const RowPair rp = row_pair(G);
  const int row = rp.row;
  if (row >= T) return;
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int g = 2 * rp.gp + half;
  const bool valid = g < G;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + row * x_stride + g * 128 + hl * 8));
  float f[8];
  unpack_bf16x8(v, f);
  if (mode != GATE_NONE) {
    uint4 gv = make_uint4(0, 0, 0, 0);
    if (valid) gv = __ldg(reinterpret_cast<const uint4*>(gate + row * gate_stride + g * 128 + hl * 8));
    float gf[8];
    unpack_bf16x8(gv, gf);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = bf16_round(f[i] * gate_activation(gf[i], mode));
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
  amax = half_warp_max(amax);
  int e = 0;
  if (amax > 0.f && isfinite(amax)) {
    frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
    e = 15 - e;        // scaled amax in [2^14, 2^15)
  }
  const float mul = ldexpf(1.0f, e);
  if (valid) {
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 p = __floats2half2_rn(f[2 * i] * mul, f[2 * i + 1] * mul);
      h[i] = *reinterpret_cast<uint32_t*>(&p);
    }
    // stored in the bank-conflict-free k order of the GEMV's B fragments
    // (dense_act_position): this lane's 8 elements stay contiguous
    const int c = hl >> 1;
    const int pos = 8 * (8 * (c >> 2) + (c & 3) + 4 * (hl & 1));
    *reinterpret_cast<uint4*>(xh + static_cast<int64_t>(row) * K + g * 128 + pos) =
        make_uint4(h[0], h[1], h[2], h[3]);
    if (hl == 0) inv[static_cast<int64_t>(row) * G + g] = ldexpf(1.0f, -e);
  }
}

// Activations of the tcgen05 dense GEMV, split exactly into two E4M3 terms.
// Per 1x128 group, xs = x * 2^s with s chosen so that max|xs| lies in
// [2^7, 2^8) (a power of two: exact), hi = e4m3(xs) (round to nearest even),
// lo = e4m3((xs - hi) * 16). An 8-bit bf16 significand rounded to its top 4
// bits leaves a remainder of at most 3 significant bits, so xs = hi + lo / 16
// exactly whenever |xs| >= 2^-6 (every element within 2^13 of its group's
// maximum); smaller elements are carried with an absolute error below
// 2^-21 times the group maximum. sc[t][g] = 2^-s. With a gate, x is first
// replaced by bf16(x * bf16(act(gate))) like dense_act_prep_kernel.
// One warp per (row, pair of groups): 16 lanes x 8 elements per group.
__global__ void dense_split_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T, int K,
                                   const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                   int mode, uint8_t* __restrict__ hi, uint8_t* __restrict__ lo,
                                   float* __restrict__ sc) {
  pdl_enter();
  const int G = K / 128;
  const RowPair rp = row_pair(G);
  const int row = rp.row;
  if (row >= T) return;
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const int g = 2 * rp.gp + half;
  const bool valid = g < G;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + row * x_stride + g * 128 + hl * 8));
  float f[8];
  unpack_bf16x8(v, f);
  if (mode != GATE_NONE) {
    uint4 gv = make_uint4(0, 0, 0, 0);
    if (valid) gv = __ldg(reinterpret_cast<const uint4*>(gate + row * gate_stride + g * 128 + hl * 8));
    float gf[8];
    unpack_bf16x8(gv, gf);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = bf16_round(f[i] * gate_activation(gf[i], mode));
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
  amax = half_warp_max(amax);
  const int sh = shift_for_amax(amax);
  const float mul = ldexpf(1.0f, sh);
  if (!valid) return;
  uint32_t h[2], l[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float xs[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) xs[j] = f[4 * i + j] * mul;
    split_e4m3x4(xs, h[i], l[i]);
  }
  const int64_t off = static_cast<int64_t>(row) * K + g * 128 + hl * 8;
  *reinterpret_cast<uint2*>(hi + off) = make_uint2(h[0], h[1]);
  *reinterpret_cast<uint2*>(lo + off) = make_uint2(l[0], l[1]);
  if (hl == 0) sc[static_cast<int64_t>(row) * G + g] = ldexpf(1.0f, -sh);
}

__device__ __forceinline__ float silu_bf16(float gate_bf16) {
  // silu(g) = g * sigmoid(g), rounded to bf16 like the reference kernel.
  return bf16_round(gate_bf16 * (1.0f / (1.0f + expf(-gate_bf16))));
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ in, int64_t in_stride, int rows,
                                int W, __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = W / 8;
  if (idx >= static_cast<int64_t>(rows) * per_row) return;
  const int row = static_cast<int>(idx / per_row), c = static_cast<int>(idx % per_row) * 8;
  const __nv_bfloat16* r = in + row * in_stride;
  float g[8], u[8];
  unpack_bf16x8(*reinterpret_cast<const uint4*>(r + c), g);
  unpack_bf16x8(*reinterpret_cast<const uint4*>(r + W + c), u);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(silu_bf16(g[2 * i]) * u[2 * i],
                                             silu_bf16(g[2 * i + 1]) * u[2 * i + 1]);
    o[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * W + c) =
      make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ in, int64_t in_stride,
                                      int rows, int W, uint8_t* __restrict__ q,
                                      float* __restrict__ scales) {
  pdl_enter();
  const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int G = W / 128;
  const int lane = threadIdx.x & 31, half = lane >> 4, hl = lane & 15;
  const __nv_bfloat16* r = in + row * in_stride;
  for (int g0 = 0; g0 < G; g0 += 2) {
    const int g = g0 + half;
    const bool valid = g < G;
    float a[8];
    if (valid) {
      float gt[8], up[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(r + g * 128 + hl * 8), gt);
      unpack_bf16x8(*reinterpret_cast<const uint4*>(r + W + g * 128 + hl * 8), up);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = silu_bf16(gt[i]) * up[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(a[i]));
    amax = half_warp_max(amax);
    const float scale = act_scale_from_amax(amax);
    if (valid) {
      *reinterpret_cast<uint2*>(q + static_cast<int64_t>(row) * W + g * 128 + hl * 8) =
          quant8(a, scale);
      if (hl == 0) scales[static_cast<int64_t>(row) * G + g] = scale;
    }
  }
}

__device__ __forceinline__ float sigmoid_gate_bf16(const __nv_bfloat16* gate) {
  const float g = __bfloat162float(*gate);
  return bf16_round(1.0f / (1.0f + expf(-g)));
}

__global__ void combine_experts_kernel(const __nv_bfloat16* __restrict__ routed,
                                       const __nv_bfloat16* __restrict__ shared,
                                       const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                       int T, int H, __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = H / 8;
  if (idx >= static_cast<int64_t>(T) * per_row) return;
  const int t = static_cast<int>(idx / per_row), c = static_cast<int>(idx % per_row) * 8;
  const float g = sigmoid_gate_bf16(gate + t * gate_stride);
  float r[8], s[8];
  const int64_t off = static_cast<int64_t>(t) * H + c;
  unpack_bf16x8(*reinterpret_cast<const uint4*>(routed + off), r);
  unpack_bf16x8(*reinterpret_cast<const uint4*>(shared + off), s);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(r[2 * i] + bf16_round(s[2 * i] * g),
                                             r[2 * i + 1] + bf16_round(s[2 * i + 1] * g));
    o[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(out + off) = make_uint4(o[0], o[1], o[2], o[3]);
}

// One thread per 4 output columns of one token. Expert rows are read in rank
// order r = 0..k-1 and summed in fp32 with the bf16 routing weight.
// 4 consecutive values of an expert row as fp32, from fp32 rows or from the
// bf16 rows of the tcgen05 path.
template <bool BF16>
__device__ __forceinline__ float4 load_row4(const void* d, int64_t row, int H, int c) {
  if constexpr (BF16) {
    const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(d) + row * H + c);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  } else {
    return *reinterpret_cast<const float4*>(static_cast<const float*>(d) + row * H + c);
  }
}

template <bool BF16>
__global__ void combine_rows_kernel(const void* __restrict__ d, int H,
                                    const int32_t* __restrict__ inv_rows,
                                    const __nv_bfloat16* __restrict__ weights, int T, int k,
                                    int with_shared, const __nv_bfloat16* __restrict__ gate,
                                    int64_t gate_stride, __nv_bfloat16* __restrict__ routed_out,
                                    __nv_bfloat16* __restrict__ shared_out,
                                    __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = H / 4;
  if (idx >= static_cast<int64_t>(T) * per_row) return;
  const int t = static_cast<int>(idx / per_row), c = static_cast<int>(idx % per_row) * 4;
  const int P = T * k;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < k; ++r) {
    const int row = inv_rows[t * k + r];
    if (row < 0) continue;  // pair whose expert id was out of range: not routed
    const float w = __bfloat162float(weights[t * k + r]);
    const float4 v = load_row4<BF16>(d, row, H, c);
    acc[0] += v.x * w;
    acc[1] += v.y * w;
    acc[2] += v.z * w;
    acc[3] += v.w * w;
  }
  float routed[4], shared[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) routed[i] = bf16_round(acc[i]);
  if (with_shared) {
    const float4 v = load_row4<BF16>(d, P + t, H, c);
    shared[0] = bf16_round(v.x);
    shared[1] = bf16_round(v.y);
    shared[2] = bf16_round(v.z);
    shared[3] = bf16_round(v.w);
  }
  const int64_t off = static_cast<int64_t>(t) * H + c;
  auto store4 = [&](__nv_bfloat16* dst, const float (&v)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
    *reinterpret_cast<uint2*>(dst + off) = u;
  };
  if (routed_out) store4(routed_out, routed);
  if (shared_out && with_shared) store4(shared_out, shared);
  if (out) {
    float o[4];
    if (with_shared && gate) {
      const float g = sigmoid_gate_bf16(gate + t * gate_stride);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = routed[i] + bf16_round(shared[i] * g);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = routed[i] + shared[i];
    }
    store4(out, o);
  }
}

// One CTA per 128x128 weight block; 256 threads x 64 elements.
__global__ void weight_quant_kernel(const __nv_bfloat16* __restrict__ w, int N, int K,
                                    uint8_t* __restrict__ q, float* __restrict__ scales) {
  pdl_enter();
  const int nb = blockIdx.x, kb = blockIdx.y, KB = K / 128;
  __shared__ float red[8];
  const int tid = threadIdx.x;
  // thread -> row tid/2, columns (tid%2)*64 .. +63
  const int row = nb * 128 + tid / 2, col = kb * 128 + (tid & 1) * 64;
  float f[64];
  const bool valid = row < N;
#pragma unroll
  for (int v = 0; v < 8; ++v) {
    float t[8];
    uint4 u = make_uint4(0, 0, 0, 0);
    if (valid) u = *reinterpret_cast<const uint4*>(w + static_cast<int64_t>(row) * K + col + v * 8);
    unpack_bf16x8(u, t);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[v * 8 + i] = t[i];
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(f[i]));
  amax = warp_max(amax);
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) amax = fmaxf(amax, red[i]);
  const float scale = __fdiv_rn(fmaxf(amax, 1e-8f), 448.0f);
  uint8_t* qrow = q + static_cast<int64_t>(row) * K + col;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    uint32_t word[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t b = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        b |= static_cast<uint32_t>(f32_to_e4m3(__fdiv_rn(f[v * 16 + j * 4 + i], scale))) << (8 * i);
      word[j] = b;
    }
    *reinterpret_cast<uint4*>(qrow + v * 16) = make_uint4(word[0], word[1], word[2], word[3]);
  }
  if (tid == 0) scales[nb * KB + kb] = scale;
}

// Expert-parallel combine on the token's own rank:
//   routed[t] = bf16( sum_r w[t,r] * rows[inv[t*k+r]] )   (fp32, r = 0..k-1)
//   out[t]    = routed + bf16(shared[t] * bf16(sigmoid(gate[t])))
__global__ void combine_pairs_kernel(const __nv_bfloat16* __restrict__ rows, int H,
                                     const int32_t* __restrict__ inv_rows,
                                     const __nv_bfloat16* __restrict__ weights, int T, int k,
                                     const __nv_bfloat16* __restrict__ shared,
                                     const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                                     __nv_bfloat16* __restrict__ out) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = H / 8;
  if (idx >= static_cast<int64_t>(T) * per_row) return;
  const int t = static_cast<int>(idx / per_row), c = static_cast<int>(idx % per_row) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < k; ++r) {
    const int row = inv_rows[t * k + r];
    if (row < 0) continue;
    const float w = __bfloat162float(weights[t * k + r]);
    float v[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(row) * H + c), v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i] * w;
  }
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = bf16_round(acc[i]);
  if (shared) {
    float sv[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(shared + static_cast<int64_t>(t) * H + c), sv);
    const float g = gate ? sigmoid_gate_bf16(gate + t * gate_stride) : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] += gate ? bf16_round(sv[i] * g) : sv[i];
  }
  uint32_t wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p2 = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    wv[i] = *reinterpret_cast<uint32_t*>(&p2);
  }
  *reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * H + c) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// Fixed-capacity EP dispatch metadata: for every destination rank d and
// token t, the routing of t restricted to the experts d owns:
//   meta_ids[d][t][j] = ids[t][j] - d*experts_per_rank if d owns ids[t][j], else -1
//   meta_w[d][t][j]   = w[t][j] if d owns ids[t][j], else 0
__global__ void ep_dispatch_meta_kernel(const int64_t* __restrict__ ids,
                                        const __nv_bfloat16* __restrict__ w, int T, int k,
                                        int experts_per_rank, int ranks,
                                        int64_t* __restrict__ meta_ids,
                                        __nv_bfloat16* __restrict__ meta_w) {
  pdl_enter();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n = static_cast<int64_t>(ranks) * T * k;
  if (idx >= n) return;
  const int d = static_cast<int>(idx / (static_cast<int64_t>(T) * k));
  const int tj = static_cast<int>(idx % (static_cast<int64_t>(T) * k));
  const int64_t e = ids[tj];
  const bool mine = e >= 0 && e / experts_per_rank == d && e < static_cast<int64_t>(experts_per_rank) * ranks;
  meta_ids[idx] = mine ? e - static_cast<int64_t>(d) * experts_per_rank : -1;
  meta_w[idx] = mine ? w[tj] : __float2bfloat16_rn(0.f);
}

// FP8 packed EP dispatch: token t is quantised once (1x128 E4M3 groups, the
// same bytes and scales the expert pipeline's own quantiser produces) and its
// row for destination rank d holds [q e4m3 H bytes | group scales f32 H/128 |
// k owner-local ids int64 (-1 where another rank owns the expert) | k bf16
// weights (0 there) | zero padding to ep_row_bytes_fp8]. The row's index in
// `send` is slot[t*ranks + d] (no row when -1), or d*T + t without a slot map
// (fixed capacity: every token to every rank). One CTA per token.
__global__ void __launch_bounds__(256)
    ep_pack_fp8_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                       const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ w, int T,
                       int k, int H, int experts_per_rank, int ranks, int row_bytes,
                       const int32_t* __restrict__ slot, uint8_t* __restrict__ send) {
  pdl_enter();
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto row_of = [&](int d) -> uint8_t* {
    const int64_t r = slot ? slot[static_cast<int64_t>(t) * ranks + d] : static_cast<int64_t>(d) * T + t;
    return r < 0 ? nullptr : send + r * row_bytes;
  };
  const int G = H / 128;
  const int half = lane >> 4, hl = lane & 15;
  for (int gp = warp; gp < (G + 1) / 2; gp += 8) {
    const int g = 2 * gp + half;
    const bool valid = g < G;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (valid) v = __ldg(reinterpret_cast<const uint4*>(x + t * x_stride + g * 128 + hl * 8));
    float f[8];
    unpack_bf16x8(v, f);
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
    amax = half_warp_max(amax);
    const float scale = act_scale_from_amax(amax);
    const uint2 qb = quant8(f, scale);
    if (!valid) continue;
    for (int d = 0; d < ranks; ++d) {
      uint8_t* row = row_of(d);
      if (!row) continue;
      *reinterpret_cast<uint2*>(row + g * 128 + hl * 8) = qb;
      if (hl == 0) reinterpret_cast<float*>(row + H)[g] = scale;
    }
  }
  const int meta = H + 4 * G;  // byte offset of the routing metadata
  const int64_t owned = static_cast<int64_t>(experts_per_rank) * ranks;
  for (int i = threadIdx.x; i < ranks * k; i += blockDim.x) {
    const int d = i / k, j = i - d * k;
    const int64_t e = ids[static_cast<int64_t>(t) * k + j];
    const bool mine = e >= 0 && e < owned && e / experts_per_rank == d;
    uint8_t* row = row_of(d);
    if (!row) continue;
    reinterpret_cast<int64_t*>(row + meta)[j] = mine ? e - static_cast<int64_t>(d) * experts_per_rank : -1;
    reinterpret_cast<__nv_bfloat16*>(row + meta + 8 * k)[j] =
        mine ? w[static_cast<int64_t>(t) * k + j] : __float2bfloat16_rn(0.f);
  }
  for (int i = meta + 10 * k + threadIdx.x; i < row_bytes; i += blockDim.x)
    for (int d = 0; d < ranks; ++d)
      if (uint8_t* row = row_of(d)) row[i] = 0;
}

// Received FP8 packed rows: group scales [rows, H/128], ids [rows, k] and
// weights [rows, k] copied out contiguous; the e4m3 bytes are read in place
// (row stride ep_row_bytes_fp8).
__global__ void ep_unpack_fp8_kernel(const uint8_t* __restrict__ recv, int rows, int k, int H,
                                     int row_bytes, float* __restrict__ scales,
                                     int64_t* __restrict__ ids, __nv_bfloat16* __restrict__ w) {
  pdl_enter();
  const int G = H / 128;
  const int per_row = G + k;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows) * per_row) return;
  const int64_t r = idx / per_row;
  const int c = static_cast<int>(idx - r * per_row);
  const uint8_t* row = recv + r * row_bytes;
  if (c < G) {
    scales[r * G + c] = reinterpret_cast<const float*>(row + H)[c];
  } else {
    const int j = c - G;
    ids[r * k + j] = reinterpret_cast<const int64_t*>(row + H + 4 * G)[j];
    w[r * k + j] = reinterpret_cast<const __nv_bfloat16*>(row + H + 4 * G + 8 * k)[j];
  }
}

inline unsigned row_blocks(int rows) { return static_cast<unsigned>((rows + kRowWarps - 1) / kRowWarps); }

// CTAs for one warp per (row, group pair).
inline unsigned pair_blocks(int rows, int cols) {
  const int64_t warps = static_cast<int64_t>(rows) * ((cols / 128 + 1) / 2);
  return static_cast<unsigned>((warps + kRowWarps - 1) / kRowWarps);
}

}  // namespace

void launch_quant_scatter(const void* x, int64_t x_stride, int T, int H, int k,
                          const int32_t* inv_rows, int P, int with_shared, uint8_t* xq, float* sx,
                          cudaStream_t s, int32_t* zero, int nzero, const RowGather& rg) {
  if (T <= 0) return;
  launch_kernel(quant_scatter_kernel, dim3(pair_blocks(T, H)), dim3(256), 0, s,
                static_cast<const __nv_bfloat16*>(x), x_stride, T, H, k, inv_rows, P, with_shared, xq,
                sx, zero, nzero, rg);
}

void launch_permute_quant(const void* x, int64_t x_stride, int T, int H, int k, const int64_t* ids,
                          int E, int with_shared, uint8_t* xq, float* sx, int32_t* counts,
                          int32_t* starts, int32_t* total, int32_t* inv_rows, int32_t* active,
                          int32_t* n_active, cudaStream_t s, int32_t* zero, int nzero,
                          const RowGather& rg) {
  if (T <= 0) return;
  launch_kernel(permute_quant_kernel, dim3(T), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(x),
                x_stride, T, H, k, ids, E, with_shared, xq, sx, counts, starts, total, inv_rows, active,
                n_active, zero, nzero, rg);
}

void launch_prequant_scatter(const uint8_t* q, int64_t q_stride, const float* qs, int transposed,
                             int T, int H, int k, const int32_t* inv_rows, uint8_t* xq, float* sx,
                             cudaStream_t s, int32_t* zero, int nzero) {
  if (T <= 0) return;
  const int64_t n = static_cast<int64_t>(T) * (H / 16);
  launch_kernel(prequant_scatter_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                q, q_stride, qs, transposed, T, H, k, inv_rows, xq, sx, zero, nzero);
}

void launch_dense_act_prep(const void* x, int64_t x_stride, int T, int K, __half* xh, float* inv,
                           cudaStream_t s, int32_t* zero, int nzero, const void* gate,
                           int64_t gate_stride, int mode) {
  if (T <= 0) return;
  launch_kernel(dense_act_prep_kernel, dim3(pair_blocks(T, K)), dim3(256), 0, s,
                static_cast<const __nv_bfloat16*>(x), x_stride, T, K, xh, inv, zero, nzero,
                static_cast<const __nv_bfloat16*>(gate), gate_stride, gate ? mode : GATE_NONE);
}

void launch_dense_split(const void* x, int64_t x_stride, int T, int K, const void* gate,
                        int64_t gate_stride, int mode, uint8_t* hi, uint8_t* lo, float* sc,
                        cudaStream_t s) {
  if (T <= 0) return;
  launch_kernel(dense_split_kernel, dim3(pair_blocks(T, K)), dim3(256), 0, s,
                static_cast<const __nv_bfloat16*>(x), x_stride, T, K,
                static_cast<const __nv_bfloat16*>(gate), gate_stride, gate ? mode : GATE_NONE, hi, lo, sc);
}

void launch_combine_rows(const float* d, int H, const int32_t* inv_rows, const void* weights,
                         int T, int k, int with_shared, const void* gate, int64_t gate_stride,
                         void* routed_out, void* shared_out, void* out, cudaStream_t s,
                         bool rows_bf16) {
  const int64_t n = static_cast<int64_t>(T) * (H / 4);
  if (n <= 0) return;
  launch_kernel(rows_bf16 ? combine_rows_kernel<true> : combine_rows_kernel<false>,
      dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
      static_cast<const void*>(d), H, inv_rows, static_cast<const __nv_bfloat16*>(weights), T, k, with_shared,
      static_cast<const __nv_bfloat16*>(gate), gate_stride,
      static_cast<__nv_bfloat16*>(routed_out), static_cast<__nv_bfloat16*>(shared_out),
      static_cast<__nv_bfloat16*>(out));
}

}  // namespace d3

using namespace d3;

extern "C" int d3_quant_act_fp8(const void* x, int64_t x_stride, int T, int H, uint8_t* q,
                                float* scales, int scales_transposed, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && H > 0 && H % 128 == 0, "quant_act_fp8: H=%d must be a positive multiple of 128", H);
  D3_REQUIRE(x_stride >= H && x_stride % 8 == 0, "quant_act_fp8: x row stride %lld must be >= H and a multiple of 8", (long long)x_stride);
  D3_REQUIRE(aligned(x, 16) && aligned(q, 16) && aligned(scales, 4), "quant_act_fp8: misaligned pointer");
  if (T == 0) return D3_OK;
  launch_kernel(quant_act_kernel, dim3(pair_blocks(T, H)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(x), x_stride, T, H, q, scales, scales_transposed);
  return check_launch("quant_act_fp8");
}

extern "C" int d3_prepare_moe_input(const void* x, int64_t x_stride, const void* router,
                                    int64_t router_stride, int T, int H, int E,
                                    const void* row_slots, int row_slots_int64,
                                    int64_t padding_start, uint8_t* q, float* scales_t,
                                    float* logits, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && H > 0 && H % 128 == 0 && E > 0, "prepare_moe_input: bad shape T=%d H=%d E=%d", T, H, E);
  D3_REQUIRE(x_stride >= H && x_stride % 8 == 0, "prepare_moe_input: x row stride must be >= H and a multiple of 8");
  D3_REQUIRE(router_stride >= E, "prepare_moe_input: router row stride must be >= E");
  D3_REQUIRE((row_slots == nullptr) == (padding_start <= 0), "prepare_moe_input: reserved padding routing needs both row_slots and padding_start > 0");
  D3_REQUIRE(aligned(x, 16) && aligned(q, 16), "prepare_moe_input: misaligned pointer");
  if (T == 0) return D3_OK;
  launch_kernel(prepare_kernel, dim3(pair_blocks(T, H)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(router),
      router_stride, T, H, E, row_slots, row_slots_int64, padding_start, q, scales_t, logits);
  return check_launch("prepare_moe_input");
}

extern "C" int d3_silu_mul(const void* in, int64_t in_stride, int rows, int W, void* out,
                           d3_stream_t stream) {
  D3_REQUIRE(rows >= 0 && W > 0 && W % 8 == 0, "silu_mul: width %d must be a positive multiple of 8", W);
  D3_REQUIRE(in_stride >= 2 * W && in_stride % 8 == 0, "silu_mul: input row stride must be >= 2W and a multiple of 8");
  D3_REQUIRE(aligned(in, 16) && aligned(out, 16), "silu_mul: misaligned pointer");
  const int64_t n = static_cast<int64_t>(rows) * (W / 8);
  if (n == 0) return D3_OK;
  launch_kernel(silu_mul_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(in), in_stride, rows, W, static_cast<__nv_bfloat16*>(out));
  return check_launch("silu_mul");
}

extern "C" int d3_silu_mul_quant(const void* in, int64_t in_stride, int rows, int W, uint8_t* q,
                                 float* scales, d3_stream_t stream) {
  D3_REQUIRE(rows >= 0 && W > 0 && W % 128 == 0, "silu_mul_quant: width %d must be a positive multiple of 128", W);
  D3_REQUIRE(in_stride >= 2 * W && in_stride % 8 == 0, "silu_mul_quant: input row stride must be >= 2W and a multiple of 8");
  D3_REQUIRE(aligned(in, 16) && aligned(q, 16), "silu_mul_quant: misaligned pointer");
  if (rows == 0) return D3_OK;
  launch_kernel(silu_mul_quant_kernel, dim3(row_blocks(rows)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(in), in_stride, rows, W, q, scales);
  return check_launch("silu_mul_quant");
}

extern "C" int d3_combine_experts(const void* routed, const void* shared, const void* gate,
                                  int64_t gate_stride, int T, int H, void* out,
                                  d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && H > 0 && H % 8 == 0, "combine_experts: H=%d must be a positive multiple of 8", H);
  D3_REQUIRE(aligned(routed, 16) && aligned(shared, 16) && aligned(out, 16), "combine_experts: misaligned pointer");
  const int64_t n = static_cast<int64_t>(T) * (H / 8);
  if (n == 0) return D3_OK;
  launch_kernel(combine_experts_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(routed), static_cast<const __nv_bfloat16*>(shared),
      static_cast<const __nv_bfloat16*>(gate), gate_stride, T, H,
      static_cast<__nv_bfloat16*>(out));
  return check_launch("combine_experts");
}

extern "C" int d3_fp8_quantize_weight(const void* w, int N, int K, uint8_t* q, float* scales,
                                      d3_stream_t stream) {
  D3_REQUIRE(N > 0 && K > 0 && K % 128 == 0, "fp8_quantize_weight: K=%d must be a positive multiple of 128", K);
  D3_REQUIRE(aligned(w, 16) && aligned(q, 16), "fp8_quantize_weight: misaligned pointer");
  dim3 grid((N + 127) / 128, K / 128);
  launch_kernel(weight_quant_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(w), N, K, q, scales);
  return check_launch("fp8_quantize_weight");
}

extern "C" int d3_combine_pairs(const void* rows, const int32_t* inv_rows, const void* weights,
                                int T, int k, int H, const void* shared, const void* gate,
                                int64_t gate_stride, void* out, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && H > 0 && H % 8 == 0, "combine_pairs: bad shape");
  D3_REQUIRE(aligned(rows, 16) && aligned(out, 16) && (!shared || aligned(shared, 16)), "combine_pairs: misaligned pointer");
  const int64_t n = static_cast<int64_t>(T) * (H / 8);
  if (n == 0) return D3_OK;
  launch_kernel(combine_pairs_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      static_cast<const __nv_bfloat16*>(rows), H, inv_rows, static_cast<const __nv_bfloat16*>(weights),
      T, k, static_cast<const __nv_bfloat16*>(shared), static_cast<const __nv_bfloat16*>(gate),
      gate_stride, static_cast<__nv_bfloat16*>(out));
  return check_launch("combine_pairs");
}

extern "C" int d3_ep_row_bytes_fp8(int H, int k, int* bytes) {
  D3_REQUIRE(bytes && H > 0 && H % 128 == 0 && k > 0, "ep_row_bytes_fp8: bad arguments");
  *bytes = (H + 4 * (H / 128) + 10 * k + 15) / 16 * 16;
  return D3_OK;
}

extern "C" int d3_ep_pack_fp8(const void* x, int64_t x_stride, const int64_t* ids, const void* weights,
                              int T, int k, int H, int experts_per_rank, int ranks, const int32_t* slot,
                              uint8_t* send, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && H > 0 && H % 128 == 0 && experts_per_rank > 0 && ranks > 0,
             "ep_pack_fp8: bad shape (H must be a multiple of 128)");
  D3_REQUIRE(x_stride >= H && x_stride % 8 == 0 && aligned(x, 16) && aligned(send, 16),
             "ep_pack_fp8: x must be 16-byte aligned with a row stride >= H, multiple of 8");
  D3_REQUIRE(ids && weights, "ep_pack_fp8: null ids or weights");
  if (T == 0) return D3_OK;
  const int row_bytes = (H + 4 * (H / 128) + 10 * k + 15) / 16 * 16;
  launch_kernel(ep_pack_fp8_kernel, dim3(T), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                static_cast<const __nv_bfloat16*>(x), x_stride, ids,
                static_cast<const __nv_bfloat16*>(weights), T, k, H, experts_per_rank, ranks, row_bytes,
                slot, send);
  return check_launch("ep_pack_fp8");
}

extern "C" int d3_ep_unpack_fp8(const uint8_t* recv, int rows, int k, int H, float* scales,
                                int64_t* ids, void* weights, d3_stream_t stream) {
  D3_REQUIRE(rows >= 0 && k > 0 && H > 0 && H % 128 == 0 && recv && scales && ids && weights,
             "ep_unpack_fp8: bad arguments");
  // the rows are read in place afterwards by TMA (16-byte aligned rows)
  D3_REQUIRE(aligned(recv, 16), "ep_unpack_fp8: the received rows must be 16-byte aligned");
  const int row_bytes = (H + 4 * (H / 128) + 10 * k + 15) / 16 * 16;
  const int64_t n = static_cast<int64_t>(rows) * (H / 128 + k);
  if (n == 0) return D3_OK;
  launch_kernel(ep_unpack_fp8_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                reinterpret_cast<cudaStream_t>(stream), recv, rows, k, H, row_bytes, scales, ids,
                static_cast<__nv_bfloat16*>(weights));
  return check_launch("ep_unpack_fp8");
}

extern "C" int d3_ep_dispatch_meta(const int64_t* ids, const void* weights, int T, int k,
                                   int experts_per_rank, int ranks, int64_t* meta_ids,
                                   void* meta_w, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && experts_per_rank > 0 && ranks > 0, "ep_dispatch_meta: bad arguments");
  const int64_t n = static_cast<int64_t>(ranks) * T * k;
  if (n == 0) return D3_OK;
  launch_kernel(ep_dispatch_meta_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), 
      ids, static_cast<const __nv_bfloat16*>(weights), T, k, experts_per_rank, ranks, meta_ids,
      static_cast<__nv_bfloat16*>(meta_w));
  return check_launch("ep_dispatch_meta");
}
