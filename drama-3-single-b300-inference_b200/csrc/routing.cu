// Routing kernels: the bf16 router projection, softmax/top-k/renormalise and
// the token->expert bucketing (stable counting sort).
#include "d3_common.cuh"
#include "d3_host.h"
#include "d3_internal.h"
#include "router_tc.cuh"

namespace d3 {

namespace {

// ------------------------------------------------------- router projection --
// logits[t, r] = bf16( sum_k x[t,k] * w[r,k] (+ bias[r]) ).
// Summation order (fixed, restated by the CPU oracle): lane l of a warp owns
// k = 256*i + 8*l + j (i ascending, then j = 0..7) and accumulates sequentially
// in fp32; the 32 lane partials are combined by an xor-butterfly with offsets
// 16, 8, 4, 2, 1. bf16*bf16 products are exact in fp32, so FMA and
// multiply-then-add give the same result and the order alone defines the sum.
// CTA: 8 warps = 8 router rows, each warp holding its weight row in registers
// and running 4 tokens at a time as independent chains (the order inside each
// chain is unchanged); x is read through the read-only cache.
constexpr int kRouterRows = 8, kRouterTokens = 8, kRouterMaxIters = 12;  // H <= 3072

__global__ void __launch_bounds__(256)
    router_logits_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                         const __nv_bfloat16* __restrict__ w, const float* __restrict__ bias,
                         int nbias, int R, int H, int T, __nv_bfloat16* __restrict__ out,
                         int64_t out_stride, RowGather rg) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [8][H]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kRouterRows + warp;
  const int t0 = blockIdx.y * kRouterTokens;
  const int nt = min(kRouterTokens, T - t0);
  const int iters = (H + 255) / 256;
  // weight row into registers first: all of its loads are in flight together
  uint4 wv[kRouterMaxIters];
  const __nv_bfloat16* wr = w + static_cast<int64_t>(r < R ? r : 0) * H;
#pragma unroll
  for (int i = 0; i < kRouterMaxIters; ++i) {
    const int k0 = 256 * i + 8 * lane;
    wv[i] = (i < iters && k0 < H) ? __ldg(reinterpret_cast<const uint4*>(wr + k0))
                                  : make_uint4(0, 0, 0, 0);
  }
  // the CTA's tokens into shared memory (every thread issues its loads at once)
  const int chunks = H / 8;
  for (int idx = threadIdx.x; idx < nt * chunks; idx += blockDim.x) {
    const int t = idx / chunks, c = idx - t * chunks;
    reinterpret_cast<uint4*>(xs + t * H)[c] =
        __ldg(reinterpret_cast<const uint4*>(x + gather_row(rg, t0 + t) * x_stride) + c);
  }
  __syncthreads();
  if (r >= R) return;
  const float b = (bias && r < nbias) ? bias[r] : 0.f;
  for (int tb = 0; tb < nt; tb += 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < kRouterMaxIters; ++i) {
      const int k0 = 256 * i + 8 * lane;
      if (i < iters && k0 < H) {
        uint4 xv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          xv[u] = reinterpret_cast<const uint4*>(xs + (tb + u < nt ? tb + u : 0) * H + k0)[0];
        const uint32_t ww[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t xx[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[u] = fma_bf16x2_seq(xx[j], ww[j], acc[u]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
    }
    if (lane < 4 && tb + lane < nt) {
      float v = acc[0];
#pragma unroll
      for (int u = 1; u < 4; ++u)
        if (lane == u) v = acc[u];
      out[(t0 + tb + lane) * out_stride + r] = __float2bfloat16_rn(v + b);
    }
  }
}

// Prefill form of the same projection, in the same summation order. A CTA of
// 8 warps computes a 32-token x 16-row tile: warp w owns tokens 4w..4w+3 and
// all 16 rows (64 independent fp32 chains per lane, lane l still owning
// k = 256*i + 8*l + j). The 256-wide k blocks of the 32 x rows and 16 weight
// rows stream through a 4-stage cp.async ring in shared memory (24 KB a
// stage), so weights are read once per 32 tokens instead of once per 8.
constexpr int kRtTok = 32, kRtRows = 16, kRtStages = 4, kRtThreads = 256;
constexpr int kRtStageElems = (kRtTok + kRtRows) * 256;
constexpr size_t kRtSmem = static_cast<size_t>(kRtStages) * kRtStageElems * 2;  // 96 KB
constexpr int kRouterTiledMinTokens = 256;
// From this many tokens the projection runs on the tensor cores (router_tc.cuh)
// unless the rows are gathered through a keep map.
constexpr int kRouterTcMinTokens = 256;

__global__ void __launch_bounds__(kRtThreads)
    router_logits_tiled_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                               const __nv_bfloat16* __restrict__ w, const float* __restrict__ bias,
                               int nbias, int R, int H, int T, __nv_bfloat16* __restrict__ out,
                               int64_t out_stride, RowGather rg) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * kRtRows, t0 = blockIdx.y * kRtTok;
  const int nt = min(kRtTok, T - t0), nr = min(kRtRows, R - r0);
  const int iters = (H + 255) / 256;

  auto fill = [&](int i) {
    __nv_bfloat16* st = ring + (i % kRtStages) * kRtStageElems;
    for (int idx = threadIdx.x; idx < (kRtTok + kRtRows) * 32; idx += kRtThreads) {
      const int row = idx >> 5, c = idx & 31;
      const int k0 = 256 * i + 8 * c;
      if (k0 >= H) continue;  // half-filled last block: those lanes skip it below
      const __nv_bfloat16* src =
          row < kRtTok ? x + gather_row(rg, t0 + min(row, nt - 1)) * x_stride + k0
                       : w + static_cast<int64_t>(r0 + min(row - kRtTok, nr - 1)) * H + k0;
      cp_async_16(st + row * 256 + 8 * c, src);
    }
  };

#pragma unroll
  for (int i = 0; i < kRtStages - 1; ++i) {
    if (i < iters) fill(i);
    cp_async_commit();
  }
  float acc[4][kRtRows];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int r = 0; r < kRtRows; ++r) acc[u][r] = 0.f;

  for (int i = 0; i < iters; ++i) {
    if (i + kRtStages - 1 < iters) fill(i + kRtStages - 1);
    cp_async_commit();
    cp_async_wait<kRtStages - 1>();
    __syncthreads();
    if (256 * i + 8 * lane < H) {
      const __nv_bfloat16* st = ring + (i % kRtStages) * kRtStageElems;
      uint32_t xx[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 v = *reinterpret_cast<const uint4*>(st + (4 * warp + u) * 256 + 8 * lane);
        xx[u][0] = v.x; xx[u][1] = v.y; xx[u][2] = v.z; xx[u][3] = v.w;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1 && nr <= 8) break;  // the tile's rows 8..15 do not exist (the last tile of R = E + 1)
        uint32_t ww[8][4];
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const uint4 v = *reinterpret_cast<const uint4*>(st + (kRtTok + 8 * h + r) * 256 + 8 * lane);
          ww[r][0] = v.x; ww[r][1] = v.y; ww[r][2] = v.z; ww[r][3] = v.w;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int r = 0; r < 8; ++r)
              acc[u][8 * h + r] = fma_bf16x2_seq(xx[u][j], ww[r][j], acc[u][8 * h + r]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
  // xor-butterfly: afterwards every lane holds every sum
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int r = 0; r < kRtRows; ++r)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[u][r] += __shfl_xor_sync(0xffffffffu, acc[u][r], o);
  // lane = (token u of this warp) * 8 + (row pair): each lane writes rows 2*(lane&7) and +1
  const int u = lane >> 3, rp = lane & 7;
  const int t = 4 * warp + u;
  if (t < nt) {
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int uu = 0; uu < 4; ++uu)
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (uu == u && q == rp) {
          v0 = acc[uu][2 * q];
          v1 = acc[uu][2 * q + 1];
        }
    const int ra = r0 + 2 * rp;
    __nv_bfloat16* o = out + static_cast<int64_t>(t0 + t) * out_stride;
    if (ra < R) o[ra] = __float2bfloat16_rn(v0 + ((bias && ra < nbias) ? bias[ra] : 0.f));
    if (ra + 1 < R) o[ra + 1] = __float2bfloat16_rn(v1 + ((bias && ra + 1 < nbias) ? bias[ra + 1] : 0.f));
  }
}

// ------------------------------------------------------------------ route --
// One warp per token. Keys order logits like the reference's packed keys
// (src/drama3/kernels.py:365-369): the sign-flipped fp32 bit pattern in the
// high word (larger logit first) and the inverted column in the low word
// (lower expert id first on ties). For bf16 logits this is the same order as
// the reference's 32-bit key; for fp32 logits it keeps the full precision.
constexpr int kMaxPerLane = 32;  // E <= 1024

__device__ __forceinline__ uint64_t route_key(float v, int col) {
  const uint32_t bits = __float_as_uint(v);
  const uint32_t ordered = bits ^ ((bits & 0x80000000u) ? 0xffffffffu : 0x80000000u);
  return (static_cast<uint64_t>(ordered) << 32) | static_cast<uint32_t>(0xffffffffu - col);
}

// Routes token t with the calling warp. Lane j < k ends with pick j; the ids
// (int64), weights and, when ids_smem != nullptr, an int32 copy of the ids are
// written out.
template <int PER_LANE>
__device__ __forceinline__ void route_token(const void* __restrict__ logits, int f32_in,
                                            int64_t stride, int t, int lt, int E, int k,
                                            const float* __restrict__ bias,
                                            int64_t* __restrict__ ids, void* __restrict__ weights,
                                            int f32_out, int* ids_smem) {
  const int lane = threadIdx.x & 31;
  float v[PER_LANE];
  uint64_t key[PER_LANE];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i) {
    const int c = lane + 32 * i;
    if (c < E) {
      float l = f32_in ? static_cast<const float*>(logits)[lt * stride + c]
                       : __bfloat162float(static_cast<const __nv_bfloat16*>(logits)[lt * stride + c]);
      if (bias) l += bias[c];
      v[i] = l;
      key[i] = route_key(l, c);
      mx = fmaxf(mx, l);
    } else {
      v[i] = -INFINITY;
      key[i] = 0;
    }
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < PER_LANE; ++i)
    if (lane + 32 * i < E) sum += expf(v[i] - mx);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);

  int sel_col = 0;
  float sel_val = 0.f;  // lane j (< k) keeps pick j
  for (int j = 0; j < k; ++j) {
    uint64_t best = 0;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) best = key[i] > best ? key[i] : best;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    const int col = static_cast<int>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffu));
    float val = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; ++i) {
      if (key[i] == best) {
        val = v[i];
        key[i] = 0;
      }
    }
    // owner lane of col holds the value; broadcast it
    val = __shfl_sync(0xffffffffu, val, col & 31);
    if (lane == j) {
      sel_col = col;
      sel_val = val;
    }
  }
  const float p = (lane < k) ? expf(sel_val - mx) / sum : 0.f;
  // renormalise over the k picks in pick order
  float psum = 0.f;
  for (int j = 0; j < k; ++j) psum += __shfl_sync(0xffffffffu, p, j);
  if (lane < k) {
    ids[static_cast<int64_t>(t) * k + lane] = sel_col;
    if (ids_smem) ids_smem[t * k + lane] = sel_col;
    const float wgt = p / psum;
    if (f32_out)
      static_cast<float*>(weights)[static_cast<int64_t>(t) * k + lane] = wgt;
    else
      static_cast<__nv_bfloat16*>(weights)[static_cast<int64_t>(t) * k + lane] =
          __float2bfloat16_rn(wgt);
  }
}

// Reserved padding rows (slot >= padding_start; src/drama3/moe_input.py:32-36)
// route with row 0's logits; their ids and weights are still written to their
// own row.
template <int PER_LANE>
__global__ void route_kernel(const void* __restrict__ logits, int f32_in, int64_t stride, int T,
                             int E, int k, const float* __restrict__ bias,
                             int64_t* __restrict__ ids, void* __restrict__ weights, int f32_out,
                             PaddingRoute pr) {
  pdl_enter();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  route_token<PER_LANE>(logits, f32_in, stride, t, padding_row(pr, t) ? 0 : t, E, k, bias, ids,
                        weights, f32_out, nullptr);
}

// ---------------------------------------------------------------- permute --
// Single CTA of 1024 threads. Histogram with shared atomics (order-free), a
// block scan of padded counts, then pairs are placed chunk by chunk (1024 pairs
// per chunk, ascending) with ranks from __match_any_sync inside a warp plus the
// counts of lower warps, so each expert's list is in ascending pair order
// (a stable counting sort, like src/drama3/kernels.py:674-699).
constexpr int kPermuteThreads = 1024;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int wv = warp_tot[lane];
    int wi = wv;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    warp_tot[lane] = wi - wv;  // exclusive prefix of warps
    if (lane == 31) warp_tot[32] = wi;
  }
  __syncthreads();
  const int excl = warp_tot[warp] + incl - v;
  total = warp_tot[32];
  __syncthreads();
  return excl;
}

// id_at(p) returns the expert of pair p, or -1 for an id outside [0, E).
template <typename IdAt>
__device__ __forceinline__ void permute_body(IdAt id_at, int P, int E, int bm, int* sm,
                                             int32_t* __restrict__ counts,
                                             int32_t* __restrict__ starts,
                                             int32_t* __restrict__ total_out,
                                             int32_t* __restrict__ sorted_ids,
                                             int32_t* __restrict__ expert_ids, int64_t max_rows,
                                             int32_t* __restrict__ inv_rows,
                                             int32_t* __restrict__ active,
                                             int32_t* __restrict__ n_active) {
  int* cnt = sm;              // [E]
  int* start = cnt + E;       // [E]
  int* cursor = start + E;    // [E]
  int* wcnt = cursor + E;     // [32][E]
  __shared__ int warp_tot[33];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kPermuteThreads) cnt[e] = cursor[e] = 0;
  for (int i = tid; i < 32 * E; i += kPermuteThreads) wcnt[i] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += kPermuteThreads) {
    const int e = id_at(p);
    if (e >= 0) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  int total = 0;
  {
    const int e = tid;
    const int c = e < E ? cnt[e] : 0;
    const int padded = (c + bm - 1) / bm * bm;
    const int excl = block_exclusive_scan(e < E ? padded : 0, warp_tot, total);
    if (e < E) start[e] = excl;
  }
  __syncthreads();
  for (int base = 0; base < P; base += kPermuteThreads) {
    const int p = base + tid;
    const int e = p < P ? id_at(p) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = rank == 0;
    if (e >= 0 && leader) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int pre = 0;
      for (int w2 = 0; w2 < warp; ++w2) pre += wcnt[w2 * E + e];
      const int pos = start[e] + cursor[e] + pre + rank;
      if (sorted_ids) sorted_ids[pos] = p;
      if (inv_rows) inv_rows[p] = pos;
    } else if (p < P && inv_rows) {
      inv_rows[p] = -1;
    }
    __syncthreads();
    if (e >= 0 && leader) {
      atomicAdd(&cursor[e], __popc(peers));
      wcnt[warp * E + e] = 0;
    }
    __syncthreads();
  }
  // padding slots of each expert, per-tile expert ids
  for (int e = warp; e < E; e += kPermuteThreads / 32) {
    const int c = cnt[e], s = start[e];
    const int padded = (c + bm - 1) / bm * bm;
    if (sorted_ids)
      for (int i = c + lane; i < padded; i += 32) sorted_ids[s + i] = P;
    if (expert_ids)
      for (int b = lane; b * bm < padded; b += 32) expert_ids[s / bm + b] = e;
    if (lane == 0) {
      counts[e] = c;
      starts[e] = s;
    }
  }
  if (sorted_ids)
    for (int64_t r = total + tid; r < max_rows; r += kPermuteThreads) sorted_ids[r] = P;
  if (expert_ids)
    for (int64_t b = total / bm + tid; b < max_rows / bm; b += kPermuteThreads) expert_ids[b] = -1;
  if (tid == 0) total_out[0] = total;
  if (active) {
    int n = 0;
    const int e = tid;
    const int flag = (e < E && cnt[e] > 0) ? 1 : 0;
    const int pos = block_exclusive_scan(flag, warp_tot, n);
    if (flag) active[pos] = e;
    if (tid == 0 && n_active) n_active[0] = n;
  }
}

__global__ void __launch_bounds__(kPermuteThreads)
    permute_kernel(const int64_t* __restrict__ ids, int P, int E, int bm,
                   int32_t* __restrict__ counts, int32_t* __restrict__ starts,
                   int32_t* __restrict__ total_out, int32_t* __restrict__ sorted_ids,
                   int32_t* __restrict__ expert_ids, int64_t max_rows,
                   int32_t* __restrict__ inv_rows, int32_t* __restrict__ active,
                   int32_t* __restrict__ n_active) {
  pdl_enter();
  extern __shared__ int sm[];
  auto id_at = [&](int p) -> int {
    const int64_t v = ids[p];
    return (v >= 0 && v < E) ? static_cast<int>(v) : -1;
  };
  permute_body(id_at, P, E, bm, sm, counts, starts, total_out, sorted_ids, expert_ids, max_rows,
               inv_rows, active, n_active);
}

// Prefill-size permute over many CTAs: the same stable counting sort as
// permute_body, split into three kernels over chunks of consecutive pairs.
//   hist:    chunk c counts its pairs per expert        -> cc[c][e]
//   scan:    one CTA: counts, padded starts, and cc[c][e] rewritten to the
//            first slot of chunk c's pairs of expert e (start[e] + sum of
//            cc[c'][e] for c' < c); padding slots, tile experts, active list
//   scatter: chunk c places its pairs from cc[c][e] on, in ascending pair
//            order (ranks from __match_any_sync and lower warps' counts)
// Ascending chunk bases + ascending order inside a chunk give the same
// sorted_ids as the single-CTA kernel.
constexpr int kMaxPermuteChunks = 256;
constexpr int kChunkedPermuteMinPairs = 8192;

inline int permute_chunk_pairs(int P) {
  const int per = (P + kMaxPermuteChunks - 1) / kMaxPermuteChunks;
  return ((per + kPermuteThreads - 1) / kPermuteThreads) * kPermuteThreads;
}

__global__ void __launch_bounds__(kPermuteThreads)
    permute_hist_kernel(const int64_t* __restrict__ ids, int P, int E, int chunk,
                        int32_t* __restrict__ cc) {
  pdl_enter();
  extern __shared__ int cnt[];
  for (int e = threadIdx.x; e < E; e += kPermuteThreads) cnt[e] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * chunk, p1 = min(P, p0 + chunk);
  for (int p = p0 + threadIdx.x; p < p1; p += kPermuteThreads) {
    const int64_t v = ids[p];
    if (v >= 0 && v < E) atomicAdd(&cnt[v], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kPermuteThreads)
    cc[static_cast<int64_t>(blockIdx.x) * E + e] = cnt[e];
}

__global__ void __launch_bounds__(kPermuteThreads)
    permute_scan_kernel(int32_t* __restrict__ cc, int chunks, int P, int E, int bm,
                        int32_t* __restrict__ counts, int32_t* __restrict__ starts,
                        int32_t* __restrict__ total_out, int32_t* __restrict__ sorted_ids,
                        int32_t* __restrict__ expert_ids, int64_t max_rows,
                        int32_t* __restrict__ active, int32_t* __restrict__ n_active) {
  pdl_enter();
  __shared__ int warp_tot[33];
  __shared__ int s_cnt[1024], s_start[1024];
  __shared__ int s_part[kPermuteThreads];  // [part][E] chunk-slice sums, then their offsets
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // parts threads per expert, each owning a contiguous slice of the chunks
  // (coalesced over e, independent loads); the slices are combined in part
  // order, so every expert's running offsets are the sequential ones.
  const int parts = E <= kPermuteThreads ? kPermuteThreads / E : 1;
  const int part = tid / E, e_mine = tid - part * E;
  const bool owner = part < parts && e_mine < E;
  const int per = (chunks + parts - 1) / parts;
  const int c0 = part * per, c1 = min(chunks, c0 + per);
  int slice = 0;
  if (owner) {
#pragma unroll 8
    for (int c = c0; c < c1; ++c) slice += cc[static_cast<int64_t>(c) * E + e_mine];
    s_part[part * E + e_mine] = slice;
  }
  __syncthreads();
  const int e = tid;
  int c_tot = 0;
  if (e < E) {
    for (int p = 0; p < parts; ++p) {
      const int v = s_part[p * E + e];
      s_part[p * E + e] = c_tot;  // exclusive offset of slice p
      c_tot += v;
    }
  }
  const int padded = (c_tot + bm - 1) / bm * bm;
  int total = 0;
  const int start = block_exclusive_scan(e < E ? padded : 0, warp_tot, total);
  if (e < E) {
    s_cnt[e] = c_tot;
    s_start[e] = start;
    counts[e] = c_tot;
    starts[e] = start;
  }
  __syncthreads();
  if (owner) {
    int run = s_start[e_mine] + s_part[part * E + e_mine];
#pragma unroll 8
    for (int c = c0; c < c1; ++c) {
      const int64_t i = static_cast<int64_t>(c) * E + e_mine;
      const int v = cc[i];
      cc[i] = run;
      run += v;
    }
  }
  for (int ee = warp; ee < E; ee += kPermuteThreads / 32) {
    const int c = s_cnt[ee], s = s_start[ee];
    const int pd = (c + bm - 1) / bm * bm;
    if (sorted_ids)
      for (int i = c + lane; i < pd; i += 32) sorted_ids[s + i] = P;
    if (expert_ids)
      for (int b = lane; b * bm < pd; b += 32) expert_ids[s / bm + b] = ee;
  }
  if (sorted_ids)
    for (int64_t r = total + tid; r < max_rows; r += kPermuteThreads) sorted_ids[r] = P;
  if (expert_ids)
    for (int64_t b = total / bm + tid; b < max_rows / bm; b += kPermuteThreads) expert_ids[b] = -1;
  if (tid == 0) total_out[0] = total;
  if (active) {
    int n = 0;
    const int flag = (e < E && c_tot > 0) ? 1 : 0;
    const int pos = block_exclusive_scan(flag, warp_tot, n);
    if (flag) active[pos] = e;
    if (tid == 0 && n_active) n_active[0] = n;
  }
}

__global__ void __launch_bounds__(kPermuteThreads)
    permute_scatter_kernel(const int64_t* __restrict__ ids, int P, int E, int chunk,
                           const int32_t* __restrict__ cc, int32_t* __restrict__ sorted_ids,
                           int32_t* __restrict__ inv_rows) {
  pdl_enter();
  extern __shared__ int sm[];
  int* cursor = sm;        // [E]
  int* wcnt = sm + E;      // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += kPermuteThreads) cursor[e] = cc[static_cast<int64_t>(blockIdx.x) * E + e];
  for (int i = tid; i < 32 * E; i += kPermuteThreads) wcnt[i] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * chunk, p1 = min(P, p0 + chunk);
  for (int base = p0; base < p1; base += kPermuteThreads) {
    const int p = base + tid;
    int e = -1;
    if (p < p1) {
      const int64_t v = ids[p];
      e = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = rank == 0;
    if (e >= 0 && leader) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int pre = 0;
      for (int w2 = 0; w2 < warp; ++w2) pre += wcnt[w2 * E + e];
      const int pos = cursor[e] + pre + rank;
      if (sorted_ids) sorted_ids[pos] = p;
      if (inv_rows) inv_rows[p] = pos;
    } else if (p < p1 && inv_rows) {
      inv_rows[p] = -1;
    }
    __syncthreads();
    if (e >= 0 && leader) {
      atomicAdd(&cursor[e], __popc(peers));
      wcnt[warp * E + e] = 0;
    }
    __syncthreads();
  }
}

constexpr int kPlanRowsThreads = 1024;
constexpr int kPlanRowsMaxRanks = 32;

// Expert-parallel dispatch plan, one packed row per (token, owning rank):
// rank d needs token t when it owns at least one of t's k experts (owner =
// id / experts_per_rank). Rows are ordered by destination rank, then token;
// slot[t*ranks + d] = the row's index in the send buffer (-1 when d needs no
// row of t) and send_counts[d] = rows for d. One CTA: pass 1 counts, pass 2
// writes the slots (a ballot + popcount scan per rank and 1024-token chunk).
__global__ void __launch_bounds__(kPlanRowsThreads)
    ep_plan_rows_kernel(const int64_t* __restrict__ ids, int T, int k, int experts_per_rank,
                        int ranks, int32_t* __restrict__ send_counts, int32_t* __restrict__ slot) {
  pdl_enter();
  __shared__ int warp_cnt[32][kPlanRowsMaxRanks];  // rows of this chunk per (warp, rank)
  __shared__ int warp_off[32][kPlanRowsMaxRanks];  // exclusive prefix over warps
  __shared__ int base[kPlanRowsMaxRanks];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t owned = static_cast<int64_t>(experts_per_rank) * ranks;
  auto need_mask = [&](int t) -> uint32_t {
    uint32_t m = 0;
    if (t < T)
      for (int j = 0; j < k; ++j) {
        const int64_t e = ids[static_cast<int64_t>(t) * k + j];
        if (e >= 0 && e < owned) m |= 1u << static_cast<int>(e / experts_per_rank);
      }
    return m;
  };
  if (tid < ranks) base[tid] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < T; c0 += kPlanRowsThreads) {  // pass 1: rows per rank
    const uint32_t m = need_mask(c0 + tid);
    for (int d = 0; d < ranks; ++d) {
      const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
      if (lane == 0) warp_cnt[warp][d] = __popc(b);
    }
    __syncthreads();
    if (tid < ranks) {
      int s = 0;
      for (int w = 0; w < kPlanRowsThreads / 32; ++w) s += warp_cnt[w][tid];
      base[tid] += s;
    }
    __syncthreads();
  }
  if (tid == 0) {
    int run = 0;
    for (int d = 0; d < ranks; ++d) {
      const int n = base[d];
      send_counts[d] = n;
      base[d] = run;
      run += n;
    }
  }
  __syncthreads();
  for (int c0 = 0; c0 < T; c0 += kPlanRowsThreads) {  // pass 2: slots
    const int t = c0 + tid;
    const uint32_t m = need_mask(t);
    for (int d = 0; d < ranks; ++d) {
      const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
      if (lane == 0) warp_cnt[warp][d] = __popc(b);
    }
    __syncthreads();
    if (warp < ranks) {  // warp d scans rank d's per-warp counts
      const int v = warp_cnt[lane][warp];
      int incl = v;
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      warp_off[lane][warp] = incl - v;
    }
    __syncthreads();
    const unsigned lt = (1u << lane) - 1u;
    for (int d = 0; d < ranks; ++d) {
      const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
      if (t < T)
        slot[static_cast<int64_t>(t) * ranks + d] =
            ((m >> d) & 1u) ? base[d] + warp_off[warp][d] + __popc(b & lt) : -1;
    }
    __syncthreads();
    if (tid < ranks) base[tid] += warp_off[31][tid] + warp_cnt[31][tid];
    __syncthreads();
  }
}

}  // namespace

namespace {

// dst bf16 [T, H] = x[keep[t]] (a keep value outside [0, x_rows) records
// kDevBadRow and reads row 0, as every row-map reader does). The tensor-core
// router reads its rows by TMA, which cannot follow the map; the reference
// materialises the kept rows the same way (x.index_select) before its router.
__global__ void gather_keep_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T,
                                        int H, RowGather rg, __nv_bfloat16* __restrict__ dst) {
  pdl_enter();
  const int per_row = H / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(T) * per_row) return;
  const int64_t t = idx / per_row;
  const int c = static_cast<int>(idx - t * per_row);
  const uint4* src = reinterpret_cast<const uint4*>(x + gather_row(rg, t) * x_stride);
  reinterpret_cast<uint4*>(dst + t * H)[c] = __ldg(src + c);
}

bool router_tc_fits(const void* x, int64_t x_stride, const void* w, int R, int H) {
  return H % 64 == 0 && x_stride % 8 == 0 && aligned(x, 16) && aligned(w, 16) && R <= 4 * kRtcMaxN;
}

// The tensor-core router (router_tc.cuh) for contiguous x with a TMA-able
// layout; false when the layout does not allow it (the caller then runs the
// CUDA-core kernel).
bool launch_router_tc(const void* x, int64_t x_stride, const void* w, const float* bias, int nbias,
                      int R, int H, int T, void* logits, int64_t logits_stride, cudaStream_t s,
                      int32_t* status) {
  if (!router_tc_fits(x, x_stride, w, R, H)) return false;
  // enough row tiles for the grid to cover the SMs (every CTA streams its
  // token tile's x once, so splitting the rows multiplies only L2 reads of x)
  const int mtiles = (T + kRtcTokens - 1) / kRtcTokens;
  const int min_tiles = (R + kRtcMaxN - 1) / kRtcMaxN;
  const int max_tiles = (R + 15) / 16;
  const int want = (sm_count() + mtiles - 1) / mtiles;
  const int ntiles = want < min_tiles ? min_tiles : (want > max_tiles ? max_tiles : want);
  const int nt = ((R + ntiles - 1) / ntiles + 15) / 16 * 16;
  int cols = 32;
  while (cols < nt) cols <<= 1;
  CUtensorMap tx, tw;
  if (encode_tmap_2d(&tx, x, 2, H, T, static_cast<uint64_t>(x_stride) * 2, 64, kRtcTokens)) return false;
  if (encode_tmap_2d(&tw, w, 2, H, R, static_cast<uint64_t>(H) * 2, 64, nt)) return false;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(RtcSmem::bytes(kRtcMaxN)));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  RouterTcArgs a{};
  a.bias = bias;
  a.nbias = nbias;
  a.R = R;
  a.T = T;
  a.KB = H / 64;
  a.nt = nt;
  a.tmem_cols = cols;
  a.out = static_cast<__nv_bfloat16*>(logits);
  a.out_stride = logits_stride;
  a.status = status;
  launch_kernel(router_tc_kernel, dim3(mtiles, (R + nt - 1) / nt), dim3(kRtcThreads),
                RtcSmem::bytes(nt), s, tx, tw, a);
  return true;
}

}  // namespace

void launch_router_logits(const void* x, int64_t x_stride, const void* w, const float* bias,
                          int nbias, int R, int H, int T, void* logits, int64_t logits_stride,
                          cudaStream_t s, const RowGather& rg, int32_t* status,
                          void* gather_scratch) {
  if (T <= 0 || R <= 0) return;
  if (T >= kRouterTcMinTokens && rg.keep == nullptr &&
      launch_router_tc(x, x_stride, w, bias, nbias, R, H, T, logits, logits_stride, s, status))
    return;
  if (T >= kRouterTcMinTokens && rg.keep != nullptr && gather_scratch &&
      router_tc_fits(gather_scratch, H, w, R, H)) {
    const int64_t n = static_cast<int64_t>(T) * (H / 8);
    launch_kernel(gather_keep_rows_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, s,
                  static_cast<const __nv_bfloat16*>(x), x_stride, T, H, rg,
                  static_cast<__nv_bfloat16*>(gather_scratch));
    if (launch_router_tc(gather_scratch, H, w, bias, nbias, R, H, T, logits, logits_stride, s, status))
      return;
  }
  if (T >= kRouterTiledMinTokens) {
    static bool configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !configured[dev]) {
      cudaFuncSetAttribute(router_logits_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kRtSmem));
      if (dev >= 0 && dev < 64) configured[dev] = true;
    }
    dim3 grid((R + kRtRows - 1) / kRtRows, (T + kRtTok - 1) / kRtTok);
    launch_kernel(router_logits_tiled_kernel, dim3(grid), dim3(kRtThreads), kRtSmem, s, 
        static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(w), bias,
        nbias, R, H, T, static_cast<__nv_bfloat16*>(logits), logits_stride, rg);
    return;
  }
  dim3 grid((R + kRouterRows - 1) / kRouterRows, (T + kRouterTokens - 1) / kRouterTokens);
  const size_t smem = static_cast<size_t>(kRouterTokens) * H * 2;  // <= 48 KB for H <= 3072
  launch_kernel(router_logits_kernel, dim3(grid), dim3(256), smem, s, 
      static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(w), bias,
      nbias, R, H, T, static_cast<__nv_bfloat16*>(logits), logits_stride, rg);
}

void launch_route_topk(const void* logits, int logits_dtype, int64_t stride, int T, int E, int k,
                       const float* bias, int64_t* ids, void* weights, int weights_dtype,
                       cudaStream_t s, const PaddingRoute& pr) {
  if (T <= 0) return;
  const unsigned grid = static_cast<unsigned>((T + 7) / 8);
  const int f32_in = logits_dtype == D3_DTYPE_F32, f32_out = weights_dtype == D3_DTYPE_F32;
  const int per_lane = (E + 31) / 32;
  if (per_lane <= 4)
    launch_kernel(route_kernel<4>, dim3(grid), dim3(256), 0, s, logits, f32_in, stride, T, E, k, bias, ids, weights, f32_out, pr);
  else if (per_lane <= 8)
    launch_kernel(route_kernel<8>, dim3(grid), dim3(256), 0, s, logits, f32_in, stride, T, E, k, bias, ids, weights, f32_out, pr);
  else
    launch_kernel(route_kernel<kMaxPerLane>, dim3(grid), dim3(256), 0, s, logits, f32_in, stride, T, E, k, bias, ids, weights, f32_out, pr);
}

int launch_route_permute(const void* logits, int logits_dtype, int64_t stride, int T, int E,
                         int k, const float* bias, int64_t* ids, void* weights, int weights_dtype,
                         int block_m, int32_t* counts, int32_t* starts, int32_t* total,
                         int32_t* sorted_ids, int32_t* expert_ids, int64_t max_rows,
                         int32_t* inv_rows, int32_t* active, int32_t* n_active, cudaStream_t s,
                         int32_t* scratch, const PaddingRoute& pr) {
  if (T <= 0) return D3_OK;
  // routing spreads tokens over many CTAs (a warp each); a single-CTA fusion
  // of routing and bucketing measured slower than the two launches
  launch_route_topk(logits, logits_dtype, stride, T, E, k, bias, ids, weights, weights_dtype, s, pr);
  int rc = check_launch("route_topk");
  if (rc) return rc;
  return launch_permute(ids, T, k, E, block_m, counts, starts, total, sorted_ids, expert_ids,
                        max_rows, inv_rows, active, n_active, s, scratch);
}

size_t permute_scratch_ints(int E) { return static_cast<size_t>(kMaxPermuteChunks) * E; }

int launch_permute(const int64_t* ids, int T, int k, int E, int block_m, int32_t* counts,
                   int32_t* starts, int32_t* total, int32_t* sorted_ids, int32_t* expert_ids,
                   int64_t max_rows, int32_t* inv_rows, int32_t* active, int32_t* n_active,
                   cudaStream_t s, int32_t* scratch) {
  const int P = T * k;
  if (scratch && P >= kChunkedPermuteMinPairs) {
    const int chunk = permute_chunk_pairs(P);
    const int chunks = (P + chunk - 1) / chunk;
    const size_t scatter_smem = static_cast<size_t>(E) * 33 * sizeof(int);
    static bool conf_scatter[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (scatter_smem > 48 * 1024 && dev >= 0 && dev < 64 && !conf_scatter[dev]) {
      if (cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               33 * 1024 * 4) != cudaSuccess)
        return set_error(D3_ECUDA, "permute: cannot raise the shared-memory limit");
      conf_scatter[dev] = true;
    }
    launch_kernel(permute_hist_kernel, dim3(chunks), dim3(kPermuteThreads), static_cast<size_t>(E) * sizeof(int), s, 
        ids, P, E, chunk, scratch);
    launch_kernel(permute_scan_kernel, dim3(1), dim3(kPermuteThreads), 0, s, scratch, chunks, P, E, block_m, counts,
                                                      starts, total, sorted_ids, expert_ids,
                                                      max_rows, active, n_active);
    launch_kernel(permute_scatter_kernel, dim3(chunks), dim3(kPermuteThreads), scatter_smem, s, ids, P, E, chunk, scratch,
                                                                         sorted_ids, inv_rows);
    return check_launch("moe_permute (chunked)");
  }
  const size_t smem = static_cast<size_t>(E) * 35 * sizeof(int);
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (smem > 48 * 1024 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             35 * 1024 * 4) != cudaSuccess)
      return set_error(D3_ECUDA, "permute: cannot raise the shared-memory limit");
    configured[dev] = true;
  }
  launch_kernel(permute_kernel, dim3(1), dim3(kPermuteThreads), smem, s, ids, T * k, E, block_m, counts, starts, total,
                                                   sorted_ids, expert_ids, max_rows, inv_rows,
                                                   active, n_active);
  return check_launch("moe_permute");
}

}  // namespace d3

using namespace d3;

extern "C" int d3_router_logits(const void* x, int64_t x_stride, const void* w, const float* bias,
                                int nbias, int R, int H, int T, void* logits, int64_t logits_stride,
                                d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && R > 0 && H > 0 && H % 128 == 0, "router_logits: bad shape R=%d H=%d", R, H);
  D3_REQUIRE(T >= kRouterTiledMinTokens || H <= 256 * kRouterMaxIters,
             "router_logits: H=%d above the %d the decode kernel holds in registers", H,
             256 * kRouterMaxIters);
  D3_REQUIRE(x_stride >= H && x_stride % 8 == 0, "router_logits: x row stride must be >= H and a multiple of 8");
  D3_REQUIRE(logits_stride >= R, "router_logits: logits row stride must be >= R");
  D3_REQUIRE(aligned(x, 16) && aligned(w, 16), "router_logits: misaligned pointer");
  D3_REQUIRE(nbias >= 0 && nbias <= R && (bias != nullptr || nbias == 0),
             "router_logits: nbias=%d must be in [0, R] with a bias pointer", nbias);
  launch_router_logits(x, x_stride, w, bias, nbias, R, H, T, logits, logits_stride,
                       reinterpret_cast<cudaStream_t>(stream));
  return check_launch("router_logits");
}

extern "C" int d3_route_topk(const void* logits, int logits_dtype, int64_t stride, int T, int E,
                             int k, const float* bias, int64_t* ids, void* weights,
                             int weights_dtype, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && E > 0 && E <= 1024, "route_topk: E=%d must be in [1, 1024]", E);
  D3_REQUIRE(k > 0 && k <= 32 && k <= E, "route_topk: k=%d must be in [1, min(32, E)]", k);
  D3_REQUIRE(stride >= E, "route_topk: logits row stride must be >= E");
  D3_REQUIRE(logits_dtype == D3_DTYPE_BF16 || logits_dtype == D3_DTYPE_F32, "route_topk: logits must be bf16 or f32");
  D3_REQUIRE(weights_dtype == D3_DTYPE_BF16 || weights_dtype == D3_DTYPE_F32, "route_topk: weights must be bf16 or f32");
  launch_route_topk(logits, logits_dtype, stride, T, E, k, bias, ids, weights, weights_dtype,
                    reinterpret_cast<cudaStream_t>(stream));
  return check_launch("route_topk");
}

extern "C" int d3_route_topk_rows(const void* logits, int logits_dtype, int64_t stride, int T,
                                  int E, int k, const float* bias, const void* row_slots,
                                  int row_slots_int64, int64_t padding_start, int64_t* ids,
                                  void* weights, int weights_dtype, d3_stream_t stream) {
  D3_REQUIRE(row_slots == nullptr || padding_start > 0,
             "route_topk_rows: padding_start must be a positive reserved-slot boundary");
  D3_REQUIRE(T >= 0 && E > 0 && E <= 1024, "route_topk: E=%d must be in [1, 1024]", E);
  D3_REQUIRE(k > 0 && k <= 32 && k <= E, "route_topk: k=%d must be in [1, min(32, E)]", k);
  D3_REQUIRE(stride >= E, "route_topk: logits row stride must be >= E");
  D3_REQUIRE(logits_dtype == D3_DTYPE_BF16 || logits_dtype == D3_DTYPE_F32, "route_topk: logits must be bf16 or f32");
  D3_REQUIRE(weights_dtype == D3_DTYPE_BF16 || weights_dtype == D3_DTYPE_F32, "route_topk: weights must be bf16 or f32");
  PaddingRoute pr;
  pr.slots = row_slots;
  pr.slots_i64 = row_slots_int64 ? 1 : 0;
  pr.padding_start = padding_start;
  launch_route_topk(logits, logits_dtype, stride, T, E, k, bias, ids, weights, weights_dtype,
                    reinterpret_cast<cudaStream_t>(stream), pr);
  return check_launch("route_topk");
}

extern "C" int d3_moe_permute(const int64_t* ids, int T, int k, int E, int block_m,
                              int32_t* counts, int32_t* starts, int32_t* total,
                              int32_t* sorted_ids, int32_t* expert_ids, int64_t max_rows,
                              int32_t* inv_rows, int32_t* active, int32_t* n_active,
                              d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && E > 0 && E <= 1024, "moe_permute: E=%d must be in [1, 1024]", E);
  D3_REQUIRE(block_m > 0, "moe_permute: block_m must be positive");
  const int64_t P = static_cast<int64_t>(T) * k;
  D3_REQUIRE(P < (1ll << 30), "moe_permute: too many pairs");
  const int64_t need = (P + (P < E ? P : E) * (block_m - 1) + block_m - 1) / block_m * block_m;
  D3_REQUIRE(max_rows >= need, "moe_permute: max_rows %lld < required %lld", (long long)max_rows, (long long)need);
  D3_REQUIRE(max_rows % block_m == 0, "moe_permute: max_rows must be a multiple of block_m");
  return launch_permute(ids, T, k, E, block_m, counts, starts, total, sorted_ids, expert_ids,
                        max_rows, inv_rows, active, n_active, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int d3_moe_permute_scratch_size(int E, size_t* bytes) {
  D3_REQUIRE(bytes != nullptr && E > 0 && E <= 1024, "moe_permute_scratch_size: bad arguments");
  *bytes = permute_scratch_ints(E) * sizeof(int32_t);
  return D3_OK;
}

extern "C" int d3_moe_permute_chunked(const int64_t* ids, int T, int k, int E, int block_m,
                                      int32_t* counts, int32_t* starts, int32_t* total,
                                      int32_t* sorted_ids, int32_t* expert_ids, int64_t max_rows,
                                      int32_t* inv_rows, int32_t* active, int32_t* n_active,
                                      int32_t* scratch, size_t scratch_bytes, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && E > 0 && E <= 1024, "moe_permute: E=%d must be in [1, 1024]", E);
  D3_REQUIRE(block_m > 0, "moe_permute: block_m must be positive");
  const int64_t P = static_cast<int64_t>(T) * k;
  D3_REQUIRE(P < (1ll << 30), "moe_permute: too many pairs");
  const int64_t need = (P + (P < E ? P : E) * (block_m - 1) + block_m - 1) / block_m * block_m;
  D3_REQUIRE(max_rows >= need, "moe_permute: max_rows %lld < required %lld", (long long)max_rows, (long long)need);
  D3_REQUIRE(max_rows % block_m == 0, "moe_permute: max_rows must be a multiple of block_m");
  D3_REQUIRE(scratch != nullptr && aligned(scratch, 16) &&
                 scratch_bytes >= permute_scratch_ints(E) * sizeof(int32_t),
             "moe_permute_chunked: scratch must hold %zu bytes", permute_scratch_ints(E) * sizeof(int32_t));
  return launch_permute(ids, T, k, E, block_m, counts, starts, total, sorted_ids, expert_ids,
                        max_rows, inv_rows, active, n_active, reinterpret_cast<cudaStream_t>(stream),
                        scratch);
}

extern "C" int d3_ep_plan_rows(const int64_t* ids, int T, int k, int experts_per_rank, int ranks,
                               int32_t* send_counts, int32_t* slot, d3_stream_t stream) {
  D3_REQUIRE(T >= 0 && k > 0 && experts_per_rank > 0 && ranks > 0 && ranks <= kPlanRowsMaxRanks,
             "ep_plan_rows: bad arguments T=%d k=%d experts_per_rank=%d ranks=%d (ranks <= %d)", T, k,
             experts_per_rank, ranks, kPlanRowsMaxRanks);
  D3_REQUIRE(ids && send_counts && slot, "ep_plan_rows: null pointer");
  D3_REQUIRE(static_cast<int64_t>(T) * ranks < (int64_t{1} << 31), "ep_plan_rows: too many rows");
  launch_kernel(ep_plan_rows_kernel, dim3(1), dim3(kPlanRowsThreads), 0, reinterpret_cast<cudaStream_t>(stream),
                ids, T, k, experts_per_rank, ranks, send_counts, slot);
  return check_launch("ep_plan_rows");
}
