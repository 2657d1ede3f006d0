// Residual update + Gemma RMSNorm epilogues (the layer's exit):
//   add_norm                  residual <- bf16(x + residual);           out = norm(residual)
//   combine_experts_add_norm  residual <- bf16(fma.rn.bf16(shared, bf16(sigmoid(g)), routed)
//                                              + residual);              out = norm(residual)
//   (expert-row form)         the same, with routed = bf16(sum_r w_r * d[row_r]) and
//                             shared = bf16(d[P + t]) read straight from the down rows, so the
//                             routed/shared bf16 tensors never go through HBM
// norm(v) = bf16(v * rsqrt(mean(v^2) + eps) * (1 + w)), fp32.
// Reference: src/drama3/kernels.py:405-423 (add_norm), :448-499
// (combine_experts_add_norm), :502-556 (the _inverse form).
//
// One 256-thread CTA per row; each thread owns W / 2048 chunks of 8 columns
// (W a multiple of 8, at most 8192), so the row stays in registers between the
// residual update and the normalisation.
#include "d3_common.cuh"
#include "d3_host.h"

namespace d3 {

namespace {

constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;  // W <= 4 * 8 * 256 = 8192

// NS_ROWS: fp32 expert rows; NS_ROWS_BF16: the bf16 expert rows of the
// tcgen05 path.
enum NormSrc { NS_ADD = 0, NS_COMBINE = 1, NS_ROWS = 2, NS_ROWS_BF16 = 3 };


__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&f)[8]) {
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    o[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 consecutive values of an expert row as fp32.
template <int SRC>
__device__ __forceinline__ void load_row8(const void* d, int64_t row, int W, int c, float (&f)[8]) {
  if constexpr (SRC == NS_ROWS_BF16) {
    load_bf16x8(static_cast<const __nv_bfloat16*>(d) + row * W + c, f);
  } else {
    const float* p = static_cast<const float*>(d) + row * W + c;
    const float4 lo = *reinterpret_cast<const float4*>(p);
    const float4 hi = *reinterpret_cast<const float4*>(p + 4);
    f[0] = lo.x; f[1] = lo.y; f[2] = lo.z; f[3] = lo.w;
    f[4] = hi.x; f[5] = hi.y; f[6] = hi.z; f[7] = hi.w;
  }
}

// combined = fma.rn.bf16(shared, gate, routed) for 8 columns (inputs are bf16
// values held in fp32; the product is exact and the sum is rounded once).
__device__ __forceinline__ void combine_fma(const float (&shared)[8], float gate,
                                            const float (&routed)[8], float (&out)[8]) {
  const __nv_bfloat16 g = __float2bfloat16_rn(gate);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    out[i] = __bfloat162float(__hfma(__float2bfloat16_rn(shared[i]), g, __float2bfloat16_rn(routed[i])));
}

__device__ __forceinline__ float sigmoid_bf16(const __nv_bfloat16* gate) {
  const float g = __bfloat162float(*gate);
  return bf16_round(1.0f / (1.0f + expf(-g)));
}

template <int SRC>
__global__ void __launch_bounds__(kNormThreads)
    add_norm_kernel(const void* __restrict__ p0, const void* __restrict__ p1,
                    const __nv_bfloat16* __restrict__ gate, int64_t gate_stride,
                    const int32_t* __restrict__ inverse, const int32_t* __restrict__ inv_rows,
                    const __nv_bfloat16* __restrict__ weights, int k, int P,
                    __nv_bfloat16* __restrict__ residual, const __nv_bfloat16* __restrict__ norm_w,
                    float eps, int W, __nv_bfloat16* __restrict__ out, RowGather rows) {
  pdl_enter();
  __shared__ float red[kNormThreads / 32];
  const int row = blockIdx.x;
  const int nchunks = W / 8;
  float v[kNormMaxChunks][8];
  float ss = 0.f;
  const int src = (SRC == NS_COMBINE && inverse) ? inverse[row]
                  : (SRC == NS_ROWS || SRC == NS_ROWS_BF16) ? static_cast<int>(gather_row(rows, row)) : row;
  float g = 0.f;
  if (SRC != NS_ADD) g = sigmoid_bf16(gate + static_cast<int64_t>(src) * gate_stride);
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int ch = threadIdx.x + kNormThreads * j;
    if (ch >= nchunks) break;
    const int c = 8 * ch;
    float res[8], val[8];
    load_bf16x8(residual + static_cast<int64_t>(row) * W + c, res);
    if constexpr (SRC == NS_ADD) {
      float a[8];
      load_bf16x8(static_cast<const __nv_bfloat16*>(p0) + static_cast<int64_t>(row) * W + c, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) val[i] = a[i];
    } else {
      float routed[8], shared[8];
      if constexpr (SRC == NS_COMBINE) {
        load_bf16x8(static_cast<const __nv_bfloat16*>(p0) + static_cast<int64_t>(src) * W + c, routed);
        load_bf16x8(static_cast<const __nv_bfloat16*>(p1) + static_cast<int64_t>(src) * W + c, shared);
      } else {
        // expert rows: fp32 rank-order sum weighted by the bf16 routing weight
        const void* d = p0;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int r = 0; r < k; ++r) {
          const int dr = inv_rows[src * k + r];
          if (dr < 0) continue;
          const float w = __bfloat162float(weights[src * k + r]);
          float v[8];
          load_row8<SRC>(d, dr, W, c, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += v[i] * w;
        }
        float sh[8];
        load_row8<SRC>(d, P + src, W, c, sh);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          routed[i] = bf16_round(acc[i]);
          shared[i] = bf16_round(sh[i]);
        }
      }
      combine_fma(shared, g, routed, val);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      val[i] = bf16_round(val[i] + res[i]);
      v[j][i] = val[i];
      ss = fmaf(val[i], val[i], ss);
    }
    *reinterpret_cast<uint4*>(residual + static_cast<int64_t>(row) * W + c) = pack_bf16x8(val);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  const float rs = rsqrtf(tot / static_cast<float>(W) + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxChunks; ++j) {
    const int ch = threadIdx.x + kNormThreads * j;
    if (ch >= nchunks) break;
    const int c = 8 * ch;
    float wn[8], o[8];
    load_bf16x8(norm_w + c, wn);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[j][i] * rs) * (1.0f + wn[i]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * W + c) = pack_bf16x8(o);
  }
}

int check_norm_args(const void* residual, const void* norm_w, const void* out, int T, int W,
                    const char* what) {
  D3_REQUIRE(T >= 0 && W > 0 && W % 8 == 0 && W <= 8 * kNormThreads * kNormMaxChunks,
             "%s: W=%d must be a positive multiple of 8 up to %d", what, W,
             8 * kNormThreads * kNormMaxChunks);
  D3_REQUIRE(residual && norm_w && out && aligned(residual, 16) && aligned(norm_w, 16) && aligned(out, 16),
             "%s: null or misaligned residual / weight / output", what);
  return D3_OK;
}

}  // namespace

int launch_combine_rows_add_norm(const float* d, int W, const int32_t* inv_rows,
                                 const void* weights, int T, int k, const void* gate,
                                 int64_t gate_stride, void* residual, const void* norm_w, float eps,
                                 void* out, cudaStream_t s, const int64_t* inverse, int T_out,
                                 int32_t* status, bool rows_bf16) {
  if (T <= 0) return D3_OK;
  RowGather rows;
  rows.keep = inverse;
  rows.x_rows = T;
  rows.status = status;
  const int nrows = inverse ? T_out : T;
  if (nrows <= 0) return D3_OK;
  launch_kernel(rows_bf16 ? add_norm_kernel<NS_ROWS_BF16> : add_norm_kernel<NS_ROWS>, dim3(nrows),
                dim3(kNormThreads), 0, s,
                static_cast<const void*>(d), static_cast<const void*>(nullptr),
                static_cast<const __nv_bfloat16*>(gate), gate_stride,
                static_cast<const int32_t*>(nullptr), inv_rows,
                static_cast<const __nv_bfloat16*>(weights), k, T * k,
                static_cast<__nv_bfloat16*>(residual), static_cast<const __nv_bfloat16*>(norm_w), eps,
                W, static_cast<__nv_bfloat16*>(out), rows);
  return check_launch("combine_rows_add_norm");
}

}  // namespace d3

using namespace d3;

extern "C" int d3_add_norm(const void* x, void* residual, const void* weight, float eps, int T,
                           int W, void* out, d3_stream_t stream) {
  int rc = check_norm_args(residual, weight, out, T, W, "add_norm");
  if (rc) return rc;
  D3_REQUIRE(x && aligned(x, 16), "add_norm: null or misaligned x");
  if (T == 0) return D3_OK;
  launch_kernel(add_norm_kernel<NS_ADD>, dim3(T), dim3(kNormThreads), 0,
                reinterpret_cast<cudaStream_t>(stream), x, static_cast<const void*>(nullptr),
                static_cast<const __nv_bfloat16*>(nullptr), int64_t{0},
                static_cast<const int32_t*>(nullptr), static_cast<const int32_t*>(nullptr),
                static_cast<const __nv_bfloat16*>(nullptr), 0, 0,
                static_cast<__nv_bfloat16*>(residual), static_cast<const __nv_bfloat16*>(weight), eps,
                W, static_cast<__nv_bfloat16*>(out), RowGather{});
  return check_launch("add_norm");
}

extern "C" int d3_combine_experts_add_norm(const void* routed, const void* shared,
                                           const void* gate, int64_t gate_stride,
                                           const int32_t* inverse, int T, int W, void* residual,
                                           const void* weight, float eps, void* out,
                                           d3_stream_t stream) {
  int rc = check_norm_args(residual, weight, out, T, W, "combine_experts_add_norm");
  if (rc) return rc;
  D3_REQUIRE(routed && shared && gate && aligned(routed, 16) && aligned(shared, 16),
             "combine_experts_add_norm: null or misaligned routed / shared / gate");
  if (T == 0) return D3_OK;
  launch_kernel(add_norm_kernel<NS_COMBINE>, dim3(T), dim3(kNormThreads), 0,
                reinterpret_cast<cudaStream_t>(stream), routed, shared,
                static_cast<const __nv_bfloat16*>(gate), gate_stride, inverse,
                static_cast<const int32_t*>(nullptr), static_cast<const __nv_bfloat16*>(nullptr), 0, 0,
                static_cast<__nv_bfloat16*>(residual), static_cast<const __nv_bfloat16*>(weight), eps,
                W, static_cast<__nv_bfloat16*>(out), RowGather{});
  return check_launch("combine_experts_add_norm");
}
