// LayerNorm over the 1024 model channels, one warp per row, statistics in fp32 from
// registers (two passes over the row held in registers, biased variance, eps 1e-5).
// Replaces tinybark/tinygrad/model.py:56-57 and layernorm_kernel of
// tinybark/mojo/bark/gpu.mojo:27-45. The fused form applies a block's norm_out in
// place and the next block's norm_feed_forward1 in the same pass over the row.
#include "common.cuh"
#include "host.h"

namespace tb {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Normalizes the row held in v (this lane's 32 values); Affine gives the parameters of
// column group i (from registers, or loaded on use).
template <typename Affine>
__device__ __forceinline__ void ln_row(float4 (&v)[8], Affine&& affine) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) * (1.0f / TB_HIDDEN);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a = v[i].x - mean, b2 = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    q += (a * a + b2 * b2) + (c * c + d * d);
  }
  const float inv = 1.0f / sqrtf(warp_sum(q) * (1.0f / TB_HIDDEN) + 1e-5f);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 g, bb;
    affine(i, g, bb);
    v[i].x = (v[i].x - mean) * inv * g.x + bb.x;
    v[i].y = (v[i].y - mean) * inv * g.y + bb.y;
    v[i].z = (v[i].z - mean) * inv * g.z + bb.z;
    v[i].w = (v[i].w - mean) * inv * g.w + bb.w;
  }
}

// PRE (small row counts, where a launch is mostly latency): the first norm's parameters
// (weights, never written by a predecessor) are loaded before waiting on the predecessor
// kernel, at the cost of registers (and so of the blocks per SM the large launches need).
template <typename OutT, bool PRE>
__global__ void __launch_bounds__(256) layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                        const float* __restrict__ b, float* x_out,
                                                        const float* __restrict__ w2, const float* __restrict__ b2,
                                                        OutT* y, int rows) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  float4 pg[PRE ? 8 : 1], pb[PRE ? 8 : 1];
  if constexpr (PRE) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      pg[i] = load4(w + (i * 32 + lane) * 4);
      pb[i] = load4(b + (i * 32 + lane) * 4);
    }
  }
  grid_dep_wait();
  grid_dep_launch();
  if (row >= rows) return;
  const float* xr = x + (long long)row * TB_HIDDEN;
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = load4(xr + (i * 32 + lane) * 4);
  auto loaded = [&](const float* wp, const float* bp) {
    return [=](int i, float4& g, float4& bb) {
      g = load4(wp + (i * 32 + lane) * 4);
      bb = load4(bp + (i * 32 + lane) * 4);
    };
  };
  if constexpr (PRE) {
    ln_row(v, [&](int i, float4& g, float4& bb) { g = pg[i], bb = pb[i]; });
  } else {
    ln_row(v, loaded(w, b));
  }
  if (x_out) {
    float* xo = x_out + (long long)row * TB_HIDDEN;
#pragma unroll
    for (int i = 0; i < 8; ++i) store4(xo + (i * 32 + lane) * 4, v[i].x, v[i].y, v[i].z, v[i].w);
  }
  if (w2) ln_row(v, loaded(w2, b2));
  OutT* yr = y + (long long)row * TB_HIDDEN;
#pragma unroll
  for (int i = 0; i < 8; ++i) store4(yr + (i * 32 + lane) * 4, v[i].x, v[i].y, v[i].z, v[i].w);
}

int layernorm(const float* x, const float* w, const float* b, float* x_out, const float* w2, const float* b2, void* y,
              int y_dtype, int rows, cudaStream_t stream) {
  if (rows <= 0) return TB_OK;
  if (!x || !w || !b || !y || (w2 && (!b2 || !x_out))) return TB_ERR_ARG;
  dim3 grid((rows + 7) / 8);
  const bool pre = (int)grid.x <= sm_count();
  if (y_dtype == TB_BF16) {
    auto* yo = reinterpret_cast<__nv_bfloat16*>(y);
    return pre ? launch_pdl(layernorm_kernel<__nv_bfloat16, true>, grid, 256, 0, stream, x, w, b, x_out, w2, b2, yo, rows)
               : launch_pdl(layernorm_kernel<__nv_bfloat16, false>, grid, 256, 0, stream, x, w, b, x_out, w2, b2, yo,
                            rows);
  }
  if (y_dtype == TB_F32) {
    auto* yo = reinterpret_cast<float*>(y);
    return pre ? launch_pdl(layernorm_kernel<float, true>, grid, 256, 0, stream, x, w, b, x_out, w2, b2, yo, rows)
               : launch_pdl(layernorm_kernel<float, false>, grid, 256, 0, stream, x, w, b, x_out, w2, b2, yo, rows);
  }
  return TB_ERR_ARG;
}

}  // namespace tb
