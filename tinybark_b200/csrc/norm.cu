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

__device__ __forceinline__ void ln_row(float4 (&v)[8], const float* w, const float* b, int lane) {
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
    const int c = (i * 32 + lane) * 4;
    float4 g = load4(w + c), bb = load4(b + c);
    v[i].x = (v[i].x - mean) * inv * g.x + bb.x;
    v[i].y = (v[i].y - mean) * inv * g.y + bb.y;
    v[i].z = (v[i].z - mean) * inv * g.z + bb.z;
    v[i].w = (v[i].w - mean) * inv * g.w + bb.w;
  }
}

template <typename OutT>
__global__ void __launch_bounds__(256) layernorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                        const float* __restrict__ b, float* x_out,
                                                        const float* __restrict__ w2, const float* __restrict__ b2,
                                                        OutT* y, int rows) {
  grid_dep_wait();
  grid_dep_launch();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + (long long)row * TB_HIDDEN;
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = load4(xr + (i * 32 + lane) * 4);
  ln_row(v, w, b, lane);
  if (x_out) {
    float* xo = x_out + (long long)row * TB_HIDDEN;
#pragma unroll
    for (int i = 0; i < 8; ++i) store4(xo + (i * 32 + lane) * 4, v[i].x, v[i].y, v[i].z, v[i].w);
  }
  if (w2) ln_row(v, w2, b2, lane);
  OutT* yr = y + (long long)row * TB_HIDDEN;
#pragma unroll
  for (int i = 0; i < 8; ++i) store4(yr + (i * 32 + lane) * 4, v[i].x, v[i].y, v[i].z, v[i].w);
}

int layernorm(const float* x, const float* w, const float* b, float* x_out, const float* w2, const float* b2, void* y,
              int y_dtype, int rows, cudaStream_t stream) {
  if (rows <= 0) return TB_OK;
  if (!x || !w || !b || !y || (w2 && (!b2 || !x_out))) return TB_ERR_ARG;
  dim3 grid((rows + 7) / 8);
  if (y_dtype == TB_BF16)
    return launch_pdl(layernorm_kernel<__nv_bfloat16>, grid, 256, 0, stream, x, w, b, x_out, w2, b2,
                      reinterpret_cast<__nv_bfloat16*>(y), rows);
  if (y_dtype == TB_F32)
    return launch_pdl(layernorm_kernel<float>, grid, 256, 0, stream, x, w, b, x_out, w2, b2,
                      reinterpret_cast<float*>(y), rows);
  return TB_ERR_ARG;
}

}  // namespace tb
