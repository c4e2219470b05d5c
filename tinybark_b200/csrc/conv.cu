// Conv module middle: depthwise conv along time (kernel 9, padding 4, BatchNorm folded
// into taps and bias) and SiLU, on the GLU output of pointwise_conv1. Replaces
// tinybark/tinygrad/model.py:121-124 and conv_kernel of tinybark/mojo/bark/gpu.mojo:78-94.
// Frames outside a clip read as zeros (the masked, zero-padded frames of the
// reference). Each thread slides one channel over DW_ROWS output frames, so every
// input value is read by one thread about (DW_ROWS + 8) / DW_ROWS times.
#include "common.cuh"
#include "host.h"

namespace tb {

constexpr int DW_ROWS = 16;

template <typename T>
__global__ void __launch_bounds__(256) depthwise_silu_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                             const float* __restrict__ b,
                                                             const int* __restrict__ row_clip,
                                                             const int* __restrict__ off, int rows, T* __restrict__ y) {
  grid_dep_wait();
  grid_dep_launch();
  const int c = blockIdx.y * 256 + threadIdx.x;
  const int r0 = blockIdx.x * DW_ROWS;
  float taps[TB_KERNEL];
#pragma unroll
  for (int k = 0; k < TB_KERNEL; ++k) taps[k] = w[c * TB_KERNEL + k];
  const float bias = b[c];
  float in[DW_ROWS + TB_KERNEL - 1];
#pragma unroll
  for (int i = 0; i < DW_ROWS + TB_KERNEL - 1; ++i) {
    const int r = r0 + i - TB_KERNEL / 2;
    in[i] = (r >= 0 && r < rows) ? to_f(x[(long long)r * TB_HIDDEN + c]) : 0.f;
  }
#pragma unroll
  for (int i = 0; i < DW_ROWS; ++i) {
    const int r = r0 + i;
    if (r >= rows) break;
    const int clip = row_clip[r];
    const int lo = off[clip] - r, hi = off[clip + 1] - r;  // valid tap offsets: lo <= k-4 < hi
    float acc = bias;
#pragma unroll
    for (int k = 0; k < TB_KERNEL; ++k) {
      const int d = k - TB_KERNEL / 2;
      if (d >= lo && d < hi) acc = fmaf(taps[k], in[i + k], acc);
    }
    y[(long long)r * TB_HIDDEN + c] = from_f<T>(siluf_(acc));
  }
}

int conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch& bt, void* out,
                   cudaStream_t stream) {
  const int rows = bt.t3_total;
  if (rows <= 0) return TB_OK;
  if (!glu || !w || !b || !out || !bt.t3_clip || !bt.t3_off) return TB_ERR_ARG;
  dim3 grid((rows + DW_ROWS - 1) / DW_ROWS, TB_HIDDEN / 256);
  if (dtype == TB_BF16)
    return launch_pdl(depthwise_silu_kernel<__nv_bfloat16>, grid, 256, 0, stream,
                      reinterpret_cast<const __nv_bfloat16*>(glu), w, b, bt.t3_clip, bt.t3_off, rows,
                      reinterpret_cast<__nv_bfloat16*>(out));
  if (dtype == TB_F32)
    return launch_pdl(depthwise_silu_kernel<float>, grid, 256, 0, stream, reinterpret_cast<const float*>(glu), w, b,
                      bt.t3_clip, bt.t3_off, rows, reinterpret_cast<float*>(out));
  return TB_ERR_ARG;
}

}  // namespace tb
