// Conv module middle: depthwise conv along time (kernel 9, padding 4, BatchNorm folded
// into taps and bias) and SiLU, on the GLU output of pointwise_conv1. Replaces
// tinybark/tinygrad/model.py:121-124 and conv_kernel of tinybark/mojo/bark/gpu.mojo:78-94.
// Frames outside a clip read as zeros (the masked, zero-padded frames of the
// reference).
#include "common.cuh"
#include "host.h"

namespace tb {

constexpr int DW_ROWS = 16;  // output frames per block (registers allow two blocks per SM)
constexpr int DW_HALO = TB_KERNEL / 2;

// SiLU: exact for the fp32 parity path, one MUFU operation for bf16.
template <typename T>
__device__ __forceinline__ float act(float x) {
  if constexpr (sizeof(T) == 4) return siluf_(x);
  return fast_silu(x);
}

template <typename T> struct Pair;
template <> struct Pair<float> {
  static __device__ __forceinline__ float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void store(float* p, float a, float b) { store2(p, a, b); }
};
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) { store2(p, a, b); }
};

// Each thread slides channels c, c + 1 over DW_ROWS output frames (input read once per
// block, DW_ROWS + 8 frames). Blocks whose frames and halo all lie in one clip (almost
// all of them) skip the per-tap clip-boundary tests.
template <typename T>
__global__ void __launch_bounds__(256, 2) depthwise_silu_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                             const float* __restrict__ b,
                                                             const int* __restrict__ row_clip,
                                                             const int* __restrict__ off, int rows, T* __restrict__ y) {
  grid_dep_wait();
  grid_dep_launch();
  const int c = (blockIdx.y * 256 + threadIdx.x) * 2;
  const int r0 = blockIdx.x * DW_ROWS;
  float ta[TB_KERNEL], tb[TB_KERNEL];
#pragma unroll
  for (int k = 0; k < TB_KERNEL; ++k) ta[k] = w[c * TB_KERNEL + k], tb[k] = w[(c + 1) * TB_KERNEL + k];
  const float ba = b[c], bb = b[c + 1];
  float ia[DW_ROWS + 2 * DW_HALO], ib[DW_ROWS + 2 * DW_HALO];
#pragma unroll
  for (int i = 0; i < DW_ROWS + 2 * DW_HALO; ++i) {
    const int r = r0 + i - DW_HALO;
    const float2 v = (r >= 0 && r < rows) ? Pair<T>::load(x + (long long)r * TB_HIDDEN + c) : make_float2(0.f, 0.f);
    ia[i] = v.x;
    ib[i] = v.y;
  }
  const bool interior = r0 >= DW_HALO && r0 + DW_ROWS + DW_HALO <= rows &&
                        row_clip[r0 - DW_HALO] == row_clip[r0 + DW_ROWS + DW_HALO - 1];
  if (interior) {
#pragma unroll
    for (int i = 0; i < DW_ROWS; ++i) {
      float acc_a = ba, acc_b = bb;
#pragma unroll
      for (int k = 0; k < TB_KERNEL; ++k) acc_a = fmaf(ta[k], ia[i + k], acc_a), acc_b = fmaf(tb[k], ib[i + k], acc_b);
      Pair<T>::store(y + (long long)(r0 + i) * TB_HIDDEN + c, act<T>(acc_a), act<T>(acc_b));
    }
  } else {
#pragma unroll
    for (int i = 0; i < DW_ROWS; ++i) {
      const int r = r0 + i;
      if (r >= rows) break;
      const int clip = row_clip[r];
      const int lo = off[clip] - r, hi = off[clip + 1] - r;  // valid tap offsets: lo <= k-4 < hi
      float acc_a = ba, acc_b = bb;
#pragma unroll
      for (int k = 0; k < TB_KERNEL; ++k) {
        const int d = k - DW_HALO;
        if (d >= lo && d < hi) acc_a = fmaf(ta[k], ia[i + k], acc_a), acc_b = fmaf(tb[k], ib[i + k], acc_b);
      }
      Pair<T>::store(y + (long long)r * TB_HIDDEN + c, act<T>(acc_a), act<T>(acc_b));
    }
  }
}

int conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch& bt, void* out,
                   cudaStream_t stream) {
  const int rows = bt.t3_total;
  if (rows <= 0) return TB_OK;
  if (!glu || !w || !b || !out || !bt.t3_clip || !bt.t3_off) return TB_ERR_ARG;
  dim3 grid((rows + DW_ROWS - 1) / DW_ROWS, TB_HIDDEN / 512);
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
