// Conv module middle: depthwise conv along time (kernel 9, padding 4, BatchNorm folded
// into taps and bias) and SiLU, on the GLU output of pointwise_conv1. Replaces
// tinybark/tinygrad/model.py:121-124 and conv_kernel of tinybark/mojo/bark/gpu.mojo:78-94.
// Frames outside a clip read as zeros (the masked, zero-padded frames of the
// reference).
#include <algorithm>

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
  const int c = (blockIdx.y * 256 + threadIdx.x) * 2;
  const int r0 = blockIdx.x * DW_ROWS;
  float ta[TB_KERNEL], tb[TB_KERNEL];
#pragma unroll
  for (int k = 0; k < TB_KERNEL; ++k) ta[k] = w[c * TB_KERNEL + k], tb[k] = w[(c + 1) * TB_KERNEL + k];
  const float ba = b[c], bb = b[c + 1];
  grid_dep_wait();  // the taps above are weights: read before the predecessor ends
  grid_dep_launch();
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

// bf16: one persistent CTA per SM streams tiles of DWS_R output frames. A tile and its
// 4-frame halo on each side are one contiguous span of [rows, 1024] bf16 (80 KB), fetched
// with a single bulk copy (no multicast) into one of two shared-memory buffers while the
// other tile is computed. Each of 512 threads slides 2 channels down the tile: the 9
// input frames of the current output frame in registers (fp32), each frame read from
// shared memory once, two-wide FMAs, and whole row segments out (a warp writes 128
// contiguous bytes per frame). Sixteen warps per SM hide the FMA and SiLU latencies. Tiles whose frames and halo all lie in one clip skip
// the per-tap clip tests.
constexpr int DWS_R = 32;
constexpr int DWS_ROWS = DWS_R + 2 * DW_HALO;
constexpr int DWS_ROW_BYTES = TB_HIDDEN * 2;
constexpr int DWS_TILE_BYTES = DWS_ROWS * DWS_ROW_BYTES;
constexpr int DWS_SMEM = 2 * DWS_TILE_BYTES + 64;
constexpr int DWS_THREADS = TB_HIDDEN / 2;  // two channels per thread

__device__ __forceinline__ void bulk_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__global__ void __launch_bounds__(DWS_THREADS, 1)
    depthwise_stream_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                            const float* __restrict__ b, const int* __restrict__ row_clip, const int* __restrict__ off,
                            int rows, __nv_bfloat16* __restrict__ y, int* err) {
  extern __shared__ __align__(128) uint8_t dws_smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(dws_smem + 2 * DWS_TILE_BYTES);
  int* abort_flag = reinterpret_cast<int*>(dws_smem + 2 * DWS_TILE_BYTES + 16);
  volatile int* abort = abort_flag;
  const int c0 = threadIdx.x * 2;
  // This thread's taps and biases for channels c0, c0 + 1.
  float2 wk[TB_KERNEL];
#pragma unroll
  for (int k = 0; k < TB_KERNEL; ++k) wk[k] = make_float2(w[c0 * TB_KERNEL + k], w[(c0 + 1) * TB_KERNEL + k]);
  const float2 bias0 = make_float2(b[c0], b[c0 + 1]);
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  grid_dep_wait();
  grid_dep_launch();
  const int tiles = (rows + DWS_R - 1) / DWS_R;
  // Tile t's frames [t*R - 4, t*R + R + 4) clipped to [0, rows), placed so that smem row i
  // holds frame t*R - 4 + i.
  auto issue = [&](int t, int s) {
    const int r0 = t * DWS_R, lo = max(0, r0 - DW_HALO), hi = min(rows, r0 + DWS_R + DW_HALO);
    uint8_t* dst = dws_smem + s * DWS_TILE_BYTES + (lo - (r0 - DW_HALO)) * DWS_ROW_BYTES;
    mbar_expect_tx(&bar[s], (uint32_t)(hi - lo) * DWS_ROW_BYTES);
    bulk_load_1d(dst, x + (long long)lo * TB_HIDDEN, (uint32_t)(hi - lo) * DWS_ROW_BYTES, &bar[s]);
  };
  if (threadIdx.x == 0 && (int)blockIdx.x < tiles) issue(blockIdx.x, 0);
  const int n_local = (int)blockIdx.x < tiles ? (tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  int k = 0, issued = n_local > 0 ? 1 : 0;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++k) {
    const int s = k & 1;
    if (t + (int)gridDim.x < tiles) {
      if (threadIdx.x == 0) issue(t + gridDim.x, s ^ 1);
      issued = k + 2;
    }
    if (!mbar_wait(&bar[s], (uint32_t)((k >> 1) & 1), err, TB_DEV_CONV_TIMEOUT, abort)) break;
    const uint8_t* tile = dws_smem + s * DWS_TILE_BYTES + c0 * 2;
    auto frame = [&](int i) {  // smem row i, this thread's 2 channels
      return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(tile + i * DWS_ROW_BYTES));
    };
    const int r0 = t * DWS_R;
    const bool interior = r0 >= DW_HALO && r0 + DWS_R + DW_HALO <= rows &&
                          row_clip[r0 - DW_HALO] == row_clip[r0 + DWS_R + DW_HALO - 1];
    float2 win[TB_KERNEL];  // frames o-4 .. o+4 of output frame o
#pragma unroll
    for (int i = 0; i < TB_KERNEL - 1; ++i) win[i] = frame(i);
    if (interior) {
#pragma unroll
      for (int o = 0; o < DWS_R; ++o) {
        win[TB_KERNEL - 1] = frame(o + TB_KERNEL - 1);
        float2 a0 = bias0;
#pragma unroll
        for (int q = 0; q < TB_KERNEL; ++q) a0 = fma2(wk[q], win[q], a0);
        a0 = silu2_tanh(a0);
        *reinterpret_cast<uint32_t*>(y + (long long)(r0 + o) * TB_HIDDEN + c0) = pack_bf16x2(a0.x, a0.y);
#pragma unroll
        for (int q = 0; q < TB_KERNEL - 1; ++q) win[q] = win[q + 1];
      }
    } else {
#pragma unroll
      for (int o = 0; o < DWS_R; ++o) {
        const int r = r0 + o;
        // Frames past the last are neither loaded nor used (their taps fall outside every clip).
        if (r + DW_HALO < rows) win[TB_KERNEL - 1] = frame(o + TB_KERNEL - 1);
        if (r < rows) {
          const int clip = row_clip[r];
          const int lo = off[clip] - r, hi = off[clip + 1] - r;  // valid tap offsets: lo <= q-4 < hi
          float2 a0 = bias0;
#pragma unroll
          for (int q = 0; q < TB_KERNEL; ++q) {
            const int d = q - DW_HALO;
            if (d >= lo && d < hi) a0 = fma2(wk[q], win[q], a0);
          }
          a0 = silu2_tanh(a0);
          *reinterpret_cast<uint32_t*>(y + (long long)r * TB_HIDDEN + c0) = pack_bf16x2(a0.x, a0.y);
        }
#pragma unroll
        for (int q = 0; q < TB_KERNEL - 1; ++q) win[q] = win[q + 1];
      }
    }
    __syncthreads();  // every thread is done with buffer s before it is refilled
  }
  // Copies still in flight (only if the loop was abandoned) land before the CTA exits.
  if (threadIdx.x == 0) {
    for (int j = k; j < issued; ++j) {
      uint64_t start = globaltimer();
      while (!mbar_try_wait(&bar[j & 1], (uint32_t)((j >> 1) & 1)))
        if (globaltimer() - start > TB_WAIT_NS) break;
    }
  }
}

// bf16 for few rows (a batch of one or two clips, where the streaming kernel would run
// a handful of CTAs): a CTA per 8 output frames and 256 channels, the frames read
// straight from global memory, the taps and bias loaded before waiting on the
// predecessor. The arithmetic is the streaming kernel's, operation for operation, so a
// clip's output does not depend on the batch it runs in.
constexpr int DWQ_R = 8, DWQ_THREADS = 128;

__global__ void __launch_bounds__(DWQ_THREADS) depthwise_small_kernel(const __nv_bfloat16* __restrict__ x,
                                                                      const float* __restrict__ w,
                                                                      const float* __restrict__ b,
                                                                      const int* __restrict__ row_clip,
                                                                      const int* __restrict__ off, int rows,
                                                                      __nv_bfloat16* __restrict__ y) {
  const int c0 = (blockIdx.y * DWQ_THREADS + threadIdx.x) * 2;
  float2 wk[TB_KERNEL];
#pragma unroll
  for (int k = 0; k < TB_KERNEL; ++k) wk[k] = make_float2(w[c0 * TB_KERNEL + k], w[(c0 + 1) * TB_KERNEL + k]);
  const float2 bias0 = make_float2(b[c0], b[c0 + 1]);
  grid_dep_wait();
  grid_dep_launch();
  const int r0 = blockIdx.x * DWQ_R;
  float2 win[DWQ_R + 2 * DW_HALO];  // frames r0-4 .. r0+R+3, zero outside [0, rows)
#pragma unroll
  for (int i = 0; i < DWQ_R + 2 * DW_HALO; ++i) {
    const int r = r0 - DW_HALO + i;
    win[i] = (r >= 0 && r < rows)
                 ? __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x + (long long)r * TB_HIDDEN + c0))
                 : make_float2(0.f, 0.f);
  }
  const bool interior = r0 >= DW_HALO && r0 + DWQ_R + DW_HALO <= rows &&
                        row_clip[r0 - DW_HALO] == row_clip[r0 + DWQ_R + DW_HALO - 1];
#pragma unroll
  for (int o = 0; o < DWQ_R; ++o) {
    const int r = r0 + o;
    if (!interior && r >= rows) break;
    float2 a0 = bias0;
    if (interior) {
#pragma unroll
      for (int q = 0; q < TB_KERNEL; ++q) a0 = fma2(wk[q], win[o + q], a0);
    } else {
      const int clip = row_clip[r];
      const int lo = off[clip] - r, hi = off[clip + 1] - r;  // valid tap offsets: lo <= q-4 < hi
#pragma unroll
      for (int q = 0; q < TB_KERNEL; ++q) {
        const int d = q - DW_HALO;
        if (d >= lo && d < hi) a0 = fma2(wk[q], win[o + q], a0);
      }
    }
    a0 = silu2_tanh(a0);
    *reinterpret_cast<uint32_t*>(y + (long long)r * TB_HIDDEN + c0) = pack_bf16x2(a0.x, a0.y);
  }
}

int conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch& bt, void* out, int* err,
                   cudaStream_t stream) {
  const int rows = bt.t3_total;
  if (rows <= 0) return TB_OK;
  if (!glu || !w || !b || !out || !bt.t3_clip || !bt.t3_off) return TB_ERR_ARG;
  if (dtype == TB_BF16) {
    if (!err) return TB_ERR_ARG;
    static bool configured[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda();
    if (!configured[dev]) {
      if (cudaFuncSetAttribute(depthwise_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DWS_SMEM) !=
          cudaSuccess)
        return fail_cuda();
      configured[dev] = true;
    }
    const int tiles = (rows + DWS_R - 1) / DWS_R;
    if (tiles < sm_budget()) {
      dim3 grid((rows + DWQ_R - 1) / DWQ_R, TB_HIDDEN / 2 / DWQ_THREADS);
      return launch_pdl(depthwise_small_kernel, grid, DWQ_THREADS, 0, stream,
                        reinterpret_cast<const __nv_bfloat16*>(glu), w, b, bt.t3_clip, bt.t3_off, rows,
                        reinterpret_cast<__nv_bfloat16*>(out));
    }
    const int grid = std::min(tiles, sm_budget());
    return launch_pdl(depthwise_stream_kernel, grid, DWS_THREADS, DWS_SMEM, stream, reinterpret_cast<const __nv_bfloat16*>(glu),
                      w, b, bt.t3_clip, bt.t3_off, rows, reinterpret_cast<__nv_bfloat16*>(out), err);
  }
  if (dtype == TB_F32) {
    dim3 grid((rows + DW_ROWS - 1) / DW_ROWS, TB_HIDDEN / 512);
    return launch_pdl(depthwise_silu_kernel<float>, grid, 256, 0, stream, reinterpret_cast<const float*>(glu), w, b,
                      bt.t3_clip, bt.t3_off, rows, reinterpret_cast<float*>(out));
  }
  return TB_ERR_ARG;
}

}  // namespace tb
