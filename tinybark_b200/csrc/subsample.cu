// dw_striding 8x subsampling: conv 3x3/2 1->256 + ReLU, then twice [depthwise 3x3/2 +
// bias, pointwise 256->256 + bias + ReLU], then the 4096->1024 linear. Replaces
// tinybark/tinygrad/model.py:87-97 (_subsample) and the subsampling kernels of
// tinybark/mojo/bark/gpu.mojo:97-143,351-397.
//
// Activations are kept as [time][frequency][channel] (channel fastest): the pointwise
// convs are then plain GEMMs over (time, frequency) rows, and the last stage is
// already the (time, 16 * 256) matrix of the linear, whose weight columns the loader
// permutes from the reference's (channel, frequency) order to (frequency, channel).
//
// The first conv is recomputed inside the first depthwise conv's tile (its halo is one
// row), so its 256-channel output never reaches HBM.
#include "epilogue.cuh"
#include "host.h"

namespace tb {

constexpr int S_T2 = 2;          // depthwise-1 output rows per block
constexpr int S_C = 32;          // channels per block (one warp)
constexpr int S_T1 = 2 * S_T2 + 1;  // conv-0 rows a block needs
constexpr int S_F1 = 64, S_F2 = 32, S_F3 = 16;
constexpr int S_FEAT_ROWS = 2 * S_T1 + 1;

template <typename T>
__global__ void __launch_bounds__(256) conv0_dw1_kernel(const float* __restrict__ feats,
                                                        const int* __restrict__ frame_off,
                                                        const int* __restrict__ t1_off, const int* __restrict__ t2_off,
                                                        const int* __restrict__ tiles, const float* __restrict__ w0,
                                                        const float* __restrict__ b0, const float* __restrict__ w1,
                                                        const float* __restrict__ b1, T* __restrict__ d1) {
  __shared__ float sf[S_FEAT_ROWS][TB_MELS + 2];    // features, frequency padded by one each side
  __shared__ float s1[S_T1][S_F1 + 2][S_C];          // conv-0 output, frequency padded by one each side
  const int clip = tiles[2 * blockIdx.x], t2a = tiles[2 * blockIdx.x + 1];
  const int c0 = blockIdx.y * S_C;
  const int F = frame_off[clip + 1] - frame_off[clip], T1 = t1_off[clip + 1] - t1_off[clip],
            T2 = t2_off[clip + 1] - t2_off[clip];
  const float* fbase = feats + (long long)frame_off[clip] * TB_MELS;
  const int t1a = 2 * t2a - 1;        // first conv-0 row
  const int fa = 2 * t1a - 1;         // first feature row

  for (int i = threadIdx.x; i < S_FEAT_ROWS * (TB_MELS + 2); i += 256) {
    const int r = i / (TB_MELS + 2), f = i % (TB_MELS + 2) - 1;
    const int t = fa + r;
    sf[r][f + 1] = (t >= 0 && t < F && f >= 0 && f < TB_MELS) ? fbase[(long long)t * TB_MELS + f] : 0.f;
  }
  const int c = threadIdx.x & (S_C - 1);
  const int lane_group = threadIdx.x >> 5;  // warp: 0..7
  float k0[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) k0[i] = w0[(c0 + c) * 9 + i];
  const float bias0 = b0[c0 + c];
  __syncthreads();

  // conv 0 (+ ReLU), zero outside the clip's rows and the frequency range.
  for (int i = lane_group; i < S_T1 * (S_F1 + 2); i += 8) {
    const int r = i / (S_F1 + 2), f1 = i % (S_F1 + 2) - 1;
    const int t1 = t1a + r;
    float v = 0.f;
    if (t1 >= 0 && t1 < T1 && f1 >= 0 && f1 < S_F1) {
      float acc = bias0;
#pragma unroll
      for (int dt = 0; dt < 3; ++dt)
#pragma unroll
        for (int df = 0; df < 3; ++df) acc = fmaf(k0[dt * 3 + df], sf[2 * r + dt][2 * f1 + df], acc);
      v = fmaxf(acc, 0.f);
    }
    s1[r][f1 + 1][c] = v;
  }
  float k1[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) k1[i] = w1[(c0 + c) * 9 + i];
  const float bias1 = b1[c0 + c];
  __syncthreads();

  // depthwise 1
  for (int i = lane_group; i < S_T2 * S_F2; i += 8) {
    const int r = i / S_F2, f2 = i % S_F2;
    const int t2 = t2a + r;
    if (t2 >= T2) continue;
    float acc = bias1;
#pragma unroll
    for (int dt = 0; dt < 3; ++dt)
#pragma unroll
      for (int df = 0; df < 3; ++df) acc = fmaf(k1[dt * 3 + df], s1[2 * r + dt][2 * f2 + df][c], acc);
    d1[((long long)(t2_off[clip] + t2) * S_F2 + f2) * TB_CHANNELS + c0 + c] = from_f<T>(acc);
  }
}

// depthwise 2: s2 [T2][32][256] -> d2 [T3][16][256]; one block per (row, frequency).
template <typename T>
__global__ void __launch_bounds__(256) dw2_kernel(const T* __restrict__ s2, const int* __restrict__ t2_off,
                                                  const int* __restrict__ t3_off, const int* __restrict__ t3_clip,
                                                  const float* __restrict__ w, const float* __restrict__ b,
                                                  T* __restrict__ d2) {
  const int row = blockIdx.x / S_F3, f3 = blockIdx.x % S_F3, c = threadIdx.x;
  const int clip = t3_clip[row];
  const int t3 = row - t3_off[clip];
  const int T2 = t2_off[clip + 1] - t2_off[clip];
  const long long base2 = t2_off[clip];
  float acc = b[c];
#pragma unroll
  for (int dt = 0; dt < 3; ++dt) {
    const int t2 = 2 * t3 + dt - 1;
    if (t2 < 0 || t2 >= T2) continue;
#pragma unroll
    for (int df = 0; df < 3; ++df) {
      const int f2 = 2 * f3 + df - 1;
      if (f2 < 0 || f2 >= S_F2) continue;
      acc = fmaf(w[c * 9 + dt * 3 + df], to_f(s2[((base2 + t2) * S_F2 + f2) * TB_CHANNELS + c]), acc);
    }
  }
  d2[((long long)row * S_F3 + f3) * TB_CHANNELS + c] = from_f<T>(acc);
}

size_t subsample_ws(int dtype, int t2_total, int t3_total) {
  const size_t e = dsize(dtype);
  return 2 * align256((size_t)t2_total * S_F2 * TB_CHANNELS * e) + 2 * align256((size_t)t3_total * S_F3 * TB_CHANNELS * e);
}

int subsample(const tb_model& m, const tb_batch& bt, const float* feats, float* x, void* ws, size_t ws_bytes, int* err,
              cudaStream_t stream) {
  if (bt.t3_total <= 0) return TB_OK;
  if (ws_bytes < subsample_ws(m.dtype, bt.t2_total, bt.t3_total)) return TB_ERR_WORKSPACE;
  if (!bt.sub_tiles || !bt.frame_off || !bt.t1_off || !bt.t2_off || !bt.t3_off || !bt.t3_clip) return TB_ERR_ARG;
  const size_t e = dsize(m.dtype);
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  void* d1 = p;
  p += align256((size_t)bt.t2_total * S_F2 * TB_CHANNELS * e);
  void* s2 = p;
  p += align256((size_t)bt.t2_total * S_F2 * TB_CHANNELS * e);
  void* d2 = p;
  p += align256((size_t)bt.t3_total * S_F3 * TB_CHANNELS * e);
  void* s3 = p;

  dim3 g1(bt.n_sub_tiles, TB_CHANNELS / S_C);
  if (m.dtype == TB_BF16)
    conv0_dw1_kernel<__nv_bfloat16><<<g1, 256, 0, stream>>>(feats, bt.frame_off, bt.t1_off, bt.t2_off, bt.sub_tiles,
                                                            m.sub0_w, m.sub0_b, m.sub_dw_w[0], m.sub_dw_b[0],
                                                            reinterpret_cast<__nv_bfloat16*>(d1));
  else
    conv0_dw1_kernel<float><<<g1, 256, 0, stream>>>(feats, bt.frame_off, bt.t1_off, bt.t2_off, bt.sub_tiles, m.sub0_w,
                                                    m.sub0_b, m.sub_dw_w[0], m.sub_dw_b[0], reinterpret_cast<float*>(d1));
  if (int rc = check_launch()) return rc;

  tb_epilogue ep = {};
  ep.kind = TB_EPI_BIAS_RELU;
  ep.out_dtype = m.dtype;
  ep.out = s2;
  ep.ldo = TB_CHANNELS;
  ep.bias = m.sub_pw_b[0];
  if (int rc = gemm(m.dtype, d1, TB_CHANNELS, m.sub_pw_w[0], bt.t2_total * S_F2, TB_CHANNELS, TB_CHANNELS, ep, err,
                    stream))
    return rc;

  if (m.dtype == TB_BF16)
    dw2_kernel<__nv_bfloat16><<<bt.t3_total * S_F3, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(s2), bt.t2_off, bt.t3_off, bt.t3_clip, m.sub_dw_w[1], m.sub_dw_b[1],
        reinterpret_cast<__nv_bfloat16*>(d2));
  else
    dw2_kernel<float><<<bt.t3_total * S_F3, 256, 0, stream>>>(reinterpret_cast<const float*>(s2), bt.t2_off, bt.t3_off,
                                                              bt.t3_clip, m.sub_dw_w[1], m.sub_dw_b[1],
                                                              reinterpret_cast<float*>(d2));
  if (int rc = check_launch()) return rc;

  ep.out = s3;
  ep.bias = m.sub_pw_b[1];
  if (int rc = gemm(m.dtype, d2, TB_CHANNELS, m.sub_pw_w[1], bt.t3_total * S_F3, TB_CHANNELS, TB_CHANNELS, ep, err,
                    stream))
    return rc;

  tb_epilogue el = {};
  el.kind = TB_EPI_STORE;
  el.out_dtype = TB_F32;
  el.out = x;
  el.ldo = TB_HIDDEN;
  el.bias = m.sub_linear_b;
  return gemm(m.dtype, s3, S_F3 * TB_CHANNELS, m.sub_linear_w, bt.t3_total, TB_HIDDEN, S_F3 * TB_CHANNELS, el, err,
              stream);
}

}  // namespace tb
