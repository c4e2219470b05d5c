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
// The first conv is computed inside the first depthwise conv's kernel, so its
// 256-channel output never reaches HBM.
#include "epilogue.cuh"
#include "host.h"

namespace tb {

constexpr int S_T2 = 8;          // depthwise-1 output rows per block: one warp each
constexpr int S_C = 64;          // channels per block: two per lane
constexpr int S_F2 = 32, S_F3 = 16;  // frequencies after depthwise 1 and 2 (conv 0 makes 64)
constexpr int S_FEAT_ROWS = 4 * S_T2 + 3;  // feature rows behind S_T2 depthwise-1 rows
constexpr int S_FEAT_COLS = TB_MELS + 2;   // frequency padded by one each side

// conv 0 (3x3/2, 1 -> 256, + ReLU) fused into depthwise 1 (3x3/2 + bias). Warp w of a
// block makes depthwise-1 row t2 = t2a + w for channels c0 + lane and c0 + 32 + lane,
// sweeping its 32 output frequencies f2 left to right. Output f2 needs conv-0 columns
// f1 = 2 f2 - 1, 2 f2, 2 f2 + 1 of conv-0 rows t1 = 2 t2 - 1 + dt (dt = 0..2); the
// first of those columns is the previous step's last, so each step computes 2 x 3
// conv-0 values per channel from a 7 x 5 window of features (the window's first
// column also carried over), all features read from shared memory (the same address
// for every lane: one broadcast per read). Conv-0 values outside the clip's rows or
// the frequency range are the zero padding of depthwise 1.
template <typename T>
__global__ void __launch_bounds__(256) conv0_dw1_kernel(const float* __restrict__ feats,
                                                        const int* __restrict__ frame_off,
                                                        const int* __restrict__ t1_off, const int* __restrict__ t2_off,
                                                        const int* __restrict__ tiles, const float* __restrict__ w0,
                                                        const float* __restrict__ b0, const float* __restrict__ w1,
                                                        const float* __restrict__ b1, T* __restrict__ d1) {
  __shared__ float sf[S_FEAT_ROWS][S_FEAT_COLS];
  const int clip = tiles[2 * blockIdx.x], t2a = tiles[2 * blockIdx.x + 1];
  const int F = frame_off[clip + 1] - frame_off[clip], T1 = t1_off[clip + 1] - t1_off[clip],
            T2 = t2_off[clip + 1] - t2_off[clip];
  const float* fbase = feats + (long long)frame_off[clip] * TB_MELS;
  const int fa = 4 * t2a - 3;  // feature row of the tile's first shared-memory row

  for (int i = threadIdx.x; i < S_FEAT_ROWS * S_FEAT_COLS; i += 256) {
    const int r = i / S_FEAT_COLS, f = i % S_FEAT_COLS - 1;
    const int t = fa + r;
    sf[r][f + 1] = (t >= 0 && t < F && f >= 0 && f < TB_MELS) ? fbase[(long long)t * TB_MELS + f] : 0.f;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ca = blockIdx.y * S_C + lane, cb = ca + 32;
  float k0a[9], k0b[9], k1a[9], k1b[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) {
    k0a[i] = w0[ca * 9 + i];
    k0b[i] = w0[cb * 9 + i];
    k1a[i] = w1[ca * 9 + i];
    k1b[i] = w1[cb * 9 + i];
  }
  const float b0a = b0[ca], b0b = b0[cb], b1a = b1[ca], b1b = b1[cb];
  __syncthreads();
  const int t2 = t2a + w;
  if (t2 >= T2) return;
  bool rowok[3];
#pragma unroll
  for (int dt = 0; dt < 3; ++dt) {
    const int t1 = 2 * t2 - 1 + dt;
    rowok[dt] = t1 >= 0 && t1 < T1;
  }
  const float* srow = &sf[4 * w][0];  // conv-0 row dt reads feature rows 2 dt .. 2 dt + 2 of these 7
  float xc[7];                        // feature column 4 f2 (padded), carried from the previous step
#pragma unroll
  for (int r = 0; r < 7; ++r) xc[r] = srow[r * S_FEAT_COLS];
  float pa[3] = {0.f, 0.f, 0.f}, pb[3] = {0.f, 0.f, 0.f};  // conv-0 column 2 f2 - 1 (zero at f2 = 0)
  T* out = d1 + (long long)(t2_off[clip] + t2) * S_F2 * TB_CHANNELS;
#pragma unroll 1
  for (int f2 = 0; f2 < S_F2; ++f2) {
    float x1[7], x2[7], x3[7], x4[7];
#pragma unroll
    for (int r = 0; r < 7; ++r) {
      const float* q = srow + r * S_FEAT_COLS + 4 * f2;
      x1[r] = q[1];
      x2[r] = q[2];
      x3[r] = q[3];
      x4[r] = q[4];
    }
    float acc_a = b1a, acc_b = b1b;
#pragma unroll
    for (int dt = 0; dt < 3; ++dt) {
      // conv 0 at columns 2 f2 (features 4 f2 .. 4 f2 + 2) and 2 f2 + 1 (4 f2 + 2 .. 4 f2 + 4)
      float va = b0a, vb = b0b, ua = b0a, ub = b0b;
#pragma unroll
      for (int dr = 0; dr < 3; ++dr) {
        const int r = 2 * dt + dr;
        va = fmaf(k0a[dr * 3], xc[r], fmaf(k0a[dr * 3 + 1], x1[r], fmaf(k0a[dr * 3 + 2], x2[r], va)));
        vb = fmaf(k0b[dr * 3], xc[r], fmaf(k0b[dr * 3 + 1], x1[r], fmaf(k0b[dr * 3 + 2], x2[r], vb)));
        ua = fmaf(k0a[dr * 3], x2[r], fmaf(k0a[dr * 3 + 1], x3[r], fmaf(k0a[dr * 3 + 2], x4[r], ua)));
        ub = fmaf(k0b[dr * 3], x2[r], fmaf(k0b[dr * 3 + 1], x3[r], fmaf(k0b[dr * 3 + 2], x4[r], ub)));
      }
      va = rowok[dt] ? fmaxf(va, 0.f) : 0.f;
      vb = rowok[dt] ? fmaxf(vb, 0.f) : 0.f;
      ua = rowok[dt] ? fmaxf(ua, 0.f) : 0.f;
      ub = rowok[dt] ? fmaxf(ub, 0.f) : 0.f;
      // depthwise 1 over conv-0 columns 2 f2 - 1, 2 f2, 2 f2 + 1
      acc_a = fmaf(k1a[dt * 3], pa[dt], fmaf(k1a[dt * 3 + 1], va, fmaf(k1a[dt * 3 + 2], ua, acc_a)));
      acc_b = fmaf(k1b[dt * 3], pb[dt], fmaf(k1b[dt * 3 + 1], vb, fmaf(k1b[dt * 3 + 2], ub, acc_b)));
      pa[dt] = ua;
      pb[dt] = ub;
    }
#pragma unroll
    for (int r = 0; r < 7; ++r) xc[r] = x4[r];
    out[f2 * TB_CHANNELS + ca] = from_f<T>(acc_a);
    out[f2 * TB_CHANNELS + cb] = from_f<T>(acc_b);
  }
}

// depthwise 2: s2 [T2][32][256] -> d2 [T3][16][256]; one block of 256 threads per output
// row t3: thread t takes channels 2 (t % 128) and 2 (t % 128) + 1 (one 4-byte access of
// two bf16 or two-wide fp32 halves) and the 8 frequencies f3 of half t / 128, sweeping f3
// upwards so each step reads two new input columns (f2 = 2 f3, 2 f3 + 1) and reuses the
// last one (2 f3 - 1).
template <typename T>
__global__ void __launch_bounds__(256) dw2_kernel(const T* __restrict__ s2, const int* __restrict__ t2_off,
                                                  const int* __restrict__ t3_off, const int* __restrict__ t3_clip,
                                                  const float* __restrict__ w, const float* __restrict__ b,
                                                  T* __restrict__ d2) {
  const int row = blockIdx.x, c = 2 * (threadIdx.x & 127), half = threadIdx.x >> 7;
  const int clip = t3_clip[row];
  const int t3 = row - t3_off[clip];
  const int T2 = t2_off[clip + 1] - t2_off[clip];
  const long long base2 = t2_off[clip];
  float wa[9], wb[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wa[i] = w[c * 9 + i], wb[i] = w[(c + 1) * 9 + i];
  const float ba = b[c], bb = b[c + 1];
  bool ok[3];
  const T* in[3];
#pragma unroll
  for (int dt = 0; dt < 3; ++dt) {
    const int t2 = 2 * t3 + dt - 1;
    ok[dt] = t2 >= 0 && t2 < T2;
    in[dt] = s2 + ((base2 + (ok[dt] ? t2 : 0)) * S_F2) * TB_CHANNELS + c;
  }
  auto load2 = [&](int dt, int f2) -> float2 {
    if (!ok[dt] || f2 < 0) return make_float2(0.f, 0.f);
    return load2f(in[dt] + f2 * TB_CHANNELS);
  };
  const int f3a = half * (S_F3 / 2);
  float2 prev[3];  // column 2 f3 - 1
#pragma unroll
  for (int dt = 0; dt < 3; ++dt) prev[dt] = load2(dt, 2 * f3a - 1);
#pragma unroll
  for (int k = 0; k < S_F3 / 2; ++k) {
    const int f3 = f3a + k;
    float acc_a = ba, acc_b = bb;
#pragma unroll
    for (int dt = 0; dt < 3; ++dt) {
      const float2 m = load2(dt, 2 * f3), r = load2(dt, 2 * f3 + 1);
      acc_a = fmaf(wa[dt * 3], prev[dt].x, fmaf(wa[dt * 3 + 1], m.x, fmaf(wa[dt * 3 + 2], r.x, acc_a)));
      acc_b = fmaf(wb[dt * 3], prev[dt].y, fmaf(wb[dt * 3 + 1], m.y, fmaf(wb[dt * 3 + 2], r.y, acc_b)));
      prev[dt] = r;
    }
    store2(d2 + ((long long)row * S_F3 + f3) * TB_CHANNELS + c, acc_a, acc_b);
  }
}

int subsample_tile_rows() { return S_T2; }

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
    dw2_kernel<__nv_bfloat16><<<bt.t3_total, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(s2), bt.t2_off, bt.t3_off, bt.t3_clip, m.sub_dw_w[1], m.sub_dw_b[1],
        reinterpret_cast<__nv_bfloat16*>(d2));
  else
    dw2_kernel<float><<<bt.t3_total, 256, 0, stream>>>(reinterpret_cast<const float*>(s2), bt.t2_off, bt.t3_off,
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
