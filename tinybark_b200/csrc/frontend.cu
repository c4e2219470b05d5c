// Log-mel front-end, replacing tinybark/audio.py:42-55 (a numpy port of transformers'
// ParakeetFeatureExtractor):
//   pre-emphasis x[n] - 0.97 x[n-1] (x[0] kept), zero padding of 256 on each side,
//   frames of 512 at hop 160 (frames = samples // 160), the 400-tap Hann window centred
//   in the frame, |rfft|^2, 128 slaney mel filters, log(. + 2^-24), then per clip and
//   per mel bin (m - mean) / (std + 1e-5), std with ddof 1.
//
// logmel_kernel: one warp per frame. The 512-point real FFT is a 256-point complex FFT
// of (even, odd) sample pairs followed by the standard split into the 257 real-input
// bins. The 256-point FFT runs in registers as 8 x 32 (four-step): each lane an 8-point
// DFT of its 8 values (n = 32 n1 + lane), a twiddle, then the 32-point DFTs across lanes
// as 4 x 8 with two transposes through shared memory. Twiddles come from sincospi in
// fp64 per block.
// stats_kernel / finish_kernel / normalize_kernel: per-clip mean and std per mel bin,
// accumulated in fp64 over frame ranges, then applied in place.
#include <mutex>

#include "common.cuh"
#include "host.h"

namespace tb {

constexpr int FE_WARPS = 8;
constexpr int FE_SPLIT = 8;  // frame ranges per clip for the statistics
constexpr float PREEMPH = 0.97f;

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 mul_neg_i(float2 a) { return make_float2(a.y, -a.x); }  // -i a

// 4-point DFT, natural order in and out: X[k] = sum_n a[n] e^{-2 pi i n k / 4}.
__device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 e0 = cadd(a0, a2), e1 = csub(a0, a2), o0 = cadd(a1, a3), o1 = mul_neg_i(csub(a1, a3));
  a0 = cadd(e0, o0);
  a2 = csub(e0, o0);
  a1 = cadd(e1, o1);
  a3 = csub(e1, o1);
}

// 8-point DFT, natural order in and out, as two 4-point DFTs (even and odd inputs).
__device__ __forceinline__ void dft8(float2 (&v)[8]) {
  constexpr float C = 0.70710678118654752f;  // cos(pi / 4)
  float2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6], o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
  dft4(e0, e1, e2, e3);
  dft4(o0, o1, o2, o3);
  o1 = make_float2(C * (o1.x + o1.y), C * (o1.y - o1.x));   // e^{-i pi/4} o1
  o2 = mul_neg_i(o2);                                         // e^{-i pi/2} o2
  o3 = make_float2(C * (o3.y - o3.x), -C * (o3.x + o3.y));  // e^{-3i pi/4} o3
  v[0] = cadd(e0, o0);
  v[4] = csub(e0, o0);
  v[1] = cadd(e1, o1);
  v[5] = csub(e1, o1);
  v[2] = cadd(e2, o2);
  v[6] = csub(e2, o2);
  v[3] = cadd(e3, o3);
  v[7] = csub(e3, o3);
}

__device__ __forceinline__ int find_clip(const int* off, int clips, int row) {
  int lo = 0, hi = clips;  // off[lo] <= row < off[hi]
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (off[mid] <= row) lo = mid; else hi = mid;
  }
  return lo;
}

// A sample as float32: float input as is, 16-bit PCM as pcm / 32768 (exact: a power of
// two), as tinybark/pytorch/__init__.py:50 converts it.
__device__ __forceinline__ float sample_f(const float* x, long long n) { return x[n]; }
__device__ __forceinline__ float sample_f(const int16_t* x, long long n) { return (float)x[n] * (1.0f / 32768.0f); }

template <typename S>
__device__ __forceinline__ float preemph_sample(const S* x, long long n, long long len) {
  if (n < 0 || n >= len) return 0.f;
  // Rounded as numpy rounds it: the product, then the difference.
  return n == 0 ? sample_f(x, 0) : __fsub_rn(sample_f(x, n), __fmul_rn(PREEMPH, sample_f(x, n - 1)));
}

template <typename S>
__global__ void __launch_bounds__(256) logmel_kernel(const S* __restrict__ samples,
                                                     const long long* __restrict__ sample_off,
                                                     const int* __restrict__ frame_off, int clips, int frames_total,
                                                     const float* __restrict__ window, const float* __restrict__ mel_w,
                                                     const int* __restrict__ mel_start, const int* __restrict__ mel_off,
                                                     float* __restrict__ feats) {
  __shared__ float2 tw256[256];     // e^{-2 pi i k / 256}
  __shared__ float2 tw512[257];     // e^{-2 pi i k / 512}
  __shared__ float2 z[FE_WARPS][264];  // per warp: the two transposes, then the spectrum
  __shared__ float pw[FE_WARPS][260];
  __shared__ float win[512];
  for (int k = threadIdx.x; k < 256; k += 256) {
    double s, c;
    sincospi(-2.0 * k / 256.0, &s, &c);
    tw256[k] = make_float2((float)c, (float)s);
  }
  for (int k = threadIdx.x; k < 257; k += 256) {
    double s, c;
    sincospi(-2.0 * k / 512.0, &s, &c);
    tw512[k] = make_float2((float)c, (float)s);
  }
  for (int k = threadIdx.x; k < 512; k += 256) win[k] = window[k];
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * FE_WARPS + warp;
  if (row >= frames_total) return;
  const int clip = find_clip(frame_off, clips, row);
  const int f = row - frame_off[clip];
  const S* x = samples + sample_off[clip];
  const long long len = sample_off[clip + 1] - sample_off[clip];
  float2* zw = z[warp];

  // Windowed frame, paired as complex z[n] = w[2n] + i w[2n+1]; lane L holds
  // z[32 n1 + L], n1 = 0..7.
  float2 v[8];
#pragma unroll
  for (int n1 = 0; n1 < 8; ++n1) {
    const int n = 32 * n1 + lane, k0 = 2 * n, k1 = 2 * n + 1;
    const long long p0 = (long long)f * 160 + k0 - 256, p1 = p0 + 1;
    const float a = win[k0] != 0.f ? __fmul_rn(preemph_sample(x, p0, len), win[k0]) : 0.f;
    const float b = win[k1] != 0.f ? __fmul_rn(preemph_sample(x, p1, len), win[k1]) : 0.f;
    v[n1] = make_float2(a, b);
  }
  // Z[k1 + 8 k2] = sum_n2 W32^(n2 k2) W256^(n2 k1) sum_n1 z[32 n1 + n2] W8^(n1 k1).
  dft8(v);  // over n1: lane L = n2 now holds Y[k1], k1 = 0..7
#pragma unroll
  for (int k1 = 1; k1 < 8; ++k1) v[k1] = cmul(v[k1], tw256[lane * k1]);
  // The 32-point DFTs over n2 (one per k1), as 4 x 8 with n2 = 8 a + b, k2 = c + 4 d:
  // Z32[c + 4 d] = sum_b W8^(b d) W32^(b c) sum_a y[8 a + b] W4^(a c).
  // Transpose 1: T1[k1][n2] (rows of 33). Lane L then takes (k1, b) = (L / 8, L % 8) and
  // (L / 8 + 4, L % 8): a 4-point DFT over a each, then the W32^(b c) twiddle.
#pragma unroll
  for (int k1 = 0; k1 < 8; ++k1) zw[k1 * 33 + lane] = v[k1];
  __syncwarp();
  const int b = lane & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k1 = (lane >> 3) + 4 * h;
    float2 a0 = zw[k1 * 33 + b], a1 = zw[k1 * 33 + 8 + b], a2 = zw[k1 * 33 + 16 + b], a3 = zw[k1 * 33 + 24 + b];
    dft4(a0, a1, a2, a3);  // now indexed by c
    v[4 * h] = a0;
    v[4 * h + 1] = cmul(a1, tw256[8 * b]);
    v[4 * h + 2] = cmul(a2, tw256[16 * b]);
    v[4 * h + 3] = cmul(a3, tw256[24 * b]);
  }
  __syncwarp();
  // Transpose 2: T2[k1][c][b]. Lane L then takes (k1, c) = (L / 4, L % 4): an 8-point DFT
  // over b, whose output d is Z[k1 + 8 c + 32 d].
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k1 = (lane >> 3) + 4 * h;
#pragma unroll
    for (int c = 0; c < 4; ++c) zw[(k1 * 4 + c) * 8 + b] = v[4 * h + c];
  }
  __syncwarp();
  {
    const int k1 = lane >> 2, c = lane & 3;
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) v[bb] = zw[(k1 * 4 + c) * 8 + bb];
  }
  dft8(v);
  __syncwarp();
#pragma unroll
  for (int d = 0; d < 8; ++d) zw[(lane >> 2) + 8 * (lane & 3) + 32 * d] = v[d];
  __syncwarp();
  // Split into the real-input spectrum, power per bin.
  for (int k = lane; k <= 256; k += 32) {
    const float2 zk = zw[k & 255], zc = zw[(256 - k) & 255];
    const float er = 0.5f * (zk.x + zc.x), ei = 0.5f * (zk.y - zc.y);   // (Z[k] + conj Z[256-k]) / 2
    const float orr = 0.5f * (zk.y + zc.y), oi = -0.5f * (zk.x - zc.x); // (Z[k] - conj Z[256-k]) / 2i
    const float2 w = tw512[k];
    const float xr = er + (w.x * orr - w.y * oi), xi = ei + (w.x * oi + w.y * orr);
    pw[warp][k] = xr * xr + xi * xi;
  }
  __syncwarp();
  float* out = feats + (long long)row * TB_MELS;
  for (int m = lane; m < TB_MELS; m += 32) {
    const int b0 = mel_start[m], o0 = mel_off[m], o1 = mel_off[m + 1];
    float acc = 0.f;
    for (int o = o0; o < o1; ++o) acc = fmaf(mel_w[o], pw[warp][b0 + o - o0], acc);
    out[m] = logf(acc + 5.9604644775390625e-8f);  // 2^-24
  }
}

// Partial sums over one of FE_SPLIT frame ranges of a clip: (sum, sum of squares) per mel.
__global__ void __launch_bounds__(TB_MELS) stats_kernel(const float* __restrict__ feats, const int* __restrict__ frame_off,
                                                        double2* __restrict__ part) {
  const int clip = blockIdx.x, split = blockIdx.y, m = threadIdx.x;
  const int base = frame_off[clip], n = frame_off[clip + 1] - base;
  const int lo = (int)((long long)n * split / FE_SPLIT), hi = (int)((long long)n * (split + 1) / FE_SPLIT);
  double s = 0.0, q = 0.0;
  for (int t = lo; t < hi; ++t) {
    const double v = feats[(long long)(base + t) * TB_MELS + m];
    s += v;
    q += v * v;
  }
  part[((long long)clip * FE_SPLIT + split) * TB_MELS + m] = make_double2(s, q);
}

__global__ void __launch_bounds__(TB_MELS) finish_kernel(const double2* __restrict__ part,
                                                         const int* __restrict__ frame_off, float2* __restrict__ stats) {
  const int clip = blockIdx.x, m = threadIdx.x;
  const double n = frame_off[clip + 1] - frame_off[clip];
  double s = 0.0, q = 0.0;
  for (int k = 0; k < FE_SPLIT; ++k) {
    const double2 p = part[((long long)clip * FE_SPLIT + k) * TB_MELS + m];
    s += p.x;
    q += p.y;
  }
  const double mean = s / n;
  double var = (q - s * mean) / (n - 1.0);
  var = var > 0.0 ? var : 0.0;
  const float stdv = (float)sqrt(var);
  stats[(long long)clip * TB_MELS + m] = make_float2((float)mean, stdv + 1e-5f);
}

__global__ void __launch_bounds__(256) normalize_kernel(float* __restrict__ feats, const int* __restrict__ frame_off,
                                                        int clips, int frames_total, const float2* __restrict__ stats) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  if (row >= frames_total) return;
  const int clip = find_clip(frame_off, clips, row);
  float* r = feats + (long long)row * TB_MELS;
  const float2* st = stats + (long long)clip * TB_MELS;
  for (int m = lane; m < TB_MELS; m += 32) {
    const float2 s = st[m];
    r[m] = (r[m] - s.x) / s.y;
  }
}

size_t frontend_ws(int clips) {
  return align256((size_t)clips * FE_SPLIT * TB_MELS * sizeof(double2)) + align256((size_t)clips * TB_MELS * sizeof(float2));
}

template <typename S>
static int frontend_t(const tb_model& m, const S* samples, const long long* sample_off, const int* frame_off,
                      int clips, int frames_total, float* feats, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (clips <= 0 || frames_total <= 0) return TB_OK;
  if (!samples || !sample_off || !frame_off || !feats || !m.window || !m.mel_w || !m.mel_start || !m.mel_off)
    return TB_ERR_ARG;
  if (ws_bytes < frontend_ws(clips)) return TB_ERR_WORKSPACE;
  double2* part = reinterpret_cast<double2*>(ws);
  float2* stats = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(ws) +
                                            align256((size_t)clips * FE_SPLIT * TB_MELS * sizeof(double2)));
  logmel_kernel<<<(frames_total + FE_WARPS - 1) / FE_WARPS, 256, 0, stream>>>(
      samples, sample_off, frame_off, clips, frames_total, m.window, m.mel_w, m.mel_start, m.mel_off, feats);
  if (int rc = check_launch()) return rc;
  stats_kernel<<<dim3(clips, FE_SPLIT), TB_MELS, 0, stream>>>(feats, frame_off, part);
  if (int rc = check_launch()) return rc;
  finish_kernel<<<clips, TB_MELS, 0, stream>>>(part, frame_off, stats);
  if (int rc = check_launch()) return rc;
  normalize_kernel<<<(frames_total + 7) / 8, 256, 0, stream>>>(feats, frame_off, clips, frames_total, stats);
  return check_launch();
}

int frontend(const tb_model& m, const float* samples, const long long* sample_off, const int* frame_off, int clips,
             int frames_total, float* feats, void* ws, size_t ws_bytes, cudaStream_t stream) {
  return frontend_t(m, samples, sample_off, frame_off, clips, frames_total, feats, ws, ws_bytes, stream);
}

int frontend_pcm16(const tb_model& m, const int16_t* pcm, const long long* sample_off, const int* frame_off,
                   int clips, int frames_total, float* feats, void* ws, size_t ws_bytes, cudaStream_t stream) {
  return frontend_t(m, pcm, sample_off, frame_off, clips, frames_total, feats, ws, ws_bytes, stream);
}

// ---------------------------------------------------------------------------
// The front-end's scratch (per-range partial sums, per-clip statistics) held by the
// library itself, for callers that cannot allocate device memory. Sized for
// TB_FRONTEND_STATIC_MAX_CLIPS clips; every GPU that loads the library keeps it until
// the process exits. Every byte is written before it is read, so nothing is cleared
// between calls.

constexpr size_t FE_STATIC_PART = ((size_t)TB_FRONTEND_STATIC_MAX_CLIPS * FE_SPLIT * TB_MELS * 16 + 255) / 256 * 256;
constexpr size_t FE_STATIC_BYTES = FE_STATIC_PART + ((size_t)TB_FRONTEND_STATIC_MAX_CLIPS * TB_MELS * 8 + 255) / 256 * 256;
static __device__ __align__(256) unsigned char g_frontend_scratch[FE_STATIC_BYTES];

// The device address of the scratch on the current device, looked up once per device.
// In host code the array's name is only a stand-in; kernels must be given this address.
static void* frontend_scratch(int* status) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = fail_cuda();
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_frontend_scratch) != cudaSuccess || !p) {
      *status = fail_cuda();
      return nullptr;
    }
    addr[dev] = p;
  }
  *status = TB_OK;
  return addr[dev];
}

int frontend_static(const tb_model& m, const float* samples, const long long* sample_off, const int* frame_off,
                    int clips, int frames_total, float* feats, cudaStream_t stream) {
  if (clips > TB_FRONTEND_STATIC_MAX_CLIPS) return TB_ERR_TOO_LARGE;
  int status = TB_OK;
  void* scratch = frontend_scratch(&status);
  if (!scratch) return status;
  return frontend(m, samples, sample_off, frame_off, clips, frames_total, feats, scratch, FE_STATIC_BYTES, stream);
}

}  // namespace tb

extern "C" int tb_frontend_static(const tb_model* m, const float* samples, const long long* sample_off,
                                  const int* frame_off, int clips, int frames_total, float* feats, void* stream) {
  if (!m) return TB_ERR_ARG;
  return tb::frontend_static(*m, samples, sample_off, frame_off, clips, frames_total, feats,
                             reinterpret_cast<cudaStream_t>(stream));
}
