// Self-test of the epilogues' fast arithmetic (no reference counterpart): evaluates one
// of the device functions over a caller's inputs so a test can bound it against exact
// arithmetic. Kinds: 0 rcp_newton (y >= 1), 1 fast_sigmoid, 2 fast_silu, 3 fast_sigmoid2,
// 4 fast_silu2 (pairs), 5 sigmoid_mufu, 6 tanh_mufu, 7 silu2_tanh (pairs).
#include "host.h"
#include "tcgemm.cuh"

namespace tb {

__global__ void selftest_math_kernel(int kind, const float* __restrict__ x, float* __restrict__ y, long long n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (kind == 3 || kind == 4 || kind == 7) {
    if (2 * i + 1 >= n + 1) return;  // pairs; an odd last element is paired with itself
    const long long j = 2 * i + 1 < n ? 2 * i + 1 : 2 * i;
    const float2 v = make_float2(x[2 * i], x[j]);
    const float2 r = kind == 3 ? fast_sigmoid2(v) : (kind == 4 ? fast_silu2(v) : silu2_tanh(v));
    y[2 * i] = r.x;
    if (j != 2 * i) y[j] = r.y;
    return;
  }
  if (i >= n) return;
  const float v = x[i];
  float r;
  switch (kind) {
    case 0: r = rcp_newton(v); break;
    case 1: r = fast_sigmoid(v); break;
    case 2: r = fast_silu(v); break;
    case 5: r = sigmoid_mufu(v); break;
    default: r = tanh_mufu(v); break;
  }
  y[i] = r;
}

int selftest_math(int kind, const float* x, float* y, long long n, cudaStream_t stream) {
  if (kind < 0 || kind > 7 || n < 0 || (n > 0 && (!x || !y))) return TB_ERR_ARG;
  if (n == 0) return TB_OK;
  const long long threads = (kind == 3 || kind == 4 || kind == 7) ? (n + 1) / 2 : n;
  const long long blocks = (threads + 255) / 256;
  if (blocks > 0x7fffffffLL) return TB_ERR_ARG;
  selftest_math_kernel<<<(unsigned)blocks, 256, 0, stream>>>(kind, x, y, n);
  return check_launch();
}

}  // namespace tb

extern "C" int tb_selftest_math(int kind, const float* x, float* y, long long n, void* stream) {
  return tb::selftest_math(kind, x, y, n, reinterpret_cast<cudaStream_t>(stream));
}
