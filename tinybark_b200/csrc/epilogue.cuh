// GEMM epilogues shared by the tensor-core (bf16) and CUDA-core (fp32) GEMMs.
// A group is 4 consecutive output columns of one row, so the interleaved weight
// layouts (GLU pairs, LSTM gate quads) keep every fused output inside one group.
#pragma once
#include "common.cuh"

namespace tb {

__device__ __forceinline__ void store4_dt(void* base, long long off, int dtype, float a, float b, float c, float d) {
  if (dtype == TB_BF16)
    store4(reinterpret_cast<__nv_bfloat16*>(base) + off, a, b, c, d);
  else
    store4(reinterpret_cast<float*>(base) + off, a, b, c, d);
}
__device__ __forceinline__ void store2_dt(void* base, long long off, int dtype, float a, float b) {
  if (dtype == TB_BF16)
    store2(reinterpret_cast<__nv_bfloat16*>(base) + off, a, b);
  else
    store2(reinterpret_cast<float*>(base) + off, a, b);
}
__device__ __forceinline__ void store1_dt(void* base, long long off, int dtype, float a) {
  if (dtype == TB_BF16)
    reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(a);
  else
    reinterpret_cast<float*>(base)[off] = a;
}

// Applies the epilogue to acc[m, n..n+3] (n % 4 == 0, m < M).
__device__ __forceinline__ void epi_group(const tb_epilogue& e, int m, int n, float v0, float v1, float v2, float v3) {
  switch (e.kind) {
    case TB_EPI_STORE: {
      if (e.bias) {
        float4 b = load4(e.bias + n);
        v0 += b.x, v1 += b.y, v2 += b.z, v3 += b.w;
      }
      store4_dt(e.out, (long long)m * e.ldo + n, e.out_dtype, v0, v1, v2, v3);
      break;
    }
    case TB_EPI_SILU:
      store4_dt(e.out, (long long)m * e.ldo + n, e.out_dtype, siluf_(v0), siluf_(v1), siluf_(v2), siluf_(v3));
      break;
    case TB_EPI_RESIDUAL: {
      float* r = reinterpret_cast<float*>(e.out) + (long long)m * e.ldo + n;
      float4 x = load4(r);
      store4(r, x.x + e.alpha * v0, x.y + e.alpha * v1, x.z + e.alpha * v2, x.w + e.alpha * v3);
      break;
    }
    case TB_EPI_BIAS_RELU: {
      float4 b = load4(e.bias + n);
      store4_dt(e.out, (long long)m * e.ldo + n, e.out_dtype, fmaxf(v0 + b.x, 0.f), fmaxf(v1 + b.y, 0.f),
                fmaxf(v2 + b.z, 0.f), fmaxf(v3 + b.w, 0.f));
      break;
    }
    case TB_EPI_GLU:
      store2_dt(e.out, (long long)m * e.ldo + (n >> 1), e.out_dtype, v0 * sigmoidf_(v1), v2 * sigmoidf_(v3));
      break;
    case TB_EPI_QKV: {
      int sec = n >> 10, c = n & 1023;
      long long off = (long long)m * e.ldo + c;
      if (sec == 0) {
        float4 u = load4(e.bias_u + c), w = load4(e.bias_v + c);
        store4_dt(e.out, off, e.out_dtype, v0 + u.x, v1 + u.y, v2 + u.z, v3 + u.w);
        if (e.out2) store4_dt(e.out2, off, e.out_dtype, v0 + w.x, v1 + w.y, v2 + w.z, v3 + w.w);
      } else {
        store4_dt(sec == 1 ? e.out3 : e.out4, off, e.out_dtype, v0, v1, v2, v3);
      }
      break;
    }
    case TB_EPI_JOINT_IN: {
      float4 b = load4(e.bias + n);
      v0 += b.x, v1 += b.y, v2 += b.z, v3 += b.w;
      store4(reinterpret_cast<float*>(e.out) + (long long)m * e.ldo + n, v0, v1, v2, v3);
      const int g = e.gather_row[m];
      if (g >= 0) {
        float4 x = load4(e.gather + (long long)g * e.ldo + n);
        store4_dt(e.out2, (long long)m * e.ldo2 + n, e.out_dtype, fmaxf(x.x + v0, 0.f), fmaxf(x.y + v1, 0.f),
                  fmaxf(x.z + v2, 0.f), fmaxf(x.w + v3, 0.f));
      }
      break;
    }
    case TB_EPI_LSTM: {
      if (e.mask && e.mask[m] == 0) break;
      int u = n >> 2;  // state rows are TB_PRED units long
      float4 b = load4(e.bias + n);
      float ig = sigmoidf_(v0 + b.x), fg = sigmoidf_(v1 + b.y), gg = tanhf(v2 + b.z), og = sigmoidf_(v3 + b.w);
      float* cp = e.c + (long long)m * TB_PRED + u;
      float c = fg * *cp + ig * gg;
      float h = og * tanhf(c);
      *cp = c;
      if (e.h) e.h[(long long)m * TB_PRED + u] = h;
      if (e.out) store1_dt(e.out, (long long)m * e.ldo + u, e.out_dtype, h);
      if (e.out2) store1_dt(e.out2, (long long)m * e.ldo2 + u, e.out_dtype, h);
      break;
    }
    default:
      break;
  }
}

// Running argmax key over the joint head's columns of one row: token columns
// [0, split) and duration columns [split, split_end).
struct ArgmaxAcc {
  unsigned long long tok = 0, dur = 0;
  __device__ __forceinline__ void add(const tb_epilogue& e, int n, float v) {
    if (n < e.split) {
      unsigned long long k = argmax_key(v + e.bias[n], n);
      tok = k > tok ? k : tok;
    } else if (n < e.split_end) {
      unsigned long long k = argmax_key(v + e.bias[n], n - e.split);
      dur = k > dur ? k : dur;
    }
  }
  __device__ __forceinline__ void flush(const tb_epilogue& e, int m) {
    if (tok) atomicMax(e.keys + m, tok);
    if (dur) atomicMax(e.keys2 + m, dur);
  }
};

}  // namespace tb
