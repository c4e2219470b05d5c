// Relative-position multi-head self-attention core, flash style: online softmax over
// key blocks, nothing of size T x T in memory. Replaces the score/softmax/PV part of
// tinybark/tinygrad/model.py:99-116 and softmax_kernel + per-head matmuls of
// tinybark/mojo/bark/gpu.mojo:202-224,308-338.
//
// score(i, j) = ((q_i + u) . k_j + (q_i + v) . r(i - j)) / sqrt(128), where r(p) is
// row max_len-1-p of the layer's projected position table: the Transformer-XL
// relative shift as an index (tinybark/mojo/bark/model.mojo:176-178). For a block of
// BQ queries from q0 and BK keys from k0 the rows needed form one band of
// BQ + BK - 1 table rows starting at max_len - BQ - q0 + k0.
//
// This is the CUDA-core form (fp32 arithmetic on fp32 or bf16 inputs).
#include "common.cuh"
#include "host.h"

namespace tb {

constexpr int AQ = 32, AK = 64, AD = TB_HEAD_DIM, APAD = 132;
constexpr int A_BAND = AQ + AK - 1;
constexpr int ATT_SMEM = (2 * AQ * APAD + AK * APAD + AK * AD + A_BAND * APAD + AQ * (AK + 1)) * 4;

template <typename T>
__device__ __forceinline__ void load_row128(float* dst, const T* src, bool valid, int t) {
  // 32 threads x 4 values.
  float4 v = valid ? load4(src + t * 4) : make_float4(0, 0, 0, 0);
  *reinterpret_cast<float4*>(dst + t * 4) = v;
}

template <typename T>
__global__ void __launch_bounds__(256) relpos_attention_simt(const T* __restrict__ qu, const T* __restrict__ qv,
                                                             const T* __restrict__ kk, const T* __restrict__ vv,
                                                             const T* __restrict__ rel, int max_len,
                                                             const int* __restrict__ t3_off,
                                                             const int* __restrict__ tiles, T* __restrict__ out) {
  extern __shared__ __align__(16) float sm[];
  float* sqU = sm;                     // [AQ][APAD]
  float* sqV = sqU + AQ * APAD;        // [AQ][APAD]
  float* sK = sqV + AQ * APAD;         // [AK][APAD]
  float* sV = sK + AK * APAD;          // [AK][AD]
  float* sR = sV + AK * AD;            // [A_BAND][APAD]
  float* sP = sR + A_BAND * APAD;      // [AQ][AK+1]

  const int clip = tiles[2 * blockIdx.x], q0 = tiles[2 * blockIdx.x + 1];
  const int head = blockIdx.y;
  const int base = t3_off[clip], T_ = t3_off[clip + 1] - base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long col = (long long)head * AD;
  const int rel_rows = 2 * max_len - 1;

  for (int r = warp; r < AQ; r += 8) {
    const bool ok = q0 + r < T_;
    const long long off = (long long)(base + q0 + r) * TB_HIDDEN + col;
    load_row128(sqU + r * APAD, qu + off, ok, lane);
    load_row128(sqV + r * APAD, qv + off, ok, lane);
  }

  // Scores: thread (qi, jg) owns query qi and keys jg, jg+8, ..., jg+56.
  const int qi = tid >> 3, jg = tid & 7;
  // PV: thread (qi, dg) owns output dims dg*16 .. dg*16+15.
  const int dg = tid & 7;
  float o[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) o[d] = 0.f;
  float row_max = -INFINITY, row_sum = 0.f;
  const float scale = rsqrtf((float)AD);

  for (int k0 = 0; k0 < T_; k0 += AK) {
    __syncthreads();
    for (int r = warp; r < AK; r += 8) {
      const bool ok = k0 + r < T_;
      const long long off = (long long)(base + k0 + r) * TB_HIDDEN + col;
      load_row128(sK + r * APAD, kk + off, ok, lane);
      float4 v = ok ? load4(vv + off + lane * 4) : make_float4(0, 0, 0, 0);
      *reinterpret_cast<float4*>(sV + r * AD + lane * 4) = v;
    }
    const int band0 = max_len - AQ - q0 + k0;
    for (int r = warp; r < A_BAND; r += 8) {
      const int row = band0 + r;
      const bool ok = row >= 0 && row < rel_rows;
      load_row128(sR + r * APAD, rel + (long long)(ok ? row : 0) * TB_HIDDEN + col, ok, lane);
    }
    __syncthreads();

    float s[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) s[c] = 0.f;
    const float* qa = sqU + qi * APAD;
    const float* qb = sqV + qi * APAD;
#pragma unroll 4
    for (int d = 0; d < AD; d += 4) {
      const float4 a = *reinterpret_cast<const float4*>(qa + d);
      const float4 b = *reinterpret_cast<const float4*>(qb + d);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int j = jg + 8 * c;
        const float4 kv = *reinterpret_cast<const float4*>(sK + j * APAD + d);
        const float4 rv = *reinterpret_cast<const float4*>(sR + (AQ - 1 - qi + j) * APAD + d);
        s[c] += a.x * kv.x + a.y * kv.y + a.z * kv.z + a.w * kv.w;
        s[c] += b.x * rv.x + b.y * rv.y + b.z * rv.z + b.w * rv.w;
      }
    }
    float blk_max = -INFINITY;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int j = k0 + jg + 8 * c;
      s[c] = j < T_ ? s[c] * scale : -INFINITY;
      blk_max = fmaxf(blk_max, s[c]);
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) blk_max = fmaxf(blk_max, __shfl_xor_sync(0xffffffffu, blk_max, off));
    const float new_max = fmaxf(row_max, blk_max);
    const float corr = row_max == -INFINITY ? 0.f : expf(row_max - new_max);
    float blk_sum = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float p = s[c] == -INFINITY ? 0.f : expf(s[c] - new_max);
      sP[qi * (AK + 1) + jg + 8 * c] = p;
      blk_sum += p;
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) blk_sum += __shfl_xor_sync(0xffffffffu, blk_sum, off);
    row_sum = row_sum * corr + blk_sum;
    row_max = new_max;
    __syncwarp();
#pragma unroll
    for (int d = 0; d < 16; ++d) o[d] *= corr;
    const int kmax = min(AK, T_ - k0);
    for (int j = 0; j < kmax; ++j) {
      const float p = sP[qi * (AK + 1) + j];
      const float* vr = sV + j * AD + dg * 16;
#pragma unroll
      for (int d = 0; d < 16; d += 4) {
        const float4 v = *reinterpret_cast<const float4*>(vr + d);
        o[d] += p * v.x, o[d + 1] += p * v.y, o[d + 2] += p * v.z, o[d + 3] += p * v.w;
      }
    }
  }
  if (q0 + qi < T_) {
    const float inv = 1.0f / row_sum;
    T* dst = out + (long long)(base + q0 + qi) * TB_HIDDEN + col + dg * 16;
#pragma unroll
    for (int d = 0; d < 16; d += 4) store4(dst + d, o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
  }
}

template <typename T>
static int launch_attn_simt(const void* qu, const void* qv, const void* k, const void* v, const void* rel, int max_len,
                            const tb_batch& b, void* out, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(relpos_attention_simt<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) !=
        cudaSuccess)
      return fail_cuda();
    configured = true;
  }
  dim3 grid(b.n_attn_tiles, TB_HEADS);
  relpos_attention_simt<T><<<grid, 256, ATT_SMEM, stream>>>(
      reinterpret_cast<const T*>(qu), reinterpret_cast<const T*>(qv), reinterpret_cast<const T*>(k),
      reinterpret_cast<const T*>(v), reinterpret_cast<const T*>(rel), max_len, b.t3_off, b.attn_tiles,
      reinterpret_cast<T*>(out));
  return check_launch();
}

int attention_tile_rows(int dtype) {
  (void)dtype;
  return AQ;
}

int relpos_attention(int dtype, const void* qu, const void* qv, const void* k, const void* v, const void* rel,
                     int max_len, const tb_batch& b, void* out, int* err, cudaStream_t stream) {
  (void)err;
  if (b.n_attn_tiles <= 0) return TB_OK;
  if (!qu || !qv || !k || !v || !rel || !out || !b.attn_tiles || !b.t3_off || b.max_t3 > max_len) return TB_ERR_ARG;
  if (dtype == TB_BF16) return launch_attn_simt<__nv_bfloat16>(qu, qv, k, v, rel, max_len, b, out, stream);
  if (dtype == TB_F32) return launch_attn_simt<float>(qu, qv, k, v, rel, max_len, b, out, stream);
  return TB_ERR_ARG;
}

}  // namespace tb
