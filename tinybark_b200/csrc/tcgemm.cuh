// Device-side pieces of the tcgen05 GEMM shared by the GEMM kernel (gemm.cu) and the
// persistent decoder (decode_tc.cu): shared-memory barriers, bounded waits and the
// fused epilogues that drain one 128-row accumulator tile from tensor memory.
#pragma once
#include "epilogue.cuh"

namespace tb {

constexpr int TC_OUT_STRIDE = 36;  // floats per staged row: 16-byte aligned, conflict-free
// Epilogue of a split-K residual GEMM (an internal kind beside tb_epilogue_kind): each
// K-split's partial product, times alpha, added to the fp32 residual with atomic adds.
constexpr int EPI_RESIDUAL_SPLIT = 64;

struct TcBars {
  uint64_t full[8], empty[8], tfull[2], tempty[2], done;
  uint32_t tmem;
  int abort;
  unsigned phase;  // persistent decoder: last phase whose grid barrier this CTA has seen
};

// Bounded wait used while winding down: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  uint64_t start = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - start > TB_WAIT_NS) break;
}

// One lane waits, the warp follows.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, TB_DEV_GEMM_TIMEOUT, abort);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// sigmoid through tanh_mufu (common.cuh), for the bf16 decoder's LSTM cells, whose inputs
// and outputs are bf16 (2^-8).
__device__ __forceinline__ float sigmoid_mufu(float x) { return fmaf(0.5f, tanh_mufu(0.5f * x), 0.5f); }

// Global values an epilogue reads, loaded by each epilogue warp for its 32 rows of a
// tile before it waits for the tile's accumulator, so their latency hides behind the
// main loop instead of adding to the epilogue. This matters for the decoder's GEMMs,
// which run one tile per CTA: there nothing else overlaps the epilogue. Lane layout as
// in epi_chunk: rows row0 + 4*it + lane/8, columns n0 + 32*ci + 4*(lane%8) .. +3.
template <int EPI, int BN>
struct EpiPre {
  __device__ __forceinline__ void load(const tb_epilogue&, int, int, int, int) {}
};

template <int BN>
struct EpiPre<TB_EPI_JOINT_IN, BN> {
  static constexpr int CH = BN / 32, PX = CH < 2 ? CH : 2;  // gathered values of the first PX chunks
  int g[8];
  float4 b[CH];
  float4 x[PX][8];
  __device__ __forceinline__ void load(const tb_epilogue& e, int row0, int n0, int lane, int M) {
    const int sub = lane >> 3, col = (lane & 7) * 4;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      g[it] = m < M ? e.gather_row[m] : -1;
    }
#pragma unroll
    for (int ci = 0; ci < CH; ++ci) b[ci] = load4(e.bias + n0 + ci * 32 + col);
#pragma unroll
    for (int ci = 0; ci < PX; ++ci)
#pragma unroll
      for (int it = 0; it < 8; ++it)
        x[ci][it] = g[it] >= 0 ? load4(e.gather + (long long)g[it] * e.ldo + n0 + ci * 32 + col)
                               : make_float4(0, 0, 0, 0);
  }
};

// Global operands of one 32-column chunk, loaded one chunk ahead (the first before the
// accumulator wait) so their latency overlaps the previous chunk's work: the residual
// rows (RESIDUAL), the bias (STORE, BIAS_RELU) or the two position biases (QKV). Lane
// layout as in epi_chunk.
template <int EPI>
struct ChunkOps {
  __device__ __forceinline__ void load(const tb_epilogue&, int, int, int, int) {}
};
template <>
struct ChunkOps<TB_EPI_RESIDUAL> {
  float4 x[8];
  __device__ __forceinline__ void load(const tb_epilogue& e, int row0, int n0, int lane, int M) {
    const int sub = lane >> 3, n = n0 + (lane & 7) * 4;
    const float* out = reinterpret_cast<const float*>(e.out);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      x[it] = m < M ? load4(out + (long long)m * e.ldo + n) : make_float4(0, 0, 0, 0);
    }
  }
};
template <int EPI>
struct BiasOps {
  float4 b;
  __device__ __forceinline__ void load(const tb_epilogue& e, int, int n0, int lane, int) {
    b = e.bias ? load4(e.bias + n0 + (lane & 7) * 4) : make_float4(0, 0, 0, 0);
  }
};
template <>
struct ChunkOps<TB_EPI_STORE> : BiasOps<TB_EPI_STORE> {};
template <>
struct ChunkOps<TB_EPI_BIAS_RELU> : BiasOps<TB_EPI_BIAS_RELU> {};
template <>
struct ChunkOps<TB_EPI_QKV> {
  float4 u, v;
  __device__ __forceinline__ void load(const tb_epilogue& e, int, int n0, int lane, int) {
    const int n = n0 + (lane & 7) * 4, c = n & 1023;
    const bool q = (n >> 10) == 0;
    u = q ? load4(e.bias_u + c) : make_float4(0, 0, 0, 0);
    v = q && e.out2 ? load4(e.bias_v + c) : make_float4(0, 0, 0, 0);
  }
};

// Stores the 8 row segments of a chunk (rows row0 + 4 it + sub, columns n .. n + 3) to
// e.out in e.out_dtype, skipping rows >= M; the dtype test is made once, not per row.
__device__ __forceinline__ void store_rows4(const tb_epilogue& e, const float4 (&v)[8], int row0, int sub, int n,
                                            int M) {
  if (e.out_dtype == TB_BF16) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(e.out);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M) store4(out + (long long)m * e.ldo + n, v[it].x, v[it].y, v[it].z, v[it].w);
    }
  } else {
    float* out = reinterpret_cast<float*>(e.out);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M) store4(out + (long long)m * e.ldo + n, v[it].x, v[it].y, v[it].z, v[it].w);
    }
  }
}

// The epilogue of one warp's 32 x 32 chunk ci of a tile, staged row-major (stride
// OUT_STRIDE) in `stage`: lane reads rows 4*it + lane/8 (it = 0..7), columns
// 4*(lane%8) .. +3. row0: global row of the chunk's first row; n0: global column of its
// first column.
template <int EPI, int BN>
__device__ __forceinline__ void epi_chunk(const tb_epilogue& e, const float* stage, int row0, int n0, int lane, int M,
                                          const EpiPre<EPI, BN>& pre, int ci, const ChunkOps<EPI>& ops) {
  constexpr int S = TC_OUT_STRIDE;
  const int sub = lane >> 3, col = (lane & 7) * 4, n = n0 + col;
  float4 v[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) v[it] = *reinterpret_cast<const float4*>(stage + (it * 4 + sub) * S + col);
  if constexpr (EPI == EPI_RESIDUAL_SPLIT) {
    float* out = reinterpret_cast<float*>(e.out);
    const float alpha = e.alpha;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m >= M) continue;
      float* p = out + (long long)m * e.ldo + n;
      atomicAdd(p, alpha * v[it].x);
      atomicAdd(p + 1, alpha * v[it].y);
      atomicAdd(p + 2, alpha * v[it].z);
      atomicAdd(p + 3, alpha * v[it].w);
    }
  } else if constexpr (EPI == TB_EPI_RESIDUAL) {
    float* out = reinterpret_cast<float*>(e.out);
    const float4* x = ops.x;
    const float alpha = e.alpha;
#pragma unroll
    for (int it = 0; it < 8; ++it)
      v[it] = make_float4(fmaf(alpha, v[it].x, x[it].x), fmaf(alpha, v[it].y, x[it].y), fmaf(alpha, v[it].z, x[it].z),
                          fmaf(alpha, v[it].w, x[it].w));
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M) store4(out + (long long)m * e.ldo + n, v[it].x, v[it].y, v[it].z, v[it].w);
    }
  } else if constexpr (EPI == TB_EPI_STORE || EPI == TB_EPI_BIAS_RELU) {
    const float4 b = ops.b;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      float4& a = v[it];
      a.x += b.x, a.y += b.y, a.z += b.z, a.w += b.w;
      if constexpr (EPI == TB_EPI_BIAS_RELU) a.x = fmaxf(a.x, 0.f), a.y = fmaxf(a.y, 0.f), a.z = fmaxf(a.z, 0.f), a.w = fmaxf(a.w, 0.f);
    }
    store_rows4(e, v, row0, sub, n, M);
  } else if constexpr (EPI == TB_EPI_SILU) {
    // All 32 activations first (independent chains the scheduler can interleave), then
    // the stores.
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const float2 lo = silu2_tanh(make_float2(v[it].x, v[it].y)), hi = silu2_tanh(make_float2(v[it].z, v[it].w));
      v[it] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    store_rows4(e, v, row0, sub, n, M);
  } else if constexpr (EPI == TB_EPI_GLU) {
    float2 g[8];
#pragma unroll
    for (int it = 0; it < 8; ++it)
      g[it] = mul2(make_float2(v[it].x, v[it].z), fast_sigmoid2(make_float2(v[it].y, v[it].w)));
    if (e.out_dtype == TB_BF16) {
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(e.out);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int m = row0 + it * 4 + sub;
        if (m < M) store2(out + (long long)m * e.ldo + (n >> 1), g[it].x, g[it].y);
      }
    } else {
      float* out = reinterpret_cast<float*>(e.out);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int m = row0 + it * 4 + sub;
        if (m < M) store2(out + (long long)m * e.ldo + (n >> 1), g[it].x, g[it].y);
      }
    }
  } else if constexpr (EPI == TB_EPI_QKV) {
    const int sec = n >> 10, c = n & 1023;
    void* dst = sec == 0 ? e.out : (sec == 1 ? e.out3 : e.out4);
    (void)c;
    const float4 u = ops.u, w = ops.v;
    if (sec == 0 && e.out2) {  // fp32 path: q + bias_v as well
      float4 qv[8];
#pragma unroll
      for (int it = 0; it < 8; ++it) qv[it] = make_float4(v[it].x + w.x, v[it].y + w.y, v[it].z + w.z, v[it].w + w.w);
      tb_epilogue e2 = e;
      e2.out = e.out2;
      store_rows4(e2, qv, row0, sub, c, M);
    }
#pragma unroll
    for (int it = 0; it < 8; ++it) v[it] = make_float4(v[it].x + u.x, v[it].y + u.y, v[it].z + u.z, v[it].w + u.w);
    tb_epilogue e1 = e;
    e1.out = dst;
    store_rows4(e1, v, row0, sub, c, M);
  } else if constexpr (EPI == TB_EPI_JOINT_IN) {
    constexpr int PX = EpiPre<EPI, BN>::PX;
    const float4 b = pre.b[ci];
    float* out = reinterpret_cast<float*>(e.out);
    float4 x[8];
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      if (ci < PX)
        x[it] = pre.x[ci < PX ? ci : 0][it];
      else
        x[it] = pre.g[it] >= 0 ? load4(e.gather + (long long)pre.g[it] * e.ldo + n) : make_float4(0, 0, 0, 0);
    }
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m >= M) continue;
      const float d0 = v[it].x + b.x, d1 = v[it].y + b.y, d2 = v[it].z + b.z, d3 = v[it].w + b.w;
      if (out) store4(out + (long long)m * e.ldo + n, d0, d1, d2, d3);
      if (pre.g[it] >= 0)
        store4_dt(e.out2, (long long)m * e.ldo2 + n, e.out_dtype, fmaxf(x[it].x + d0, 0.f), fmaxf(x[it].y + d1, 0.f),
                  fmaxf(x[it].z + d2, 0.f), fmaxf(x[it].w + d3, 0.f));
    }
  }
}

// The new h of one warp's 32 rows (lane = row, in `tile`, 32 rows x 33 floats) out to
// e.h (fp32), e.out and e.out2 (out_dtype) as row segments: U units of a row per warp
// store. Only rows whose bit is set in `steps` (and below M) are written.
template <int BN>
__device__ __forceinline__ void lstm_store_h(const tb_epilogue& e, const float* tile, int row0, int n0, int lane,
                                             int M, unsigned steps) {
  constexpr int U = BN / 4, RPI = 32 / U, TS = 33;
  const int u0 = n0 >> 2, j = lane % U, rsub = lane / U;
  float* const hst = e.h;
  void* const out = e.out;
  void* const out2 = e.out2;
  const int dt = e.out_dtype;
  const long long ldo = e.ldo, ldo2 = e.ldo2;
  if (U == 32 && dt == TB_BF16 && !hst) {
    // 16-byte stores: lane l writes units 8q .. 8q+7 (q = l % 4) of rows l/4 + 8i, so one
    // warp store covers 8 row segments (4 stores per warp instead of 32).
    const int q = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = (lane >> 2) + 8 * i, m = row0 + row;
      const float* t = tile + row * TS + 8 * q;
      uint4 pk;
      pk.x = pack_bf16x2(t[0], t[1]);
      pk.y = pack_bf16x2(t[2], t[3]);
      pk.z = pack_bf16x2(t[4], t[5]);
      pk.w = pack_bf16x2(t[6], t[7]);
      if (((steps >> row) & 1u) && m < M) {
        if (out) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + (long long)m * ldo + u0 + 8 * q) = pk;
        if (out2)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out2) + (long long)m * ldo2 + u0 + 8 * q) = pk;
      }
    }
    return;
  }
  float v[U];
#pragma unroll
  for (int it = 0; it < U; ++it) v[it] = tile[(it * RPI + rsub) * TS + j];
  auto row_ok = [&](int it) {
    const int row = it * RPI + rsub;
    return ((steps >> row) & 1u) && row0 + row < M;
  };
  auto at = [&](int it, long long ld) { return (long long)(row0 + it * RPI + rsub) * ld + u0 + j; };
  if (hst) {
#pragma unroll
    for (int it = 0; it < U; ++it)
      if (row_ok(it)) hst[at(it, TB_PRED)] = v[it];
  }
  if (dt == TB_BF16) {
    if (out) {
#pragma unroll
      for (int it = 0; it < U; ++it)
        if (row_ok(it)) reinterpret_cast<__nv_bfloat16*>(out)[at(it, ldo)] = __float2bfloat16_rn(v[it]);
    }
    if (out2) {
#pragma unroll
      for (int it = 0; it < U; ++it)
        if (row_ok(it)) reinterpret_cast<__nv_bfloat16*>(out2)[at(it, ldo2)] = __float2bfloat16_rn(v[it]);
    }
  } else {
    if (out) {
#pragma unroll
      for (int it = 0; it < U; ++it)
        if (row_ok(it)) reinterpret_cast<float*>(out)[at(it, ldo)] = v[it];
    }
    if (out2) {
#pragma unroll
      for (int it = 0; it < U; ++it)
        if (row_ok(it)) reinterpret_cast<float*>(out2)[at(it, ldo2)] = v[it];
    }
  }
}

// The LSTM cell epilogue for one warp's 32 rows of a tile. W rows are gate-interleaved,
// so columns n0 .. n0+BN-1 hold the gates (i, f, g, o) of units u0 = n0/4 .. u0+U-1,
// U = BN/4. Each lane computes the cells of one row (tensor-memory lane = row) straight
// from its 32-column chunks; the previous cell state comes in (cp.async, issued before
// the accumulator wait) and the new c and h go out through `tile` (32 rows x 33 floats
// of shared memory), so that global loads and stores are whole row segments (one
// 128-byte line per row for U = 32) rather than a 32-byte piece per row and chunk.
// Loops are kept rolled: in the persistent decoder every phase runs its epilogue once
// per iteration, and compact code stays in the instruction cache between iterations.
// Rows with mask[m] == 0 (and rows >= M) are left as they are.
//
// CREG: the cell state of the lane's row lives in the caller's registers `creg` instead
// of e.c (the persistent decoder runs a tile's rows on the same warp every step): no
// loads or stores of c, and one pass over the accumulator.
template <int BN, bool CREG = false>
__device__ __forceinline__ bool lstm_tile(const tb_epilogue& e, float* tile, uint32_t taddr, int row0, int n0,
                                          int lane, int M, uint64_t* tfull, uint32_t ph, int* err,
                                          volatile int* abort, float (*creg)[BN / 4] = nullptr) {
  static_assert(BN == 64 || BN == 128, "LSTM tiles cover 16 or 32 units");
  constexpr int U = BN / 4, RPI = 32 / U, TS = 33;  // units per row, rows per warp access, tile stride
  const int u0 = n0 >> 2, j = lane % U, rsub = lane / U;
  if constexpr (CREG) {
    const float4 bl = load4(e.bias + n0 + 4 * (lane % U));
    const int my_m = row0 + lane;
    const int step = my_m < M && (!e.mask || e.mask[my_m] != 0);
    if (!warp_wait(tfull, ph, err, abort)) return false;
    tc_fence_after();
    const unsigned steps = __ballot_sync(0xffffffffu, step);
    float* c = *creg;
#pragma unroll
    for (int ci = 0; ci < BN / 32; ++ci) {
      uint32_t r[32];
      tmem_ld32(taddr + ci * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int uu = ci * 8 + k;
        const float ig = sigmoid_mufu(__uint_as_float(r[4 * k]) + __shfl_sync(0xffffffffu, bl.x, uu));
        const float fg = sigmoid_mufu(__uint_as_float(r[4 * k + 1]) + __shfl_sync(0xffffffffu, bl.y, uu));
        const float gg = tanh_mufu(__uint_as_float(r[4 * k + 2]) + __shfl_sync(0xffffffffu, bl.z, uu));
        const float og = sigmoid_mufu(__uint_as_float(r[4 * k + 3]) + __shfl_sync(0xffffffffu, bl.w, uu));
        const float cn = fg * c[uu] + ig * gg;
        if (step) c[uu] = cn;
        tile[lane * TS + uu] = og * tanh_mufu(cn);
      }
    }
    __syncwarp();
    lstm_store_h<BN>(e, tile, row0, n0, lane, M, steps);
    __syncwarp();
    return true;
  }
  float* const cst = e.c;
  const float* const bias = e.bias;
#pragma unroll 1
  for (int it = 0; it < U; ++it) {
    const int row = it * RPI + rsub, m = row0 + row;
    if (m < M) cp_async4(tile + row * TS + j, cst + (long long)m * TB_PRED + u0 + j);
  }
  cp_async_commit();
  // Lane l holds the four gate biases of unit u0 + l (l < U); the cells take them by shuffle.
  const float4 bl = load4(bias + n0 + 4 * (lane % U));
  const int my_m = row0 + lane;
  const int step = my_m < M && (!e.mask || e.mask[my_m] != 0);
  if (!warp_wait(tfull, ph, err, abort)) {
    cp_async_wait_all();
    return false;
  }
  tc_fence_after();
  cp_async_wait_all();
  const unsigned steps = __ballot_sync(0xffffffffu, step);  // bit r: row row0 + r is updated
  __syncwarp();
  // Pass 1: the new cell state, into the tile, then out to e.c.
#pragma unroll 1
  for (int ci = 0; ci < BN / 32; ++ci) {
    uint32_t r[32];
    tmem_ld32(taddr + ci * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int uu = ci * 8 + k;
      const float ig = sigmoid_mufu(__uint_as_float(r[4 * k]) + __shfl_sync(0xffffffffu, bl.x, uu));
      const float fg = sigmoid_mufu(__uint_as_float(r[4 * k + 1]) + __shfl_sync(0xffffffffu, bl.y, uu));
      const float gg = tanh_mufu(__uint_as_float(r[4 * k + 2]) + __shfl_sync(0xffffffffu, bl.z, uu));
      float* t = tile + lane * TS + uu;
      *t = fg * *t + ig * gg;
    }
  }
  __syncwarp();
  // Row segments out: every tile read first, then the stores (program order keeps the
  // loads from waiting behind stores the compiler cannot prove disjoint).
  float v[U];
#pragma unroll
  for (int it = 0; it < U; ++it) v[it] = tile[(it * RPI + rsub) * TS + j];
#pragma unroll
  for (int it = 0; it < U; ++it) {
    const int row = it * RPI + rsub, m = row0 + row;
    if (((steps >> row) & 1u) && m < M) cst[(long long)m * TB_PRED + u0 + j] = v[it];
  }
  __syncwarp();
  // Pass 2: h = o * tanh(c), the output gate read again from tensor memory (the
  // accumulator is not released until this epilogue returns), into the tile and out.
#pragma unroll 1
  for (int ci = 0; ci < BN / 32; ++ci) {
    uint32_t r[32];
    tmem_ld32(taddr + ci * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int uu = ci * 8 + k;
      const float og = sigmoid_mufu(__uint_as_float(r[4 * k + 3]) + __shfl_sync(0xffffffffu, bl.w, uu));
      float* t = tile + lane * TS + uu;
      *t = og * tanh_mufu(*t);
    }
  }
  __syncwarp();
  lstm_store_h<BN>(e, tile, row0, n0, lane, M, steps);
  __syncwarp();
  return true;
}

// The joint head's epilogue for one row (one lane) of a tile: the largest token logit
// and the largest duration logit with their first column, merged into the row's keys.
// `bias` holds the tile's BN bias values. Padding columns have bias -inf and never win.
// Token columns go in 64-column chunks (two tensor-memory loads per wait; a load is
// warp-collective, so every lane reads the same columns) through four running maxima
// (columns j = 0..3 mod 4). Each keeps its first column: fmaxf gives the new maximum,
// and the column changes only when the maximum did, so a tie keeps the earlier column
// and each chain's dependence is one fmaxf per column. The columns from the last whole
// chunk on (the token/duration boundary) are compared one by one, in column order.
template <int BN>
__device__ __forceinline__ void argmax_tile(const tb_epilogue& e, const float* bias, uint32_t taddr, int m, int n0,
                                            int M) {
  const float neg_inf = __int_as_float(0xff800000);
  const int split = e.split, split_end = e.split_end;
  int tok_end = split - n0;  // token columns of this tile: [0, tok_end)
  tok_end = tok_end < 0 ? 0 : (tok_end > BN ? BN : tok_end);
  const int whole = tok_end & ~63;
  float best[4] = {neg_inf, neg_inf, neg_inf, neg_inf};
  int idx[4] = {-1, -1, -1, -1};
#pragma unroll 1
  for (int c = 0; c < whole; c += 64) {
    uint32_t r[2][32];
    tmem_ld32(taddr + c, r[0]);
    tmem_ld32(taddr + c + 32, r[1]);
    tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 b = *reinterpret_cast<const float4*>(bias + c + 32 * h + j);
        const int n = n0 + c + 32 * h + j;
        const float x[4] = {__uint_as_float(r[h][j]) + b.x, __uint_as_float(r[h][j + 1]) + b.y,
                            __uint_as_float(r[h][j + 2]) + b.z, __uint_as_float(r[h][j + 3]) + b.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float nb = fmaxf(best[k], x[k]);
          idx[k] = nb != best[k] ? n + k : idx[k];
          best[k] = nb;
        }
      }
  }
  float tb = best[0];
  int ti = idx[0];
#pragma unroll
  for (int k = 1; k < 4; ++k)
    if (idx[k] >= 0 && (ti < 0 || best[k] > tb || (best[k] == tb && idx[k] < ti))) tb = best[k], ti = idx[k];
  float dbest = neg_inf;
  int di = -1;
  const int cols = split_end - n0 < BN ? split_end - n0 : BN;
#pragma unroll 1
  for (int c = whole; c < cols; c += 32) {  // the boundary: token, duration and padding columns
    const int n = n0 + c;
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float x = __uint_as_float(r[j]) + bias[c + j];
      if (n + j < split) {
        if (x > tb) tb = x, ti = n + j;
      } else if (n + j < split_end) {
        if (x > dbest) dbest = x, di = n + j - split;
      }
    }
  }
  if (m < M) {
    if (ti >= 0) atomicMax(e.keys + m, argmax_key(tb, ti));
    if (di >= 0) atomicMax(e.keys2 + m, argmax_key(dbest, di));
  }
}

// The epilogue of one accumulator tile for the calling epilogue warp: its 32 rows
// row0 .. row0+31 (tensor-memory lanes of the warp's quarter, at `taddr`), columns
// n0 .. n0+BN-1. Loads the epilogue's global operands, waits for the accumulator
// (`tfull`, parity `ph`), then drains it in 32-column chunks through the warp's staging
// rows `stage` (32 x TC_OUT_STRIDE floats). Rows >= M are not written. False if the
// wait gave up (error recorded in `err`).
template <int BN, int EPI>
__device__ __forceinline__ bool epilogue_tile(const tb_epilogue& e, float* stage, uint32_t taddr, int row0, int n0,
                                              int lane, int M, uint64_t* tfull, uint32_t ph, int* err,
                                              volatile int* abort) {
  if constexpr (EPI == TB_EPI_LSTM) {
    return lstm_tile<BN>(e, stage, taddr, row0, n0, lane, M, tfull, ph, err, abort);
  } else if constexpr (EPI == TB_EPI_ARGMAX) {
    // The tile's bias, loaded before the wait, then kept in the warp's staging rows.
    float bias[BN / 32];
#pragma unroll
    for (int ci = 0; ci < BN / 32; ++ci) bias[ci] = e.bias[n0 + ci * 32 + lane];
    if (!warp_wait(tfull, ph, err, abort)) return false;
    tc_fence_after();
#pragma unroll
    for (int ci = 0; ci < BN / 32; ++ci) stage[ci * 32 + lane] = bias[ci];
    __syncwarp();
    argmax_tile<BN>(e, stage, taddr, row0 + lane, n0, M);
    __syncwarp();
  } else {
    EpiPre<EPI, BN> pre;
    pre.load(e, row0, n0, lane, M);
    // Operands two chunks ahead: the residual rows come from HBM, whose latency is
    // longer than one chunk's work.
    ChunkOps<EPI> ops, ops1;
    ops.load(e, row0, n0, lane, M);
    if (BN / 32 > 1) ops1.load(e, row0, n0 + 32, lane, M);
    if (!warp_wait(tfull, ph, err, abort)) return false;
    tc_fence_after();
    auto chunk = [&](int ci) {
      ChunkOps<EPI> next;  // chunk ci + 2's operands, in flight during this one
      if (ci + 2 < BN / 32) next.load(e, row0, n0 + (ci + 2) * 32, lane, M);
      uint32_t r[32];
      tmem_ld32(taddr + ci * 32, r);
      tmem_wait_ld();
      float4* srow = reinterpret_cast<float4*>(stage + lane * TC_OUT_STRIDE);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        srow[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                              __uint_as_float(r[4 * j + 3]));
      __syncwarp();
      epi_chunk<EPI, BN>(e, stage, row0, n0 + ci * 32, lane, M, pre, ci, ops);
      __syncwarp();
      ops = ops1;
      ops1 = next;
    };
    if constexpr (EPI == TB_EPI_JOINT_IN) {
#pragma unroll
      for (int ci = 0; ci < BN / 32; ++ci) chunk(ci);  // prefetched values indexed by ci
    } else {
#pragma unroll 1
      for (int ci = 0; ci < BN / 32; ++ci) chunk(ci);
    }
  }
  return true;
}

}  // namespace tb
