// Linear layers: C = A (M x K, row-major) * W (N x K, row-major)^T with a fused
// epilogue. Replaces tinybark/tinygrad/model.py:37-40 (linear) and the MAX matmul calls
// of tinybark/mojo/bark/gpu.mojo:429-436.
//
// bf16: a persistent, warp-specialized tcgen05 kernel. Warp 0 issues TMA tile loads
// into a STAGES-deep shared-memory ring, warp 1 issues tcgen05.mma (128 x BN x 16 per
// instruction) into one of two tensor-memory accumulators, warps 2-5 drain the other
// accumulator through the epilogue, so a tile's epilogue overlaps the next tile's
// main loop. The epilogue is a template parameter; each warp moves its 32 rows x 32
// columns from tensor memory through a shared-memory transpose, so global loads and
// stores are whole row segments (8 lanes per row) instead of one row per lane.
// BN is 256, 128 or 64: small-M GEMMs (the decoder's) take narrow tiles to spread
// over more SMs.
// fp32: a CUDA-core kernel, 128 x 128 tiles, 8 x 8 outputs per thread, for the fp32
// parity path.
#include "epilogue.cuh"
#include "host.h"

namespace tb {

// ---------------------------------------------------------------------------
// tcgen05 bf16 kernel

template <int BN>
struct TcCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int OUT_STRIDE = 36;  // floats per staged row: 16-byte aligned, conflict-free
  static constexpr int OUT_BYTES = 4 * 32 * OUT_STRIDE * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + OUT_BYTES + BAR_BYTES;
};

struct TcBars {
  uint64_t full[8], empty[8], tfull[2], tempty[2], done;
  uint32_t tmem;
  int abort;
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

__device__ __forceinline__ float fast_sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float fast_silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
// The PTX tanh.approx.f32 instruction (one MUFU operation, about 2^-11 relative error).
// Used in the bf16 decoder's LSTM cell, whose inputs and outputs are bf16 (2^-8).
__device__ __forceinline__ float tanh_mufu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
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
struct EpiPre<TB_EPI_LSTM, BN> {
  static constexpr int CH = BN / 32;
  float cp[CH][8];  // previous cell state of unit n/4
  float4 b[CH];
  unsigned step;    // bit it: row 4*it + lane/8 is updated
  __device__ __forceinline__ void load(const tb_epilogue& e, int row0, int n0, int lane, int M) {
    const int sub = lane >> 3, col = (lane & 7) * 4;
    step = 0;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M && (!e.mask || e.mask[m] != 0)) step |= 1u << it;
    }
#pragma unroll
    for (int ci = 0; ci < CH; ++ci) {
      const int n = n0 + ci * 32 + col;
      b[ci] = load4(e.bias + n);
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        const int m = row0 + it * 4 + sub;
        cp[ci][it] = m < M ? e.c[(long long)m * TB_PRED + (n >> 2)] : 0.f;
      }
    }
  }
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

// The epilogue of one warp's 32 x 32 chunk ci of a tile, staged row-major (stride
// OUT_STRIDE) in `stage`: lane reads rows 4*it + lane/8 (it = 0..7), columns
// 4*(lane%8) .. +3. row0: global row of the chunk's first row; n0: global column of its
// first column.
template <int EPI, int BN>
__device__ __forceinline__ void epi_chunk(const tb_epilogue& e, const float* stage, int row0, int n0, int lane, int M,
                                          const EpiPre<EPI, BN>& pre, int ci) {
  constexpr int S = 36;
  const int sub = lane >> 3, col = (lane & 7) * 4, n = n0 + col;
  float4 v[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) v[it] = *reinterpret_cast<const float4*>(stage + (it * 4 + sub) * S + col);
  if constexpr (EPI == TB_EPI_RESIDUAL) {
    float* out = reinterpret_cast<float*>(e.out);
    float4 x[8];
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      x[it] = m < M ? load4(out + (long long)m * e.ldo + n) : make_float4(0, 0, 0, 0);
    }
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M)
        store4(out + (long long)m * e.ldo + n, x[it].x + e.alpha * v[it].x, x[it].y + e.alpha * v[it].y,
               x[it].z + e.alpha * v[it].z, x[it].w + e.alpha * v[it].w);
    }
  } else if constexpr (EPI == TB_EPI_STORE || EPI == TB_EPI_BIAS_RELU) {
    const float4 b = e.bias ? load4(e.bias + n) : make_float4(0, 0, 0, 0);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m >= M) continue;
      float a0 = v[it].x + b.x, a1 = v[it].y + b.y, a2 = v[it].z + b.z, a3 = v[it].w + b.w;
      if constexpr (EPI == TB_EPI_BIAS_RELU) a0 = fmaxf(a0, 0.f), a1 = fmaxf(a1, 0.f), a2 = fmaxf(a2, 0.f), a3 = fmaxf(a3, 0.f);
      store4_dt(e.out, (long long)m * e.ldo + n, e.out_dtype, a0, a1, a2, a3);
    }
  } else if constexpr (EPI == TB_EPI_SILU) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M)
        store4_dt(e.out, (long long)m * e.ldo + n, e.out_dtype, fast_silu(v[it].x), fast_silu(v[it].y),
                  fast_silu(v[it].z), fast_silu(v[it].w));
    }
  } else if constexpr (EPI == TB_EPI_GLU) {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m < M)
        store2_dt(e.out, (long long)m * e.ldo + (n >> 1), e.out_dtype, v[it].x * fast_sigmoid(v[it].y),
                  v[it].z * fast_sigmoid(v[it].w));
    }
  } else if constexpr (EPI == TB_EPI_QKV) {
    const int sec = n >> 10, c = n & 1023;
    void* dst = sec == 0 ? e.out : (sec == 1 ? e.out3 : e.out4);
    const float4 u = sec == 0 ? load4(e.bias_u + c) : make_float4(0, 0, 0, 0);
    const float4 w = sec == 0 ? load4(e.bias_v + c) : make_float4(0, 0, 0, 0);
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int m = row0 + it * 4 + sub;
      if (m >= M) continue;
      const long long off = (long long)m * e.ldo + c;
      store4_dt(dst, off, e.out_dtype, v[it].x + u.x, v[it].y + u.y, v[it].z + u.z, v[it].w + u.w);
      if (sec == 0 && e.out2)
        store4_dt(e.out2, off, e.out_dtype, v[it].x + w.x, v[it].y + w.y, v[it].z + w.z, v[it].w + w.w);
    }
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
      store4(out + (long long)m * e.ldo + n, d0, d1, d2, d3);
      if (pre.g[it] >= 0)
        store4_dt(e.out2, (long long)m * e.ldo2 + n, e.out_dtype, fmaxf(x[it].x + d0, 0.f), fmaxf(x[it].y + d1, 0.f),
                  fmaxf(x[it].z + d2, 0.f), fmaxf(x[it].w + d3, 0.f));
    }
  } else if constexpr (EPI == TB_EPI_LSTM) {
    // Columns n..n+3 are the gates i, f, g, o of unit n / 4.
    const int u = n >> 2;
    const float4 b = pre.b[ci];
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      if (!((pre.step >> it) & 1u)) continue;
      const int m = row0 + it * 4 + sub;
      const float ig = sigmoid_mufu(v[it].x + b.x), fg = sigmoid_mufu(v[it].y + b.y);
      const float gg = tanh_mufu(v[it].z + b.z), og = sigmoid_mufu(v[it].w + b.w);
      const float c = fg * pre.cp[ci][it] + ig * gg;
      const float h = og * tanh_mufu(c);
      e.c[(long long)m * TB_PRED + u] = c;
      e.h[(long long)m * TB_PRED + u] = h;
      if (e.out) store1_dt(e.out, (long long)m * e.ldo + u, e.out_dtype, h);
      if (e.out2) store1_dt(e.out2, (long long)m * e.ldo2 + u, e.out_dtype, h);
    }
  }
}

// The joint head's epilogue for one row (one lane) of a tile: the largest token logit
// and the largest duration logit with their first column, merged into the row's keys.
// `bias` holds the tile's BN bias values. Padding columns have bias -inf and never win.
template <int BN>
__device__ __forceinline__ void argmax_tile(const tb_epilogue& e, const float* bias, uint32_t taddr, int m, int n0,
                                            int M) {
  const float neg_inf = __int_as_float(0xff800000);
  float best = neg_inf, dbest = neg_inf;
  int bi = -1, di = -1;
  const bool tokens_only = n0 + BN <= e.split;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
    if (tokens_only) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 b = *reinterpret_cast<const float4*>(bias + c + j);
        const float x0 = __uint_as_float(r[j]) + b.x, x1 = __uint_as_float(r[j + 1]) + b.y;
        const float x2 = __uint_as_float(r[j + 2]) + b.z, x3 = __uint_as_float(r[j + 3]) + b.w;
        // Strictly greater, columns ascending: the first of equal values wins.
        if (x0 > best) best = x0, bi = n0 + c + j;
        if (x1 > best) best = x1, bi = n0 + c + j + 1;
        if (x2 > best) best = x2, bi = n0 + c + j + 2;
        if (x3 > best) best = x3, bi = n0 + c + j + 3;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + c + j;
        const float x = __uint_as_float(r[j]) + bias[c + j];
        if (n < e.split) {
          if (x > best) best = x, bi = n;
        } else if (n < e.split_end) {
          if (x > dbest) dbest = x, di = n - e.split;
        }
      }
    }
  }
  if (m < M) {
    if (bi >= 0) atomicMax(e.keys + m, argmax_key(best, bi));
    if (di >= 0) atomicMax(e.keys2 + m, argmax_key(dbest, di));
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
                   const tb_epilogue e, int* err) {
  using C = TcCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* out_stage = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
  TcBars* bars = reinterpret_cast<TcBars*>(smem + C::STAGES * C::STAGE_BYTES + C::OUT_BYTES);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);
      mbar_init(&bars->tempty[a], 4);
    }
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  grid_dep_wait();
  grid_dep_launch();

  if (e.rows) M = min(M, *e.rows);
  const int m_tiles = (M + C::BM - 1) / C::BM, n_tiles = N / BN, tiles = m_tiles * n_tiles, kb_count = K / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mt = t / n_tiles, nt = t % n_tiles;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars->empty[s], ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          mbar_expect_tx(&bars->full[s], C::STAGE_BYTES);
          tma_load_2d(sa, &ta, &bars->full[s], kb * C::BK, mt * C::BM);
          tma_load_2d(sa + C::A_BYTES, &tw, &bars->full[s], kb * C::BK, nt * BN);
          ++issued;
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA exits.
        long long back = issued < C::STAGES ? issued : C::STAGES;
        for (long long i = 1; i <= back; ++i) {
          long long idx = issued - i;
          drain_wait(&bars->full[idx % C::STAGES], (uint32_t)((idx / C::STAGES) & 1));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(C::BM, BN);
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&bars->tempty[acc], acc_ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars->full[s], ph, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t ad = sdesc_sw128(sa), bd = sdesc_sw128(sa + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) umma_f16(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit(&bars->empty[s]);
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
        if (!ok) break;
        umma_commit(&bars->tfull[acc]);
        if (++acc == 2) acc = 0, acc_ph ^= 1;
      }
      // Every MMA issued has completed once this commit arrives.
      umma_commit(&bars->done);
      drain_wait(&bars->done, 0);
    }
  } else {
    const int q = warp & 3;  // tensor-memory lane quarter this warp may access
    float* stage = out_stage + q * 32 * C::OUT_STRIDE;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mt = t / n_tiles, nt = t % n_tiles;
      const int row0 = mt * C::BM + q * 32, n0 = nt * BN;
      if constexpr (EPI == TB_EPI_ARGMAX) {
        // The tile's bias, loaded before the wait, then kept in the warp's staging rows.
        float bias[BN / 32];
#pragma unroll
        for (int ci = 0; ci < BN / 32; ++ci) bias[ci] = e.bias[n0 + ci * 32 + lane];
        if (!warp_wait(&bars->tfull[acc], acc_ph, err, abort)) break;
        tc_fence_after();
#pragma unroll
        for (int ci = 0; ci < BN / 32; ++ci) stage[ci * 32 + lane] = bias[ci];
        __syncwarp();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
        argmax_tile<BN>(e, stage, taddr, row0 + lane, n0, M);
        __syncwarp();
      } else {
        EpiPre<EPI, BN> pre;
        pre.load(e, row0, n0, lane, M);
        if (!warp_wait(&bars->tfull[acc], acc_ph, err, abort)) break;
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * BN;
        auto chunk = [&](int ci) {
          uint32_t r[32];
          tmem_ld32(taddr + ci * 32, r);
          tmem_wait_ld();
          float4* srow = reinterpret_cast<float4*>(stage + lane * C::OUT_STRIDE);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            srow[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                  __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          __syncwarp();
          epi_chunk<EPI, BN>(e, stage, row0, n0 + ci * 32, lane, M, pre, ci);
          __syncwarp();
        };
        if constexpr (EPI == TB_EPI_LSTM || EPI == TB_EPI_JOINT_IN) {
#pragma unroll
          for (int ci = 0; ci < BN / 32; ++ci) chunk(ci);  // prefetched values indexed by ci
        } else {
#pragma unroll 1
          for (int ci = 0; ci < BN / 32; ++ci) chunk(ci);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[acc]);
      if (++acc == 2) acc = 0, acc_ph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// fp32 CUDA-core kernel

constexpr int SG_BM = 128, SG_BN = 128, SG_BK = 16, SG_PAD = 4;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, long long lda,
                                                       const float* __restrict__ W, int M, int N, int K,
                                                       const tb_epilogue e) {
  __shared__ __align__(16) float As[2][SG_BK][SG_BM + SG_PAD];
  __shared__ __align__(16) float Ws[2][SG_BK][SG_BN + SG_PAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  grid_dep_wait();
  grid_dep_launch();
  if (e.rows) M = min(M, *e.rows);
  if (m0 >= M) return;
  // Loader mapping: rows lr and lr + 64, k offset lk.
  const int lr = tid >> 2, lk = (tid & 3) * 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float4 ra[2], rw[2];
  auto load = [&](int k0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int m = m0 + lr + h * 64;
      ra[h] = m < M ? *reinterpret_cast<const float4*>(A + (long long)m * lda + k0 + lk) : make_float4(0, 0, 0, 0);
      int n = n0 + lr + h * 64;
      rw[h] = *reinterpret_cast<const float4*>(W + (long long)n * K + k0 + lk);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int r = lr + h * 64;
      As[buf][lk + 0][r] = ra[h].x, As[buf][lk + 1][r] = ra[h].y, As[buf][lk + 2][r] = ra[h].z,
      As[buf][lk + 3][r] = ra[h].w;
      Ws[buf][lk + 0][r] = rw[h].x, Ws[buf][lk + 1][r] = rw[h].y, Ws[buf][lk + 2][r] = rw[h].z,
      Ws[buf][lk + 3][r] = rw[h].w;
    }
  };

  load(0);
  stash(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += SG_BK) {
    const bool more = k0 + SG_BK < K;
    if (more) load(k0 + SG_BK);
#pragma unroll
    for (int k = 0; k < SG_BK; ++k) {
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
      float4 w0 = *reinterpret_cast<const float4*>(&Ws[buf][k][tx * 4]);
      float4 w1 = *reinterpret_cast<const float4*>(&Ws[buf][k][64 + tx * 4]);
      float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    if (more) {
      stash(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

  if (e.kind == TB_EPI_ARGMAX) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
      ArgmaxAcc am;
#pragma unroll
      for (int j = 0; j < 8; ++j) am.add(e, n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4), acc[i][j]);
      // Reduce over the 16 threads sharing this row (same ty, a half warp).
#pragma unroll
      for (int o = 8; o; o >>= 1) {
        unsigned long long t1 = __shfl_xor_sync(0xffffffffu, am.tok, o), t2 = __shfl_xor_sync(0xffffffffu, am.dur, o);
        am.tok = t1 > am.tok ? t1 : am.tok;
        am.dur = t2 > am.dur ? t2 : am.dur;
      }
      if (tx == 0 && m < M) am.flush(e, m);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (m >= M) continue;
    epi_group(e, m, n0 + tx * 4, acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    epi_group(e, m, n0 + 64 + tx * 4, acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
  }
}

// ---------------------------------------------------------------------------
// Host side

bool encode_tmap_2d(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld_elems,
                    int box_cols, int box_rows) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld_elems * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static bool encode_tmap(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld_elems,
                        int box_rows) {
  return encode_tmap_2d(map, ptr, rows, cols, ld_elems, 64, box_rows);
}

template <int BN, int EPI>
static int launch_tc(const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e, int* err,
                     cudaStream_t stream) {
  using C = TcCfg<BN>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return fail_cuda();
    configured = true;
  }
  CUtensorMap ta, tw;
  if (!encode_tmap(&ta, a, m, k, lda, C::BM) || !encode_tmap(&tw, w, n, k, k, BN)) return TB_ERR_CUDA;
  const int tiles = ((m + C::BM - 1) / C::BM) * (n / BN);
  const int grid = tiles < sm_budget() ? tiles : sm_budget();
  return launch_pdl(gemm_tc_kernel<BN, EPI>, grid, 192, C::SMEM, stream, ta, tw, m, n, k, e, err);
}

template <int BN>
static int launch_tc_kind(const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e,
                          int* err, cudaStream_t s) {
  switch (e.kind) {
    case TB_EPI_STORE: return launch_tc<BN, TB_EPI_STORE>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_SILU: return launch_tc<BN, TB_EPI_SILU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_RESIDUAL: return launch_tc<BN, TB_EPI_RESIDUAL>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_BIAS_RELU: return launch_tc<BN, TB_EPI_BIAS_RELU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_GLU: return launch_tc<BN, TB_EPI_GLU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_QKV: return launch_tc<BN, TB_EPI_QKV>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_ARGMAX: return launch_tc<BN, TB_EPI_ARGMAX>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_LSTM: return launch_tc<BN, TB_EPI_LSTM>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_JOINT_IN: return launch_tc<BN, TB_EPI_JOINT_IN>(a, lda, w, m, n, k, e, err, s);
    default: return TB_ERR_ARG;
  }
}

static int pick_bn(int m, int n, int k) {
  // Tile width with the least operand traffic into the busiest SM: waves x (A + B bytes
  // per k-block), plus a per-wave allowance for the prologue and epilogue (about two
  // k-blocks). Wide tiles re-read A less; narrow ones spread small-M GEMMs over more SMs.
  const long long m_tiles = (m + 127) / 128, sms = sm_budget(), kb = k / 64;
  int best = 0;
  long long best_cost = 0;
  for (int bn : {256, 128, 64}) {
    if (n % bn) continue;
    const long long tiles = m_tiles * (n / bn), waves = (tiles + sms - 1) / sms;
    const long long cost = waves * (kb + 2) * (128 * 128 + bn * 128);
    if (!best || cost < best_cost) best = bn, best_cost = cost;
  }
  return best;
}

int gemm(int dtype, const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e, int* err,
         cudaStream_t stream) {
  if (m <= 0) return TB_OK;
  if (n <= 0 || k <= 0 || !a || !w) return TB_ERR_ARG;
  if (e.kind < TB_EPI_STORE || e.kind > TB_EPI_JOINT_IN) return TB_ERR_ARG;
  if (e.kind == TB_EPI_JOINT_IN && (!e.bias || !e.gather || !e.gather_row || !e.out2)) return TB_ERR_ARG;
  if (e.kind == TB_EPI_ARGMAX && (!e.keys || !e.keys2 || !e.bias)) return TB_ERR_ARG;
  if (dtype == TB_BF16) {
    if (k % 64 || lda % 8 || (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
      return TB_ERR_UNSUPPORTED;
    switch (pick_bn(m, n, k)) {
      case 256: return launch_tc_kind<256>(a, lda, w, m, n, k, e, err, stream);
      case 128: return launch_tc_kind<128>(a, lda, w, m, n, k, e, err, stream);
      case 64: return launch_tc_kind<64>(a, lda, w, m, n, k, e, err, stream);
      default: return TB_ERR_UNSUPPORTED;
    }
  }
  if (dtype != TB_F32) return TB_ERR_ARG;
  if (k % SG_BK || n % SG_BN || lda % 4) return TB_ERR_UNSUPPORTED;
  dim3 grid(n / SG_BN, (m + SG_BM - 1) / SG_BM);
  return launch_pdl(gemm_f32_kernel, grid, 256, 0, stream, reinterpret_cast<const float*>(a), lda,
                    reinterpret_cast<const float*>(w), m, n, k, e);
}

}  // namespace tb
