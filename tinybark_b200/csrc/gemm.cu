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
// parity path; at most 8 rows (the fp32 decoder at small batch), a matrix-vector kernel.
#include <algorithm>

#include "host.h"
#include "tcgemm.cuh"

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
  static constexpr int OUT_STRIDE = TC_OUT_STRIDE;
  static constexpr int OUT_BYTES = 4 * 32 * OUT_STRIDE * 4;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + OUT_BYTES + BAR_BYTES;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
                   const tb_epilogue e, int* err, int splits) {
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
  const int n_tiles = N / BN, kb_count = K / C::BK / splits;
  // W holds weights, never written by the predecessor kernel: for a few rows (a batch of
  // one or two clips, where a launch is mostly latency) and a row count fixed at launch,
  // the producer starts the weight copies of its first item's first stages before waiting
  // on the predecessor (the A copies of those stages follow after the wait). Each such
  // stage's `full` barrier expects the weight bytes now, and the A bytes with its arrival.
  int pre = 0;
  if (warp == 0 && lane == 0 && !e.rows && M <= 2 * C::BM &&
      (int)blockIdx.x < (M + C::BM - 1) / C::BM * n_tiles * splits) {
    prefetch_tmap(&tw);
    const int t = blockIdx.x, nt = (t / splits) % n_tiles, kb0 = (t % splits) * kb_count;
    pre = kb_count < C::STAGES ? kb_count : C::STAGES;
    for (int kb = 0; kb < pre; ++kb) {
      mbar_expect_tx_only(&bars->full[kb], C::B_BYTES);
      tma_load_2d(smem + kb * C::STAGE_BYTES + C::A_BYTES, &tw, &bars->full[kb], (kb0 + kb) * C::BK, nt * BN);
    }
  }
  grid_dep_wait();
  grid_dep_launch();

  if (e.rows) M = min(M, *e.rows);
  // Work item t: output tile t / splits, K range t % splits of `splits` equal ranges (split
  // K only with the EPI_RESIDUAL_SPLIT epilogue, whose atomic adds sum the ranges).
  const int m_tiles = (M + C::BM - 1) / C::BM, tiles = m_tiles * n_tiles * splits;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int tile = t / splits, mt = tile / n_tiles, nt = tile % n_tiles, kb0 = (t % splits) * kb_count;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars->empty[s], ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          if (issued < pre) {  // the weights of this stage are on their way already
            mbar_expect_tx(&bars->full[s], C::A_BYTES);
            tma_load_2d(sa, &ta, &bars->full[s], (kb0 + kb) * C::BK, mt * C::BM);
          } else {
            mbar_expect_tx(&bars->full[s], C::STAGE_BYTES);
            tma_load_2d(sa, &ta, &bars->full[s], (kb0 + kb) * C::BK, mt * C::BM);
            tma_load_2d(sa + C::A_BYTES, &tw, &bars->full[s], (kb0 + kb) * C::BK, nt * BN);
          }
          ++issued;
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
      }
      // Stages whose weights were prefetched but whose A copy was never issued (the loop
      // was abandoned): their arrival completes them once the weights land.
      for (long long i = issued; i < pre; ++i) mbar_arrive(&bars->full[i]);
      if (issued < pre) issued = pre, ok = false;
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
      const int tile = t / splits, mt = tile / n_tiles, nt = tile % n_tiles;
      const int row0 = mt * C::BM + q * 32, n0 = nt * BN;
      if (!epilogue_tile<BN, EPI>(e, stage, tmem + ((uint32_t)(q * 32) << 16) + acc * BN, row0, n0, lane, M,
                                  &bars->tfull[acc], acc_ph, err, abort))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&bars->tempty[acc]);
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
// tcgen05 bf16 kernel on CTA pairs: 256 x 256 tiles, each SM of the pair loading its
// 128 rows of A and 128 of the 256 W rows per k-block (32 KB instead of the 48 KB a
// 128 x 256 tile on one SM needs), the leader issuing 256-row MMAs over both SMs'
// shared memory. Roles as in gemm_tc_kernel; the loads of both CTAs complete on the
// leader's `full` barriers, the leader's commits arrive on both CTAs' `empty` and
// `tfull` barriers, and both CTAs' epilogue warps release an accumulator on the
// leader's `tempty`. Every CTA runs the epilogue of its own 128 rows, with eight
// warps: two per tensor-memory lane quarter, each taking 128 of the 256 columns (a
// pair waits for the slower of its two epilogues, so they must keep well ahead of the
// main loop).

struct Tc2Cfg {
  static constexpr int BM = 128, BN = 256, BK = 64, STAGES = 5, EPI_WARPS = 8, THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int OUT_BYTES = EPI_WARPS * 32 * TC_OUT_STRIDE * 4;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + OUT_BYTES + 256;
};

template <int EPI>
__global__ void __launch_bounds__(Tc2Cfg::THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw, int M, int N, int K,
                    const tb_epilogue e, int* err) {
  using C = Tc2Cfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* out_stage = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);
  TcBars* bars = reinterpret_cast<TcBars*>(smem + C::STAGES * C::STAGE_BYTES + C::OUT_BYTES);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->full[s], 1);   // the leader's: its producer's arrival + both CTAs' bytes
      mbar_init(&bars->empty[s], 1);  // the leader's commit
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);   // the leader's commit
      mbar_init(&bars->tempty[a], 2 * C::EPI_WARPS);  // the leader's: every epilogue warp of both CTAs
    }
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(&bars->tmem, C::TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // barriers initialised and tensor memory allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  grid_dep_wait();
  grid_dep_launch();

  const int m_pairs = (M + 2 * C::BM - 1) / (2 * C::BM), n_tiles = N / C::BN, tiles = m_pairs * n_tiles;
  const int kb_count = K / C::BK;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      int s = 0;
      uint32_t ph = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        const int mt = t / n_tiles, nt = t % n_tiles;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars->empty[s], ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          if (rank == 0) mbar_expect_tx(&bars->full[s], 2 * C::STAGE_BYTES);
          const uint32_t full = cluster_addr(&bars->full[s], 0);
          tma_load_2d_pair(sa, &ta, full, kb * C::BK, mt * 2 * C::BM + (int)rank * C::BM);
          tma_load_2d_pair(sa + C::A_BYTES, &tw, full, kb * C::BK, nt * C::BN + (int)rank * (C::BN / 2));
          ++issued;
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
      }
      if (!ok && rank == 0) {
        // Let the copies already in flight land before the CTA exits (both CTAs' copies
        // complete on the leader's barriers; the peer stays until the final cluster
        // barrier).
        long long back = issued < C::STAGES ? issued : C::STAGES;
        for (long long i = 1; i <= back; ++i) {
          long long idx = issued - i;
          drain_wait(&bars->full[idx % C::STAGES], (uint32_t)((idx / C::STAGES) & 1));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16(2 * C::BM, C::BN);
      int s = 0, acc = 0;
      uint32_t ph = 0, acc_ph = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        if (!mbar_wait(&bars->tempty[acc], acc_ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * C::BN;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(&bars->full[s], ph, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t ad = sdesc_sw128(sa), bd = sdesc_sw128(sa + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < C::BK / 16; ++k) umma_f16_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair(cluster_addr(&bars->empty[s], 0));
          umma_commit_pair(cluster_addr(&bars->empty[s], 1));
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
        if (!ok) break;
        umma_commit_pair(cluster_addr(&bars->tfull[acc], 0));
        umma_commit_pair(cluster_addr(&bars->tfull[acc], 1));
        if (++acc == 2) acc = 0, acc_ph ^= 1;
      }
      // Every MMA issued has completed once this commit arrives.
      umma_commit_pair(cluster_addr(&bars->done, 0));
      drain_wait(&bars->done, 0);
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;      // tensor-memory lane quarter this warp may access
    const int half = ew >> 2;    // which 128 of the 256 columns
    float* stage = out_stage + ew * 32 * TC_OUT_STRIDE;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int t = pair; t < tiles; t += pairs) {
      const int mt = t / n_tiles, nt = t % n_tiles;
      const int row0 = mt * 2 * C::BM + (int)rank * C::BM + q * 32, n0 = nt * C::BN + half * (C::BN / 2);
      if (!epilogue_tile<C::BN / 2, EPI>(e, stage,
                                         tmem + ((uint32_t)(q * 32) << 16) + acc * C::BN + half * (C::BN / 2), row0,
                                         n0, lane, M, &bars->tfull[acc], acc_ph, err, abort))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(cluster_addr(&bars->tempty[acc], 0));
      if (++acc == 2) acc = 0, acc_ph ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// fp32 CUDA-core kernel

constexpr int SG_BM = 128, SG_BN = 128, SG_BK = 16, SG_PAD = 4;

// K range blockIdx.z of gridDim.z equal ranges: with more than one (the residual epilogue
// only), each range's product is added to the residual rows atomically.
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
  const int k_len = K / gridDim.z, k_base = blockIdx.z * k_len;
  A += k_base;
  W += k_base;
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
  for (int k0 = 0; k0 < k_len; k0 += SG_BK) {
    const bool more = k0 + SG_BK < k_len;
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
  if (gridDim.z > 1) {  // split K: residual rows += alpha * this range's product
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
      if (m >= M) continue;
      float* r = reinterpret_cast<float*>(e.out) + (long long)m * e.ldo;
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(r + n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4), e.alpha * acc[i][j]);
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

// The same product on 64 x 64 tiles (4 x 4 outputs per thread), for a clip or two, whose
// 128 x 128 tiles would leave most SMs idle: each output sums over k in the same order
// as in the kernel above, so the results are the same bits.
constexpr int SS_BM = 64, SS_BN = 64, SS_BK = 16, SS_PAD = 4;

__global__ void __launch_bounds__(256) gemm_f32_small_kernel(const float* __restrict__ A, long long lda,
                                                             const float* __restrict__ W, int M, int N, int K,
                                                             const tb_epilogue e) {
  __shared__ __align__(16) float As[2][SS_BK][SS_BM + SS_PAD];
  __shared__ __align__(16) float Ws[2][SS_BK][SS_BN + SS_PAD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * SS_BM, n0 = blockIdx.x * SS_BN;
  const int lr = tid >> 2, lk = (tid & 3) * 4;  // loader: row lr, k offset lk
  float4 rw = *reinterpret_cast<const float4*>(W + (long long)(n0 + lr) * K + lk);  // weights: before the wait
  grid_dep_wait();
  grid_dep_launch();
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const int am = m0 + lr;
  float4 ra = am < M ? *reinterpret_cast<const float4*>(A + (long long)am * lda + lk) : make_float4(0, 0, 0, 0);
  auto stash = [&](int buf) {
    As[buf][lk + 0][lr] = ra.x, As[buf][lk + 1][lr] = ra.y, As[buf][lk + 2][lr] = ra.z, As[buf][lk + 3][lr] = ra.w;
    Ws[buf][lk + 0][lr] = rw.x, Ws[buf][lk + 1][lr] = rw.y, Ws[buf][lk + 2][lr] = rw.z, Ws[buf][lk + 3][lr] = rw.w;
  };
  stash(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += SS_BK) {
    const bool more = k0 + SS_BK < K;
    if (more) {
      ra = am < M ? *reinterpret_cast<const float4*>(A + (long long)am * lda + k0 + SS_BK + lk) : make_float4(0, 0, 0, 0);
      rw = *reinterpret_cast<const float4*>(W + (long long)(n0 + lr) * K + k0 + SS_BK + lk);
    }
#pragma unroll
    for (int k = 0; k < SS_BK; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
    }
    if (more) {
      stash(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m < M) epi_group(e, m, n0 + tx * 4, acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
}

// ---------------------------------------------------------------------------
// fp32 matrix-vector kernel for a few rows (the fp32 decoder's GEMMs at batch 1-8): a CTA
// of four warps per epilogue group of 4 output columns, warp j taking column n0 + j over
// all of K for every row. Each lane holds its K / 128 16-byte pieces of the weight row in
// registers, loaded before waiting on the predecessor kernel (W is weights), so one memory
// round trip brings the whole row; the rows of A are staged in shared memory. Per column
// the sum runs in the same order as one warp's (lane l takes k = 4l + 128i, i ascending;
// a butterfly over the lanes). A 128 x 128 tile of the GEMM kernel would compute up to
// 127 rows of nothing here.

constexpr int GV_MAX_ROWS = 8, GV_MAX_K = 1280, GV_THREADS = 128;

__global__ void __launch_bounds__(GV_THREADS) gemv_f32_kernel(const float* __restrict__ A, long long lda,
                                                             const float* __restrict__ W, int M, int N, int K,
                                                             const tb_epilogue e) {
  extern __shared__ __align__(16) float As[];  // [M, K], sized by the launch
  __shared__ float red[GV_MAX_ROWS][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 4, n = n0 + warp;
  float4 w[GV_MAX_K / 128];
#pragma unroll
  for (int i = 0; i < GV_MAX_K / 128; ++i) {
    const int k = i * 128 + lane * 4;
    w[i] = (n < N && k < K) ? *reinterpret_cast<const float4*>(W + (long long)n * K + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  grid_dep_wait();
  grid_dep_launch();
  if (e.rows) M = min(M, *e.rows);
  if (M <= 0) return;
  for (int i = threadIdx.x * 4; i < M * K; i += GV_THREADS * 4) {
    const int m = i / K, k = i - m * K;
    *reinterpret_cast<float4*>(As + i) = *reinterpret_cast<const float4*>(A + (long long)m * lda + k);
  }
  __syncthreads();
  float acc[GV_MAX_ROWS];
#pragma unroll
  for (int m = 0; m < GV_MAX_ROWS; ++m) acc[m] = 0.f;
#pragma unroll
  for (int i = 0; i < GV_MAX_K / 128; ++i) {
    const int k = i * 128 + lane * 4;
    if (k >= K) break;
#pragma unroll
    for (int m = 0; m < GV_MAX_ROWS; ++m) {
      if (m >= M) break;
      const float4 a = *reinterpret_cast<const float4*>(As + m * K + k);
      acc[m] = fmaf(a.w, w[i].w, fmaf(a.z, w[i].z, fmaf(a.y, w[i].y, fmaf(a.x, w[i].x, acc[m]))));
    }
  }
#pragma unroll
  for (int m = 0; m < GV_MAX_ROWS; ++m)
#pragma unroll
    for (int o = 16; o; o >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], o);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < GV_MAX_ROWS; ++m) red[m][warp] = acc[m];
  }
  __syncthreads();
  const int m = threadIdx.x;
  if (m >= M || n0 >= N) return;
  if (e.kind == TB_EPI_ARGMAX) {
    ArgmaxAcc am;
#pragma unroll
    for (int j = 0; j < 4; ++j) am.add(e, n0 + j, red[m][j]);
    am.flush(e, m);
  } else {
    epi_group(e, m, n0, red[m][0], red[m][1], red[m][2], red[m][3]);
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
                     cudaStream_t stream, int splits = 1) {
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
  const int tiles = ((m + C::BM - 1) / C::BM) * (n / BN) * splits;
  const int grid = tiles < sm_budget() ? tiles : sm_budget();
  return launch_pdl(gemm_tc_kernel<BN, EPI>, grid, 192, C::SMEM, stream, ta, tw, m, n, k, e, err, splits);
}

// The pair kernel: clusters of two CTAs, as many pairs as can be resident at once (at
// most one per two SMs of the budget) looping over the 256 x 256 tiles.
template <int EPI>
static int launch_tc2(const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e, int* err,
                      cudaStream_t stream) {
  using C = Tc2Cfg;
  static int max_pairs = -1;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (max_pairs < 0) {
    if (cudaFuncSetAttribute(gemm_tc2_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return fail_cuda();
    int clusters = 0;
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    if (cudaOccupancyMaxActiveClusters(&clusters, gemm_tc2_kernel<EPI>, &cfg) != cudaSuccess) return fail_cuda();
    max_pairs = clusters;
  }
  if (max_pairs < 1) return TB_ERR_UNSUPPORTED;
  CUtensorMap ta, tw;
  if (!encode_tmap(&ta, a, m, k, lda, C::BM) || !encode_tmap(&tw, w, n, k, k, C::BN / 2)) return TB_ERR_CUDA;
  const int tiles = ((m + 2 * C::BM - 1) / (2 * C::BM)) * (n / C::BN);
  int pairs = std::min(std::min(tiles, max_pairs), sm_budget() / 2);
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(2 * pairs);
  cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<EPI>, ta, tw, m, n, k, e, err);
  return check_launch();
}

// K splits for a residual GEMM of at most 256 rows (a clip or two) whose tiles leave most
// SMs idle (three quarters of them or more): the largest power of two up to 8 that keeps at least
// 4 k-blocks per split and at most one work item per SM. Split sums land in an order the
// atomic adds choose, so such a GEMM is not bit-reproducible; larger ones never split.
static int residual_splits(int m, int n, int k, int bn) {
  const int tiles = ((m + 127) / 128) * (n / bn), kb = k / 64, sms = sm_budget();
  if (m > 256 || 4 * tiles > sms) return 1;
  int s = 1;
  while (s < 8 && kb % (2 * s) == 0 && kb / (2 * s) >= 4 && tiles * 2 * s <= sms) s *= 2;
  return s;
}

template <int BN>
static int launch_tc_kind(const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e,
                          int* err, cudaStream_t s) {
  if (e.kind == TB_EPI_RESIDUAL && !e.rows) {
    const int splits = residual_splits(m, n, k, BN);
    if (splits > 1) return launch_tc<BN, EPI_RESIDUAL_SPLIT>(a, lda, w, m, n, k, e, err, s, splits);
  }
  switch (e.kind) {
    case TB_EPI_STORE: return launch_tc<BN, TB_EPI_STORE>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_SILU: return launch_tc<BN, TB_EPI_SILU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_RESIDUAL: return launch_tc<BN, TB_EPI_RESIDUAL>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_BIAS_RELU: return launch_tc<BN, TB_EPI_BIAS_RELU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_GLU: return launch_tc<BN, TB_EPI_GLU>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_QKV: return launch_tc<BN, TB_EPI_QKV>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_ARGMAX: return launch_tc<BN, TB_EPI_ARGMAX>(a, lda, w, m, n, k, e, err, s);
    case TB_EPI_LSTM:
      if constexpr (BN <= 128) return launch_tc<BN, TB_EPI_LSTM>(a, lda, w, m, n, k, e, err, s);
      return TB_ERR_UNSUPPORTED;
    case TB_EPI_JOINT_IN: return launch_tc<BN, TB_EPI_JOINT_IN>(a, lda, w, m, n, k, e, err, s);
    default: return TB_ERR_ARG;
  }
}

// Rows from which a GEMM runs on CTA pairs: below, 128-row tiles spread further.
constexpr int GEMM_PAIR_MIN_ROWS = 2048;

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
    // Large GEMMs of the encoder on CTA pairs (half the operand traffic per SM); the
    // decoder's (row bound read at run time, per-row epilogues) on single CTAs.
    const bool pair_kind = e.kind == TB_EPI_STORE || e.kind == TB_EPI_SILU || e.kind == TB_EPI_RESIDUAL ||
                           e.kind == TB_EPI_BIAS_RELU || e.kind == TB_EPI_GLU || e.kind == TB_EPI_QKV;
    if (gemm_pairs() && pair_kind && !e.rows && n % 256 == 0 && m >= GEMM_PAIR_MIN_ROWS) {
      switch (e.kind) {
        case TB_EPI_STORE: return launch_tc2<TB_EPI_STORE>(a, lda, w, m, n, k, e, err, stream);
        case TB_EPI_SILU: return launch_tc2<TB_EPI_SILU>(a, lda, w, m, n, k, e, err, stream);
        case TB_EPI_RESIDUAL: return launch_tc2<TB_EPI_RESIDUAL>(a, lda, w, m, n, k, e, err, stream);
        case TB_EPI_BIAS_RELU: return launch_tc2<TB_EPI_BIAS_RELU>(a, lda, w, m, n, k, e, err, stream);
        case TB_EPI_GLU: return launch_tc2<TB_EPI_GLU>(a, lda, w, m, n, k, e, err, stream);
        default: return launch_tc2<TB_EPI_QKV>(a, lda, w, m, n, k, e, err, stream);
      }
    }
    int bn = pick_bn(m, n, k);
    if (e.kind == TB_EPI_LSTM && bn > 128) bn = n % 128 ? 64 : 128;  // the cell epilogue covers <= 32 units
    switch (bn) {
      case 256: return launch_tc_kind<256>(a, lda, w, m, n, k, e, err, stream);
      case 128: return launch_tc_kind<128>(a, lda, w, m, n, k, e, err, stream);
      case 64: return launch_tc_kind<64>(a, lda, w, m, n, k, e, err, stream);
      default: return TB_ERR_UNSUPPORTED;
    }
  }
  if (dtype != TB_F32) return TB_ERR_ARG;
  if (m <= GV_MAX_ROWS && k <= GV_MAX_K && k % 128 == 0 && n % 4 == 0 && lda % 4 == 0 &&
      !(reinterpret_cast<uintptr_t>(a) & 15) && !(reinterpret_cast<uintptr_t>(w) & 15)) {
    // Shared memory for the launch's M rows only (at most 40 KB), so more CTAs share an SM.
    return launch_pdl(gemv_f32_kernel, dim3(n / 4), GV_THREADS, (size_t)m * k * sizeof(float), stream,
                      reinterpret_cast<const float*>(a), lda, reinterpret_cast<const float*>(w), m, n, k, e);
  }
  if (k % SG_BK || n % SG_BN || lda % 4) return TB_ERR_UNSUPPORTED;
  dim3 grid(n / SG_BN, (m + SG_BM - 1) / SG_BM);
  if (e.kind != TB_EPI_RESIDUAL && e.kind != TB_EPI_ARGMAX && !e.rows && m <= 256 &&
      (int)(2 * grid.x * grid.y) <= sm_budget())
    return launch_pdl(gemm_f32_small_kernel, dim3(n / SS_BN, (m + SS_BM - 1) / SS_BM), 256, 0, stream,
                      reinterpret_cast<const float*>(a), lda, reinterpret_cast<const float*>(w), m, n, k, e);
  // A residual GEMM of a clip or two whose tiles leave most SMs idle splits K (a power of
  // two up to 16, at least 64 of K per range, at most one CTA per SM). The ranges' sums
  // land in the order the atomic adds take, so such a GEMM is not bit-reproducible.
  if (e.kind == TB_EPI_RESIDUAL && !e.rows && m <= 256) {
    const int sms = sm_budget();
    while (grid.z < 16 && k % (2 * grid.z * SG_BK) == 0 && k / (2 * (int)grid.z) >= 64 &&
           (int)(grid.x * grid.y * grid.z * 2) <= sms)
      grid.z *= 2;
  }
  return launch_pdl(gemm_f32_kernel, grid, 256, 0, stream, reinterpret_cast<const float*>(a), lda,
                    reinterpret_cast<const float*>(w), m, n, k, e);
}

}  // namespace tb
