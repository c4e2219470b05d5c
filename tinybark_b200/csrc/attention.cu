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

// ---------------------------------------------------------------------------
// tcgen05 form (bf16): one CTA per (clip, head, 128 queries), key tiles of 64.
//
// Warp 0 loads Q, K and band tiles with TMA, warp 6 the V tiles, warp 1 issues the MMAs,
// warps 2-5 (one query row per thread) run the softmax. Per key tile, into tensor memory:
//   S  = Qu K^T          (128 x 64)
//   BD = Qu R_band^T     (128 x 192), R_band the 192 table rows the tile's relative
//                        positions span (191 used)
// The positional term of the reference, (q + bias_v) . r, is computed as
// (q + bias_u) . r + (bias_v - bias_u) . r: the second product depends only on the
// head and the relative position and comes precomputed per layer (rel_c), so Qu is the
// only query operand. Each softmax warp copies the 96 BD columns its 32 rows need into
// shared memory (a 64-column ring per row) and reads its row's window shifted by its row
// index (the relative shift). K and the band are double-buffered: tile g + 1's copies land
// while tile g's S and BD are computed. P (bf16) is written back into the tensor memory of S and the PV MMA reads
// it from there; V is an MN-major operand straight from the [frames, 1024] V tensor.
// O accumulates in tensor memory, rescaled by the softmax threads when the row max
// grows.

namespace att {
constexpr int TQ = 128, TK = 64, D = 128, BAND = 192;
constexpr int Q_BYTES = TQ * D * 2, K_BYTES = TK * D * 2, R_BYTES = BAND * D * 2, V_BYTES = TK * D * 2;
constexpr int Q_SUB = TQ * 128, K_SUB = TK * 128, R_SUB = BAND * 128, V_SUB = TK * 128;  // 64-column halves
// A softmax warp stages its rows' 96 BD columns in a 64-column ring per row (columns 64-95
// land on 0-31 once the first 32 keys no longer need them), so K and the band fit twice.
constexpr int ST_STRIDE = 68, WIN = 96;
constexpr int ST_BYTES = 4 * 32 * ST_STRIDE * 4, C_BYTES = 4 * WIN * 4;
constexpr int OFF_Q = 0, OFF_K = OFF_Q + Q_BYTES, OFF_R = OFF_K + 2 * K_BYTES, OFF_V = OFF_R + 2 * R_BYTES,
              OFF_ST = OFF_V + V_BYTES, OFF_C = OFF_ST + ST_BYTES, OFF_BAR = OFF_C + C_BYTES;
constexpr int SMEM = 1024 + OFF_BAR + 256;
constexpr uint32_t COL_S = 0, COL_BD = 64, COL_O = 256, COL_P = 384, TMEM_COLS = 512;
// log2(e) / sqrt(128): scores are kept in the base-2 exponent domain.
constexpr float SCALE_LOG2 = 0.12751743074f;
constexpr int V_WARP = 6, THREADS = 32 * (V_WARP + 1);  // TMA, MMA, 4 softmax warps, the V loader

struct Bars {
  uint64_t q_full, q_empty, kr_full[2], kr_empty[2], v_full, v_empty, sbd_full, sbd_empty, p_full, o_done, o_empty,
      done;
  uint32_t tmem;
  int abort;
};
}  // namespace att

__device__ __forceinline__ void att_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t start = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - start > TB_WAIT_NS) break;
}

__device__ __forceinline__ bool att_warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err, TB_DEV_ATTN_TIMEOUT, abort);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Persistent: one CTA per SM walks the (query tile, head) items t = blockIdx.x + k * gridDim.x
// (query tiles come longest clips first, so the strided walk balances the SMs). Every
// per-tile barrier counts key tiles across items (g below, this CTA's running tile index),
// so the next item's Q, K and band loads and its first S and BD products overlap the
// current item's last softmax and its output; q_empty (the item's last S and BD products
// have read Q) and o_empty (the softmax warps have read the finished O) hand Q's buffer
// and O's columns to the next item.
__global__ void __launch_bounds__(att::THREADS, 1)
    relpos_attention_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tr,
                        const float* __restrict__ rel_c, int max_len, const int* __restrict__ t3_off,
                        const int* __restrict__ tiles, int n_items, __nv_bfloat16* __restrict__ out, int* err) {
  using namespace att;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + OFF_BAR);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dep_wait();
  grid_dep_launch();
  struct Item {
    int q0, head, base, T, nk, col0;
  };
  auto item = [&](int t) {
    Item it;
    const int tile = t / TB_HEADS, clip = tiles[2 * tile];
    it.q0 = tiles[2 * tile + 1];
    it.head = t % TB_HEADS;
    it.base = t3_off[clip];
    it.T = t3_off[clip + 1] - it.base;
    it.nk = (it.T + TK - 1) / TK;
    it.col0 = it.head * D;
    return it;
  };

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kr_full[i], 1);
      mbar_init(&bars->kr_empty[i], 1);
    }
    mbar_init(&bars->v_full, 1);
    mbar_init(&bars->v_empty, 1);
    mbar_init(&bars->sbd_full, 1);
    mbar_init(&bars->sbd_empty, 4);
    mbar_init(&bars->p_full, 4);
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->o_empty, 4);
    mbar_init(&bars->done, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tr);
      int kr_issued = 0, q_issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_items && ok; t += gridDim.x) {
        const Item it = item(t);
        // Q's buffer is free once the previous item's last S and BD products are done.
        if (q_issued > 0 && !mbar_wait(&bars->q_empty, (q_issued - 1) & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) break;
        mbar_expect_tx(&bars->q_full, Q_BYTES);
        tma_load_2d(smem + OFF_Q, &tq, &bars->q_full, it.col0, it.base + it.q0);
        tma_load_2d(smem + OFF_Q + Q_SUB, &tq, &bars->q_full, it.col0 + 64, it.base + it.q0);
        ++q_issued;
        for (int j = 0; j < it.nk; ++j) {
          const int k0 = j * TK;
          const int band0 = max_len - TQ - it.q0 + k0;  // may be negative: TMA fills zeros
          // K and the band in one of two stages (tile kr_issued uses stage kr_issued % 2).
          const int ks = kr_issued & 1;
          if (!mbar_wait(&bars->kr_empty[ks], ((kr_issued >> 1) & 1) ^ 1, err, TB_DEV_ATTN_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          uint8_t* sk = smem + OFF_K + ks * K_BYTES;
          uint8_t* sr = smem + OFF_R + ks * R_BYTES;
          mbar_expect_tx(&bars->kr_full[ks], K_BYTES + R_BYTES);
          tma_load_2d(sk, &tk, &bars->kr_full[ks], it.col0, it.base + k0);
          tma_load_2d(sk + K_SUB, &tk, &bars->kr_full[ks], it.col0 + 64, it.base + k0);
          tma_load_2d(sr, &tr, &bars->kr_full[ks], it.col0, band0);
          tma_load_2d(sr + R_SUB, &tr, &bars->kr_full[ks], it.col0 + 64, band0);
          ++kr_issued;
        }
      }
      // Let the copies in flight land before the CTA exits (all have, unless the loop was
      // abandoned).
      if (q_issued) att_drain(&bars->q_full, (q_issued - 1) & 1);
      for (int i = kr_issued - 1; i >= 0 && i >= kr_issued - 2; --i) att_drain(&bars->kr_full[i & 1], (i >> 1) & 1);
    }
  } else if (warp == V_WARP) {
    // V has a producer of its own: its single buffer frees only when a tile's PV is done,
    // and waiting for that in the K / band producer would hold back the next tiles'
    // K and band copies.
    if (lane == 0) {
      int v_issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < n_items && ok; t += gridDim.x) {
        const Item it = item(t);
        for (int j = 0; j < it.nk; ++j) {
          if (!mbar_wait(&bars->v_empty, (v_issued & 1) ^ 1, err, TB_DEV_ATTN_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars->v_full, V_BYTES);
          tma_load_2d(smem + OFF_V, &tv, &bars->v_full, it.col0, it.base + j * TK);
          tma_load_2d(smem + OFF_V + V_SUB, &tv, &bars->v_full, it.col0 + 64, it.base + j * TK);
          ++v_issued;
        }
      }
      if (v_issued) att_drain(&bars->v_full, (v_issued - 1) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16(TQ, TK), id_bd = idesc_bf16(TQ, BAND), id_pv = idesc_bf16_bmn(TQ, D);
      const uint32_t qa = smem_u32(smem + OFF_Q), ka0 = smem_u32(smem + OFF_K), ra0 = smem_u32(smem + OFF_R),
                     va = smem_u32(smem + OFF_V);
      // S and BD of tile g + 1 are issued as soon as the softmax has read tile g's (before
      // tile g's PV), so they overlap the softmax of tile g; P has its own columns. Tile gg's
      // K and band are in stage gg % 2.
      auto sbd = [&](int gg) {
        const uint32_t ka = ka0 + (gg & 1) * K_BYTES, ra = ra0 + (gg & 1) * R_BYTES;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + COL_S, sdesc_sw128(qa + s * Q_SUB) + 2 * k, sdesc_sw128(ka + s * K_SUB) + 2 * k, id_s,
                     (s | k) != 0);
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + COL_BD, sdesc_sw128(qa + s * Q_SUB) + 2 * k, sdesc_sw128(ra + s * R_SUB) + 2 * k, id_bd,
                     (s | k) != 0);
        umma_commit(&bars->sbd_full);
        umma_commit(&bars->kr_empty[gg & 1]);
      };
      bool ok = true;
      int g = 0, n = 0;  // key tiles and items this CTA has done
      // Item `items`'s first key tile (this CTA's tile gg), issued as soon as possible: Q
      // loaded, the tile's K and band loaded, the softmax done reading the S and BD before.
      auto first_sbd = [&](int items, int gg) {
        if (!mbar_wait(&bars->q_full, items & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) return false;
        if (!mbar_wait(&bars->kr_full[gg & 1], (gg >> 1) & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) return false;
        if (gg > 0 && !mbar_wait(&bars->sbd_empty, (gg - 1) & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) return false;
        sbd(gg);
        return true;
      };
      int t = blockIdx.x;
      if (t < n_items) ok = first_sbd(0, 0);
      for (; t < n_items && ok; t += gridDim.x, ++n) {
        const int nk = item(t).nk;
        for (int j = 0; j < nk && ok; ++j, ++g) {
          if (j + 1 < nk) {
            if (!mbar_wait(&bars->kr_full[(g + 1) & 1], ((g + 1) >> 1) & 1, err, TB_DEV_ATTN_TIMEOUT, abort) ||
                !mbar_wait(&bars->sbd_empty, g & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) {  // tile g read
              ok = false;
              break;
            }
            sbd(g + 1);
          } else {
            umma_commit(&bars->q_empty);  // this item's S and BD products are issued: Q is free after them
          }
          if (!mbar_wait(&bars->p_full, g & 1, err, TB_DEV_ATTN_TIMEOUT, abort) ||
              !mbar_wait(&bars->v_full, g & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          // O's columns hold the previous item's result until its softmax warps read it.
          if (j == 0 && n > 0 && !mbar_wait(&bars->o_empty, (n - 1) & 1, err, TB_DEV_ATTN_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < TK / 16; ++kk)
            umma_f16_ts(tmem + COL_O, tmem + COL_P + 8 * kk, sdesc_sw128_mn(va + 2048 * kk, V_SUB), id_pv,
                        (j | kk) != 0);
          umma_commit(&bars->o_done);
          umma_commit(&bars->v_empty);
          // After this item's last PV, start the next item's first S and BD.
          if (j + 1 == nk && t + (int)gridDim.x < n_items) ok = first_sbd(n + 1, g + 1);
        }
      }
      umma_commit(&bars->done);
      att_drain(&bars->done, 0);
    }
  } else {
    // Warps 2-5 (V_WARP is 6).
    const int q = warp & 3;  // tensor-memory lane quarter: query rows 32q .. 32q+31
    const int il = q * 32 + lane;
    float* stage = reinterpret_cast<float*>(smem + OFF_ST) + q * 32 * ST_STRIDE;
    float* cband = reinterpret_cast<float*>(smem + OFF_C) + q * WIN;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
    const int wcol = 96 - 32 * q;  // first BD column this warp's rows need
    const int rel_rows = 2 * max_len - 1;
    bool ok = true;
    uint32_t r[32];
    int g = 0;  // key tiles this CTA has done
    for (int t = blockIdx.x; t < n_items && ok; t += gridDim.x) {
      const Item it = item(t);
      float m_run = -INFINITY, l_run = 0.f;
      // This warp's window of the (bias_v - bias_u) . r term for key tile j, loaded one
      // tile ahead so its latency hides behind the previous tile.
      float cnext[WIN / 32];
      auto load_cband = [&](int j) {
        const int band0 = max_len - TQ - it.q0 + j * TK;
#pragma unroll
        for (int u = 0; u < WIN / 32; ++u) {
          const int nn = band0 + wcol + u * 32 + lane;
          cnext[u] = (nn >= 0 && nn < rel_rows) ? rel_c[(long long)nn * 128 + it.head] : 0.f;
        }
      };
      load_cband(0);
      for (int j = 0; j < it.nk; ++j, ++g) {
        const int k0 = j * TK;
        __syncwarp();  // every lane is done with the previous tile's cband
#pragma unroll
        for (int u = 0; u < WIN / 32; ++u) cband[u * 32 + lane] = cnext[u];
        __syncwarp();
        if (j + 1 < it.nk) load_cband(j + 1);
        if (!att_warp_wait(&bars->sbd_full, g & 1, err, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // S (64 columns) and this warp's 96 BD columns out of tensor memory before any
        // arithmetic, so the next tile's S and BD products can start right away. BD columns
        // 0-63 of the window go to the row's ring; columns 64-95 stay in registers until
        // the first 32 keys are scored. (Adding the (bias_v - bias_u) . r term into the
        // ring here, from broadcast reads, measured slower than adding it per score.)
        uint32_t s0[32], s1[32];
        tmem_ld32(tl + COL_S, s0);
        tmem_ld32(tl + COL_S + 32, s1);
        tmem_ld32(tl + COL_BD + wcol, r);
        tmem_wait_ld();
        float* ring = stage + lane * ST_STRIDE;
        auto to_ring = [&](int slot) {
          float4* dst = reinterpret_cast<float4*>(ring + slot);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k] = make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]),
                                 __uint_as_float(r[4 * k + 2]), __uint_as_float(r[4 * k + 3]));
        };
        to_ring(0);
        tmem_ld32(tl + COL_BD + wcol + 32, r);
        tmem_wait_ld();
        to_ring(32);
        tmem_ld32(tl + COL_BD + wcol + 64, r);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->sbd_empty);  // S and BD read: the next tile's may go
        // Scores: content + shifted position terms. Key jj reads window column
        // 31 - lane + jj: columns 0-62 for the first 32 keys; then columns 64-95 take ring
        // slots 0-31 (each lane's ring is its own row), and the last 32 keys read column x
        // at slot x & 63 (one load, conflict-free: lane L's slot lands in bank 3L + c).
        // Keys at or past the clip's end score -inf; only a clip's last tile can have
        // them, so whole tiles run loops without the test. The maxima run in four
        // independent chains.
        const int lim = it.T - k0;  // keys of this tile inside the clip
        const bool partial = lim < TK;
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        const float* row_lo = ring + (31 - lane);
        const float* crow = cband + (31 - lane);
        if (!partial) {
#pragma unroll
          for (int jj = 0; jj < TK / 2; jj += 2) {
            const float v0 = __uint_as_float(s0[jj]) + row_lo[jj] + crow[jj];
            const float v1 = __uint_as_float(s0[jj + 1]) + row_lo[jj + 1] + crow[jj + 1];
            s0[jj] = __float_as_uint(v0);
            s0[jj + 1] = __float_as_uint(v1);
            mx4[(jj >> 1) & 3] = max3(mx4[(jj >> 1) & 3], v0, v1);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < TK / 2; ++jj) {
            float v = __uint_as_float(s0[jj]) + row_lo[jj] + crow[jj];
            if (jj >= lim) v = -INFINITY;
            s0[jj] = __float_as_uint(v);
            mx4[jj & 3] = fmaxf(mx4[jj & 3], v);
          }
        }
        to_ring(0);  // slots 0-31 are only this lane's row: its reads above are done
        if (!partial) {
#pragma unroll
          for (int jj = 0; jj < TK / 2; jj += 2) {
            const int kk = TK / 2 + jj;
            const float v0 = __uint_as_float(s1[jj]) + ring[(31 - lane + kk) & 63] + crow[kk];
            const float v1 = __uint_as_float(s1[jj + 1]) + ring[(32 - lane + kk) & 63] + crow[kk + 1];
            s1[jj] = __float_as_uint(v0);
            s1[jj + 1] = __float_as_uint(v1);
            mx4[(jj >> 1) & 3] = max3(mx4[(jj >> 1) & 3], v0, v1);
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < TK / 2; ++jj) {
            const int kk = TK / 2 + jj;
            float v = __uint_as_float(s1[jj]) + ring[(31 - lane + kk) & 63] + crow[kk];
            if (kk >= lim) v = -INFINITY;
            s1[jj] = __float_as_uint(v);
            mx4[jj & 3] = fmaxf(mx4[jj & 3], v);
          }
        }
        // In the base-2 exponent domain (scores times log2(e) / sqrt(128)). The running
        // max moves only when the row max grows by more than 8 (a factor 256 in the
        // exponentials, which bf16 P and the fp32 sums hold exactly): O is rescaled far less
        // often, and the final O / l is the same for any reference max.
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * SCALE_LOG2;
        float corr = 1.0f;
        if (mx > m_run + 8.0f) {
          corr = ex2_approx(m_run - mx);
          m_run = mx;
        }
        const float m_new = m_run;
        // Two scores per packed FMA (each half rounds as fmaf would).
        const float2 scale2 = make_float2(SCALE_LOG2, SCALE_LOG2), negm2 = make_float2(-m_new, -m_new);
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int jj = 0; jj < TK / 2; jj += 2) {
          const float2 e = fma2(make_float2(__uint_as_float(s0[jj]), __uint_as_float(s0[jj + 1])), scale2, negm2);
          const float p0 = ex2_approx(e.x), p1 = ex2_approx(e.y);
          sum4[(jj >> 1) & 1] += p0 + p1;
          __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          r[jj >> 1] = *reinterpret_cast<uint32_t*>(&b2);
        }
#pragma unroll
        for (int jj = 0; jj < TK / 2; jj += 2) {
          const float2 e = fma2(make_float2(__uint_as_float(s1[jj]), __uint_as_float(s1[jj + 1])), scale2, negm2);
          const float p0 = ex2_approx(e.x), p1 = ex2_approx(e.y);
          sum4[2 + ((jj >> 1) & 1)] += p0 + p1;
          __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          r[16 + (jj >> 1)] = *reinterpret_cast<uint32_t*>(&b2);
        }
        const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        l_run = l_run * corr + sum;
        if (j > 0) {
          if (!att_warp_wait(&bars->o_done, (g - 1) & 1, err, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(0xffffffffu, corr != 1.0f)) {
            uint32_t o[32];
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              tmem_ld32(tl + COL_O + 32 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * corr);
              tmem_st32(tl + COL_O + 32 * c, o);
            }
          }
        }
        tmem_st32(tl + COL_P, r);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full);
      }
      if (!ok || !att_warp_wait(&bars->o_done, (g - 1) & 1, err, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = 1.0f / l_run;
      const bool valid = it.q0 + il < it.T;
      __nv_bfloat16* dst = out + (long long)(it.base + it.q0 + il) * TB_HIDDEN + it.col0;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tl + COL_O + 32 * c, r);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int k = 0; k < 32; k += 4)
            store4(dst + 32 * c + k, __uint_as_float(r[k]) * inv, __uint_as_float(r[k + 1]) * inv,
                   __uint_as_float(r[k + 2]) * inv, __uint_as_float(r[k + 3]) * inv);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_empty);  // O's columns are free for the next item
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, att::TMEM_COLS);
  }
}

static int launch_attn_tc(const void* qu, const void* k, const void* v, const void* rel, const float* rel_c,
                          int max_len, const tb_batch& b, void* out, int* err, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(relpos_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, att::SMEM) !=
        cudaSuccess)
      return fail_cuda();
    configured = true;
  }
  for (const void* p : {qu, k, v, rel})
    if (reinterpret_cast<uintptr_t>(p) & 15) return TB_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv, mr;
  const long long rows = b.t3_total;
  if (!encode_tmap_2d(&mq, qu, rows, TB_HIDDEN, TB_HIDDEN, 64, att::TQ) ||
      !encode_tmap_2d(&mk, k, rows, TB_HIDDEN, TB_HIDDEN, 64, att::TK) ||
      !encode_tmap_2d(&mv, v, rows, TB_HIDDEN, TB_HIDDEN, 64, att::TK) ||
      !encode_tmap_2d(&mr, rel, 2LL * max_len - 1, TB_HIDDEN, TB_HIDDEN, 64, att::BAND))
    return TB_ERR_CUDA;
  const int items = b.n_attn_tiles * TB_HEADS;
  const int grid = items < sm_budget() ? items : sm_budget();
  return launch_pdl(relpos_attention_tc, grid, att::THREADS, att::SMEM, stream, mq, mk, mv, mr, rel_c, max_len, b.t3_off,
                    b.attn_tiles, items, reinterpret_cast<__nv_bfloat16*>(out), err);
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

int attention_tile_rows(int dtype) { return dtype == TB_BF16 ? att::TQ : AQ; }

int relpos_attention(int dtype, const void* qu, const void* qv, const void* k, const void* v, const void* rel,
                     const float* rel_c, int max_len, const tb_batch& b, void* out, int* err, cudaStream_t stream) {
  if (b.n_attn_tiles <= 0) return TB_OK;
  if (!qu || !k || !v || !rel || !out || !b.attn_tiles || !b.t3_off || b.max_t3 > max_len) return TB_ERR_ARG;
  if (dtype == TB_BF16) {
    if (!rel_c || !err) return TB_ERR_ARG;
    return launch_attn_tc(qu, k, v, rel, rel_c, max_len, b, out, err, stream);
  }
  if (dtype == TB_F32) {
    if (!qv) return TB_ERR_ARG;
    return launch_attn_simt<float>(qu, qv, k, v, rel, max_len, b, out, stream);
  }
  return TB_ERR_ARG;
}

}  // namespace tb
