// Block-scaled FP8 (MXFP8) GEMM for the FFN layers: C = A * W^T with A [M, K] and W [N, K]
// stored as E4M3 codes, each run of 32 values along K sharing one E8M0 scale (OCP
// Microscaling v1.0: value = code * 2^(scale - 127)), fp32 accumulation, the bf16 GEMM's
// fused epilogues. The block-scaled weights are the low-precision option of
// tinybark/docs/2026-10-24-learnings.md:133-146; the bf16 GEMM stays the default path.
//
// mx_quantize_kernel: rows of bf16 or fp32 values to E4M3 codes and E8M0 scales, one
// thread per 32-value block: scale exponent e = floor(log2 max|x|) - 8 (the largest E4M3
// binade is 2^8), clamped to [-127, 127], -127 for an all-zero block; codes = E4M3 of
// x * 2^-e, rounded to nearest even and saturated to +-448.
//
// Scales are stored tiled, one chunk per 128 rows and 512 values of K:
// [rows / 128][K / 512][128 rows][16 bytes], byte j of a row's 16 the scale of its 32-value
// block j of that 512 (k-block j / 4, MMA j % 4). In tensor memory a chunk takes 4 columns
// for A and 4 for W per k-block (the layout at sf_store), byte b of a cell the scale of MMA
// b, selected by the instruction descriptor's scale-factor ids.
//
// mx_gemm_kernel: the persistent warp-specialized layout of the bf16 GEMM (gemm.cu) with
// 128 x 128 tiles and k-blocks of 128 E4M3 values (one 128-byte swizzled row per tile
// row): warp 0 loads A and W tiles with TMA and, once per 512 values of K, both tiles'
// 2 KB scale chunks with bulk copies; warps 6-9 write each chunk into one of two
// tensor-memory scale buffers (tcgen05.st, each warp its lane quarter); warp 1 issues
// kind::mxf8f6f4 block-scaled MMAs into one of two accumulators; warps 2-5 drain the
// other accumulator through the epilogue.
#include <cuda_fp8.h>

#include "host.h"
#include "tcgemm.cuh"

namespace tb {

namespace {

struct MxCfg {
  static constexpr int BM = 128, BN = 128, BK = 128, STAGES = 6;
  static constexpr int THREADS = 32 * 10;  // producer, MMA, 4 epilogue warps, 4 SF warps
  static constexpr uint32_t SF_COLS = 32;  // a scale buffer: 16 columns for A, then 16 for W
  static constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK, STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SF_BYTES = 128 * 16;  // one 128-row x 512-value scale chunk
  static constexpr int SF_SLOTS = 2;
  static constexpr int OUT_BYTES = 4 * 32 * TC_OUT_STRIDE * 4;
  static constexpr int OFF_SF = STAGES * STAGE_BYTES, OFF_OUT = OFF_SF + SF_SLOTS * 2 * SF_BYTES,
                       OFF_BAR = OFF_OUT + OUT_BYTES;
  static constexpr int SMEM = 1024 + OFF_BAR + 256;
  static constexpr uint32_t TMEM_COLS = 512, COL_SF = 2 * BN;  // scale buffers after the two accumulators
};

struct MxBars {
  TcBars tc;
  uint64_t sf_full[2], sf_empty[2];  // a group's scale chunks in shared memory
  uint64_t st_full[2], st_empty[2];  // a group's scales in a tensor-memory buffer
};
static_assert(sizeof(MxBars) <= 256, "mx barriers");

// Instruction descriptor of kind::mxf8f6f4 with block scaling: E4M3 A and B (K-major),
// E8M0 scales, f32 accumulator of 128 x n; the scale-factor ids (which byte of the scale
// column) for A at bits 29-30 and for B at bits 4-5.
__host__ __device__ constexpr uint32_t idesc_mx(int n, int sf_id) {
  return ((uint32_t)sf_id << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) | (1u << 23) |
         ((128u >> 4) << 24) | ((uint32_t)sf_id << 29);
}

__device__ __forceinline__ void umma_mx(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                        uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(sfa), "r"(sfb), "r"(acc)
      : "memory");
}

// One-dimensional bulk copy global -> shared (16-byte aligned, size a multiple of 16),
// completion counted on `bar`; no multicast.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <typename T>
__global__ void __launch_bounds__(256) mx_quantize_kernel(const T* __restrict__ src, long long ld, int rows,
                                                          int rows_pad, int k, uint8_t* __restrict__ codes,
                                                          uint8_t* __restrict__ sf) {
  const int blocks_per_row = k / 32;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)rows_pad * blocks_per_row) return;
  const int r = (int)(idx / blocks_per_row), j = (int)(idx % blocks_per_row);
  float v[32];
  float amax = 0.f;
  if (r < rows) {
    const T* p = src + (long long)r * ld + j * 32;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 q = load4(p + i);
      v[i] = q.x, v[i + 1] = q.y, v[i + 2] = q.z, v[i + 3] = q.w;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
  }
  // floor(log2(amax)) from the exponent field (amax below the normal range floors to
  // at most -127 and clamps there, as does zero).
  const int biased = (int)((__float_as_uint(amax) >> 23) & 0xFF);
  int e = biased == 0 ? -127 : biased - 127 - 8;
  e = e < -127 ? -127 : (e > 127 ? 127 : e);
  // x * 2^-e, a power of two: e is at most 119 (floats stay below 2^128), so 2^-e is a
  // normal float; a product too small for a normal float is far below E4M3's smallest
  // subnormal (2^-9) and rounds to zero either way. Then E4M3, round to nearest even,
  // saturated.
  const float inv = __uint_as_float((uint32_t)(127 - e) << 23);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    uint32_t word = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float x = v[i + u] * inv;
      const __nv_fp8_storage_t c = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
      word |= (uint32_t)c << (8 * u);
    }
    w[i / 4] = word;
  }
  uint4* dst = reinterpret_cast<uint4*>(codes + (long long)r * k + j * 32);
  dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
  dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  // Tiled scale layout: [r / 128][j / 16][r % 128][j % 16].
  const long long groups = k / 512;
  sf[(((long long)(r >> 7) * groups + (j >> 4)) * 128 + (r & 127)) * 16 + (j & 15)] = (uint8_t)(e + 127);
}

// Where a block-scaled MMA (M = 128, N = 128) reads its E8M0 scales in tensor memory, as
// measured on the B200 with one-MMA experiments (each scale cell holding a distinct value,
// in-bounds addresses only): for scale-buffer column `col` and scale-factor id k (the
// byte of a cell), row m of A reads (lane m, column col + m / 32, byte k), and column n of
// W reads (lane n % 32 + 32 * (m / 32), column col + n / 32, byte k) for output row m: every
// lane quarter needs its own copy of W's scales. So a k-block of 128 values (four MMAs,
// k = 0..3) takes 4 columns for A and 4 for W, lane r + 32 q of column col + g holding the
// 4 scales of row r + 32 g (the copies in other quarters are read only for W).
//
// sf_store: SF warp q writes its lanes' cells for one 512-value group (4 k-blocks: 16
// columns for A at col_a, 16 for W at col_w) from the group's shared-memory chunks
// ([128 rows][16 bytes], bytes 4 kb .. 4 kb + 3 of a row the scales of k-block kb).
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void sf_store(const uint8_t* chunk_a, const uint8_t* chunk_w, uint32_t tmem_quarter,
                                         uint32_t col_a, uint32_t col_w, int q, int lane) {
  uint32_t v[16];
  // A: lane 32 q + r's own row; column col_a + 4 kb + q is the one read, the others of
  // the k-block's four get the same word.
  const uint4 a = *reinterpret_cast<const uint4*>(chunk_a + (q * 32 + lane) * 16);
  const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = aw[i / 4];
  tmem_st_x16(tmem_quarter + col_a, v);
  // W: column col_w + 4 kb + g holds row r + 32 g, in every quarter.
  uint4 w[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) w[g] = *reinterpret_cast<const uint4*>(chunk_w + (lane + 32 * g) * 16);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    v[0 + g] = w[g].x;
    v[4 + g] = w[g].y;
    v[8 + g] = w[g].z;
    v[12 + g] = w[g].w;
  }
  tmem_st_x16(tmem_quarter + col_w, v);
}

template <int EPI>
__global__ void __launch_bounds__(MxCfg::THREADS, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tw,
                   const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfw, int M, int N, int K,
                   const tb_epilogue e, int* err) {
  using C = MxCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* out_stage = reinterpret_cast<float*>(smem + C::OFF_OUT);
  MxBars* mb = reinterpret_cast<MxBars*>(smem + C::OFF_BAR);
  TcBars* bars = &mb->tc;
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
      mbar_init(&mb->sf_full[a], 1);
      mbar_init(&mb->sf_empty[a], 4);
      mbar_init(&mb->st_full[a], 4);
      mbar_init(&mb->st_empty[a], 1);
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

  const int m_tiles = (M + C::BM - 1) / C::BM, n_tiles = N / C::BN, tiles = m_tiles * n_tiles;
  const int kb_count = K / C::BK, groups = K / 512;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&ta);
      prefetch_tmap(&tw);
      int s = 0, f = 0;
      uint32_t ph = 0, fph = 0;
      long long issued = 0, sf_issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mt = t / n_tiles, nt = t % n_tiles;
        for (int kb = 0; kb < kb_count; ++kb) {
          if ((kb & 3) == 0) {
            if (!mbar_wait(&mb->sf_empty[f], fph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) {
              ok = false;
              break;
            }
            uint8_t* dst = smem + C::OFF_SF + f * 2 * C::SF_BYTES;
            mbar_expect_tx(&mb->sf_full[f], 2 * C::SF_BYTES);
            bulk_load(dst, sfa + ((long long)mt * groups + (kb >> 2)) * C::SF_BYTES, C::SF_BYTES, &mb->sf_full[f]);
            bulk_load(dst + C::SF_BYTES, sfw + ((long long)nt * groups + (kb >> 2)) * C::SF_BYTES, C::SF_BYTES,
                      &mb->sf_full[f]);
            ++sf_issued;
            if (++f == C::SF_SLOTS) f = 0, fph ^= 1;
          }
          if (!mbar_wait(&bars->empty[s], ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * C::STAGE_BYTES;
          mbar_expect_tx(&bars->full[s], C::STAGE_BYTES);
          tma_load_2d(sa, &ta, &bars->full[s], kb * C::BK, mt * C::BM);
          tma_load_2d(sa + C::A_BYTES, &tw, &bars->full[s], kb * C::BK, nt * C::BN);
          ++issued;
          if (++s == C::STAGES) s = 0, ph ^= 1;
        }
      }
      if (!ok) {
        // Let the copies already in flight land before the CTA exits.
        const long long back = issued < C::STAGES ? issued : C::STAGES;
        for (long long i = 1; i <= back; ++i) {
          const long long idx = issued - i;
          drain_wait(&bars->full[idx % C::STAGES], (uint32_t)((idx / C::STAGES) & 1));
        }
        const long long sback = sf_issued < C::SF_SLOTS ? sf_issued : C::SF_SLOTS;
        for (long long i = 1; i <= sback; ++i) {
          const long long idx = sf_issued - i;
          drain_wait(&mb->sf_full[idx % C::SF_SLOTS], (uint32_t)((idx / C::SF_SLOTS) & 1));
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0, acc = 0, b = 0;
      uint32_t ph = 0, acc_ph = 0, bph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&bars->tempty[acc], acc_ph ^ 1, err, TB_DEV_GEMM_TIMEOUT, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * C::BN;
        uint32_t sf_col = 0;
        for (int kb = 0; kb < kb_count; ++kb) {
          if ((kb & 3) == 0) {
            // This group's scales, written into tensor-memory buffer b by the SF warps.
            if (!mbar_wait(&mb->st_full[b], bph, err, TB_DEV_GEMM_TIMEOUT, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            sf_col = tmem + C::COL_SF + C::SF_COLS * b;
          }
          if (!mbar_wait(&bars->full[s], ph, err, TB_DEV_GEMM_TIMEOUT, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t ad = sdesc_sw128(sa), bd = sdesc_sw128(sa + C::A_BYTES);
          const uint32_t col = sf_col + 4 * (kb & 3);  // this k-block's 4 columns of A, then of W
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_mx(d, ad + 2 * k, bd + 2 * k, idesc_mx(C::BN, k), col, col + C::SF_COLS / 2, (kb | k) != 0);
          umma_commit(&bars->empty[s]);
          if (++s == C::STAGES) s = 0, ph ^= 1;
          if ((kb & 3) == 3 || kb + 1 == kb_count) {
            umma_commit(&mb->st_empty[b]);  // the buffer is free once these MMAs are done
            if (++b == 2) b = 0, bph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&bars->tfull[acc]);
        if (++acc == 2) acc = 0, acc_ph ^= 1;
      }
      umma_commit(&bars->done);
      drain_wait(&bars->done, 0);
    }
  } else if (warp < 6) {
    const int q = warp & 3;
    float* stage = out_stage + q * 32 * TC_OUT_STRIDE;
    int acc = 0;
    uint32_t acc_ph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int mt = t / n_tiles, nt = t % n_tiles;
      const int row0 = mt * C::BM + q * 32, n0 = nt * C::BN;
      if (!epilogue_tile<C::BN, EPI>(e, stage, tmem + ((uint32_t)(q * 32) << 16) + acc * C::BN, row0, n0, lane, M,
                                     &bars->tfull[acc], acc_ph, err, abort))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&bars->tempty[acc]);
      if (++acc == 2) acc = 0, acc_ph ^= 1;
    }
  } else {
    // SF warps (6-9): each group's scale chunks from shared memory into a tensor-memory
    // scale buffer, for the 32 lanes of this warp's quarter.
    const int q = warp & 3;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    int f = 0, b = 0;
    uint32_t fph = 0, bph = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int g = 0; g < groups; ++g) {
        if (!warp_wait(&mb->sf_full[f], fph, err, abort) || !warp_wait(&mb->st_empty[b], bph ^ 1, err, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* chunk = smem + C::OFF_SF + f * 2 * C::SF_BYTES;
        const uint32_t col = C::COL_SF + C::SF_COLS * b;
        sf_store(chunk, chunk + C::SF_BYTES, tq, col, col + C::SF_COLS / 2, q, lane);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&mb->st_full[b]);
          mbar_arrive(&mb->sf_empty[f]);
        }
        if (++f == C::SF_SLOTS) f = 0, fph ^= 1;
        if (++b == 2) b = 0, bph ^= 1;
      }
    }
    if (!ok) *abort = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// 2-D E4M3 tensor map: rows x cols bytes (row stride ld bytes), boxes of 128 x 128 bytes,
// 128-byte swizzle (the layout sdesc_sw128 describes).
bool encode_tmap_fp8(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld) {
  auto fn = tensor_map_encoder();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI>
int launch_mx(const uint8_t* a, const uint8_t* sfa, const uint8_t* w, const uint8_t* sfw, int m, int n, int k,
              const tb_epilogue& e, int* err, cudaStream_t stream) {
  using C = MxCfg;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda();
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(mx_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) != cudaSuccess)
      return fail_cuda();
    configured[dev] = true;
  }
  CUtensorMap ta, tw;
  if (!encode_tmap_fp8(&ta, a, m, k, k) || !encode_tmap_fp8(&tw, w, n, k, k)) return TB_ERR_CUDA;
  const int tiles = ((m + C::BM - 1) / C::BM) * (n / C::BN);
  const int grid = tiles < sm_budget() ? tiles : sm_budget();
  return launch_pdl(mx_gemm_kernel<EPI>, grid, C::THREADS, C::SMEM, stream, ta, tw, sfa, sfw, m, n, k, e, err);
}

}  // namespace

size_t mx_scale_bytes(int rows, int k) { return (size_t)((rows + 127) / 128) * 128 * (size_t)(k / 32); }

int mx_quantize(int src_dtype, const void* src, long long ld, int rows, int k, uint8_t* codes, uint8_t* sf,
                cudaStream_t stream) {
  if (rows <= 0) return TB_OK;
  if (!src || !codes || !sf || k <= 0 || k % 512 || ld < k || ld % 4 || (reinterpret_cast<uintptr_t>(codes) & 15) ||
      (src_dtype != TB_F32 && src_dtype != TB_BF16) || (reinterpret_cast<uintptr_t>(src) & 15))
    return TB_ERR_ARG;
  const int rows_pad = (rows + 127) / 128 * 128;
  const long long n = (long long)rows_pad * (k / 32);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  // Codes of padding rows land past `rows` rows: the caller's code buffer holds rows_pad rows.
  if (src_dtype == TB_BF16)
    mx_quantize_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), ld, rows,
                                                                  rows_pad, k, codes, sf);
  else
    mx_quantize_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float*>(src), ld, rows, rows_pad, k, codes,
                                                          sf);
  return check_launch();
}

int gemm_mx(const uint8_t* a, const uint8_t* sfa, const uint8_t* w, const uint8_t* sfw, int m, int n, int k,
            const tb_epilogue& e, int* err, cudaStream_t stream) {
  if (m <= 0) return TB_OK;
  if (!a || !sfa || !w || !sfw || n <= 0 || n % 128 || k <= 0 || k % 512) return TB_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(sfa) & 15) || (reinterpret_cast<uintptr_t>(sfw) & 15))
    return TB_ERR_ARG;
  if (e.rows) return TB_ERR_UNSUPPORTED;
  switch (e.kind) {
    case TB_EPI_STORE: return launch_mx<TB_EPI_STORE>(a, sfa, w, sfw, m, n, k, e, err, stream);
    case TB_EPI_SILU: return launch_mx<TB_EPI_SILU>(a, sfa, w, sfw, m, n, k, e, err, stream);
    case TB_EPI_RESIDUAL: return launch_mx<TB_EPI_RESIDUAL>(a, sfa, w, sfw, m, n, k, e, err, stream);
    default: return TB_ERR_UNSUPPORTED;
  }
}

}  // namespace tb

extern "C" {

size_t tb_mx_scale_bytes(int rows, int k) { return tb::mx_scale_bytes(rows, k); }

int tb_mx_quantize(int src_dtype, const void* src, long long ld, int rows, int k, void* codes, void* scales,
                   void* stream) {
  return tb::mx_quantize(src_dtype, src, ld, rows, k, static_cast<uint8_t*>(codes), static_cast<uint8_t*>(scales),
                         reinterpret_cast<cudaStream_t>(stream));
}

int tb_gemm_mx(const void* a, const void* a_scales, const void* w, const void* w_scales, int m, int n, int k,
               const tb_epilogue* e, int* err, void* stream) {
  if (!e) return TB_ERR_ARG;
  return tb::gemm_mx(static_cast<const uint8_t*>(a), static_cast<const uint8_t*>(a_scales),
                     static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(w_scales), m, n, k, *e, err,
                     reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
