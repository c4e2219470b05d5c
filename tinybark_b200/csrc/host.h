// Host-side helpers shared by the .cu files of libtbcuda.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/tbcuda.h"

namespace tb {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tensor_map_encoder();
// 2-D bf16 tensor map, 128-byte swizzle, box of box_cols x box_rows (box_cols * 2 <= 128).
bool encode_tmap_2d(CUtensorMap* map, const void* ptr, long long rows, long long cols, long long ld_elems,
                    int box_cols, int box_rows);
int sm_count();
// SMs a GEMM launched from this thread may plan for (all by default): kernels that run
// concurrently on several streams each take a share.
int sm_budget();
void set_sm_budget(int n);  // 0: all
// Whether large bf16 GEMMs may run on CTA pairs (this thread's setting; on by default).
bool gemm_pairs();
void set_gemm_pairs(bool on);
int fail_cuda();     // records cudaGetLastError() and returns TB_ERR_CUDA
int check_launch();  // TB_OK, or fail_cuda() if the last launch failed; counts the launch
void count_launches(long long n);  // adds kernels run by a graph replay (or removes captured ones)
long long launch_count();

int gemm(int dtype, const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue& e, int* err,
         cudaStream_t stream);
int layernorm(const float* x, const float* w, const float* b, float* x_out, const float* w2, const float* b2, void* y,
              int y_dtype, int rows, cudaStream_t stream);
int relpos_attention(int dtype, const void* qu, const void* qv, const void* k, const void* v, const void* rel,
                     const float* rel_c, int max_len, const tb_batch& batch, void* out, int* err, cudaStream_t stream);
int conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch& batch, void* out, int* err,
                   cudaStream_t stream);
int subsample(const tb_model& m, const tb_batch& batch, const float* feats, float* x, void* ws, size_t ws_bytes,
              int* err, cudaStream_t stream);
size_t subsample_ws(int dtype, int t2_total, int t3_total);
int subsample_tile_rows();  // depthwise-1 rows per work item of the fused conv-0 kernel
int attention_tile_rows(int dtype);
int text_offsets(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off, int vocab,
                 long long* text_off, int* err, cudaStream_t stream);
int text_bytes(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off,
               const uint8_t* piece_bytes, long long piece_bytes_len, int vocab, const long long* text_off,
               uint8_t* text, long long text_len, cudaStream_t stream);
int repack(const tb_repack_job* jobs, int n_jobs, void* jobs_dev, const void* src, size_t src_bytes, void* dst,
           size_t dst_bytes, cudaStream_t stream);

// Launches `kernel` with programmatic stream serialization (see grid_dep_wait in
// common.cuh): its prologue may overlap the end of the previous kernel on the stream.
template <typename... Params, typename... Args>
int launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
  return check_launch();
}

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }
inline size_t dsize(int dtype) { return dtype == TB_BF16 ? 2 : 4; }

}  // namespace tb
