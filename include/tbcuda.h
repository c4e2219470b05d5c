/* tbcuda: the C ABI of the B200 (sm_100a) inference path for the
 * Parakeet-TDT-0.6B-v3 / Underdog Bark speech-to-text model.
 *
 * Plain C types only: device pointers, sizes and a cudaStream_t passed as void*.
 * The library allocates no device memory: the caller passes every buffer, including
 * a workspace whose size the *_workspace_bytes functions give. Every function returns
 * TB_OK (0) or a TB_ERR_* status; kernels that wait on hardware barriers report a
 * timeout by or-ing a TB_DEV_* bit into the caller's device error word `err`
 * (int32, zeroed by the caller) instead of hanging.
 *
 * Threading: functions are reentrant; calls on one stream are ordered. Use one
 * process per GPU.
 */
#ifndef TBCUDA_H
#define TBCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tb_status {
  TB_OK = 0,
  TB_ERR_ARG = 1,         /* bad size, pointer or enum */
  TB_ERR_CUDA = 2,        /* a CUDA runtime call failed (see tb_last_cuda_error) */
  TB_ERR_UNSUPPORTED = 3, /* no kernel for this shape / dtype */
  TB_ERR_WORKSPACE = 4,   /* workspace smaller than *_workspace_bytes */
  TB_ERR_TOO_LARGE = 5    /* more than the library's own scratch holds (tb_frontend_static) */
};

/* Bits a kernel or-s into the device error word. */
enum tb_device_error {
  TB_DEV_GEMM_TIMEOUT = 1 << 0,
  TB_DEV_ATTN_TIMEOUT = 1 << 1,
  TB_DEV_DECODE_TIMEOUT = 1 << 2,
  TB_DEV_CONV_TIMEOUT = 1 << 3,
  TB_DEV_TEXT_TOKEN = 1 << 4 /* tb_text_offsets: a token id outside the piece table (it adds no bytes) */
};

/* Arithmetic type of a path: fp32 everywhere, or bf16 operands with fp32
 * accumulation, fp32 residual stream and fp32 LayerNorm/softmax statistics. */
enum tb_dtype { TB_F32 = 0, TB_BF16 = 1 };

/* Model dimensions, fixed by the architecture (tinybark/mojo/bark/model.mojo:29-43). */
#define TB_HIDDEN 1024
#define TB_HEADS 8
#define TB_HEAD_DIM 128
#define TB_FFN 4096
#define TB_KERNEL 9
#define TB_CHANNELS 256
#define TB_MELS 128
#define TB_VOCAB 8193
#define TB_BLANK 8192
#define TB_EOS 3
#define TB_DURATIONS 5
#define TB_PRED 640
#define TB_TOKEN_ROWS 8256 /* token head padded to a multiple of 64 (tinybark/weights.py:24,84-86) */
#define TB_JOINT_ROWS 8448 /* token rows, then the 5 duration rows at TB_TOKEN_ROWS, zero rows to a multiple of 256 */

/* GEMM epilogues: C = A(M x K) * W(N x K)^T, then one of: */
enum tb_epilogue_kind {
  TB_EPI_STORE = 0,     /* out[m,n] = acc (+ bias[n])                                     */
  TB_EPI_SILU = 1,      /* out[m,n] = silu(acc)                                            */
  TB_EPI_RESIDUAL = 2,  /* res[m,n] += alpha * acc (res is fp32 `out`)                     */
  TB_EPI_BIAS_RELU = 3, /* out[m,n] = relu(acc + bias[n])                                  */
  TB_EPI_GLU = 4,       /* W rows interleaved (a0,g0,a1,g1..): out[m,n/2] = a*sigmoid(g)   */
  TB_EPI_QKV = 5,       /* N = 3072: out = q+bias_u, out2 = q+bias_v, out3 = k, out4 = v    */
  TB_EPI_ARGMAX = 6,    /* joint head: argmax of acc+bias over [0,split) into keys[m] and
                           over [split, split_end) into keys2[m]; first index wins ties   */
  TB_EPI_LSTM = 7,      /* W rows gate-interleaved (row 4u+g, gates i,f,g,o): LSTM cell for
                           rows with mask[m] != 0: c[m,u], h[m,u] updated, h also written
                           to out[m*ldo+u] and out2[m*ldo2+u] (out_dtype)                  */
  TB_EPI_JOINT_IN = 8   /* the decoder projector: out[m,n] = acc + bias[n] (fp32; out may be NULL), and for
                           rows with gather_row[m] >= 0 the joint's next input
                           out2[m*ldo2+n] = relu(gather[gather_row[m]*ldo + n] + out[m,n])
                           (out_dtype)                                                    */
};

typedef struct tb_epilogue {
  int kind;
  int out_dtype; /* tb_dtype of out/out2/out3/out4 (RESIDUAL: out is always fp32) */
  void* out;
  long long ldo; /* elements */
  const float* bias;
  float alpha;
  void* out2;
  long long ldo2;
  void* out3;
  void* out4;
  const float* bias_u;
  const float* bias_v;
  unsigned long long* keys;
  unsigned long long* keys2;
  int split;
  int split_end;
  float* c;
  float* h;
  const int* mask;
  const int* rows; /* if not NULL: only rows below *rows (device int, read at run time) are computed */
  const float* gather;    /* TB_EPI_JOINT_IN: rows of N values (the encoder frames) */
  const int* gather_row;  /* TB_EPI_JOINT_IN: row of `gather` for each output row, < 0 to skip */
} tb_epilogue;

/* One conformer layer, device pointers. Matrices are tb_model.dtype; vectors fp32. */
typedef struct tb_layer {
  const float* norm_w[5]; /* norm_feed_forward1, norm_self_att, norm_conv, norm_feed_forward2, norm_out */
  const float* norm_b[5];
  const void* ff1_w1; /* [4096, 1024] */
  const void* ff1_w2; /* [1024, 4096] */
  const void* ff2_w1;
  const void* ff2_w2;
  const void* qkv;    /* [3072, 1024]: q, k, v rows */
  const void* o_proj; /* [1024, 1024] */
  const void* pw1;    /* [2048, 1024]: pointwise_conv1 rows interleaved (a0, g0, a1, g1, ...) */
  const void* pw2;    /* [1024, 1024] */
  const float* bias_u; /* [8, 128] */
  const float* bias_v;
  const float* dw_w;  /* [1024, 9] depthwise taps with BatchNorm folded in */
  const float* dw_b;  /* [1024] */
  const void* rel;    /* [2*max_len-1, 1024]: positions(max_len) @ relative_k_proj^T */
  const float* rel_c; /* [2*max_len-1, 128]: column h < 8 = (bias_v - bias_u)_h . rel (bf16 attention) */
} tb_layer;

typedef struct tb_model {
  int dtype;
  int layers;
  int max_len; /* encoder frames the rel tables cover */
  /* subsampling (dw_striding, 8x) */
  const float* sub0_w;  /* [256, 9] conv 1->256, 3x3 */
  const float* sub0_b;
  const float* sub_dw_w[2]; /* [256, 9] depthwise 3x3 */
  const float* sub_dw_b[2];
  const void* sub_pw_w[2];  /* [256, 256] pointwise */
  const float* sub_pw_b[2];
  const void* sub_linear_w; /* [1024, 4096], columns in (frequency, channel) order */
  const float* sub_linear_b;
  const tb_layer* layer;    /* host array of `layers` entries */
  const void* enc_proj_w;   /* [640, 1024] */
  const float* enc_proj_b;
  /* prediction network and joint */
  const void* embedding;    /* [8193, 640] */
  const void* lstm_w[2];    /* [2560, 1280] = [W_ih | W_hh], rows gate-interleaved (4u+g) */
  const float* lstm_b[2];   /* [2560] = b_ih + b_hh, same row order */
  const void* dec_proj_w;   /* [640, 640] */
  const float* dec_proj_b;
  const void* joint_w;      /* [TB_JOINT_ROWS, 640] */
  const float* joint_b;     /* [TB_JOINT_ROWS], -inf on padding rows */
  /* front-end tables */
  const float* window;      /* [512] */
  const float* mel_w;       /* packed non-zero filter weights */
  const int* mel_start;     /* [128] first FFT bin of each filter */
  const int* mel_off;       /* [129] offsets of each filter's weights in mel_w */
  /* persistent decoder (bf16): layer 0's LSTM split in its two inputs */
  const void* lstm0_hh;     /* [2560, 640]: the h columns of lstm_w[0] (its last 640), contiguous */
  const float* lstm0_emb;   /* [8193, 2560] fp32: embedding . (the x columns of lstm_w[0])^T,
                               the input term of layer 0's gates for every token */
  /* block-scaled FFN (bf16 models only; NULL: the bf16 FFN): 4 per layer, ff1_w1, ff1_w2,
     ff2_w1, ff2_w2, each in tb_mx_quantize's form */
  const struct tb_mx_weight* ffn_mx;
} tb_model;

/* One weight matrix [n, k] in MXFP8 (tb_mx_quantize): E4M3 codes and tiled E8M0 scales. */
typedef struct tb_mx_weight {
  const void* codes;
  const void* scales;
} tb_mx_weight;

/* A batch of clips, packed end to end at every stage (no padding between clips).
 * Offsets are cumulative row counts, [clips + 1], on the device; *_total are the
 * last entries, also passed by value. */
typedef struct tb_batch {
  int clips;
  int frames_total; /* feature frames */
  int t1_total;     /* after the first stride-2 conv */
  int t2_total;     /* after the second */
  int t3_total;     /* encoder frames */
  const int* frame_off;
  const int* t1_off;
  const int* t2_off;
  const int* t3_off;
  const int* t2_clip;  /* [t2_total] clip of each row */
  const int* t3_clip;  /* [t3_total] clip of each row */
  const int* sub_tiles;  /* [n_sub_tiles * 2]: (clip, first t2 row in clip) */
  int n_sub_tiles;
  const int* attn_tiles; /* [n_attn_tiles * 2]: (clip, first query row in clip) */
  int n_attn_tiles;
  int max_t3;
} tb_batch;

/* ---- library ---- */
int tb_version(void);
/* Rows per work item in tb_batch.sub_tiles (second-stage frames) and
 * tb_batch.attn_tiles (query frames) for the given dtype. */
int tb_tile_rows(int dtype, int* sub_rows, int* attn_rows);
/* Kernels this process has launched through the library so far. */
long long tb_launch_count(void);
const char* tb_last_cuda_error(void);
int tb_sm_count(int device, int* out);

/* ---- front-end: tinybark/audio.py:42-55 (features) ----
 * samples: float32, clips packed end to end (sample_off [clips+1], device, int64).
 * feats: [frames_total, 128] float32; frame_off [clips+1] device, frames = samples // 160,
 * every clip at least 2 frames. stats: workspace of tb_frontend_workspace_bytes. */
size_t tb_frontend_workspace_bytes(int clips, int frames_total);
int tb_frontend(const tb_model* m, const float* samples, const long long* sample_off, const int* frame_off,
                int clips, int frames_total, int max_frames, float* feats, void* ws, size_t ws_bytes, void* stream);
/* The same from 16-bit PCM (s16le as transcribe_pcm takes it, tinybark/tinygrad/__init__.py:33-35),
 * converted on the device as pcm / 32768 (tinybark/pytorch/__init__.py:50): half the bytes
 * to move, the same features. */
int tb_frontend_pcm16(const tb_model* m, const int16_t* pcm, const long long* sample_off, const int* frame_off,
                      int clips, int frames_total, int max_frames, float* feats, void* ws, size_t ws_bytes,
                      void* stream);

/* ---- front-end without a caller-supplied workspace (no counterpart in the reference) ----
 * The same features as tb_frontend, for callers that cannot allocate device memory:
 * a real-time audio thread, where cudaMalloc can synchronize the device and stall the
 * stream, or a host whose device memory is all owned by another allocator. The scratch
 * lives in a fixed device array inside the library (about 1.1 MB on every GPU that loads
 * it, kept until the process exits), so at most TB_FRONTEND_STATIC_MAX_CLIPS clips per
 * call; more returns TB_ERR_TOO_LARGE before anything runs. The caller still allocates
 * samples, offsets and feats. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current: make it before any stream
 * capture. The address is kept for the life of the process: after a device reset
 * (cudaDeviceReset), which unloads the library's device code, do not call it again. All calls share the array: calls that can overlap on the GPU (other streams,
 * other threads) race and must be serialized by the caller. Nothing in it needs to start
 * at zero: every scratch value is written before it is read. Allocates nothing. */
#define TB_FRONTEND_STATIC_MAX_CLIPS 64
int tb_frontend_static(const tb_model* m, const float* samples, const long long* sample_off, const int* frame_off,
                       int clips, int frames_total, float* feats, void* stream);

/* ---- LayerNorm over 1024: tinybark/tinygrad/model.py:56-57 (layernorm) ----
 * y = LN(x) (y_dtype), fp32 statistics, eps 1e-5. If x_out != NULL, LN(x) is also
 * written there in fp32 (x_out may be x). If w2 != NULL (needs x_out), y = LN2(LN(x)):
 * a block's norm_out fused with the next block's norm_feed_forward1. */
int tb_layernorm(const float* x, const float* w, const float* b, float* x_out, const float* w2, const float* b2,
                 void* y, int y_dtype, int rows, void* stream);

/* ---- linear layers: tinybark/tinygrad/model.py:37-40 (linear), tinybark/mojo/bark/gpu.mojo:429-436 (mm) ----
 * A [M, K] (lda elements) times W [N, K] transposed, epilogue `epi`. dtype TB_BF16 runs
 * the tcgen05 tensor-core kernel (K % 64 == 0, N % 256 == 0 or N % 128 == 0); TB_F32 a
 * CUDA-core fp32 kernel (K % 16 == 0, N % 128 == 0). W is read as constant: for M <= 256
 * (bf16) or M <= 8 (fp32) the kernel may start reading it before the kernel launched just
 * before it on the stream has finished, so W must not be the output of that kernel (the
 * library's kernels let their successor start early). A RESIDUAL GEMM of at most 256 rows
 * whose tiles would leave most SMs idle splits K over several CTAs that add their sums
 * into out atomically: its last bits depend on the order of those adds. */
int tb_gemm(int dtype, const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue* epi,
            int* err, void* stream);
/* Large bf16 GEMMs (at least 2048 rows, N % 256 == 0, no run-time row bound, epilogue
 * STORE, SILU, RESIDUAL, BIAS_RELU, GLU or QKV) run on CTA pairs, 256 x 256 tiles with
 * 256-row MMAs over two SMs' shared memory. on = 0 makes the calling thread's later
 * GEMMs take one CTA per 128-row tile instead (the same results, bit for bit); returns
 * the previous setting. No reference counterpart: a tuning and test switch. */
int tb_set_gemm_pairs(int on);

/* ---- relative-position MHSA core: tinybark/tinygrad/model.py:99-116 (_attention),
 * tinybark/mojo/bark/gpu.mojo:202-224 (softmax_kernel) ----
 * qu = q + bias_u, qv = q + bias_v, k, v: [t3_total, 1024] (dtype) packed by clip;
 * rel: [2*max_len-1, 1024]; out: [t3_total, 1024] (dtype), heads side by side.
 * fp32 reads qv; bf16 (tensor cores) reads rel_c instead: [2*max_len-1, 128] fp32,
 * column h < 8 = (bias_v - bias_u)_h . rel[row, head h] (qv may then be NULL).
 * tb_batch.attn_tiles must use tb_tile_rows(dtype) query rows per item. */
int tb_relpos_attention(int dtype, const void* qu, const void* qv, const void* k, const void* v, const void* rel,
                        const float* rel_c, int max_len, const tb_batch* batch, void* out, int* err, void* stream);

/* ---- conv module middle: tinybark/tinygrad/model.py:121-124 (_conv: GLU output,
 * depthwise k=9 with folded BatchNorm, SiLU) ----
 * glu: [t3_total, 1024] (dtype) = a * sigmoid(g); out = silu(dw(glu) + b) (dtype).
 * err: device error word (TB_DEV_CONV_TIMEOUT if the bf16 kernel's bounded wait gave up). */
int tb_conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch* batch, void* out,
                      int* err, void* stream);

/* ---- subsampling: tinybark/tinygrad/model.py:87-97 (_subsample) ----
 * feats [frames_total, 128] fp32 -> x [t3_total, 1024] fp32. */
size_t tb_subsample_workspace_bytes(int dtype, int t2_total, int t3_total);
int tb_subsample(const tb_model* m, const tb_batch* batch, const float* feats, float* x, void* ws, size_t ws_bytes,
                 int* err, void* stream);

/* ---- whole encoder: tinybark/tinygrad/model.py:140-158 (_encode),
 * tinybark/mojo/bark/gpu.mojo:399-426 (GpuEncoder.encode) ----
 * feats -> enc [t3_total, 640] fp32 (encoder frames projected for the joint). With
 * tb_model.ffn_mx set, each FFN's input and hidden activations are quantized to MXFP8
 * (tb_mx_quantize) and both FFN GEMMs run block-scaled (tb_gemm_mx). */
size_t tb_encoder_workspace_bytes(int dtype, int t2_total, int t3_total);
/* The workspace of a bf16 model with block-scaled FFN weights (tb_model.ffn_mx set): the
 * bf16 one plus the MXFP8 activations of the FFN GEMMs. */
size_t tb_encoder_workspace_bytes_mx(int t2_total, int t3_total);
int tb_encoder_forward(const tb_model* m, const tb_batch* batch, const float* feats, float* enc, void* ws,
                       size_t ws_bytes, int* err, void* stream);

/* ---- TDT greedy decode: tinybark/tinygrad/model.py:162-233 (_step, generate),
 * tinybark/mojo/bark/model.mojo:294-318 (decode) ----
 * One lane per clip, all lanes stepped together. enc [t3_total, 640] fp32 packed by
 * clip (enc_off [lanes+1]); cap [lanes] = 10 * subsampled(frames + 1, 3) - 1.
 * tokens: [lanes, max_cap] int32; counts: [lanes].
 * groups = 0 (bf16): one persistent kernel runs the whole loop over all lanes, its
 * phases separated by a grid-wide barrier; it stops once no lane runs. fp32, or
 * groups = 1..8: the loop is replayed as CUDA graphs of 32 iterations, one GEMM kernel
 * per step, with the lanes split into `groups` contiguous groups decoded concurrently,
 * group 0 on `stream` and the others on the library's own streams, joined back into
 * `stream` before return: group g holds ceil((lanes - g) / groups) lanes, so dealing
 * clips (longest first) round-robin into groups gives balanced groups. host_flag:
 * pinned host memory (may be NULL). Graph decoder: 2 ints per group, used to stop a group
 * early once all its lanes are done (NULL: every group runs its longest cap). Persistent
 * decoder: every 32 iterations it stores [1] = the iteration and then [0] = a row bound
 * R such that every lane >= R has stopped with its tokens and counts[] final (the caller
 * may copy those lanes out while the loop goes on; set [0] = lanes before the call).
 * Lanes ordered longest first let the GEMMs shrink to the lanes still running. Both
 * decoders give the same tokens. */
/* Self-test of the failure handling; no reference counterpart. Launches one CTA that
 * waits on something nothing will complete: kind 0 an mbarrier (the wait between the
 * warps of every tcgen05 kernel here), kind 1 the persistent decoder's grid barrier
 * (counter and abort flag in `scratch`, 256 device bytes this call zeroes). The wait
 * gives up after the library's limit (2 s), or-s TB_DEV_GEMM_TIMEOUT (kind 0) or
 * TB_DEV_DECODE_TIMEOUT (kind 1) into *err and the kernel returns: no hang, no fault, and
 * the context stays usable. */
int tb_selftest_wait(int kind, void* scratch, int* err, void* stream);
/* Self-test of the epilogues' fast arithmetic (no reference counterpart): y[i] = f(x[i])
 * for n float32 values on the device, f by kind: 0 the Newton reciprocal (x >= 1),
 * 1 sigmoid and 2 SiLU with one special-function operation, 3 and 4 their two-wide forms,
 * 5 the tanh-based sigmoid and 6 the hardware tanh of the LSTM cells, 7 the tanh-based
 * two-wide SiLU of the FFN-up and depthwise-conv epilogues. */
int tb_selftest_math(int kind, const float* x, float* y, long long n, void* stream);

size_t tb_decode_workspace_bytes(int dtype, int lanes, int groups);
/* After a tb_tdt_decode with groups 0 or 1 on this workspace (and stream): the greedy-loop
 * iterations each lane ran (tinybark/tinygrad/model.py:222-233 counts them against the
 * cap), copied into iters [lanes] (device int32). The algorithmic work of a decode is these
 * iterations times the work of one (joint on every iteration, prediction step on each
 * emitted token); measurement only. TB_ERR_ARG for other groups. */
int tb_decode_lane_iterations(const void* ws, int dtype, int lanes, int groups, int* iters, void* stream);
int tb_tdt_decode(const tb_model* m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                  int groups, int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err,
                  void* stream);

/* ---- block-scaled FP8 FFN GEMM (MXFP8): the low-precision weight option of
 * tinybark/docs/2026-10-24-learnings.md:133-146 (no reference kernel; the bf16 GEMM,
 * tb_gemm, is the default path) ----
 * tb_mx_quantize: rows x k values (src_dtype TB_F32 or TB_BF16, row stride ld elements,
 * 16-byte aligned, k a multiple of 512) to E4M3 codes [ceil(rows / 128) * 128, k] (row
 * stride k; rows past `rows` get zero codes) and E8M0 scales, one per 32 values along k:
 * e = floor(log2 max |x|) - 8 clamped to [-127, 127] (-127 for an all-zero block), codes
 * E4M3(x * 2^-e) rounded to nearest even, saturated to +-448, scale byte e + 127. The
 * scales are stored tiled as [rows / 128][k / 512][128][16] bytes: tb_mx_scale_bytes.
 * tb_gemm_mx: C = A * W^T from two such matrices (m rows of A, n of W, n a multiple of
 * 128, k a multiple of 512), fp32 accumulation, epilogue TB_EPI_STORE, TB_EPI_SILU or
 * TB_EPI_RESIDUAL as tb_gemm's (no run-time row bound). */
size_t tb_mx_scale_bytes(int rows, int k);
int tb_mx_quantize(int src_dtype, const void* src, long long ld, int rows, int k, void* codes, void* scales,
                   void* stream);
int tb_gemm_mx(const void* a, const void* a_scales, const void* w, const void* w_scales, int m, int n, int k,
               const tb_epilogue* e, int* err, void* stream);

/* ---- weight loading: the fp16 cache (tinybark/weights.py:92-120), read whole as
 * tinybark/tinygrad/weights.py:10-26 reads it, then split into the kernels' layout ----
 * tb_repack writes the packed weights from one source buffer: the cache file's data block
 * uploaded as is (or any buffer of f16 / f32 tensors). Job j writes one contiguous
 * destination tensor at dst + dst_off of extents dims[0..3] (dims[3] innermost): element
 * (i0, i1, i2, i3) is source element src_off / size + i0 * stride[0] + i1 * stride[1] +
 * i2 * stride[2] + i3 * stride[3], converted to dst_type (bf16 rounded to nearest even), or
 * `value` when fill is 1. Reorderings (gate interleaving, column permutations, slices)
 * are strides; padding rows are fill jobs.
 * Every job is checked against src_bytes and dst_bytes before anything runs (TB_ERR_ARG:
 * a type, an offset not a multiple of its element size, a negative stride, a read or a
 * write out of range, more than 2^31 - 1 elements). The table is then copied into
 * jobs_dev (device, at least n_jobs * sizeof(tb_repack_job) bytes, 8-byte aligned) and one
 * kernel runs, in chunks of TB_REPACK_CHUNK elements spread over the SMs. first_chunk is
 * filled in by the library. */
#define TB_REPACK_CHUNK 16384
enum tb_src_type { TB_SRC_F16 = 0, TB_SRC_F32 = 1 };
typedef struct {
  long long src_off;     /* source byte offset */
  long long dst_off;     /* destination byte offset */
  long long stride[4];   /* source element stride of each destination index, >= 0 */
  long long first_chunk; /* set by tb_repack */
  int dims[4];           /* destination extents, >= 0 */
  int src_type;          /* TB_SRC_F16 or TB_SRC_F32 (ignored by fill jobs) */
  int dst_type;          /* TB_F32 or TB_BF16 */
  int fill;              /* 1: every element is `value` */
  float value;
} tb_repack_job;
int tb_repack(const tb_repack_job* jobs, int n_jobs, void* jobs_dev, const void* src, size_t src_bytes, void* dst,
              size_t dst_bytes, void* stream);

/* ---- text: tinybark/text.py:19-34 (Tokenizer.decode, special tokens skipped) ----
 * Token rows to UTF-8 bytes. The piece table gives each id's bytes as the text joins them:
 * a SentencePiece piece with "\u2581" as a space, a byte-fallback piece <0xNN> as the byte
 * NN, a special token as nothing (piece_off [vocab + 1] and piece_bytes, device). Lane l's
 * bytes are those of tokens[l * ld + t] for t < counts[l] (clamped to [0, ld]), joined;
 * decoded as UTF-8 with invalid sequences replaced, "\u2581" turned into a space and the
 * ends stripped, they are the reference's text for those ids.
 * tb_text_offsets writes text_off [lanes + 1] (int64, device): lane l's bytes are
 * [text_off[l], text_off[l + 1]). An id outside [0, vocab) adds nothing and sets
 * TB_DEV_TEXT_TOKEN in err (may be NULL). tb_text_bytes then writes the bytes into text
 * (text_len bytes, at least text_off[lanes]; nothing is written past it or read outside
 * piece_bytes [piece_bytes_len]). */
int tb_text_offsets(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off, int vocab,
                    long long* text_off, int* err, void* stream);
int tb_text_bytes(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off,
                  const uint8_t* piece_bytes, long long piece_bytes_len, int vocab, const long long* text_off,
                  uint8_t* text, long long text_len, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TBCUDA_H */
