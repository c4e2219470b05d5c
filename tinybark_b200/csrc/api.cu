// The extern "C" entry points of libtbcuda (declared in include/tbcuda.h) and the
// encoder orchestration: subsampling, the conformer layers and the encoder projector,
// as tinybark/tinygrad/model.py:140-158 (_encode) and tinybark/mojo/bark/gpu.mojo:399-426
// (GpuEncoder.encode) run them.
#include <atomic>
#include <mutex>
#include <string>

#include "decode.cuh"
#include "host.h"

namespace tb {

int frontend(const tb_model& m, const float* samples, const long long* sample_off, const int* frame_off, int clips,
             int frames_total, float* feats, void* ws, size_t ws_bytes, cudaStream_t stream);
size_t frontend_ws(int clips);
int frontend_pcm16(const tb_model& m, const int16_t* pcm, const long long* sample_off, const int* frame_off,
                   int clips, int frames_total, float* feats, void* ws, size_t ws_bytes, cudaStream_t stream);
size_t decode_ws_groups(int dtype, int lanes, int groups);
int selftest_wait(int kind, unsigned* scratch, int* err, cudaStream_t stream);
size_t mx_scale_bytes(int rows, int k);
int mx_quantize(int src_dtype, const void* src, long long ld, int rows, int k, uint8_t* codes, uint8_t* sf,
                cudaStream_t stream);
int gemm_mx(const uint8_t* a, const uint8_t* sfa, const uint8_t* w, const uint8_t* sfw, int m, int n, int k,
            const tb_epilogue& e, int* err, cudaStream_t stream);
int tdt_decode(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
               int groups, int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err,
               cudaStream_t stream);

static thread_local std::string g_last_error;

int fail_cuda() {
  cudaError_t e = cudaGetLastError();
  g_last_error = cudaGetErrorString(e);
  return TB_ERR_CUDA;
}

static std::atomic<long long> g_launches{0};

void count_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(); }

int check_launch() {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TB_OK;
  g_last_error = cudaGetErrorString(e);
  return TB_ERR_CUDA;
}

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static thread_local int g_sm_budget = 0;
void set_sm_budget(int n) { g_sm_budget = n; }
static thread_local bool g_gemm_pairs = true;
bool gemm_pairs() { return g_gemm_pairs; }
void set_gemm_pairs(bool on) { g_gemm_pairs = on; }
int sm_budget() {
  const int s = sm_count();
  return g_sm_budget > 0 && g_sm_budget < s ? g_sm_budget : s;
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!count[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = n > 0 ? n : 148;
  }
  return count[dev];
}

// ---------------------------------------------------------------------------
// Encoder

struct EncWs {
  float* x;
  void *xn, *hid, *qu, *qv, *k, *v, *att, *glu, *dwo;
  uint8_t *xq, *xs, *hq, *hs;  // block-scaled FFN: MXFP8 codes and scales of its two inputs
  void* sub;
  size_t sub_bytes;
};

static EncWs carve_encoder(void* ws, int dtype, int t2_total, int t3_total, bool mx = false) {
  const size_t e = dsize(dtype), R = t3_total;
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  auto take = [&](size_t bytes) {
    void* q = p;
    p += align256(bytes);
    return q;
  };
  EncWs w;
  w.x = (float*)take(R * TB_HIDDEN * 4);
  w.xn = take(R * TB_HIDDEN * e);
  w.hid = take(R * TB_FFN * e);
  w.qu = take(R * TB_HIDDEN * e);
  w.qv = take(R * TB_HIDDEN * e);
  w.k = take(R * TB_HIDDEN * e);
  w.v = take(R * TB_HIDDEN * e);
  w.att = take(R * TB_HIDDEN * e);
  w.glu = take(R * TB_HIDDEN * e);
  w.dwo = take(R * TB_HIDDEN * e);
  w.xq = w.xs = w.hq = w.hs = nullptr;
  if (mx) {
    const size_t pad = (R + 127) / 128 * 128;
    w.xq = (uint8_t*)take(pad * TB_HIDDEN);
    w.xs = (uint8_t*)take(mx_scale_bytes(t3_total, TB_HIDDEN));
    w.hq = (uint8_t*)take(pad * TB_FFN);
    w.hs = (uint8_t*)take(mx_scale_bytes(t3_total, TB_FFN));
  }
  w.sub_bytes = subsample_ws(dtype, t2_total, t3_total);
  w.sub = take(w.sub_bytes);
  return w;
}

static size_t encoder_ws(int dtype, int t2_total, int t3_total, bool mx = false) {
  uint8_t* base = nullptr;
  EncWs w = carve_encoder(base, dtype, t2_total, t3_total, mx);
  return (size_t)(reinterpret_cast<uint8_t*>(w.sub) - base) + align256(w.sub_bytes);
}

static int encoder_forward(const tb_model& m, const tb_batch& b, const float* feats, float* enc, void* ws,
                           size_t ws_bytes, int* err, cudaStream_t s) {
  if (b.t3_total <= 0) return TB_OK;
  if (!m.layer || m.layers <= 0 || !feats || !enc || !ws) return TB_ERR_ARG;
  const bool mx = m.ffn_mx != nullptr;
  if (mx && m.dtype != TB_BF16) return TB_ERR_ARG;
  if (ws_bytes < encoder_ws(m.dtype, b.t2_total, b.t3_total, mx)) return TB_ERR_WORKSPACE;
  if (b.max_t3 > m.max_len) return TB_ERR_ARG;
  const int dt = m.dtype, R = b.t3_total;
  EncWs w = carve_encoder(ws, dt, b.t2_total, b.t3_total, mx);

  if (int rc = subsample(m, b, feats, w.x, w.sub, w.sub_bytes, err, s)) return rc;

  tb_epilogue silu = {};
  silu.kind = TB_EPI_SILU;
  silu.out_dtype = dt;
  silu.out = w.hid;
  silu.ldo = TB_FFN;
  tb_epilogue half = {};
  half.kind = TB_EPI_RESIDUAL;
  half.out = w.x;
  half.ldo = TB_HIDDEN;
  half.alpha = 0.5f;
  tb_epilogue full = half;
  full.alpha = 1.0f;
  tb_epilogue glu = {};
  glu.kind = TB_EPI_GLU;
  glu.out_dtype = dt;
  glu.out = w.glu;
  glu.ldo = TB_HIDDEN;
  tb_epilogue qkv = {};
  qkv.kind = TB_EPI_QKV;
  qkv.out_dtype = dt;
  qkv.out = w.qu;
  qkv.out2 = dt == TB_F32 ? w.qv : nullptr;  // the bf16 attention takes the bias_v term from rel_c
  qkv.out3 = w.k;
  qkv.out4 = w.v;
  qkv.ldo = TB_HIDDEN;

  // One macaron FFN: x += 0.5 * W2 silu(W1 xn), xn the normalised input in w.xn; block
  // scaled when the model has MXFP8 FFN weights (j: 0 for the first FFN, 1 the second).
  auto ffn = [&](int i, int j) -> int {
    const tb_layer& L = m.layer[i];
    if (!mx) {
      if (int rc = gemm(dt, w.xn, TB_HIDDEN, j ? L.ff2_w1 : L.ff1_w1, R, TB_FFN, TB_HIDDEN, silu, err, s)) return rc;
      return gemm(dt, w.hid, TB_FFN, j ? L.ff2_w2 : L.ff1_w2, R, TB_HIDDEN, TB_FFN, half, err, s);
    }
    const tb_mx_weight& w1 = m.ffn_mx[4 * i + 2 * j];
    const tb_mx_weight& w2 = m.ffn_mx[4 * i + 2 * j + 1];
    if (int rc = mx_quantize(TB_BF16, w.xn, TB_HIDDEN, R, TB_HIDDEN, w.xq, w.xs, s)) return rc;
    if (int rc = gemm_mx(w.xq, w.xs, static_cast<const uint8_t*>(w1.codes), static_cast<const uint8_t*>(w1.scales),
                         R, TB_FFN, TB_HIDDEN, silu, err, s))
      return rc;
    if (int rc = mx_quantize(TB_BF16, w.hid, TB_FFN, R, TB_FFN, w.hq, w.hs, s)) return rc;
    return gemm_mx(w.hq, w.hs, static_cast<const uint8_t*>(w2.codes), static_cast<const uint8_t*>(w2.scales), R,
                   TB_HIDDEN, TB_FFN, half, err, s);
  };

  const tb_layer& first = m.layer[0];
  if (int rc = layernorm(w.x, first.norm_w[0], first.norm_b[0], nullptr, nullptr, nullptr, w.xn, dt, R, s)) return rc;
  for (int i = 0; i < m.layers; ++i) {
    const tb_layer& L = m.layer[i];
    // x += 0.5 * FF1(LN(x))  (the LN was applied at the end of the previous layer)
    if (int rc = ffn(i, 0)) return rc;
    // x += MHSA(LN(x))
    if (int rc = layernorm(w.x, L.norm_w[1], L.norm_b[1], nullptr, nullptr, nullptr, w.xn, dt, R, s)) return rc;
    qkv.bias_u = L.bias_u;
    qkv.bias_v = L.bias_v;
    if (int rc = gemm(dt, w.xn, TB_HIDDEN, L.qkv, R, 3 * TB_HIDDEN, TB_HIDDEN, qkv, err, s)) return rc;
    if (int rc = relpos_attention(dt, w.qu, w.qv, w.k, w.v, L.rel, L.rel_c, m.max_len, b, w.att, err, s)) return rc;
    if (int rc = gemm(dt, w.att, TB_HIDDEN, L.o_proj, R, TB_HIDDEN, TB_HIDDEN, full, err, s)) return rc;
    // x += Conv(LN(x))
    if (int rc = layernorm(w.x, L.norm_w[2], L.norm_b[2], nullptr, nullptr, nullptr, w.xn, dt, R, s)) return rc;
    if (int rc = gemm(dt, w.xn, TB_HIDDEN, L.pw1, R, 2 * TB_HIDDEN, TB_HIDDEN, glu, err, s)) return rc;
    if (int rc = conv_depthwise(dt, w.glu, L.dw_w, L.dw_b, b, w.dwo, err, s)) return rc;
    if (int rc = gemm(dt, w.dwo, TB_HIDDEN, L.pw2, R, TB_HIDDEN, TB_HIDDEN, full, err, s)) return rc;
    // x += 0.5 * FF2(LN(x))
    if (int rc = layernorm(w.x, L.norm_w[3], L.norm_b[3], nullptr, nullptr, nullptr, w.xn, dt, R, s)) return rc;
    if (int rc = ffn(i, 1)) return rc;
    // x = LN_out(x), fused with the next layer's first LN (or, after the last layer, the
    // projector's input cast).
    if (i + 1 < m.layers) {
      const tb_layer& N = m.layer[i + 1];
      if (int rc = layernorm(w.x, L.norm_w[4], L.norm_b[4], w.x, N.norm_w[0], N.norm_b[0], w.xn, dt, R, s)) return rc;
    } else {
      if (int rc = layernorm(w.x, L.norm_w[4], L.norm_b[4], w.x, nullptr, nullptr, w.xn, dt, R, s)) return rc;
    }
  }
  tb_epilogue pj = {};
  pj.kind = TB_EPI_STORE;
  pj.out_dtype = TB_F32;
  pj.out = enc;
  pj.ldo = TB_PRED;
  pj.bias = m.enc_proj_b;
  return gemm(dt, w.xn, TB_HIDDEN, m.enc_proj_w, R, TB_PRED, TB_HIDDEN, pj, err, s);
}

}  // namespace tb

using namespace tb;

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

int tb_version(void) { return 1; }

long long tb_launch_count(void) { return g_launches.load(); }

int tb_tile_rows(int dtype, int* sub_rows, int* attn_rows) {
  if (!sub_rows || !attn_rows || (dtype != TB_F32 && dtype != TB_BF16)) return TB_ERR_ARG;
  *sub_rows = subsample_tile_rows();
  *attn_rows = attention_tile_rows(dtype);
  return TB_OK;
}

const char* tb_last_cuda_error(void) { return g_last_error.c_str(); }

int tb_sm_count(int device, int* out) {
  if (!out) return TB_ERR_ARG;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return fail_cuda();
  *out = n;
  return TB_OK;
}

size_t tb_frontend_workspace_bytes(int clips, int frames_total) {
  (void)frames_total;
  return frontend_ws(clips);
}

int tb_frontend(const tb_model* m, const float* samples, const long long* sample_off, const int* frame_off, int clips,
                int frames_total, int max_frames, float* feats, void* ws, size_t ws_bytes, void* stream) {
  (void)max_frames;
  if (!m) return TB_ERR_ARG;
  return frontend(*m, samples, sample_off, frame_off, clips, frames_total, feats, ws, ws_bytes, as_stream(stream));
}

int tb_frontend_pcm16(const tb_model* m, const int16_t* pcm, const long long* sample_off, const int* frame_off,
                      int clips, int frames_total, int max_frames, float* feats, void* ws, size_t ws_bytes,
                      void* stream) {
  (void)max_frames;
  if (!m) return TB_ERR_ARG;
  return frontend_pcm16(*m, pcm, sample_off, frame_off, clips, frames_total, feats, ws, ws_bytes, as_stream(stream));
}

int tb_layernorm(const float* x, const float* w, const float* b, float* x_out, const float* w2, const float* b2,
                 void* y, int y_dtype, int rows, void* stream) {
  return layernorm(x, w, b, x_out, w2, b2, y, y_dtype, rows, as_stream(stream));
}

int tb_gemm(int dtype, const void* a, long long lda, const void* w, int m, int n, int k, const tb_epilogue* epi,
            int* err, void* stream) {
  if (!epi) return TB_ERR_ARG;
  return gemm(dtype, a, lda, w, m, n, k, *epi, err, as_stream(stream));
}

int tb_text_offsets(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off, int vocab,
                    long long* text_off, int* err, void* stream) {
  return text_offsets(tokens, ld, counts, lanes, piece_off, vocab, text_off, err, as_stream(stream));
}

int tb_text_bytes(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off,
                  const uint8_t* piece_bytes, long long piece_bytes_len, int vocab, const long long* text_off,
                  uint8_t* text, long long text_len, void* stream) {
  return text_bytes(tokens, ld, counts, lanes, piece_off, piece_bytes, piece_bytes_len, vocab, text_off, text,
                    text_len, as_stream(stream));
}

int tb_repack(const tb_repack_job* jobs, int n_jobs, void* jobs_dev, const void* src, size_t src_bytes, void* dst,
              size_t dst_bytes, void* stream) {
  return repack(jobs, n_jobs, jobs_dev, src, src_bytes, dst, dst_bytes, as_stream(stream));
}

int tb_set_gemm_pairs(int on) {
  const int was = gemm_pairs() ? 1 : 0;
  set_gemm_pairs(on != 0);
  return was;
}

int tb_relpos_attention(int dtype, const void* qu, const void* qv, const void* k, const void* v, const void* rel,
                        const float* rel_c, int max_len, const tb_batch* batch, void* out, int* err, void* stream) {
  if (!batch) return TB_ERR_ARG;
  return relpos_attention(dtype, qu, qv, k, v, rel, rel_c, max_len, *batch, out, err, as_stream(stream));
}

int tb_conv_depthwise(int dtype, const void* glu, const float* w, const float* b, const tb_batch* batch, void* out,
                      int* err, void* stream) {
  if (!batch) return TB_ERR_ARG;
  return conv_depthwise(dtype, glu, w, b, *batch, out, err, as_stream(stream));
}

size_t tb_subsample_workspace_bytes(int dtype, int t2_total, int t3_total) {
  return subsample_ws(dtype, t2_total, t3_total);
}

int tb_subsample(const tb_model* m, const tb_batch* batch, const float* feats, float* x, void* ws, size_t ws_bytes,
                 int* err, void* stream) {
  if (!m || !batch) return TB_ERR_ARG;
  return subsample(*m, *batch, feats, x, ws, ws_bytes, err, as_stream(stream));
}

size_t tb_encoder_workspace_bytes(int dtype, int t2_total, int t3_total) {
  return encoder_ws(dtype, t2_total, t3_total);
}

size_t tb_encoder_workspace_bytes_mx(int t2_total, int t3_total) {
  return encoder_ws(TB_BF16, t2_total, t3_total, true);
}

int tb_encoder_forward(const tb_model* m, const tb_batch* batch, const float* feats, float* enc, void* ws,
                       size_t ws_bytes, int* err, void* stream) {
  if (!m || !batch) return TB_ERR_ARG;
  return encoder_forward(*m, *batch, feats, enc, ws, ws_bytes, err, as_stream(stream));
}

size_t tb_decode_workspace_bytes(int dtype, int lanes, int groups) {
  if (lanes <= 0) return 0;  // groups <= 0: the persistent decoder's workspace, that of one group
  groups = groups < 1 ? 1 : (groups > 8 ? 8 : groups);
  return decode_ws_groups(dtype, lanes, groups < lanes ? groups : lanes);
}

int tb_decode_lane_iterations(const void* ws, int dtype, int lanes, int groups, int* iters, void* stream) {
  if (!ws || !iters || lanes <= 0 || groups > 1 || (dtype != TB_F32 && dtype != TB_BF16)) return TB_ERR_ARG;
  const DecodeWs w = carve(const_cast<void*>(ws), dtype, lanes);
  if (cudaMemcpyAsync(iters, w.it, (size_t)lanes * sizeof(int), cudaMemcpyDeviceToDevice, as_stream(stream)) !=
      cudaSuccess)
    return fail_cuda();
  return TB_OK;
}

int tb_selftest_wait(int kind, void* scratch, int* err, void* stream) {
  return selftest_wait(kind, reinterpret_cast<unsigned*>(scratch), err, as_stream(stream));
}

int tb_tdt_decode(const tb_model* m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                  int groups, int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err,
                  void* stream) {
  if (!m) return TB_ERR_ARG;
  return tdt_decode(*m, enc, enc_off, cap, lanes, max_cap, groups, tokens, counts, ws, ws_bytes, host_flag, err,
                    as_stream(stream));
}

}  // extern "C"
