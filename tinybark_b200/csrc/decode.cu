// TDT greedy decoding for a batch of clips, one lane per clip, all lanes stepped
// together. Replaces the prediction network step, joint and greedy loop of
// tinybark/tinygrad/model.py:162-233 (= tinybark/ort/__init__.py:55-86,
// tinybark/mojo/bark/model.mojo:250-318), which run one clip and one host round trip
// per emitted token.
//
// Per iteration, for every lane still running:
//   prep:  z = relu(enc[frame] + dec)                          (the joint's input)
//   joint: argmax over 8193 token logits and 5 duration logits  (GEMM, ARGMAX epilogue)
//   step:  the loop body of the reference: blank -> frame += max(d, 1); otherwise emit,
//          stop on EOS, else frame += d and the LSTM steps on the token; stop when
//          frame >= valid or after `cap` iterations
//   lstm0, lstm1: gates GEMM with the LSTM cell fused into the epilogue (masked lanes
//          keep their state)
//   proj:  dec = h1 W_p^T + b_p
// The LSTM inputs [embedding(token) | h] are assembled from the fp32 state by the step
// kernel, so no GEMM reads a buffer that its own epilogue writes.
#include <algorithm>
#include <chrono>
#include <thread>
#include <vector>

#include "epilogue.cuh"
#include "host.h"

namespace tb {

constexpr int DECODE_CHUNK = 32;       // iterations per captured graph
constexpr int DECODE_MAX_CHUNKS = 8192;  // so max_cap <= 262144

struct DecodeWs {
  unsigned long long *keys, *keys2;
  void *z, *x0, *x1, *hp;
  float *h, *c, *dec;
  int *frame, *it, *done, *mask, *count, *active;
  int* m_chunk;  // [DECODE_MAX_CHUNKS]: only lanes below this index can run in chunk c
  int* m_cur;    // [0]: the current chunk's bound, [1]: the current chunk
};

static DecodeWs carve(void* ws, int dtype, int lanes) {
  const size_t e = dsize(dtype), L = lanes;
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  DecodeWs w;
  auto take = [&](size_t bytes) {
    void* q = p;
    p += align256(bytes);
    return q;
  };
  w.keys = (unsigned long long*)take(L * 8);
  w.keys2 = (unsigned long long*)take(L * 8);
  w.z = take(L * TB_PRED * e);
  w.x0 = take(L * 2 * TB_PRED * e);
  w.x1 = take(L * 2 * TB_PRED * e);
  w.hp = take(L * TB_PRED * e);
  w.h = (float*)take(2 * L * TB_PRED * 4);
  w.c = (float*)take(2 * L * TB_PRED * 4);
  w.dec = (float*)take(L * TB_PRED * 4);
  w.frame = (int*)take(L * 4);
  w.it = (int*)take(L * 4);
  w.done = (int*)take(L * 4);
  w.mask = (int*)take(L * 4);
  w.count = (int*)take(L * 4);
  w.active = (int*)take(256);
  w.m_chunk = (int*)take(DECODE_MAX_CHUNKS * 4);
  w.m_cur = (int*)take(256);
  return w;
}

size_t decode_ws(int dtype, int lanes) {
  uint8_t* base = nullptr;
  DecodeWs w = carve(base, dtype, lanes);
  return (size_t)(reinterpret_cast<uint8_t*>(w.m_cur) - base) + 256;
}

// Lane state initialisation and the inputs of the first step (token = blank, zero state).
template <typename T>
__global__ void decode_init_kernel(DecodeWs w, const T* __restrict__ emb, const int* __restrict__ enc_off,
                                   const int* __restrict__ cap, int lanes) {
  const int l = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (l >= lanes) return;
  const long long L = lanes;
  for (int j = lane; j < TB_PRED; j += 32) {
    w.h[l * TB_PRED + j] = 0.f;
    w.h[(L + l) * TB_PRED + j] = 0.f;
    w.c[l * TB_PRED + j] = 0.f;
    w.c[(L + l) * TB_PRED + j] = 0.f;
  }
  T* x0 = reinterpret_cast<T*>(w.x0) + (long long)l * 2 * TB_PRED;
  T* x1 = reinterpret_cast<T*>(w.x1) + (long long)l * 2 * TB_PRED;
  for (int j = lane; j < TB_PRED; j += 32) {
    x0[j] = emb[(long long)TB_BLANK * TB_PRED + j];
    x0[TB_PRED + j] = from_f<T>(0.f);
    x1[TB_PRED + j] = from_f<T>(0.f);
  }
  if (lane == 0) {
    const int valid = enc_off[l + 1] - enc_off[l];
    w.frame[l] = 0;
    w.it[l] = 0;
    w.count[l] = 0;
    w.done[l] = (valid <= 0 || cap[l] <= 0) ? 1 : 0;
    w.mask[l] = 1;
  }
}

// z = relu(enc[frame] + dec) for running lanes; clears the argmax keys.
template <typename T>
__global__ void decode_prep_kernel(DecodeWs w, const float* __restrict__ enc, const int* __restrict__ enc_off,
                                   int lanes) {
  const int l = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (l >= lanes || l >= w.m_cur[0]) return;
  T* z = reinterpret_cast<T*>(w.z) + (long long)l * TB_PRED;
  if (lane == 0) w.keys[l] = 0ull, w.keys2[l] = 0ull;
  if (w.done[l]) return;
  const float* er = enc + (long long)(enc_off[l] + w.frame[l]) * TB_PRED;
  const float* dr = w.dec + (long long)l * TB_PRED;
  for (int j = lane * 4; j < TB_PRED; j += 128) {
    float4 a = load4(er + j), b = load4(dr + j);
    store4(z + j, fmaxf(a.x + b.x, 0.f), fmaxf(a.y + b.y, 0.f), fmaxf(a.z + b.z, 0.f), fmaxf(a.w + b.w, 0.f));
  }
}

// The loop body for each lane, then the LSTM inputs of lanes that step.
template <typename T>
__global__ void decode_step_kernel(DecodeWs w, const T* __restrict__ emb, const int* __restrict__ enc_off,
                                   const int* __restrict__ cap, int lanes, int max_cap, int* __restrict__ tokens) {
  const int l = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (l >= lanes || l >= w.m_cur[0]) return;  // lanes past the bound finished before this chunk
  int step = 0, tok = 0;
  if (lane == 0) {
    if (!w.done[l]) {
      tok = argmax_index(w.keys[l]);
      int d = argmax_index(w.keys2[l]);  // durations are 0, 1, 2, 3, 4
      // The joint always sets both keys; an index out of range can only come from a
      // key the joint never wrote, and is read as a blank of duration 1.
      if (tok < 0 || tok >= TB_VOCAB) tok = TB_BLANK;
      if (d < 0 || d >= TB_DURATIONS) d = 1;
      const int valid = enc_off[l + 1] - enc_off[l];
      int frame = w.frame[l], it = w.it[l] + 1, done = 0;
      if (tok == TB_BLANK) {
        frame += d > 1 ? d : 1;
      } else {
        const int n = w.count[l];
        if (n < max_cap) tokens[(long long)l * max_cap + n] = tok;
        w.count[l] = n + 1;
        if (tok == TB_EOS) {
          done = 1;
        } else {
          step = 1;
          frame += d;
        }
      }
      if (it >= cap[l] || frame >= valid) done = 1;
      if (done) step = 0;
      w.frame[l] = frame;
      w.it[l] = it;
      w.done[l] = done;
      if (!done) atomicAdd(w.active, 1);
    }
    w.mask[l] = step;
  }
  step = __shfl_sync(0xffffffffu, step, 0);
  tok = __shfl_sync(0xffffffffu, tok, 0);
  if (!step) return;
  const long long L = lanes;
  T* __restrict__ x0 = reinterpret_cast<T*>(w.x0) + (long long)l * 2 * TB_PRED;
  T* __restrict__ x1 = reinterpret_cast<T*>(w.x1) + (long long)l * 2 * TB_PRED;
  const T* __restrict__ er = emb + (long long)tok * TB_PRED;
  const float* __restrict__ h0 = w.h + (long long)l * TB_PRED;
  const float* __restrict__ h1 = w.h + (L + l) * TB_PRED;
  // 640 = 5 x 32 lanes x 4 values; all loads first, then the stores.
  float4 e4[5], a4[5], b4[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int j = (i * 32 + lane) * 4;
    e4[i] = load4(er + j);
    a4[i] = load4(h0 + j);
    b4[i] = load4(h1 + j);
  }
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    const int j = (i * 32 + lane) * 4;
    store4(x0 + j, e4[i].x, e4[i].y, e4[i].z, e4[i].w);
    store4(x0 + TB_PRED + j, a4[i].x, a4[i].y, a4[i].z, a4[i].w);
    store4(x1 + TB_PRED + j, b4[i].x, b4[i].y, b4[i].z, b4[i].w);
  }
}

// Ends a chunk of iterations: publishes (lanes still running, summed over the chunk's
// iterations; chunk number) to pinned host memory when asked, resets the count and
// moves the GEMMs' row bound to the next chunk's.
__global__ void decode_chunk_end_kernel(int* active, int* m_cur, const int* m_chunk, int chunks,
                                        volatile int* host_flag) {
  const int chunk = m_cur[1];
  if (host_flag) {
    host_flag[0] = active[0];
    __threadfence_system();
    host_flag[1] = chunk;
  }
  active[0] = 0;
  m_cur[0] = chunk + 1 < chunks ? m_chunk[chunk + 1] : 0;
  m_cur[1] = chunk + 1;
}

// A non-blocking stream per thread and device, used only to record graphs.
static cudaStream_t capture_stream() {
  static thread_local cudaStream_t streams[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!streams[dev] && cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking) != cudaSuccess)
    return nullptr;
  return streams[dev];
}

template <typename T>
static int decode_impl(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                       int* tokens, int* counts, void* ws, int* host_flag, int* err, cudaStream_t stream) {
  const int dt = m.dtype;
  DecodeWs w = carve(ws, dt, lanes);
  const T* emb = reinterpret_cast<const T*>(m.embedding);
  const int lane_blocks = (lanes + 7) / 8;
  const long long L = lanes;

  // Row bound per chunk: lane l runs iterations [0, cap[l]), so it can run in chunk c
  // only if 32c < cap[l]. With lanes ordered by length the bound shrinks as clips finish
  // and the GEMMs stop computing finished lanes.
  const int chunks = (max_cap + DECODE_CHUNK - 1) / DECODE_CHUNK;
  if (chunks > DECODE_MAX_CHUNKS) return TB_ERR_ARG;
  std::vector<int> caps(lanes), bound(chunks, 0);
  if (cudaMemcpyAsync(caps.data(), cap, (size_t)lanes * sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return fail_cuda();
  for (int l = 0; l < lanes; ++l) {
    const int last = std::min(chunks, (std::max(caps[l], 0) + DECODE_CHUNK - 1) / DECODE_CHUNK);
    for (int c = 0; c < last; ++c) bound[c] = l + 1;
  }
  const int head[2] = {bound[0], 0};
  if (cudaMemcpyAsync(w.m_chunk, bound.data(), (size_t)chunks * sizeof(int), cudaMemcpyHostToDevice, stream) !=
          cudaSuccess ||
      cudaMemcpyAsync(w.m_cur, head, sizeof(head), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return fail_cuda();

  tb_epilogue l0 = {};
  l0.kind = TB_EPI_LSTM;
  l0.out_dtype = dt;
  l0.bias = m.lstm_b[0];
  l0.c = w.c;
  l0.h = w.h;
  l0.mask = w.mask;
  l0.rows = w.m_cur;
  l0.out = w.x1;  // h0 -> first half of layer 1's input
  l0.ldo = 2 * TB_PRED;
  tb_epilogue l1 = l0;
  l1.bias = m.lstm_b[1];
  l1.c = w.c + L * TB_PRED;
  l1.h = w.h + L * TB_PRED;
  l1.out = w.hp;  // h1 -> the projector's input
  l1.ldo = TB_PRED;
  tb_epilogue pj = {};
  pj.kind = TB_EPI_STORE;
  pj.out_dtype = TB_F32;
  pj.out = w.dec;
  pj.ldo = TB_PRED;
  pj.bias = m.dec_proj_b;
  pj.rows = w.m_cur;
  tb_epilogue jt = {};
  jt.rows = w.m_cur;
  jt.kind = TB_EPI_ARGMAX;
  jt.bias = m.joint_b;
  jt.keys = w.keys;
  jt.keys2 = w.keys2;
  jt.split = TB_TOKEN_ROWS;
  jt.split_end = TB_TOKEN_ROWS + TB_DURATIONS;

  auto lstm_and_proj = [&](cudaStream_t s) -> int {
    if (int rc = gemm(dt, w.x0, 2 * TB_PRED, m.lstm_w[0], lanes, 4 * TB_PRED, 2 * TB_PRED, l0, err, s)) return rc;
    if (int rc = gemm(dt, w.x1, 2 * TB_PRED, m.lstm_w[1], lanes, 4 * TB_PRED, 2 * TB_PRED, l1, err, s)) return rc;
    return gemm(dt, w.hp, TB_PRED, m.dec_proj_w, lanes, TB_PRED, TB_PRED, pj, err, s);
  };

  if (cudaMemsetAsync(tokens, 0xff, (size_t)lanes * max_cap * sizeof(int), stream) != cudaSuccess) return fail_cuda();
  if (cudaMemsetAsync(w.active, 0, 2 * sizeof(int), stream) != cudaSuccess) return fail_cuda();
  decode_init_kernel<T><<<lane_blocks, 256, 0, stream>>>(w, emb, enc_off, cap, lanes);
  if (int rc = check_launch()) return rc;
  if (int rc = lstm_and_proj(stream)) return rc;

  auto iteration = [&](cudaStream_t s) -> int {
    decode_prep_kernel<T><<<lane_blocks, 256, 0, s>>>(w, enc, enc_off, lanes);
    if (int rc = check_launch()) return rc;
    if (int rc = gemm(dt, w.z, TB_PRED, m.joint_w, lanes, TB_JOINT_ROWS, TB_PRED, jt, err, s)) return rc;
    decode_step_kernel<T><<<lane_blocks, 256, 0, s>>>(w, emb, enc_off, cap, lanes, max_cap, tokens);
    if (int rc = check_launch()) return rc;
    return lstm_and_proj(s);
  };

  // Early exit: the device publishes per chunk into pinned host memory.
  int* flag_dev = nullptr;
  if (host_flag && cudaHostGetDevicePointer(reinterpret_cast<void**>(&flag_dev), host_flag, 0) != cudaSuccess) {
    cudaGetLastError();
    flag_dev = nullptr;  // not mapped: run every chunk
  }

  // Every iteration launches the same kernels on the same buffers (the loop state is
  // in device memory), so one chunk of iterations is captured once and replayed on the
  // caller's stream. Capture runs nothing, so it uses a stream of its own: the
  // caller's may be the legacy default stream, which cannot be captured.
  constexpr int AHEAD = 3;
  const cudaStream_t cap_stream = capture_stream();
  if (!cap_stream) return fail_cuda();
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  const long long launches_before = launch_count();
  if (cudaStreamBeginCapture(cap_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return fail_cuda();
  int rc = TB_OK;
  for (int i = 0; i < DECODE_CHUNK && rc == TB_OK; ++i) rc = iteration(cap_stream);
  if (rc == TB_OK) {
    decode_chunk_end_kernel<<<1, 1, 0, cap_stream>>>(w.active, w.m_cur, w.m_chunk, chunks, flag_dev);
    rc = check_launch();
  }
  const cudaError_t captured = cudaStreamEndCapture(cap_stream, &graph);
  count_launches(launches_before - launch_count());  // recorded, not run
  if (rc != TB_OK || captured != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    return rc != TB_OK ? rc : fail_cuda();
  }
  if (cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
    cudaGraphDestroy(graph);
    return fail_cuda();
  }
  size_t nodes = 0;
  cudaGraphGetNodes(graph, nullptr, &nodes);
  if (flag_dev) host_flag[0] = 1, host_flag[1] = -1;
  for (int c = 0; c < chunks && rc == TB_OK; ++c) {
    if (flag_dev) {
      // Stay at most AHEAD chunks ahead of the device; stop once a finished chunk
      // reports that no lane was running.
      const auto start = std::chrono::steady_clock::now();
      bool stop = false;
      while (true) {
        volatile int* hf = host_flag;
        const int seen = hf[1];
        if (seen >= 0 && hf[0] == 0) {
          stop = true;
          break;
        }
        if (seen >= c - AHEAD) break;
        if (std::chrono::steady_clock::now() - start > std::chrono::seconds(60)) {
          rc = TB_ERR_CUDA;
          break;
        }
        std::this_thread::yield();
      }
      if (stop || rc != TB_OK) break;
    }
    if (cudaGraphLaunch(exec, stream) != cudaSuccess) rc = fail_cuda();
    count_launches((long long)nodes);
  }
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  if (rc != TB_OK) return rc;
  if (cudaMemcpyAsync(counts, w.count, (size_t)lanes * sizeof(int), cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
    return fail_cuda();
  return TB_OK;
}

int tdt_decode(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
               int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err, cudaStream_t stream) {
  if (lanes <= 0) return TB_OK;
  if (!enc || !enc_off || !cap || !tokens || !counts || !ws || max_cap <= 0) return TB_ERR_ARG;
  if (ws_bytes < decode_ws(m.dtype, lanes)) return TB_ERR_WORKSPACE;
  if (m.dtype == TB_BF16)
    return decode_impl<__nv_bfloat16>(m, enc, enc_off, cap, lanes, max_cap, tokens, counts, ws, host_flag, err, stream);
  if (m.dtype == TB_F32)
    return decode_impl<float>(m, enc, enc_off, cap, lanes, max_cap, tokens, counts, ws, host_flag, err, stream);
  return TB_ERR_ARG;
}

}  // namespace tb
