// TDT greedy decoding for a batch of clips, one lane per clip, all lanes stepped
// together. Replaces the prediction network step, joint and greedy loop of
// tinybark/tinygrad/model.py:162-233 (= tinybark/ort/__init__.py:55-86,
// tinybark/mojo/bark/model.mojo:250-318), which run one clip and one host round trip
// per emitted token.
//
// Per iteration, for every lane still running:
//   joint: argmax over 8193 token logits and 5 duration logits of z (GEMM, ARGMAX epilogue)
//   step:  the loop body of the reference: blank -> frame += max(d, 1); otherwise emit,
//          stop on EOS, else frame += d and the LSTM steps on the token; stop when
//          frame >= valid or after `cap` iterations
//   lstm0, lstm1: gates GEMM with the LSTM cell fused into the epilogue (masked lanes
//          keep their state)
//   proj:  dec = h1 W_p^T + b_p, and in the same epilogue the next joint input
//          z = relu(enc[frame] + dec)
// The LSTM inputs [embedding(token) | h] are assembled from the fp32 state by the step
// kernel, so no GEMM reads a buffer that its own epilogue writes.
#include <algorithm>
#include <chrono>
#include <thread>
#include <vector>

#include "decode.cuh"

namespace tb {

// Lane state initialisation and the inputs of the first step (token blank, zero state).
template <typename T>
__global__ void decode_init_kernel(DecodeWs w, const T* __restrict__ emb, const int* __restrict__ enc_off,
                                   const int* __restrict__ cap, int lanes) {
  grid_dep_wait();
  grid_dep_launch();
  const int l = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (l >= lanes) return;
  lane_init<T>(w, emb, enc_off, cap, l, lanes, lane);
}

// The loop body for each lane, then the LSTM inputs of lanes that step.
template <typename T>
__global__ void decode_step_kernel(DecodeWs w, const T* __restrict__ emb, const int* __restrict__ enc_off,
                                   const int* __restrict__ cap, int lanes, int max_cap, int* __restrict__ tokens) {
  grid_dep_wait();
  grid_dep_launch();
  const int l = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (l >= lanes || l >= w.m_cur[0]) return;  // lanes past the bound finished before this chunk
  if (lane_step<T>(w, emb, enc_off, cap, l, lanes, max_cap, tokens, lane) && lane == 0) atomicAdd(w.active, 1);
}

// Ends a chunk of iterations: publishes (lanes still running, summed over the chunk's
// iterations; chunk number) to pinned host memory when asked, resets the count and
// moves the GEMMs' row bound to the next chunk's.
__global__ void decode_chunk_end_kernel(int* active, int* m_cur, const int* m_chunk, int chunks,
                                        volatile int* host_flag) {
  grid_dep_wait();
  grid_dep_launch();
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

// Streams and events the decoder owns on each device: one to record graphs on (capture
// runs nothing, and the caller's stream may be the legacy default stream, which cannot
// be captured) and one per extra lane group, with fork/join events.
struct DecodeStreams {
  cudaStream_t capture = nullptr;
  cudaStream_t group[DECODE_MAX_GROUPS] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[DECODE_MAX_GROUPS] = {};
};

static DecodeStreams* decode_streams() {
  static thread_local DecodeStreams per_device[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  DecodeStreams& d = per_device[dev];
  if (!d.capture) {
    if (cudaStreamCreateWithFlags(&d.capture, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    for (int g = 1; g < DECODE_MAX_GROUPS; ++g)
      if (cudaStreamCreateWithFlags(&d.group[g], cudaStreamNonBlocking) != cudaSuccess ||
          cudaEventCreateWithFlags(&d.join[g], cudaEventDisableTiming) != cudaSuccess)
        return nullptr;
    if (cudaEventCreateWithFlags(&d.fork, cudaEventDisableTiming) != cudaSuccess) return nullptr;
  }
  return &d;
}

struct SmBudget {  // GEMMs of concurrent groups each plan for a share of the SMs
  explicit SmBudget(int n) { set_sm_budget(n); }
  ~SmBudget() { set_sm_budget(0); }
};

// Lane group g of `groups`: lanes [group_first(g), group_first(g) + group_size(g)).
// Sizes follow a round-robin deal of `lanes` lanes, so a caller that deals its clips
// (longest first) round-robin and lays the groups out one after another gets balanced
// groups, each still ordered longest first.
static int group_size(int lanes, int groups, int g) { return (lanes - g + groups - 1) / groups; }
static int group_first(int lanes, int groups, int g) {
  int first = 0;
  for (int i = 0; i < g; ++i) first += group_size(lanes, groups, i);
  return first;
}

size_t decode_ws_groups(int dtype, int lanes, int groups) {
  size_t total = 0;
  for (int g = 0; g < groups; ++g) total += align256(decode_ws(dtype, group_size(lanes, groups, g)));
  return total;
}

struct DecodeGroup {
  int first = 0, lanes = 0, chunks = 0;
  DecodeWs w;
  cudaStream_t stream = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  size_t nodes = 0;
  int* flag = nullptr;      // host view of this group's two progress ints
  int* flag_dev = nullptr;  // device view, or NULL
  bool finished = false;
};

template <typename T>
static int decode_impl(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                       int groups, int* tokens, int* counts, void* ws, int* host_flag, int* err,
                       cudaStream_t stream) {
  const int dt = m.dtype;
  const T* emb = reinterpret_cast<const T*>(m.embedding);
  const int max_chunks = (max_cap + DECODE_CHUNK - 1) / DECODE_CHUNK;
  if (max_chunks > DECODE_MAX_CHUNKS) return TB_ERR_ARG;
  DecodeStreams* ds = decode_streams();
  if (!ds) return fail_cuda();
  const SmBudget budget(std::max(1, sm_count() / groups));

  // Every lane's cap, to bound each chunk's GEMMs to the lanes that can still run.
  std::vector<int> caps(lanes);
  if (cudaMemcpyAsync(caps.data(), cap, (size_t)lanes * sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return fail_cuda();

  int* flag_dev = nullptr;
  if (host_flag && cudaHostGetDevicePointer(reinterpret_cast<void**>(&flag_dev), host_flag, 0) != cudaSuccess) {
    cudaGetLastError();
    flag_dev = nullptr;  // not mapped: every chunk runs
  }

  std::vector<DecodeGroup> gs(groups);
  std::vector<std::vector<int>> bounds(groups);
  uint8_t* wp = reinterpret_cast<uint8_t*>(ws);
  for (int g = 0; g < groups; ++g) {
    DecodeGroup& G = gs[g];
    G.first = group_first(lanes, groups, g);
    G.lanes = group_size(lanes, groups, g);
    G.w = carve(wp, dt, G.lanes);
    wp += align256(decode_ws(dt, G.lanes));
    G.stream = g == 0 ? stream : ds->group[g];
    if (flag_dev) G.flag = host_flag + 2 * g, G.flag_dev = flag_dev + 2 * g;
    // Lane l runs iterations [0, cap[l]), so it can run in chunk c only if 32c < cap[l].
    std::vector<int>& bound = bounds[g];
    bound.assign(max_chunks, 0);
    for (int l = 0; l < G.lanes; ++l) {
      const int last = std::min(max_chunks, (std::max(caps[G.first + l], 0) + DECODE_CHUNK - 1) / DECODE_CHUNK);
      for (int c = 0; c < last; ++c) bound[c] = l + 1;
    }
    G.chunks = 0;
    while (G.chunks < max_chunks && bound[G.chunks] > 0) ++G.chunks;
  }

  // The other groups' streams start after the work already queued on the caller's.
  if (cudaEventRecord(ds->fork, stream) != cudaSuccess) return fail_cuda();
  for (int g = 1; g < groups; ++g)
    if (cudaStreamWaitEvent(gs[g].stream, ds->fork, 0) != cudaSuccess) return fail_cuda();

  int rc = TB_OK;
  const long long launches_before = launch_count();
  for (int g = 0; g < groups && rc == TB_OK; ++g) {
    DecodeGroup& G = gs[g];
    DecodeWs& w = G.w;
    const int* g_off = enc_off + G.first;
    const int* g_cap = cap + G.first;
    int* g_tokens = tokens + (long long)G.first * max_cap;
    const int L = G.lanes, lane_blocks = (L + 7) / 8;

    tb_epilogue l0 = {};
    l0.kind = TB_EPI_LSTM;
    l0.out_dtype = dt;
    l0.bias = m.lstm_b[0];
    l0.c = w.c;
    l0.mask = w.mask;
    l0.rows = w.m_cur;
    l0.out = w.x1;  // h0 -> first half of layer 1's input
    l0.ldo = 2 * TB_PRED;
    tb_epilogue l1 = l0;
    l1.bias = m.lstm_b[1];
    l1.c = w.c + (long long)L * TB_PRED;
    l1.out = w.hp;  // h1 -> the projector's input
    l1.ldo = TB_PRED;
    tb_epilogue pj = {};  // dec, and the next joint input z = relu(enc[frame] + dec)
    pj.kind = TB_EPI_JOINT_IN;
    pj.out_dtype = dt;
    pj.out = w.dec;
    pj.ldo = TB_PRED;
    pj.out2 = w.z;
    pj.ldo2 = TB_PRED;
    pj.bias = m.dec_proj_b;
    pj.gather = enc;
    pj.gather_row = w.erow;
    pj.rows = w.m_cur;
    tb_epilogue jt = {};
    jt.kind = TB_EPI_ARGMAX;
    jt.bias = m.joint_b;
    jt.keys = w.keys;
    jt.keys2 = w.keys2;
    jt.split = TB_TOKEN_ROWS;
    jt.split_end = TB_TOKEN_ROWS + TB_DURATIONS;
    jt.rows = w.m_cur;

    auto lstm_and_proj = [&](cudaStream_t s) -> int {
      if (int r = gemm(dt, w.x0, 2 * TB_PRED, m.lstm_w[0], L, 4 * TB_PRED, 2 * TB_PRED, l0, err, s)) return r;
      if (int r = gemm(dt, w.x1, 2 * TB_PRED, m.lstm_w[1], L, 4 * TB_PRED, 2 * TB_PRED, l1, err, s)) return r;
      return gemm(dt, w.hp, TB_PRED, m.dec_proj_w, L, TB_PRED, TB_PRED, pj, err, s);
    };
    auto iteration = [&](cudaStream_t s) -> int {
      if (int r = gemm(dt, w.z, TB_PRED, m.joint_w, L, TB_JOINT_ROWS, TB_PRED, jt, err, s)) return r;
      if (int r = launch_pdl(decode_step_kernel<T>, lane_blocks, 256, 0, s, w, emb, g_off, g_cap, L, max_cap,
                             g_tokens))
        return r;
      return lstm_and_proj(s);
    };

    // Set-up on the group's stream: bounds, lane state, the first prediction step.
    const int head[2] = {bounds[g][0], 0};
    if (cudaMemsetAsync(g_tokens, 0xff, (size_t)L * max_cap * sizeof(int), G.stream) != cudaSuccess ||
        cudaMemsetAsync(w.active, 0, sizeof(int), G.stream) != cudaSuccess ||
        cudaMemcpyAsync(w.m_chunk, bounds[g].data(), (size_t)max_chunks * sizeof(int), cudaMemcpyHostToDevice,
                        G.stream) != cudaSuccess ||
        cudaMemcpyAsync(w.m_cur, head, sizeof(head), cudaMemcpyHostToDevice, G.stream) != cudaSuccess ||
        cudaStreamSynchronize(G.stream) != cudaSuccess) {
      rc = fail_cuda();
      break;
    }
    if ((rc = launch_pdl(decode_init_kernel<T>, lane_blocks, 256, 0, G.stream, w, emb, g_off, g_cap, L))) break;
    if ((rc = lstm_and_proj(G.stream))) break;

    // Every iteration launches the same kernels on the same buffers (the loop state is
    // in device memory), so one chunk of iterations is captured once and replayed.
    const long long before_capture = launch_count();
    if (cudaStreamBeginCapture(ds->capture, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
      rc = fail_cuda();
      break;
    }
    for (int i = 0; i < DECODE_CHUNK && rc == TB_OK; ++i) rc = iteration(ds->capture);
    if (rc == TB_OK)
      rc = launch_pdl(decode_chunk_end_kernel, 1, 1, 0, ds->capture, w.active, w.m_cur, w.m_chunk, max_chunks,
                      G.flag_dev);
    const cudaError_t captured = cudaStreamEndCapture(ds->capture, &G.graph);
    count_launches(before_capture - launch_count());  // recorded, not run
    if (rc == TB_OK && captured != cudaSuccess) rc = fail_cuda();
    if (rc == TB_OK && cudaGraphInstantiate(&G.exec, G.graph, 0) != cudaSuccess) rc = fail_cuda();
    if (rc == TB_OK) cudaGraphGetNodes(G.graph, nullptr, &G.nodes);
    if (G.flag) G.flag[0] = 1, G.flag[1] = -1;
  }
  (void)launches_before;

  // Chunks of all groups, interleaved so the groups' kernels overlap on the GPU. A group
  // stays at most AHEAD chunks ahead of its progress on the device and stops once a
  // finished chunk reports that none of its lanes was running.
  constexpr int AHEAD = 3;
  for (int c = 0; c < max_chunks && rc == TB_OK; ++c) {
    for (int g = 0; g < groups && rc == TB_OK; ++g) {
      DecodeGroup& G = gs[g];
      if (G.finished || c >= G.chunks) continue;
      if (G.flag) {
        const auto start = std::chrono::steady_clock::now();
        while (true) {
          volatile int* hf = G.flag;
          const int seen = hf[1];
          if (seen >= 0 && hf[0] == 0) {
            G.finished = true;
            break;
          }
          if (seen >= c - AHEAD) break;
          if (std::chrono::steady_clock::now() - start > std::chrono::seconds(60)) {
            rc = TB_ERR_CUDA;
            break;
          }
          std::this_thread::yield();
        }
        if (G.finished || rc != TB_OK) continue;
      }
      if (cudaGraphLaunch(G.exec, G.stream) != cudaSuccess) rc = fail_cuda();
      count_launches((long long)G.nodes);
    }
  }

  for (int g = 0; g < groups; ++g) {
    DecodeGroup& G = gs[g];
    if (G.lanes > 0 && rc == TB_OK &&
        cudaMemcpyAsync(counts + G.first, G.w.count, (size_t)G.lanes * sizeof(int), cudaMemcpyDeviceToDevice,
                        G.stream) != cudaSuccess)
      rc = fail_cuda();
    // The caller's stream waits for every group, also after a failure.
    if (g > 0 && (cudaEventRecord(ds->join[g], G.stream) != cudaSuccess ||
                  cudaStreamWaitEvent(stream, ds->join[g], 0) != cudaSuccess) && rc == TB_OK)
      rc = fail_cuda();
    if (G.exec) cudaGraphExecDestroy(G.exec);
    if (G.graph) cudaGraphDestroy(G.graph);
  }
  return rc;
}

int tdt_decode_tc(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                  int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err, cudaStream_t stream);

int tdt_decode(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
               int groups, int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err,
               cudaStream_t stream) {
  if (lanes <= 0) return TB_OK;
  if (!enc || !enc_off || !cap || !tokens || !counts || !ws || max_cap <= 0) return TB_ERR_ARG;
  if (groups <= 0 && m.dtype == TB_BF16)
    return tdt_decode_tc(m, enc, enc_off, cap, lanes, max_cap, tokens, counts, ws, ws_bytes, host_flag, err,
                         stream);
  groups = std::max(1, std::min(std::min(groups, DECODE_MAX_GROUPS), lanes));
  if (ws_bytes < decode_ws_groups(m.dtype, lanes, groups)) return TB_ERR_WORKSPACE;
  if (m.dtype == TB_BF16)
    return decode_impl<__nv_bfloat16>(m, enc, enc_off, cap, lanes, max_cap, groups, tokens, counts, ws, host_flag,
                                      err, stream);
  if (m.dtype == TB_F32)
    return decode_impl<float>(m, enc, enc_off, cap, lanes, max_cap, groups, tokens, counts, ws, host_flag, err,
                              stream);
  return TB_ERR_ARG;
}

}  // namespace tb
