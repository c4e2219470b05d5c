// Lane state of the TDT greedy decoder and the per-lane loop body, shared by the
// graph-replayed decoder (decode.cu: one kernel per GEMM, used for fp32) and the
// persistent tcgen05 decoder (decode_tc.cu: bf16). The loop body follows
// tinybark/tinygrad/model.py:218-233.
#pragma once
#include "epilogue.cuh"
#include "host.h"

namespace tb {

constexpr int DECODE_CHUNK = 32;         // iterations per captured graph
constexpr int DECODE_MAX_CHUNKS = 8192;  // so max_cap <= 262144
constexpr int DECODE_MAX_GROUPS = 8;     // lane groups decoded concurrently
constexpr int DECODE_MAX_ITERS = DECODE_MAX_CHUNKS * DECODE_CHUNK;

struct DecodeWs {
  unsigned long long *keys, *keys2;
  void *z, *x0, *x1, *hp;
  float *c, *dec;  // LSTM cell state [2][lanes][640]; projector output
  float* pre0;     // persistent decoder: [lanes][2560] W_hh0 . h0 + b0 for the next step
  int *frame, *it, *done, *mask, *count, *active;
  int* erow;     // [lanes]: encoder row the joint reads next (enc_off + frame), -1 once done
  int* m_chunk;  // [DECODE_MAX_CHUNKS]: only lanes below this index can run in chunk c
  int* bounds;   // [DECODE_MAX_ITERS + 1]: persistent decoder, [0] = lanes, [i + 1] = 1 + the
                 // last lane still running after iteration i (written once, never reused)
  int* m_cur;    // [64]: the graph decoder's chunk bound ([0]) and chunk ([1]); the
                 // persistent decoder's grid barrier ([8]: arrivals, [9]: abort)
};

inline DecodeWs carve(void* ws, int dtype, int lanes) {
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
  w.c = (float*)take(2 * L * TB_PRED * 4);
  w.dec = (float*)take(L * TB_PRED * 4);
  w.pre0 = (float*)take(L * 4 * TB_PRED * 4);
  w.frame = (int*)take(L * 4);
  w.it = (int*)take(L * 4);
  w.done = (int*)take(L * 4);
  w.mask = (int*)take(L * 4);
  w.count = (int*)take(L * 4);
  w.active = (int*)take(256);
  w.erow = (int*)take(L * 4);
  w.m_chunk = (int*)take(DECODE_MAX_CHUNKS * 4);
  w.bounds = (int*)take((DECODE_MAX_ITERS + 1) * 4);
  w.m_cur = (int*)take(256);
  return w;
}

inline size_t decode_ws(int dtype, int lanes) {
  uint8_t* base = nullptr;
  DecodeWs w = carve(base, dtype, lanes);
  return (size_t)(reinterpret_cast<uint8_t*>(w.m_cur) - base) + 256;
}

// Lane l's state before the first step (token blank, zero LSTM state) and the inputs of
// the first prediction step. One warp per lane.
template <typename T>
__device__ __forceinline__ void lane_init(const DecodeWs& w, const T* __restrict__ emb, const int* __restrict__ enc_off,
                                          const int* __restrict__ cap, int l, int lanes, int lane) {
  const long long L = lanes;
  for (int j = lane; j < TB_PRED; j += 32) {
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
    const int done = (valid <= 0 || cap[l] <= 0) ? 1 : 0;
    w.frame[l] = 0;
    w.it[l] = 0;
    w.count[l] = 0;
    w.done[l] = done;
    w.mask[l] = 1;
    w.keys[l] = 0ull;
    w.keys2[l] = 0ull;
    w.erow[l] = done ? -1 : enc_off[l];
  }
}

// One iteration of the greedy loop for lane l, run by one thread: reads the joint's argmax
// keys (and clears them for the next joint), then blank -> frame += max(d, 1); otherwise
// emit, stop on EOS, else frame += d and the LSTM steps on the token; the lane stops when
// frame >= valid or after cap[l] iterations. Returns whether lane l still runs; sets
// `step` (the LSTM steps) and `tok`. counts_out (if not NULL) receives the lane's token
// count when it stops.
__device__ __forceinline__ bool lane_scalar(const DecodeWs& w, const int* __restrict__ enc_off,
                                            const int* __restrict__ cap, int l, int max_cap,
                                            int* __restrict__ tokens, int& step, int& tok,
                                            int* __restrict__ counts_out) {
  step = 0;
  tok = 0;
  int running = 0;
  // Every scalar the step needs, loaded at once (one memory round trip), then used.
  const int was_done = w.done[l];
  const unsigned long long k1 = w.keys[l], k2 = w.keys2[l];
  const int frame0 = w.frame[l], it0 = w.it[l], n0 = w.count[l], cap_l = cap[l];
  const int off0 = enc_off[l], off1 = enc_off[l + 1];
  if (!was_done) {
    tok = argmax_index(k1);
    int d = argmax_index(k2);  // durations are 0, 1, 2, 3, 4
    w.keys[l] = 0ull;  // cleared for the next joint
    w.keys2[l] = 0ull;
    // The joint always sets both keys; an index out of range can only come from a
    // key the joint never wrote, and is read as a blank of duration 1.
    if (tok < 0 || tok >= TB_VOCAB) tok = TB_BLANK;
    if (d < 0 || d >= TB_DURATIONS) d = 1;
    const int valid = off1 - off0;
    int frame = frame0, it = it0 + 1, done = 0, n = n0;
    if (tok == TB_BLANK) {
      frame += d > 1 ? d : 1;
    } else {
      if (n0 < max_cap) tokens[(long long)l * max_cap + n0] = tok;
      n = n0 + 1;
      w.count[l] = n;
      if (tok == TB_EOS) {
        done = 1;
      } else {
        step = 1;
        frame += d;
      }
    }
    if (it >= cap_l || frame >= valid) done = 1;
    if (done) step = 0;
    if (done && counts_out) counts_out[l] = n;
    w.frame[l] = frame;
    w.it[l] = it;
    w.done[l] = done;
    w.erow[l] = done ? -1 : off0 + frame;
    running = !done;
  }
  w.mask[l] = step;
  return running != 0;
}

// lane_scalar for lane l on one warp (lane 0 does the work); the results on every lane.
__device__ __forceinline__ bool lane_scalar_step(const DecodeWs& w, const int* __restrict__ enc_off,
                                                 const int* __restrict__ cap, int l, int max_cap,
                                                 int* __restrict__ tokens, int lane, int& step_out, int& tok_out,
                                                 int* __restrict__ counts_out = nullptr) {
  int step = 0, tok = 0, running = 0;
  if (lane == 0) running = lane_scalar(w, enc_off, cap, l, max_cap, tokens, step, tok, counts_out) ? 1 : 0;
  step_out = __shfl_sync(0xffffffffu, step, 0);
  tok_out = __shfl_sync(0xffffffffu, tok, 0);
  return __shfl_sync(0xffffffffu, running, 0) != 0;
}

// The loop body (lane_scalar_step) and, for a lane that steps, its LSTM inputs
// [embedding(token) | h0] and [. | h1] assembled from the hidden states the LSTM
// epilogues last wrote for it: h0 in x1[:, :640], h1 in hp. Returns whether lane l
// still runs.
template <typename T>
__device__ __forceinline__ bool lane_step(const DecodeWs& w, const T* __restrict__ emb,
                                          const int* __restrict__ enc_off, const int* __restrict__ cap, int l,
                                          int lanes, int max_cap, int* __restrict__ tokens, int lane) {
  int step, tok;
  const bool running = lane_scalar_step(w, enc_off, cap, l, max_cap, tokens, lane, step, tok);
  if (!step) return running;
  T* __restrict__ x0 = reinterpret_cast<T*>(w.x0) + (long long)l * 2 * TB_PRED;
  T* __restrict__ x1 = reinterpret_cast<T*>(w.x1) + (long long)l * 2 * TB_PRED;
  const T* __restrict__ er = emb + (long long)tok * TB_PRED;
  const T* __restrict__ h0 = x1;
  const T* __restrict__ h1 = reinterpret_cast<const T*>(w.hp) + (long long)l * TB_PRED;
  (void)lanes;
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
  return running;
}

}  // namespace tb
