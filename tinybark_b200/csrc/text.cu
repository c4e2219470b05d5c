// Token rows to text bytes (tinybark/text.py:19-34, Tokenizer.decode with
// skip_special_tokens): each id's bytes come from a piece table (a SentencePiece piece with
// "▁" already a space, a byte-fallback piece <0xNN> as the byte NN, a special token as
// nothing), and a lane's text is its pieces' bytes joined. Decoded once as UTF-8 with
// invalid sequences replaced, "▁" turned into a space and stripped, that is the
// reference's text: it decodes each run of byte pieces on its own, but a run is always
// followed by a whole piece, whose first byte ends any sequence the run left open.
//
// Three small kernels: per-lane byte counts (one CTA per lane), a scan of those counts
// into offsets (one CTA), and the copy (one CTA per lane, each token's bytes at its
// prefix within the lane).
#include <cstdint>

#include "host.h"

namespace tb {
namespace {

constexpr int TEXT_THREADS = 128;
constexpr int SCAN_THREADS = 1024;

// Bytes of token `id`, or -1 if the id is outside the table.
__device__ __forceinline__ int piece_len(const int* __restrict__ piece_off, int vocab, int id) {
  if (id < 0 || id >= vocab) return -1;
  const int n = piece_off[id + 1] - piece_off[id];
  return n > 0 ? n : 0;
}

__device__ __forceinline__ int lane_tokens(const int* counts, int lane, int ld) {
  const int n = counts[lane];
  return n < 0 ? 0 : (n > ld ? ld : n);
}

template <int THREADS, typename T>
__device__ __forceinline__ T block_inclusive(T x, T* part, T& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) part[warp] = x;
  __syncthreads();
  T before = 0, sum = 0;
#pragma unroll
  for (int w = 0; w < THREADS / 32; ++w) {
    before += w < warp ? part[w] : T(0);
    sum += part[w];
  }
  __syncthreads();  // part is reused by the next call
  total = sum;
  return before + x;
}

__global__ void __launch_bounds__(TEXT_THREADS)
    text_len_kernel(const int* __restrict__ tokens, int ld, const int* __restrict__ counts,
                    const int* __restrict__ piece_off, int vocab, long long* __restrict__ text_off, int* err) {
  __shared__ long long part[TEXT_THREADS / 32];
  const int lane = blockIdx.x, n = lane_tokens(counts, lane, ld);
  const int* row = tokens + static_cast<long long>(lane) * ld;
  long long s = 0;
  bool bad = false;
  for (int t = threadIdx.x; t < n; t += TEXT_THREADS) {
    const int len = piece_len(piece_off, vocab, row[t]);
    bad |= len < 0;
    s += len > 0 ? len : 0;
  }
  long long total;
  block_inclusive<TEXT_THREADS>(s, part, total);
  if (threadIdx.x == 0) {
    text_off[lane + 1] = total;
    if (lane == 0) text_off[0] = 0;
  }
  if (bad && err) atomicOr(err, TB_DEV_TEXT_TOKEN);
}

// In place: text_off[1..lanes] from per-lane counts to running offsets.
__global__ void __launch_bounds__(SCAN_THREADS) text_scan_kernel(long long* __restrict__ text_off, int lanes) {
  __shared__ long long part[SCAN_THREADS / 32];
  long long carry = 0;
  for (int base = 0; base < lanes; base += SCAN_THREADS) {
    const int i = base + threadIdx.x;
    long long total;
    const long long x = block_inclusive<SCAN_THREADS>(i < lanes ? text_off[i + 1] : 0LL, part, total);
    if (i < lanes) text_off[i + 1] = carry + x;
    carry += total;
  }
}

__global__ void __launch_bounds__(TEXT_THREADS)
    text_bytes_kernel(const int* __restrict__ tokens, int ld, const int* __restrict__ counts,
                      const int* __restrict__ piece_off, const uint8_t* __restrict__ piece_bytes,
                      long long piece_bytes_len, int vocab, const long long* __restrict__ text_off,
                      uint8_t* __restrict__ text, long long text_bytes) {
  __shared__ int part[TEXT_THREADS / 32];
  const int lane = blockIdx.x, n = lane_tokens(counts, lane, ld);
  const int* row = tokens + static_cast<long long>(lane) * ld;
  long long at = text_off[lane];
  const long long end = text_off[lane + 1] < text_bytes ? text_off[lane + 1] : text_bytes;
  for (int base = 0; base < n; base += TEXT_THREADS) {  // n is the same for the whole CTA
    const int t = base + threadIdx.x;
    const int id = t < n ? row[t] : -1;
    int len = t < n ? piece_len(piece_off, vocab, id) : 0;
    len = len > 0 ? len : 0;
    int total;
    const long long o = at + block_inclusive<TEXT_THREADS>(len, part, total) - len;
    const long long src = len ? piece_off[id] : 0;
    for (int k = 0; k < len; ++k)
      if (o + k >= 0 && o + k < end && src + k >= 0 && src + k < piece_bytes_len) text[o + k] = piece_bytes[src + k];
    at += total;
  }
}

}  // namespace

int text_offsets(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off, int vocab,
                 long long* text_off, int* err, cudaStream_t stream) {
  if (lanes < 0 || ld < 0 || vocab <= 0 || !text_off || (lanes > 0 && (!tokens || !counts || !piece_off)))
    return TB_ERR_ARG;
  if (lanes == 0) return cudaMemsetAsync(text_off, 0, sizeof(long long), stream) == cudaSuccess ? TB_OK : fail_cuda();
  text_len_kernel<<<lanes, TEXT_THREADS, 0, stream>>>(tokens, ld, counts, piece_off, vocab, text_off, err);
  if (int s = check_launch()) return s;
  text_scan_kernel<<<1, SCAN_THREADS, 0, stream>>>(text_off, lanes);
  return check_launch();
}

int text_bytes(const int* tokens, int ld, const int* counts, int lanes, const int* piece_off,
               const uint8_t* piece_bytes, long long piece_bytes_len, int vocab, const long long* text_off,
               uint8_t* text, long long text_len, cudaStream_t stream) {
  if (lanes < 0 || ld < 0 || vocab <= 0 || piece_bytes_len < 0 || text_len < 0 ||
      (lanes > 0 && (!tokens || !counts || !piece_off || !text_off || (piece_bytes_len && !piece_bytes) ||
                     (text_len && !text))))
    return TB_ERR_ARG;
  if (lanes == 0 || text_len == 0) return TB_OK;
  text_bytes_kernel<<<lanes, TEXT_THREADS, 0, stream>>>(tokens, ld, counts, piece_off, piece_bytes, piece_bytes_len,
                                                        vocab, text_off, text, text_len);
  return check_launch();
}

}  // namespace tb
