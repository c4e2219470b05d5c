// Weight loading: tinybark keeps the converted weights as one fp16 safetensors file
// (tinybark/weights.py:92-120) and uploads its data block in one read, then splits it into
// one GPU buffer per tensor (tinybark/tinygrad/weights.py:10-26). Here the data block is
// uploaded as is and one kernel writes every tensor of the packed layout the kernels read,
// converting f16 (or f32) to the engine's type and applying the reorderings of that layout
// (gate interleaving, column permutations, slices) as strided reads, padding as fills.
//
// The work is HBM-bound element copying: the kernel walks chunks of TB_REPACK_CHUNK
// destination elements, each CTA finding its job by binary search over the jobs' first
// chunks; destination writes are contiguous, source reads follow the job's strides.
// A thread keeps several 16-byte loads in flight: with one 2-byte load per thread at a
// time, a full SM holds about 4 KB in flight, which caps the copy near 0.75 TB/s.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdint>
#include <vector>

#include "host.h"

namespace tb {
namespace {

constexpr int REPACK_THREADS = 256;
constexpr int REPACK_CTAS_PER_SM = 3;  // 80 registers a thread; 48 KB of loads in flight per SM
constexpr int REPACK_BATCH = 4;  // loads a thread issues before its stores

// The last job whose first chunk is at or below c: jobs without elements share their first
// chunk with the job after them, so they are never picked.
__device__ __forceinline__ int find_job(const tb_repack_job* __restrict__ jobs, int n, long long c) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (jobs[mid].first_chunk <= c)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

struct Job {
  const char* src;
  char* dst;
  long long s0, s1, s2, s3;
  int d1, d2, d3, n, fill, f16, bf16;
  float value;
  // Source element of destination element e.
  __device__ __forceinline__ long long at(int e) const {
    const int i3 = e % d3;
    e /= d3;
    const int i2 = e % d2;
    e /= d2;
    return (e / d1) * s0 + (e % d1) * s1 + i2 * s2 + i3 * s3;
  }
};

__device__ __forceinline__ void store1(const Job& j, int e, float v) {
  if (j.bf16)
    reinterpret_cast<__nv_bfloat16*>(j.dst)[e] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(j.dst)[e] = v;
}

// Eight converted values to destination elements e..e+7 (16- or 32-byte aligned).
template <bool BF16>
__device__ __forceinline__ void store8(char* dst, int e, const float (&v)[8]) {
  if constexpr (BF16) {
    uint4 raw;
    __nv_bfloat162* b = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) b[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + e) = raw;
  } else {
    float* d = reinterpret_cast<float*>(dst) + e;
    *reinterpret_cast<float4*>(d) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(d + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// Groups of 8 elements with 16-byte accesses. The loads of a batch are issued before its
// stores and held raw (4 registers per f16 group), converted only when stored.
template <bool F16, bool BF16>
__device__ __forceinline__ void copy_groups(const Job& j, int e0, int e1) {
  constexpr int STEP = REPACK_THREADS * 8;
  constexpr int BATCH = F16 ? REPACK_BATCH : REPACK_BATCH / 2;  // f32 groups are 32 bytes
  for (int base = e0 + threadIdx.x * 8; base < e1; base += STEP * BATCH) {
    uint4 raw[BATCH][F16 ? 1 : 2];
#pragma unroll
    for (int b = 0; b < BATCH; ++b)
      if (base + b * STEP < e1) {
        const uint4* p = reinterpret_cast<const uint4*>(j.src + j.at(base + b * STEP) * (F16 ? 2 : 4));
        raw[b][0] = p[0];
        if constexpr (!F16) raw[b][F16 ? 0 : 1] = p[1];
      }
#pragma unroll
    for (int b = 0; b < BATCH; ++b)
      if (base + b * STEP < e1) {
        float v[8];
        if constexpr (F16) {
          const __half2* h = reinterpret_cast<const __half2*>(&raw[b][0]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
          }
        } else {
          const float* f = reinterpret_cast<const float*>(&raw[b][0]);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = f[i];
        }
        store8<BF16>(j.dst, base + b * STEP, v);
      }
  }
}

// Element by element (strided rows, fills), REPACK_BATCH * 2 loads in flight per thread.
__device__ __forceinline__ void copy_elements(const Job& j, int e0, int e1) {
  constexpr int PER = REPACK_BATCH * 2;
  for (int base = e0 + threadIdx.x; base < e1; base += REPACK_THREADS * PER) {
    float v[PER];
#pragma unroll
    for (int b = 0; b < PER; ++b) {
      const int e = base + b * REPACK_THREADS;
      v[b] = j.value;
      if (!j.fill && e < e1)
        v[b] = j.f16 ? __half2float(reinterpret_cast<const __half*>(j.src)[j.at(e)])
                     : reinterpret_cast<const float*>(j.src)[j.at(e)];
    }
#pragma unroll
    for (int b = 0; b < PER; ++b)
      if (base + b * REPACK_THREADS < e1) store1(j, base + b * REPACK_THREADS, v[b]);
  }
}

// Each CTA takes chunks c = blockIdx.x, blockIdx.x + gridDim.x, ... A job whose rows are
// contiguous in the source (innermost stride 1, every other stride and the row length
// multiples of 8, both ends 16-byte aligned) moves groups of 8 elements with 16-byte
// accesses; any other job element by element.
__global__ void __launch_bounds__(REPACK_THREADS, REPACK_CTAS_PER_SM)
    repack_kernel(const tb_repack_job* __restrict__ jobs, int n_jobs, long long n_chunks, const char* __restrict__ src,
                  char* __restrict__ dst) {
  for (long long c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const tb_repack_job& t = jobs[find_job(jobs, n_jobs, c)];
    Job j;
    j.src = src + t.src_off;
    j.dst = dst + t.dst_off;
    j.s0 = t.stride[0], j.s1 = t.stride[1], j.s2 = t.stride[2], j.s3 = t.stride[3];
    j.d1 = t.dims[1], j.d2 = t.dims[2], j.d3 = t.dims[3];
    j.n = t.dims[0] * j.d1 * j.d2 * j.d3;  // below 2^31, checked by the host
    j.fill = t.fill, j.f16 = t.src_type == TB_SRC_F16, j.bf16 = t.dst_type == TB_BF16;
    j.value = t.value;
    const int e0 = static_cast<int>((c - t.first_chunk) * TB_REPACK_CHUNK);
    const int e1 = min(j.n, e0 + TB_REPACK_CHUNK);
    const bool vec = !j.fill && j.s3 == 1 && j.d3 % 8 == 0 && (j.s0 | j.s1 | j.s2) % 8 == 0 &&
                     reinterpret_cast<uintptr_t>(j.src) % 16 == 0 && reinterpret_cast<uintptr_t>(j.dst) % 16 == 0;
    // With vec, e0 and e1 are multiples of 8 and a group of 8 never crosses a row.
    if (!vec)
      copy_elements(j, e0, e1);
    else if (j.f16)
      j.bf16 ? copy_groups<true, true>(j, e0, e1) : copy_groups<true, false>(j, e0, e1);
    else
      j.bf16 ? copy_groups<false, true>(j, e0, e1) : copy_groups<false, false>(j, e0, e1);
  }
}

// Checks one job against the buffers and returns its element count, or -1.
long long check_job(const tb_repack_job& j, bool have_src, size_t src_bytes, size_t dst_bytes) {
  long long n = 1;
  for (int k = 0; k < 4; ++k) {
    if (j.dims[k] < 0) return -1;
    n *= j.dims[k];  // each factor below 2^31 and the running product below 2^31: no overflow
    if (n > INT_MAX) return -1;
  }
  if (j.dst_type != TB_F32 && j.dst_type != TB_BF16) return -1;
  const long long dsz = j.dst_type == TB_BF16 ? 2 : 4;
  if (j.dst_off < 0 || j.dst_off % dsz) return -1;
  if (n == 0) return 0;
  if (static_cast<unsigned long long>(j.dst_off) > dst_bytes ||
      static_cast<unsigned long long>(n * dsz) > dst_bytes - static_cast<unsigned long long>(j.dst_off))
    return -1;
  if (j.fill) return n;
  if (j.src_type != TB_SRC_F16 && j.src_type != TB_SRC_F32) return -1;
  const long long ssz = j.src_type == TB_SRC_F16 ? 2 : 4;
  if (!have_src || j.src_off < 0 || j.src_off % ssz || static_cast<unsigned long long>(j.src_off) >= src_bytes)
    return -1;
  const long long avail = static_cast<long long>((src_bytes - static_cast<size_t>(j.src_off)) / ssz);
  long long last = 0;  // the largest source element index the job reads, kept below avail
  for (int k = 0; k < 4; ++k) {
    if (j.stride[k] < 0) return -1;
    const long long steps = j.dims[k] - 1;
    if (steps > 0 && j.stride[k] > 0) {
      if (j.stride[k] > (avail - 1 - last) / steps) return -1;
      last += steps * j.stride[k];
    }
  }
  return last < avail ? n : -1;
}

}  // namespace

int repack(const tb_repack_job* jobs, int n_jobs, void* jobs_dev, const void* src, size_t src_bytes, void* dst,
           size_t dst_bytes, cudaStream_t stream) {
  if (n_jobs < 0) return TB_ERR_ARG;
  if (n_jobs == 0) return TB_OK;
  if (!jobs || !jobs_dev || !dst || reinterpret_cast<uintptr_t>(jobs_dev) % 8 || reinterpret_cast<uintptr_t>(dst) % 4 ||
      reinterpret_cast<uintptr_t>(src) % 4)
    return TB_ERR_ARG;
  std::vector<tb_repack_job> table(jobs, jobs + n_jobs);
  long long chunks = 0;
  for (tb_repack_job& j : table) {
    const long long n = check_job(j, src != nullptr, src_bytes, dst_bytes);
    if (n < 0) return TB_ERR_ARG;
    j.first_chunk = chunks;
    chunks += (n + TB_REPACK_CHUNK - 1) / TB_REPACK_CHUNK;
  }
  if (chunks == 0) return TB_OK;
  // From pageable memory: the call returns once the table is staged, so `table` may go.
  if (cudaMemcpyAsync(jobs_dev, table.data(), table.size() * sizeof(tb_repack_job), cudaMemcpyHostToDevice, stream) !=
      cudaSuccess)
    return fail_cuda();
  const long long cap = static_cast<long long>(sm_count()) * REPACK_CTAS_PER_SM;
  const int grid = static_cast<int>(chunks < cap ? chunks : cap);
  repack_kernel<<<grid, REPACK_THREADS, 0, stream>>>(static_cast<const tb_repack_job*>(jobs_dev), n_jobs, chunks,
                                                     static_cast<const char*>(src), static_cast<char*>(dst));
  return check_launch();
}

}  // namespace tb
