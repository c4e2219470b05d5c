// Shared device helpers for the sm_100a kernels: error reporting, bounded waits,
// mbarriers, TMA tile loads and the tcgen05 (5th-generation tensor core + tensor
// memory) instructions, written as inline PTX.
//
// Every wait in these kernels is bounded: after TB_WAIT_NS nanoseconds without
// progress it records an error code in the caller's error word and returns false, and
// the kernel then winds down (its own copies drained, tensor memory freed) instead of
// spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tbcuda.h"

#define TB_WAIT_NS 2000000000ull  // 2 s without progress is a hang

namespace tb {

// ---------------------------------------------------------------------------
// Element conversion

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Stores 4 consecutive values.
__device__ __forceinline__ void store4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&lo);
  u.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = u;
}
// Two values rounded to bf16 in one 32-bit word (a in the low half, as memory order).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void store2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }
__device__ __forceinline__ void store2(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
__device__ __forceinline__ float2 load2f(const float* p) { return *reinterpret_cast<const float2*>(p); }
__device__ __forceinline__ float2 load2f(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&u.x), hi = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + expf(-x)); }
// 1/y for normal y >= 1 on the FMA pipe. The initial estimate is the integer-subtraction
// reciprocal of J. F. Blinn, "Floating-point tricks", IEEE Computer Graphics and
// Applications 17(4), 1997: reading a float's bits as an integer approximates a scaled,
// offset log2, so C - bits(y) approximates bits(1/y). The constant is this file's own
// choice: RCP_SEED minimises max |1 - y r0| over every float mantissa (an exhaustive
// minimax search; 0.0505 at the optimum). Two Newton-Raphson steps r <- r (2 - y r) then
// square the error twice: relative error below 7e-6 (plus rounding). Epilogues whose
// throughput is set by the special-function unit use it instead of a second MUFU
// operation. Checked against division on the host (every mantissa) and on the GPU
// (tb_selftest_math).
constexpr int RCP_SEED = 0x7EF311C2;
__device__ __forceinline__ float rcp_newton(float y) {
  float r = __int_as_float(RCP_SEED - __float_as_int(y));
  r = r * fmaf(-y, r, 2.0f);
  return r * fmaf(-y, r, 2.0f);
}
// sigmoid and SiLU with one MUFU operation (the exponential); for bf16 outputs.
__device__ __forceinline__ float fast_sigmoid(float x) { return rcp_newton(1.0f + __expf(fminf(-x, 80.0f))); }
__device__ __forceinline__ float fast_silu(float x) { return x * fast_sigmoid(x); }

// Two-wide fp32 arithmetic (sm_100 packed f32x2 instructions; each half rounds as the
// scalar instruction would).
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  return (unsigned long long)__float_as_uint(v.x) | ((unsigned long long)__float_as_uint(v.y) << 32);
}
__device__ __forceinline__ float2 f2_from(unsigned long long b) {
  return make_float2(__uint_as_float((uint32_t)b), __uint_as_float((uint32_t)(b >> 32)));
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}
// Largest of three (sm_100 three-input max.f32: one instruction where two fmaxf would be).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_from(r);
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// Sigmoid of two values: 1 / (1 + 2^(-x log2 e)), the exponential on the MUFU unit (its
// argument capped at 80 log2 e, where the sigmoid is 0 in fp32 anyway), the reciprocal by
// the bit-level estimate and two Newton-Raphson steps as rcp_newton, the rest two-wide.
__device__ __forceinline__ float2 fast_sigmoid2(float2 x) {
  const float2 t = mul2(x, make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 y = add2(make_float2(ex2_approx(fminf(t.x, 115.415f)), ex2_approx(fminf(t.y, 115.415f))),
                        make_float2(1.0f, 1.0f));
  float2 r = make_float2(__int_as_float(RCP_SEED - __float_as_int(y.x)), __int_as_float(RCP_SEED - __float_as_int(y.y)));
  const float2 ny = make_float2(-y.x, -y.y), two = make_float2(2.0f, 2.0f);
  r = mul2(r, fma2(ny, r, two));
  return mul2(r, fma2(ny, r, two));
}
__device__ __forceinline__ float2 fast_silu2(float2 x) { return mul2(x, fast_sigmoid2(x)); }
// The PTX tanh.approx.f32 instruction (one MUFU operation, at most 2^-10.987 relative error
// as the PTX ISA documents it).
__device__ __forceinline__ float tanh_mufu(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// SiLU of two values for bf16 outputs: x sigmoid(x) with sigmoid(x) = (1 + tanh(x/2)) / 2,
// i.e. h + h tanh(h) with h = x/2: one MUFU operation and one two-wide FMA per value, the
// cheapest form (the SiLU epilogue of FFN up and the depthwise conv are bound by their
// arithmetic, not by memory). Its absolute error is about |x| 2^-12 (the tanh's), below
// a bf16 output's resolution except where the SiLU is near zero.
__device__ __forceinline__ float2 silu2_tanh(float2 x) {
  const float2 h = mul2(x, make_float2(0.5f, 0.5f));
  return fma2(h, make_float2(tanh_mufu(h.x), tanh_mufu(h.y)), h);
}

// Float to an unsigned key whose unsigned order is the float order.
__device__ __forceinline__ uint32_t order_key(float v) {
  uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// (value, index) packed so that an unsigned max picks the largest value and, among
// equal values, the smallest index: the first-index tie rule of torch.argmax.
__device__ __forceinline__ unsigned long long argmax_key(float v, int index) {
  return ((unsigned long long)order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)index);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) { return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)); }

// ---------------------------------------------------------------------------
// Programmatic dependent launch. Kernels launched with programmatic stream
// serialization may start before their predecessor on the stream has finished: each
// kernel here runs only its prologue (barrier init, tensor-memory allocation, descriptor
// prefetch) before grid_dep_wait(), which returns once the predecessor has completed and
// its writes are visible; grid_dep_launch() then lets the successor start its own
// prologue. Without that launch attribute both are no-ops.

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Timers, shared-memory addresses, mbarriers

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Arrival that orders none of this thread's memory operations (for "tensor memory read"
// signals, whose reads completed at tcgen05.wait::ld).
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Adds `bytes` to the transaction count the barrier's current phase waits for, without an
// arrival (the phase completes only after its arrival, too).
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread until the phase completes, for at most
// `suspend_ns`: a waiting warp then takes no issue slots from the warps sharing its SM
// sub-partition, and still resumes as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `bar` with the given parity to complete. Returns false, with
// `code` or-ed into *err, after TB_WAIT_NS without completion, or at once if the
// kernel has already given up (*abort set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = globaltimer();
  for (;;) {
    if (mbar_try_wait_suspend(bar, parity, 20000)) return true;
    if (*abort) return false;
    if (globaltimer() - start > TB_WAIT_NS) {
      atomicOr(err, code);
      *abort = 1;
      return false;
    }
  }
}

// Asynchronous 4-byte global -> shared copies (no registers held while they fly).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------------------
// TMA (tensor memory accelerator) tile loads, no multicast.

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA issue, commit, loads.

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, f32 accumulation.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T: the A operand (K-major, bf16 pairs packed in
// 32-bit columns, one row per lane) read from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (a cluster of two CTAs): one 256-row MMA over both CTAs' shared memory.
// Each CTA holds half of A (its 128 rows) and half of B (128 of the N columns) at the
// same shared-memory offsets; the leader (rank 0) issues the MMA, and each CTA's tensor
// memory receives its own 128 rows x N accumulator.

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Every thread of both CTAs: all shared-memory writes before are visible to the peer.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of either CTA of the cluster, with no ordering of this thread's
// memory operations: for signals that only say "tensor memory read" (the reads have
// completed at tcgen05.wait::ld), so the arrival does not wait for the thread's global
// stores to become visible.
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (no multicast).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// D (each CTA's tensor memory, its 128 rows) (+)= A * B^T over the pair: M = 256.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on the mbarrier at `bar_cluster` (either CTA) once the pair MMAs this thread
// issued before have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A and B (both K-major) and an f32
// accumulator of M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4)                        // accumulator format: f32
         | (1u << 7)                      // A format: bf16
         | (1u << 10)                     // B format: bf16
         | ((uint32_t)(n >> 3) << 17)     // N / 8
         | ((uint32_t)(m >> 4) << 24);    // M / 16
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with 128-byte
// swizzling: rows of 128 bytes, 8-row atoms 1024 bytes apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4)   // start address
         | ((uint64_t)1 << 16)                 // leading byte offset (unused for swizzled K-major)
         | ((uint64_t)(1024 >> 4) << 32)       // stride byte offset: next 8-row atom
         | ((uint64_t)1 << 46)                 // descriptor version for sm_100
         | ((uint64_t)2 << 61);                // layout: 128-byte swizzle
}

// Descriptor for an MN-major operand written by TMA with 128-byte swizzling: each row
// (one K index) holds 64 consecutive MN elements; 8-row K groups are 1024 bytes apart
// and consecutive 64-element MN chunks `mn_chunk_bytes` apart.
__device__ __forceinline__ uint64_t sdesc_sw128_mn(uint32_t saddr, uint32_t mn_chunk_bytes) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4)                 // start address
         | ((uint64_t)((mn_chunk_bytes >> 4) & 0x3FFFu) << 16)  // leading byte offset: next MN chunk
         | ((uint64_t)(1024 >> 4) << 32)                     // stride byte offset: next 8 K rows
         | ((uint64_t)1 << 46)
         | ((uint64_t)2 << 61);
}

// Instruction descriptor for kind::f16, bf16 inputs, f32 accumulator, K-major A and
// MN-major B.
__host__ __device__ constexpr uint32_t idesc_bf16_bmn(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit columns to tensor memory; one row per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns to tensor memory; one row per thread.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns from tensor memory; one row per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tb
