// TDT greedy decoding in bf16 as ONE persistent kernel: every SM runs one CTA for the
// whole loop, and the phases of an iteration are separated by a grid-wide barrier
// instead of kernel launches. Replaces the prediction network, joint and greedy loop
// of tinybark/tinygrad/model.py:162-233 (one clip and one host round trip per token in
// the reference) for a batch of clips, one lane per clip, all lanes stepped together.
//
// Layer 0 of the LSTM is split in its two inputs: its gates are E[token] + P0, with
// E = embedding . W_ih0^T precomputed for every token (tb_model.lstm0_emb) and
// P0 = W_hh0 . h0 + b0 computed one iteration ahead, from the h0 the cell just made.
// That leaves no GEMM between the argmax and layer 1:
//
// Phases (q counts them from 0; every CTA takes part in every phase):
//   q = 0             INIT   lane state, h = 0, P0 = b0
//   q = 1, 2, 3       CELL, LSTM, PROJ of the first prediction step (token blank)
//   q = 4 + 4i + r    iteration i: r = 0 JOINT, 1 CELL, 2 LSTM, 3 PROJ
// JOINT  z [lanes x 640] . joint_w^T [8448 x 640] -> per-lane argmax keys (BN = 256)
// CELL   the loop body of each lane (lane_scalar: token, duration, frame, stop; 32 lanes
//        at a time per warp, one per thread) and, for a lane that emitted a token, the
//        layer-0 cell from E[token] + P0 (a warp per lane): c0 and h0 (into x1[:, :640]),
//        and h1 (hp) copied into x1[:, 640:]
// LSTM   layer 1: x1 . W1^T [2560 x 1280] with the cell in the epilogue (BN = 128), and
//        on the SMs it leaves idle, the next P0 = x1[:, :640] . W_hh0^T + b0
// PROJ   hp . dec_proj^T [640 x 640] -> dec, and z = relu(enc[frame] + dec) (BN = 64)
// Split layer 1 (when its tiles fit one per SM, up to 896 lanes): the h1 half of layer
// 1's product, hp . W_hh1^T, does not wait for the token. PROJ computes it on the SMs
// the projector leaves idle, into a tensor-memory accumulator that the SM keeps through
// JOINT and CELL; LSTM then adds h0 . W_ih1^T (K = 640 instead of 1280) into the same
// accumulator, so layer 1 reads half the bytes on the critical path.
// The GEMM phases use the tcgen05 pipeline of the GEMM kernel (gemm.cu): warp 0 loads
// A and W tiles with TMA into a shared-memory ring, warp 1 issues the MMAs into one of
// two tensor-memory accumulators, warps 2-5 run the epilogue (tcgemm.cuh) and the
// INIT/CELL work.
//
// Each iteration only covers lanes below the row bound M_i = 1 + the last lane still
// running after CELL i (lanes are ordered longest first, so M shrinks as clips end);
// the loop ends when no lane runs. The barrier is a global arrival counter: after a
// phase every CTA adds 1, and phase q starts once the counter reaches q * gridDim.
// Every wait is bounded (TB_WAIT_NS): a CTA that gives up sets TB_DEV_DECODE_TIMEOUT in
// the error word and a global abort flag, and every CTA then leaves the loop.
#include <algorithm>

#include "decode.cuh"
#include "decode_tiles.cuh"
#include "tcgemm.cuh"

namespace tb {

namespace {

constexpr int DT_OUT_BYTES = 4 * 32 * TC_OUT_STRIDE * 4;
constexpr int DT_SMEM = 1024 + DT_RING_BYTES + DT_OUT_BYTES + 256;
constexpr int DT_ACC_COLS = 256;  // tensor-memory columns per accumulator
constexpr int DT_CARRY_COL = 384;  // split layer 1: the accumulator kept from PROJ to LSTM


struct DecodeTcArgs {
  CUtensorMap a[5], w[5];  // A operand and weights of the joint, LSTM1, next-P0, projector, W_hh1 GEMMs
  tb_epilogue e[4];        // epilogues of the first four (the W_hh1 product has none)
  int split;               // 1: layer 1 split in its h0 and h1 halves (see above)
  DecodeWs ws;
  const float* emb_gates;  // [8193, 2560] E = embedding . W_ih0^T
  const float* b0;         // [2560] layer 0's bias
  const int* enc_off;
  const int* cap;
  int lanes, max_cap, max_iters;
  int* tokens;
  int* counts;    // each lane's count, written when the lane stops
  int* progress;  // host-mapped (may be NULL): [0] row bound, [1] iteration
  int* err;
};

// Rows a phase covers: JOINT and CELL of iteration i read M_{i-1}, the rest M_i. Each
// bound is written during one CELL phase and read only after its barrier, so every
// role of every CTA reads the same value, however late it reads it.
__device__ __forceinline__ int phase_rows(const Phase& p, const int* bounds) {
  if (p.kind == P_INIT) return 0;
  if (p.iter < 0) return bounds[0];
  const int i = (p.kind == P_CELL || p.kind == P_JOINT) ? p.iter - 1 : p.iter;
  return bounds[i + 1];
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Waits until `count` phase arrivals are in (every CTA finished the phases before).
// False if the decoder gave up: abort set by another CTA, or this wait timed out.
__device__ bool grid_wait(unsigned* sync, unsigned count, int* err, volatile int* abort) {
  const uint64_t start = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire(sync) >= count) {
      fence_proxy_async_global();  // TMA reads issued after this see the phase's writes
      return true;
    }
    if ((i & 15) == 15) {
      if (*abort || reinterpret_cast<volatile unsigned*>(sync)[1]) {
        *abort = 1;
        return false;
      }
      if (globaltimer() - start > TB_WAIT_NS) {
        atomicOr(err, TB_DEV_DECODE_TIMEOUT);
        atomicExch(sync + 1, 1u);
        *abort = 1;
        return false;
      }
    }
  }
}

// The CTA's view of the grid barrier: the producer thread is the only one that polls
// global memory; it publishes each phase it has seen here, and the MMA thread and the
// epilogue warps wait on that (release/acquire at CTA scope, after the producer's
// acquire at GPU scope, so the phase's writes are visible to them too).
__device__ __forceinline__ void post_phase(unsigned* slot, unsigned q) {
  asm volatile("st.release.cta.shared.u32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(q) : "memory");
}
__device__ bool cta_phase_wait(unsigned* slot, unsigned q, int* err, volatile int* abort, unsigned* sync) {
  const uint64_t start = globaltimer();
  for (uint32_t i = 0;; ++i) {
    unsigned v;
    asm volatile("ld.acquire.cta.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(slot)) : "memory");
    if (v >= q) return true;
    // After a few quick polls, back off briefly between polls: the issue slots go to the
    // epilogue warp on the same SM sub-partition.
    if (i >= 8) __nanosleep(32);
    if ((i & 15) == 15) {
      if (*abort) return false;
      if (globaltimer() - start > TB_WAIT_NS) {
        atomicOr(err, TB_DEV_DECODE_TIMEOUT);
        atomicExch(sync + 1, 1u);
        *abort = 1;
        return false;
      }
    }
  }
}

// Named barrier of the four epilogue warps (128 threads) with an OR of `pred`.
__device__ __forceinline__ bool epi_bar_or(bool pred) {
  int r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n barrier.red.or.pred q, 1, 128, p;\n selp.s32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((int)pred)
      : "memory");
  return r != 0;
}

// Brings the descriptors a GEMM phase uses into the TMA unit's cache (issued while the
// producer waits for the phase's barrier).
__device__ __forceinline__ void prefetch_phase_maps(const DecodeTcArgs& args, int kind) {
  if (kind == P_JOINT) {
    prefetch_tmap(&args.a[G_JOINT]);
    prefetch_tmap(&args.w[G_JOINT]);
  } else if (kind == P_LSTM) {
    prefetch_tmap(&args.a[a_map(G_LSTM1, args.split)]);
    prefetch_tmap(&args.w[G_LSTM1]);
    prefetch_tmap(&args.a[G_PRE0]);
    prefetch_tmap(&args.w[G_PRE0]);
  } else if (kind == P_PROJ) {
    prefetch_tmap(&args.a[G_PROJ]);
    prefetch_tmap(&args.w[G_PROJ]);
    if (args.split) {
      prefetch_tmap(&args.w[G_HH1]);
      prefetch_tmap(&args.w[G_PRE0]);  // next-P0 tiles moved into this phase
    }
  }
}

// The two tensor-memory accumulators the GEMM tiles alternate between, with one phase bit
// each. With layer 1 split, the joint's 256-column tiles always take buffer 0 (buffer 1
// then has 128 columns; the carried accumulator holds the other 128). The MMA thread and
// the epilogue warps walk the same tiles in the same order, so they pick alike.
struct AccPick {
  int next = 0;
  uint32_t ph = 0;  // bit b: parity of buffer b's next use
  __device__ __forceinline__ int pick(bool first_only) {
    const int b = first_only ? 0 : next;
    if (!first_only) next ^= 1;
    return b;
  }
  __device__ __forceinline__ uint32_t parity(int b) const { return (ph >> b) & 1u; }
  __device__ __forceinline__ void used(int b) { ph ^= 1u << b; }
};

// Barriers beyond the GEMM kernel's: the carried accumulator of split layer 1 is full
// (layer 1's MMAs done) and empty (its epilogue has read it).
struct DtBars {
  TcBars tc;
  uint64_t cfull, cempty;
};
static_assert(sizeof(DtBars) <= 256, "decoder barriers");

// Lane l's state before the first step: zero LSTM state (h0, h1 in x1, c), P0 = b0 (its
// value at h0 = 0), counters. One warp per lane.
__device__ __forceinline__ void lane_init_tc(const DecodeTcArgs& args, int l, int lane) {
  const DecodeWs& w = args.ws;
  const long long L = args.lanes;
  __nv_bfloat16* x1 = reinterpret_cast<__nv_bfloat16*>(w.x1) + (long long)l * 2 * TB_PRED;
  for (int j = lane; j < TB_PRED; j += 32) {
    w.c[l * TB_PRED + j] = 0.f;
    w.c[(L + l) * TB_PRED + j] = 0.f;
  }
  for (int j = lane; j < 2 * TB_PRED; j += 32) x1[j] = __float2bfloat16_rn(0.f);
  float* p0 = w.pre0 + (long long)l * 4 * TB_PRED;
  for (int j = lane; j < 4 * TB_PRED; j += 32) p0[j] = args.b0[j];
  if (lane == 0) {
    const int valid = args.enc_off[l + 1] - args.enc_off[l];
    const int done = (valid <= 0 || args.cap[l] <= 0) ? 1 : 0;
    w.frame[l] = 0;
    w.it[l] = 0;
    w.count[l] = 0;
    w.done[l] = done;
    w.mask[l] = 1;
    w.keys[l] = 0ull;
    w.keys2[l] = 0ull;
    w.erow[l] = done ? -1 : args.enc_off[l];
    args.counts[l] = 0;
  }
}

// Layer 0's cell for lane l, which steps on token `tok` (one warp): gates E[tok] + P0,
// c0 and h0 (into x1[:, :640]), and h1 (hp) copied into x1[:, 640:] unless layer 1 is
// split (it then reads h1 from hp itself) or this is the first prediction step (h1 = 0,
// as INIT wrote it).
__device__ __forceinline__ void lane_cell(const DecodeTcArgs& args, int l, int tok, int iter, int lane) {
  const DecodeWs& w = args.ws;
  const float4* __restrict__ eg = reinterpret_cast<const float4*>(args.emb_gates + (long long)tok * 4 * TB_PRED);
  const float4* __restrict__ p0 = reinterpret_cast<const float4*>(w.pre0 + (long long)l * 4 * TB_PRED);
  float* __restrict__ c0 = w.c + (long long)l * TB_PRED;
  __nv_bfloat16* __restrict__ x1 = reinterpret_cast<__nv_bfloat16*>(w.x1) + (long long)l * 2 * TB_PRED;
  const __nv_bfloat16* __restrict__ hp = reinterpret_cast<const __nv_bfloat16*>(w.hp) + (long long)l * TB_PRED;
  float4 ge[TB_PRED / 32], gp[TB_PRED / 32];
  float cv[TB_PRED / 32];
#pragma unroll
  for (int k = 0; k < TB_PRED / 32; ++k) {
    const int u = k * 32 + lane;
    ge[k] = eg[u];
    gp[k] = p0[u];
    cv[k] = c0[u];
  }
  uint2 h1v[TB_PRED / 128];
  const bool copy_h1 = iter >= 0 && !args.split;
  if (copy_h1) {
#pragma unroll
    for (int k = 0; k < TB_PRED / 128; ++k) h1v[k] = reinterpret_cast<const uint2*>(hp)[k * 32 + lane];
  }
#pragma unroll
  for (int k = 0; k < TB_PRED / 32; ++k) {
    const int u = k * 32 + lane;
    const float ig = sigmoid_mufu(ge[k].x + gp[k].x), fg = sigmoid_mufu(ge[k].y + gp[k].y);
    const float gg = tanh_mufu(ge[k].z + gp[k].z), og = sigmoid_mufu(ge[k].w + gp[k].w);
    const float c = fg * cv[k] + ig * gg;
    c0[u] = c;
    x1[u] = __float2bfloat16_rn(og * tanh_mufu(c));
  }
  if (copy_h1) {
#pragma unroll
    for (int k = 0; k < TB_PRED / 128; ++k) reinterpret_cast<uint2*>(x1 + TB_PRED)[k * 32 + lane] = h1v[k];
  }
}

// The CELL phase for this warp's lanes l = first + t * stride (t = 0, 1, ...) below `rows`:
// the loop body of 32 lanes at a time, one lane per thread (their scalars in one memory
// round trip), then layer 0's cell of each lane that steps, the whole warp on one lane.
// The first prediction step (iter < 0) feeds the blank token to every lane still running.
// The row bound of iteration `iter` rises to 1 + the last lane still running.
__device__ __forceinline__ void cell_phase(const DecodeTcArgs& args, int first, int stride, int rows, int iter,
                                           int lane, int* bounds) {
  const DecodeWs& w = args.ws;
  for (int base = first; base < rows; base += 32 * stride) {
    const int l = base + lane * stride;
    int step = 0, tok = TB_BLANK;
    bool running = false;
    if (l < rows) {
      if (iter < 0) {
        running = !w.done[l];
        step = running;
      } else {
        running = lane_scalar(w, args.enc_off, args.cap, l, args.max_cap, args.tokens, step, tok, args.counts);
      }
    }
    const unsigned run_mask = __ballot_sync(0xffffffffu, running);
    if (iter >= 0 && run_mask && lane == 31 - __clz(run_mask)) atomicMax(bounds + iter + 1, l + 1);
    unsigned step_mask = __ballot_sync(0xffffffffu, step != 0);
    while (step_mask) {
      const int t = __ffs(step_mask) - 1;
      step_mask &= step_mask - 1;
      lane_cell(args, base + t * stride, __shfl_sync(0xffffffffu, tok, t), iter, lane);
    }
  }
}

}  // namespace

__global__ void __launch_bounds__(192, 1) decode_tc_kernel(const __grid_constant__ DecodeTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* out_stage = reinterpret_cast<float*>(smem + DT_RING_BYTES);
  DtBars* dbars = reinterpret_cast<DtBars*>(smem + DT_RING_BYTES + DT_OUT_BYTES);
  TcBars* bars = &dbars->tc;
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DecodeWs& w = args.ws;
  int* bounds = w.bounds;
  unsigned* sync = reinterpret_cast<unsigned*>(w.m_cur + 8);
  const unsigned G = gridDim.x;
  int* err = args.err;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 8; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);
      mbar_init(&bars->tempty[a], 4);
    }
    mbar_init(&bars->done, 1);
    mbar_init(&dbars->cfull, 1);
    mbar_init(&dbars->cempty, 4);
    bars->abort = 0;
    bars->phase = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem, 2 * DT_ACC_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;
  // Phases run while q < q_end; the last iteration ends after its STEP.
  const int q_end = 4 + 4 * args.max_iters;

  if (warp == 0) {
    if (lane == 0) {
      for (int g = 0; g < 5; ++g) {
        prefetch_tmap(&args.a[g]);
        prefetch_tmap(&args.w[g]);
      }
      uint32_t use = 0, used = 0;  // per ring slot: parity of its next use; slots ever used
      int last = -1;               // the slot filled last
      bool ok = true;
      for (int q = 1; q < q_end && ok; ++q) {
        const Phase p = phase_of(q);
        prefetch_phase_maps(args, p.kind);
        if (!grid_wait(sync, (unsigned)q * G, err, abort)) break;
        post_phase(&bars->phase, (unsigned)q);
        const int rows = phase_rows(p, bounds);
        if (rows <= 0) break;  // no lane runs: the loop is over
        if (p.kind == P_CELL) continue;
        const int sg = phase_stage_gemm(p.kind, args.split, rows, blockIdx.x, G), sb = stage_bytes(sg), slots = ring_slots(sg);
        // The new cut may overlap stages of the old one: wait until the MMAs have
        // released every stage in use. They complete in issue order, so the release of
        // the stage filled last implies all the others.
        if (last >= 0) ok = mbar_wait(&bars->empty[last], ((use >> last) & 1) ^ 1, err, TB_DEV_DECODE_TIMEOUT, abort);
        int s = 0, g, mt, nt;
        for (int k = 0; ok && phase_tile(p.kind, rows, blockIdx.x, G, k, args.split, g, mt, nt); ++k) {
          const int bn = gemm_bn(g), kb_count = gemm_k(g, args.split) / 64;
          for (int kb = 0; kb < kb_count; ++kb) {
            if (!mbar_wait(&bars->empty[s], ((use >> s) & 1) ^ 1, err, TB_DEV_DECODE_TIMEOUT, abort)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + s * sb;
            mbar_expect_tx(&bars->full[s], DT_A_BYTES + bn * 64 * 2);
            tma_load_2d(sa, &args.a[a_map(g, args.split)], &bars->full[s], kb * 64, mt * 128);
            tma_load_2d(sa + DT_A_BYTES, &args.w[g], &bars->full[s], kb * 64, nt * bn);
            use ^= 1u << s;
            used |= 1u << s;
            last = s;
            if (++s == slots) s = 0;
          }
        }
      }
      // Let the copies in flight land before the CTA exits (all of them have landed
      // unless the loop was abandoned).
      for (int s = 0; s < 8; ++s)
        if ((used >> s) & 1) drain_wait(&bars->full[s], ((use >> s) & 1) ^ 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      AccPick ap;
      uint32_t use = 0, cph = 0;  // per ring slot: parity of its next use; carried accumulator's parity
      bool ok = true;
      for (int q = 1; q < q_end && ok; ++q) {
        const Phase p = phase_of(q);
        if (!cta_phase_wait(&bars->phase, (unsigned)q, err, abort, sync)) break;
        const int rows = phase_rows(p, bounds);
        if (rows <= 0) break;
        if (p.kind == P_CELL) continue;
        const int sg = phase_stage_gemm(p.kind, args.split, rows, blockIdx.x, G), sb = stage_bytes(sg), slots = ring_slots(sg);
        int s = 0, g, mt, nt;
        for (int k = 0; ok && phase_tile(p.kind, rows, blockIdx.x, G, k, args.split, g, mt, nt); ++k) {
          const int kb_count = gemm_k(g, args.split) / 64;
          const uint32_t idesc = g == G_JOINT ? idesc_bf16(128, 256) : (g == G_PROJ ? idesc_bf16(128, 64) : idesc_bf16(128, 128));
          // Split layer 1: the W_hh1 product starts the carried accumulator once the last
          // layer-1 epilogue has read it; layer 1's MMAs then add to it (except at the
          // first step, where h1 = 0 and nothing was carried).
          const bool carried = g == G_HH1 || (g == G_LSTM1 && args.split);
          const bool add = g == G_LSTM1 && args.split && p.iter >= 0;
          int b = 0;
          bool waited;
          if (g == G_HH1) {
            waited = mbar_wait(&dbars->cempty, cph ^ 1, err, TB_DEV_DECODE_TIMEOUT, abort);
          } else if (carried) {
            waited = true;
          } else {
            b = ap.pick(args.split && g == G_JOINT);
            waited = mbar_wait(&bars->tempty[b], ap.parity(b) ^ 1, err, TB_DEV_DECODE_TIMEOUT, abort);
          }
          if (!waited) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (carried ? DT_CARRY_COL : b * DT_ACC_COLS);
          for (int kb = 0; kb < kb_count; ++kb) {
            if (!mbar_wait(&bars->full[s], (use >> s) & 1, err, TB_DEV_DECODE_TIMEOUT, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * sb);
            const uint64_t ad = sdesc_sw128(sa), bd = sdesc_sw128(sa + DT_A_BYTES);
#pragma unroll
            for (int k4 = 0; k4 < 4; ++k4) umma_f16(d, ad + 2 * k4, bd + 2 * k4, idesc, add || (kb | k4) != 0);
            umma_commit(&bars->empty[s]);
            use ^= 1u << s;
            if (++s == slots) s = 0;
          }
          if (!ok) break;
          if (g == G_HH1) continue;  // read by layer 1's MMAs, issued after these
          if (carried) {
            umma_commit(&dbars->cfull);
            cph ^= 1;
          } else {
            umma_commit(&bars->tfull[b]);
            ap.used(b);
          }
        }
      }
      if (!ok) *abort = 1;
      // Every MMA issued has completed once this commit arrives.
      umma_commit(&bars->done);
      drain_wait(&bars->done, 0);
    }
  } else {
    const int ew = warp - 2;       // epilogue warp 0..3
    const int quarter = warp & 3;  // tensor-memory lane quarter this warp may access
    float* stage = out_stage + quarter * 32 * TC_OUT_STRIDE;
    AccPick ap;
    uint32_t cph = 0;  // carried accumulator's parity
    // Split layer 1: the cell state of this warp's 32 rows of the CTA's layer-1 tile (the
    // tile never moves to another SM), one row per lane.
    float c1[32];
#pragma unroll
    for (int u = 0; u < 32; ++u) c1[u] = 0.f;
    for (int q = 0; q < q_end; ++q) {
      const Phase p = phase_of(q);
      bool ok = true;
      int rows = args.lanes;
      if (q > 0) {
        if (ew == 0 && lane == 0) ok = cta_phase_wait(&bars->phase, (unsigned)q, err, abort, sync);
        if (epi_bar_or(!ok || *abort)) break;
        rows = phase_rows(p, bounds);
        if (rows <= 0) break;
      }
      if (p.kind == P_JOINT && args.progress && blockIdx.x == 0 && ew == 0 && lane == 0 && (p.iter & 31) == 0) {
        // Every lane at or above `rows` has stopped, its tokens and count written before
        // the last barrier: publish the bound to the host, which may copy those lanes out
        // while the loop goes on.
        __threadfence_system();
        *reinterpret_cast<volatile int*>(args.progress + 1) = p.iter;
        *reinterpret_cast<volatile int*>(args.progress) = rows;
      }
      if (p.kind == P_INIT) {
        for (int l = blockIdx.x * 4 + ew; l < args.lanes; l += G * 4) lane_init_tc(args, l, lane);
      } else if (p.kind == P_CELL) {
        cell_phase(args, blockIdx.x * 4 + ew, G * 4, rows, p.iter, lane, bounds);
      } else {
        int g, mt, nt;
        for (int k = 0; phase_tile(p.kind, rows, blockIdx.x, G, k, args.split, g, mt, nt); ++k) {
          if (g == G_HH1) continue;  // no epilogue: layer 1 reads it from tensor memory
          const bool carried = g == G_LSTM1 && args.split;
          const int b = carried ? 0 : ap.pick(args.split && g == G_JOINT);
          uint64_t* full = carried ? &dbars->cfull : &bars->tfull[b];
          const uint32_t ph = carried ? cph : ap.parity(b);
          const int row0 = mt * 128 + quarter * 32, n0 = nt * gemm_bn(g);
          const uint32_t taddr =
              tmem + ((uint32_t)(quarter * 32) << 16) + (carried ? DT_CARRY_COL : b * DT_ACC_COLS);
          if (ok) {
            // Constant indices: the epilogue's operands are then read straight from the
            // kernel parameters, never through a pointer that the stores might alias.
            if (g == G_JOINT)
              ok = epilogue_tile<256, TB_EPI_ARGMAX>(args.e[G_JOINT], stage, taddr, row0, n0, lane, rows, full, ph,
                                                     err, abort);
            else if (g == G_PROJ)
              ok = epilogue_tile<64, TB_EPI_JOINT_IN>(args.e[G_PROJ], stage, taddr, row0, n0, lane, rows, full, ph,
                                                      err, abort);
            else if (carried)
              ok = lstm_tile<128, true>(args.e[G_LSTM1], stage, taddr, row0, n0, lane, rows, full, ph, err, abort,
                                        &c1);
            else if (g == G_LSTM1)
              ok = epilogue_tile<128, TB_EPI_LSTM>(args.e[G_LSTM1], stage, taddr, row0, n0, lane, rows, full, ph,
                                                   err, abort);
            else
              ok = epilogue_tile<128, TB_EPI_STORE>(args.e[G_PRE0], stage, taddr, row0, n0, lane, rows, full, ph,
                                                    err, abort);
          }
          tc_fence_before();
          __syncwarp();
          if (ok && lane == 0) mbar_arrive_relaxed(carried ? &dbars->cempty : &bars->tempty[b]);
          if (carried)
            cph ^= 1;
          else
            ap.used(b);
        }
      }
      // The phase's writes, visible to the other CTAs' loads and TMA reads, then one
      // arrival for this CTA: each writer orders its stores before later async-proxy
      // reads, the named barrier orders every epilogue thread's stores before thread 0's
      // GPU-scope fence, and that fence (cumulative over what the barrier ordered) before
      // the arrival. A fence in every thread as well costs ~2 us per iteration and orders
      // nothing more (the same pattern as a cooperative grid sync).
      fence_proxy_async_global();
      if (epi_bar_or(!ok)) {
        *abort = 1;
        break;
      }
      if (ew == 0 && lane == 0) {
        __threadfence();
        atomicAdd(sync, 1u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * DT_ACC_COLS);
  }
}

// Self-test of the bounded waits (no reference counterpart): one CTA waits on a
// shared-memory barrier that nothing completes (kind 0: the wait every tcgen05 kernel
// here uses between its warps) or on the decoder's grid barrier with a counter nothing
// increments (kind 1). Each gives up after TB_WAIT_NS, or-s its TB_DEV_* bit into *err
// and returns; nothing hangs and nothing faults.
__global__ void selftest_wait_kernel(int kind, unsigned* counter, int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort;
  if (threadIdx.x != 0) return;
  abort = 0;
  if (kind == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, err, TB_DEV_GEMM_TIMEOUT, &abort);  // phase 0 never completes
  } else {
    grid_wait(counter, 1u, err, &abort);  // the counter stays 0
  }
}

int selftest_wait(int kind, unsigned* scratch, int* err, cudaStream_t stream) {
  if ((kind != 0 && kind != 1) || !err || !scratch) return TB_ERR_ARG;
  // scratch: 256 zeroed bytes for the counter and the abort flag of kind 1.
  if (cudaMemsetAsync(scratch, 0, 256, stream) != cudaSuccess) return fail_cuda();
  selftest_wait_kernel<<<1, 32, 0, stream>>>(kind, scratch, err);
  return check_launch();
}

int tdt_decode_tc(const tb_model& m, const float* enc, const int* enc_off, const int* cap, int lanes, int max_cap,
                  int* tokens, int* counts, void* ws, size_t ws_bytes, int* host_flag, int* err, cudaStream_t stream) {
  if (lanes <= 0) return TB_OK;
  if (m.dtype != TB_BF16 || !m.lstm0_hh || !m.lstm0_emb) return TB_ERR_ARG;
  if (!enc || !enc_off || !cap || !tokens || !counts || !ws || max_cap <= 0) return TB_ERR_ARG;
  if (ws_bytes < decode_ws(TB_BF16, lanes)) return TB_ERR_WORKSPACE;
  static bool configured[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail_cuda();
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DT_SMEM) != cudaSuccess)
      return fail_cuda();
    configured[dev] = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_tc_kernel, 192, DT_SMEM) != cudaSuccess)
    return fail_cuda();
  if (per_sm < 1) return TB_ERR_UNSUPPORTED;
  const int grid = sm_count();

  DecodeTcArgs args = {};
  DecodeWs& w = args.ws;
  w = carve(ws, TB_BF16, lanes);
  // Layer 1 splits when its tiles fit one per SM with SMs left for the next P0.
  args.split = lstm1_tiles(lanes) < grid ? 1 : 0;
  // A operands [lanes x K] and weights [N x K], 64-column boxes of 128 rows (A) or BN rows
  // (W). The next-P0 GEMM and split layer 1 read the h0 half of layer 1's input x1; the
  // W_hh1 product reads h1 (hp) and the right half of layer 1's weights.
  const void* a_ptr[5] = {w.z, w.x1, w.x1, w.hp, w.hp};
  const long long a_ld[5] = {TB_PRED, 2 * TB_PRED, 2 * TB_PRED, TB_PRED, TB_PRED};
  const void* w_ptr[5] = {m.joint_w, m.lstm_w[1], m.lstm0_hh, m.dec_proj_w,
                          static_cast<const __nv_bfloat16*>(m.lstm_w[1]) + TB_PRED};
  const long long w_ld[5] = {TB_PRED, 2 * TB_PRED, TB_PRED, TB_PRED, 2 * TB_PRED};
  for (int g = 0; g < 5; ++g) {
    const int k = gemm_k(g, args.split);
    if (!encode_tmap_2d(&args.a[g], a_ptr[g], lanes, k, a_ld[g], 64, 128) ||
        !encode_tmap_2d(&args.w[g], w_ptr[g], gemm_n(g), k, w_ld[g], 64, gemm_bn(g)))
      return TB_ERR_CUDA;
  }
  tb_epilogue& jt = args.e[G_JOINT];
  jt.kind = TB_EPI_ARGMAX;
  jt.bias = m.joint_b;
  jt.keys = w.keys;
  jt.keys2 = w.keys2;
  jt.split = TB_TOKEN_ROWS;
  jt.split_end = TB_TOKEN_ROWS + TB_DURATIONS;
  tb_epilogue& l1 = args.e[G_LSTM1];
  l1.kind = TB_EPI_LSTM;
  l1.out_dtype = TB_BF16;
  l1.bias = m.lstm_b[1];
  l1.c = w.c + (long long)lanes * TB_PRED;
  l1.mask = w.mask;
  l1.out = w.hp;  // h1 -> the projector's input
  l1.ldo = TB_PRED;
  tb_epilogue& p0 = args.e[G_PRE0];
  p0.kind = TB_EPI_STORE;
  p0.out_dtype = TB_F32;
  p0.out = w.pre0;
  p0.ldo = 4 * TB_PRED;
  p0.bias = m.lstm_b[0];
  tb_epilogue& pj = args.e[G_PROJ];
  pj.kind = TB_EPI_JOINT_IN;
  pj.out_dtype = TB_BF16;
  pj.out = nullptr;  // dec itself is not needed again: PROJ recomputes it every iteration
  pj.ldo = TB_PRED;  // the gather's row stride
  pj.out2 = w.z;
  pj.ldo2 = TB_PRED;
  pj.bias = m.dec_proj_b;
  pj.gather = enc;
  pj.gather_row = w.erow;
  args.emb_gates = m.lstm0_emb;
  args.b0 = m.lstm_b[0];
  args.enc_off = enc_off;
  args.cap = cap;
  args.lanes = lanes;
  args.max_cap = max_cap;
  args.max_iters = max_cap;  // every lane stops after at most cap <= max_cap iterations
  if (max_cap > DECODE_MAX_ITERS) return TB_ERR_ARG;
  args.tokens = tokens;
  args.counts = counts;
  args.progress = nullptr;
  if (host_flag && cudaHostGetDevicePointer(reinterpret_cast<void**>(&args.progress), host_flag, 0) != cudaSuccess)
    return fail_cuda();
  args.err = err;

  // Row bounds: [0] = every lane, the rest zero until their iteration; barrier counter
  // and abort flag zero.
  if (cudaMemsetAsync(tokens, 0xff, (size_t)lanes * max_cap * sizeof(int), stream) != cudaSuccess ||
      cudaMemsetAsync(w.bounds, 0, (size_t)(max_cap + 1) * sizeof(int), stream) != cudaSuccess ||
      cudaMemsetAsync(w.m_cur, 0, 256, stream) != cudaSuccess ||
      cudaMemcpyAsync(w.bounds, &lanes, sizeof(int), cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return fail_cuda();

  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = DT_SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, decode_tc_kernel, args);
  return check_launch();
}

}  // namespace tb
