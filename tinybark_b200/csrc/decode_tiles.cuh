// Work distribution of the persistent decoder (decode_tc.cu): the GEMMs of its phases,
// their tile sizes, which CTA runs which tile, and how each CTA cuts its shared-memory
// ring in a phase. Host and device code: the kernel uses it, and a host test checks that
// every tile of every phase runs exactly once and fits the ring stage of its CTA.
#pragma once

#include "../../include/tbcuda.h"

namespace tb {
namespace {

constexpr int DT_A_BYTES = 128 * 64 * 2;
constexpr int DT_RING_BYTES = 4 * (DT_A_BYTES + 256 * 64 * 2);  // 4 stages of the widest (joint) tiles
enum { G_JOINT = 0, G_LSTM1 = 1, G_PRE0 = 2, G_PROJ = 3, G_HH1 = 4 };
enum { P_INIT = 0, P_CELL = 1, P_JOINT = 2, P_LSTM = 3, P_PROJ = 4 };
__host__ __device__ constexpr int gemm_n(int g) { return g == G_JOINT ? TB_JOINT_ROWS : (g == G_PROJ ? TB_PRED : 4 * TB_PRED); }
__host__ __device__ constexpr int gemm_k(int g, int split) { return g == G_LSTM1 && !split ? 2 * TB_PRED : TB_PRED; }
__host__ __device__ constexpr int gemm_bn(int g) { return g == G_JOINT ? 256 : (g == G_PROJ ? 64 : 128); }
// Layer 1's tiles for `rows` lanes (mtiles x 20); the split needs them one per SM.
__host__ __device__ constexpr int lstm1_tiles(int rows) { return (rows + 127) / 128 * (4 * TB_PRED / 128); }
// The shared-memory ring is re-cut at every GEMM phase into as many stages of that
// phase's tile size as fit (4 x 48 KB joint, 6 x 32 KB LSTM and split PROJ, 8 x 24 KB
// projector): the narrower the tiles, the deeper the pipeline. Before a re-cut the
// producer waits until the MMAs have released every stage of the previous cut (only the
// W_hh1 product, which has no epilogue, can still be running then).
__host__ __device__ constexpr int stage_bytes(int g) { return DT_A_BYTES + gemm_bn(g) * 64 * 2; }
__host__ __device__ constexpr int ring_slots(int g) {
  return DT_RING_BYTES / stage_bytes(g) < 8 ? DT_RING_BYTES / stage_bytes(g) : 8;
}

struct Phase {
  int kind;  // P_*
  int iter;  // greedy-loop iteration (-1 for the first prediction step)
};

__host__ __device__ __forceinline__ Phase phase_of(int q) {
  if (q == 0) return {P_INIT, -1};
  if (q < 4) return {q == 1 ? P_CELL : (q == 2 ? P_LSTM : P_PROJ), -1};
  const int i = (q - 4) / 4, r = (q - 4) % 4;
  return {r == 0 ? P_JOINT : (r == 1 ? P_CELL : (r == 2 ? P_LSTM : P_PROJ)), i};
}

// Split layer 1 with more next-P0 tiles than CTAs left over in LSTM: the P0 tiles beyond
// one per free CTA run in PROJ instead, on the CTAs past the projector's tiles (P0 reads h0,
// which CELL wrote, and is read in the next CELL), so no CTA runs two of them in LSTM.
__host__ __device__ constexpr bool p0_in_proj(int mtiles, int G) {
  return G - mtiles * 20 > 0 && mtiles * 20 > G - mtiles * 20 &&
         mtiles * 20 - (G - mtiles * 20) <= (G - mtiles * 20) - mtiles * 10;
}

// The k-th GEMM tile of this CTA in a phase, as (gemm, m tile, n tile); false if none.
// JOINT and PROJ: tile t = cta + k * gridDim. LSTM: layer 1's tiles (the critical path)
// go one per CTA, and the next-P0 tiles (half the work each) to the CTAs left over, at
// most two per CTA; with too few CTAs left, both lists are dealt round-robin.
// Split layer 1: layer 1's tile t always runs on CTA t, in LSTM and, for its h1 half,
// in the PROJ before it (so the accumulator stays on that SM); the projector's tiles
// then start at CTA t1 and the next-P0 tiles are dealt to CTAs t1 and up.
__host__ __device__ __forceinline__ bool phase_tile(int kind, int rows, int cta, int G, int k, int split, int& g, int& mt,
                                           int& nt) {
  const int mtiles = (rows + 127) / 128;
  const int ntc = gemm_n(G_LSTM1) / gemm_bn(G_LSTM1), t1 = mtiles * ntc, free = G - t1;
  int t;
  if (kind == P_JOINT || (kind == P_PROJ && !split)) {
    g = kind == P_JOINT ? G_JOINT : G_PROJ;
    const int nc = gemm_n(g) / gemm_bn(g);
    t = cta + k * G;
    if (t >= mtiles * nc) return false;
    mt = t / nc;
    nt = t % nc;
    return true;
  }
  if (kind == P_PROJ) {
    const int nc = gemm_n(G_PROJ) / gemm_bn(G_PROJ), pt = mtiles * nc;
    const int base = (cta - t1 % G + G) % G;  // this CTA's first projector tile
    const int np = base < pt ? (pt - 1 - base) / G + 1 : 0;
    if (k < np) {
      g = G_PROJ;
      t = base + k * G;
      mt = t / nc;
      nt = t % nc;
      return true;
    }
    if (p0_in_proj(mtiles, G) && cta >= t1 + pt && cta < t1 + pt + (t1 - free)) {
      if (k != np) return false;
      g = G_PRE0;
      t = free + (cta - t1 - pt);
    } else {
      if (k > np || cta >= t1) return false;
      g = G_HH1;
      t = cta;
    }
  } else if (split) {
    if (cta < t1) {
      if (k > 0) return false;
      g = G_LSTM1;
      t = cta;
    } else {
      t = (cta - t1) + k * free;
      if (t >= (p0_in_proj(mtiles, G) ? free : t1)) return false;
      g = G_PRE0;
    }
  } else if (free > 0 && (t1 + free - 1) / free <= 2) {
    if (cta < t1) {
      if (k > 0) return false;
      g = G_LSTM1;
      t = cta;
    } else {
      t = (cta - t1) + k * free;
      if (t >= t1) return false;
      g = G_PRE0;
    }
  } else {
    t = cta + k * G;
    if (t >= 2 * t1) return false;
    g = t < t1 ? G_LSTM1 : G_PRE0;
    if (t >= t1) t -= t1;
  }
  mt = t / ntc;
  nt = t % ntc;
  return true;
}

// The ring's stage size for this CTA in a GEMM phase (both LSTM-phase GEMMs have
// BN = 128, and so have the W_hh1 product that joins the projector's phase, on CTAs below
// layer 1's tile count, when layer 1 is split, and next-P0 tiles moved into that phase).
__host__ __device__ __forceinline__ int phase_stage_gemm(int kind, int split, int rows, int cta, int G) {
  if (kind == P_JOINT) return G_JOINT;
  if (kind == P_PROJ) {
    const int mtiles = (rows + 127) / 128, t1 = lstm1_tiles(rows);
    if (split && cta < t1) return G_HH1;
    if (split && p0_in_proj(mtiles, G) && cta >= t1 + mtiles * 10) return G_PRE0;  // BN = 128 tiles
    return G_PROJ;
  }
  return G_LSTM1;
}

// The A-operand descriptor of GEMM g. With layer 1 split, layer 1 and the next-P0 GEMM
// read the same x1 columns, and the W_hh1 product and the projector the same hp: they
// share one descriptor, so fewer descriptors compete for the TMA unit's cache.
__host__ __device__ __forceinline__ int a_map(int g, int split) {
  if (!split) return g;
  return g == G_LSTM1 ? G_PRE0 : (g == G_HH1 ? G_PROJ : g);
}


}  // namespace
}  // namespace tb
