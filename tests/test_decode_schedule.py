"""The persistent decoder's work distribution checked on the host, with the code the kernel
runs (csrc/decode_tiles.cuh compiled into a host program): in every GEMM phase, for every
row count and grid size, each tile of each GEMM runs exactly once; a CTA's tiles come
without gaps (once it has none, it has no more); no tile is larger than the ring stage its
CTA cuts for the phase; with layer 1 split, its tile t runs on CTA t both in LSTM and in
the PROJ phase before it (the accumulator stays on that SM), as that CTA's last tile of
PROJ; and every next-P0 tile runs once, in LSTM or (the surplus beyond one per free CTA)
in PROJ."""

import shutil
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "tinybark_b200" / "csrc"

HARNESS = r"""
#include <cstdio>
#include <map>
#include <tuple>

#include "decode_tiles.cuh"

using namespace tb;

int main() {
  int bad = 0, checked = 0;
  const int grids[] = {148, 132, 100, 64};
  for (int G : grids)
    for (int split = 0; split < 2; ++split)
      for (int mtiles = 1; mtiles <= 10; ++mtiles)
        for (int part = 0; part < 2; ++part) {
          if (split && lstm1_tiles(mtiles * 128) >= G) continue;  // the host splits only below the grid
          const int rows = part ? mtiles * 128 - 77 : mtiles * 128;
          const int kinds[] = {P_JOINT, P_LSTM, P_PROJ};
          std::map<std::tuple<int, int, int>, int> pre0_seen;  // next-P0 tiles, in LSTM or PROJ
          for (int kind : kinds) {
            std::map<std::tuple<int, int, int>, int> seen;
            for (int cta = 0; cta < G; ++cta) {
              const int sg = phase_stage_gemm(kind, split, rows, cta, G);
              bool ended = false;
              int last = -1;
              for (int k = 0; k < 64; ++k) {
                int g = -1, mt = -1, nt = -1;
                if (!phase_tile(kind, rows, cta, G, k, split, g, mt, nt)) {
                  ended = true;
                  continue;
                }
                if (ended) ++bad, printf("G %d split %d rows %d kind %d cta %d: tile after a gap\n", G, split, rows, kind, cta);
                if (stage_bytes(g) > stage_bytes(sg))
                  ++bad, printf("G %d rows %d kind %d cta %d: gemm %d larger than the stage\n", G, rows, kind, cta, g);
                if (split && (g == G_LSTM1 || g == G_HH1) && mt * (gemm_n(G_LSTM1) / gemm_bn(G_LSTM1)) + nt != cta)
                  ++bad, printf("G %d rows %d kind %d: layer-1 tile (%d,%d) on cta %d\n", G, rows, kind, mt, nt, cta);
                if (last == G_HH1) ++bad, printf("G %d rows %d cta %d: a tile after the W_hh1 product\n", G, rows, cta);
                last = g;
                if (g == G_PRE0)
                  ++pre0_seen[std::make_tuple(g, mt, nt)];
                else
                  ++seen[std::make_tuple(g, mt, nt)];
              }
            }
            std::map<std::tuple<int, int, int>, int> want;
            auto add = [&](int g) {
              for (int mt = 0; mt < mtiles; ++mt)
                for (int nt = 0; nt < gemm_n(g) / gemm_bn(g); ++nt) want[std::make_tuple(g, mt, nt)] = 1;
            };
            if (kind == P_JOINT) add(G_JOINT);
            if (kind == P_LSTM) add(G_LSTM1);
            if (kind == P_PROJ) {
              add(G_PROJ);
              if (split) add(G_HH1);
            }
            if (seen != want)
              ++bad, printf("G %d split %d rows %d kind %d: %zu tiles run, %zu expected (or some twice)\n", G, split,
                            rows, kind, seen.size(), want.size());
            ++checked;
          }
          std::map<std::tuple<int, int, int>, int> pre0_want;
          for (int mt = 0; mt < mtiles; ++mt)
            for (int nt = 0; nt < gemm_n(G_PRE0) / gemm_bn(G_PRE0); ++nt) pre0_want[std::make_tuple(G_PRE0, mt, nt)] = 1;
          if (pre0_seen != pre0_want)
            ++bad, printf("G %d split %d rows %d: %zu next-P0 tiles run, %zu expected (or some twice)\n", G, split, rows,
                          pre0_seen.size(), pre0_want.size());
          // With the surplus P0 tiles moved into PROJ, no CTA runs two of them in LSTM.
          if (split && p0_in_proj(mtiles, G))
            for (int cta = 0; cta < G; ++cta) {
              int n0 = 0, g, mt, nt;
              for (int k = 0; k < 64; ++k)
                if (phase_tile(P_LSTM, rows, cta, G, k, split, g, mt, nt) && g == G_PRE0) ++n0;
              if (n0 > 1) ++bad, printf("G %d rows %d cta %d: %d next-P0 tiles in LSTM\n", G, rows, cta, n0);
            }
        }
  printf("checked %d phases, %d problems\n", checked, bad);
  return bad ? 1 : 0;
}
"""


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="needs nvcc (host code only; no GPU)")
def test_every_decoder_tile_runs_once_on_a_fitting_cta(tmp_path):
    src = tmp_path / "schedule.cu"
    src.write_text(HARNESS)
    exe = tmp_path / "schedule"
    subprocess.run(["nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I", str(CSRC), "-o",
                    str(exe), str(src)], check=True, capture_output=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0, run.stdout[-2000:]
    assert "0 problems" in run.stdout
