"""The z-streaming convolution's work split, checked on the CPU.

``csrc/zs_schedule.cuh`` decides which output planes of which brick columns each CTA computes; every role
of the kernel walks the same sequence, so a plane computed twice or never is a wrong result.  The header is
plain integer arithmetic, so a host build of it (g++) is run here over launch geometries of the benchmark
and test shapes and grid sizes, and checked: every (column, plane) exactly once, per-CTA plane counts
within one of each other, whole-column rounds first (CTA i takes column 148 k + i in round k on 148 SMs),
and the loaded input planes covering each segment's halo.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parent.parent / "nnunet-mlx_b200" / "csrc"

DRIVER = r"""
#include <cstdio>
#include <cstdlib>
#include <vector>
#include "zs_schedule.cuh"
using namespace nnb::tc;
int main(int argc, char** argv) {
  const int ncols = atoi(argv[1]), D = atoi(argv[2]), cap = atoi(argv[3]);
  const long long total = (long long)ncols * D;
  const int ncta = (int)(total < cap ? total : cap);
  std::vector<int> hits(total, 0);
  long long mn = 1LL << 62, mx = 0;
  int bad = 0;
  for (int cta = 0; cta < ncta; ++cta) {
    ZsRun r = zs_run(total, D, cta, ncta);
    ZsSegment s;
    long long planes = 0;
    int k = 0;
    while (zs_next(r, s, D, D, cta, ncta)) {
      if (s.col < 0 || s.col >= ncols || s.z0 < 0 || s.z1 > D || s.z0 >= s.z1) { ++bad; break; }
      if (s.ua != (s.z0 > 0 ? s.z0 - 1 : 0) || s.ub != (s.z1 < D ? s.z1 : D - 1)) ++bad;
      if (k < r.rounds && (s.col != k * ncta + cta || s.z0 != 0 || s.z1 != D)) ++bad;  // whole-column rounds
      for (int z = s.z0; z < s.z1; ++z) hits[(long long)s.col * D + z]++;
      planes += s.z1 - s.z0;
      ++k;
    }
    if (planes < mn) mn = planes;
    if (planes > mx) mx = planes;
  }
  for (int h : hits) if (h != 1) { ++bad; break; }
  if (mx - mn > 1) ++bad;
  printf("%d %lld %lld\n", bad, mn, mx);
  return 0;
}
"""

# (brick columns, output planes): 8 views of 128^3 (8 x 16 bricks -> 128 columns per view), one view, 64^3,
# the benchmark-size test shapes and small edge cases
GEOMETRIES = [(1024, 128), (128, 128), (2048, 128), (256, 64), (148, 4), (300, 9), (30, 5), (6, 40), (12, 4),
              (1, 1), (1, 7), (149, 3), (295, 17), (1036, 101)]


@pytest.fixture(scope="module")
def schedule_binary(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    d = tmp_path_factory.mktemp("zs")
    src = d / "zs_check.cpp"
    src.write_text(DRIVER)
    exe = d / "zs_check"
    subprocess.run([cxx, "-O1", "-std=c++17", f"-I{CSRC}", str(src), "-o", str(exe)], check=True)
    return exe


@pytest.mark.parametrize("cols,depth", GEOMETRIES)
@pytest.mark.parametrize("sms", [148, 132, 7, 1])
def test_every_plane_once_and_balanced(schedule_binary, cols, depth, sms):
    out = subprocess.run([str(schedule_binary), str(cols), str(depth), str(sms)], check=True,
                         capture_output=True, text=True).stdout.split()
    bad, lo, hi = (int(v) for v in out)
    assert bad == 0
    assert hi - lo <= 1
    assert lo + hi > 0
