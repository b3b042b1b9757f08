// The z-streaming convolution's work split: which output planes of which brick columns each CTA computes.
// Plain integer arithmetic shared by the kernel's roles (they all walk the same sequence) and by a host
// build of the same functions that checks the split on the CPU.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__
#define __host__
#define __device__
#define __forceinline__ inline
#endif

namespace nnb {
namespace tc {

// A CTA's share of the output planes.  Whole columns first, in rounds: in round k CTA i takes column
// k * ncta + i from plane 0 to the last, so at any time the CTAs work on neighbouring columns at about the same
// depth, and the halo rows one CTA loads of its neighbours' columns are the rows those neighbours are loading
// (L2 hits instead of a second trip to DRAM).  The columns left after the last full round are split evenly as
// contiguous runs of their column-major, z-fastest plane sequence, so every CTA gets the same number of planes
// to within one.
struct ZsRun {
  int round, rounds;  // whole-column rounds taken / to take
  int64_t idx, end;   // then [idx, end) of the column-major, z-fastest output-plane sequence
};

struct ZsSegment {
  int col, z0, z1;  // output planes [z0, z1) of brick column col
  int ua, ub;       // input planes loaded: [ua, ub]
};

// total: brick columns x OD output planes of the launch; cta / ncta: this CTA and the grid size.
__host__ __device__ __forceinline__ ZsRun zs_run(int64_t total, int OD, int cta, int ncta) {
  const int64_t ncols = total / OD;
  const int rounds = (int)(ncols / ncta);
  const int64_t base = (int64_t)rounds * ncta * OD, tail = total - base;
  return ZsRun{0, rounds, base + tail * cta / ncta, base + tail * (cta + 1) / ncta};
}

// The CTA's next segment (one column's planes [z0, z1) and the input planes it loads); false when done.
__host__ __device__ __forceinline__ bool zs_next(ZsRun& r, ZsSegment& s, int OD, int ID, int cta, int ncta) {
  if (r.round < r.rounds) {
    s.col = r.round * ncta + cta;
    s.z0 = 0;
    s.z1 = OD;
    ++r.round;
  } else {
    if (r.idx >= r.end) return false;
    s.col = (int)(r.idx / OD);
    s.z0 = (int)(r.idx - (int64_t)s.col * OD);
    const int64_t stop = r.end < (int64_t)(s.col + 1) * OD ? r.end : (int64_t)(s.col + 1) * OD;
    s.z1 = s.z0 + (int)(stop - r.idx);
    r.idx = stop;
  }
  s.ua = s.z0 - 1 > 0 ? s.z0 - 1 : 0;
  s.ub = s.z1 < ID - 1 ? s.z1 : ID - 1;
  return true;
}

}  // namespace tc
}  // namespace nnb
