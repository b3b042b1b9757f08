// Device restoration of class labels: trilinear (order-1, half-pixel grid,
// edge-clamped indices) resampling of class logits to the cropped original
// grid, first-argmax over classes, uncrop and inverse axis transpose, fused in
// one pass over the output label volume.  A streaming kernel: each warp owns
// output rows in output order (coalesced label stores), reads the corners of
// each class (neighbouring lanes share corners through L1 and L2), and does
// the interpolation in float64 with the host spline path's exact operation
// order, so the rounded values equal that path's bit for bit.
//
// Reference: the fused Metal restoration
// src/nnunet_mlx/kernels/metal_restore.py:71-139 (kernel), :462-495 (axis
// metadata), and the host order-1 spline path it reproduces,
// src/nnunet_mlx/data/resampling.py:476-502 (skimage resize -> scipy zoom,
// grid_mode, mode "nearest", float64), plus the uncrop + transpose_backward of
// src/nnunet_mlx/prediction/export.py:363-373.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"

namespace nnb {

struct RestoreGeometry {
  int32_t src[3];
  int32_t tgt[3];
  double ratio[3];     // S / T per axis, IEEE-divided on the host (Python's `source / target`)
  int64_t cstride;
  int64_t sstride[3];
  int32_t lo[3];       // crop box start
  int32_t out[3];      // output dims: vol[axes[i]]
  int32_t axes[3];
  int32_t classes;
  int32_t vec4;        // identity grid whose row axis is the logits' contiguous axis, rows 4-element aligned
};

// One axis of the half-pixel order-1 grid: c = (t + 0.5) * (S / T) - 0.5 with
// one rounding per operation (the products are not fused: __dmul_rn /
// __dsub_rn forbid contraction into an FMA), floor(c) and its right neighbour
// clamped into [0, S - 1] (mode "nearest"), weights (1 - f, f) with f = c - floor(c).
struct AxisTap {
  int i0, i1;
  double w0, w1;
};

__device__ __forceinline__ AxisTap axis_tap(int t, int size, double ratio) {
  const double c = __dsub_rn(__dmul_rn((double)t + 0.5, ratio), 0.5);
  const double f = floor(c);
  const int lo = (int)f;
  AxisTap a;
  a.w1 = __dsub_rn(c, f);
  a.w0 = __dsub_rn(1.0, a.w1);
  a.i0 = min(max(lo, 0), size - 1);
  a.i1 = min(max(lo + 1, 0), size - 1);
  return a;
}

// One rounding of the float64 interpolant to the logits' precision (round to
// nearest even, directly from float64), returned as the float it compares as.
template <typename In>
__device__ __forceinline__ float round_to_input(double v);

template <>
__device__ __forceinline__ float round_to_input<float>(double v) {
  return __double2float_rn(v);
}

template <>
__device__ __forceinline__ float round_to_input<__half>(double v) {
  return __half2float(__double2half(v));
}

constexpr int kSmallClasses = 4;    // identity grids with up to this many classes: all loads of a step in flight
constexpr int kIdentityVoxels = 8;  // voxels per lane per step on an identity grid

template <typename In>
__device__ __forceinline__ float load_raw(const In* p, int64_t i);

template <>
__device__ __forceinline__ float load_raw<float>(const float* p, int64_t i) {
  return __ldg(p + i);
}

template <>
__device__ __forceinline__ float load_raw<__half>(const __half* p, int64_t i) {
  return __half2float(__ldg(p + i));
}

// v[i] for a runtime i in 0..2 without indexing a parameter array (which would
// copy the whole parameter block to local memory).
__device__ __forceinline__ int sel3(const int32_t (&v)[3], int i) { return i == 0 ? v[0] : (i == 1 ? v[1] : v[2]); }
__device__ __forceinline__ int64_t sel3(const int64_t (&v)[3], int i) {
  return i == 0 ? v[0] : (i == 1 ? v[1] : v[2]);
}

// First-maximum update of a running argmax; non-finite values mark the voxel invalid.
__device__ __forceinline__ void argmax_step(float value, int c, float& best, int& winner, bool& invalid) {
  invalid |= !isfinite(value);
  if (c == 0 || value > best) {
    best = value;
    winner = c;
  }
}

// Four consecutive logits of one class along a contiguous row whose address is
// 16-byte (float) or 8-byte (half) aligned, as floats.
template <typename In>
__device__ __forceinline__ void load4(const In* p, float (&v)[4]);

template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  const float4 q = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = q.x, v[1] = q.y, v[2] = q.z, v[3] = q.w;
}

template <>
__device__ __forceinline__ void load4<__half>(const __half* p, float (&v)[4]) {
  const uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
  v[0] = __half2float(__ushort_as_half((unsigned short)(q.x & 0xFFFFu)));
  v[1] = __half2float(__ushort_as_half((unsigned short)(q.x >> 16)));
  v[2] = __half2float(__ushort_as_half((unsigned short)(q.y & 0xFFFFu)));
  v[3] = __half2float(__ushort_as_half((unsigned short)(q.y >> 16)));
}

// One identity-grid row read with 4-element vector loads (g.vec4): the crop's
// `extent` voxels start at element `rowbase` (class 0) and land at output
// positions x_lo + x.  Each lane takes 2 x 4 consecutive voxels per step; the
// extent's last (extent % 4) voxels are read one by one.  Returns the row's
// count of non-finite voxels.
template <int CS, typename In, typename LabelT>
__device__ __forceinline__ int identity_row_vec(const In* __restrict__ logits, const RestoreGeometry& g,
                                                LabelT* __restrict__ row, int lane, int64_t rowbase, int extent,
                                                int x_lo, LabelT invalid_label) {
  constexpr int U = 2;
  const int nvec = extent >> 2;
  int invalid_voxels = 0;
  for (int o2 = lane; o2 < x_lo; o2 += 32) row[o2] = (LabelT)0;
  for (int o2 = x_lo + extent + lane; o2 < g.out[2]; o2 += 32) row[o2] = (LabelT)0;
  for (int kb = lane; kb < nvec; kb += 32 * U) {
    float best[U][4];
    int winner[U][4];
    bool invalid[U][4];
    int vx[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      vx[u] = 4 * min(kb + 32 * u, nvec - 1);  // a step past the row re-reads its last vector
#pragma unroll
      for (int j = 0; j < 4; ++j) best[u][j] = 0.f, winner[u][j] = 0, invalid[u][j] = false;
    }
    if constexpr (CS > 0) {
      float val[U][CS][4];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int c = 0; c < CS; ++c) load4<In>(logits + rowbase + min(c, g.classes - 1) * g.cstride + vx[u], val[u][c]);
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int c = 0; c < CS; ++c)
          if (c < g.classes)
#pragma unroll
            for (int j = 0; j < 4; ++j) argmax_step(val[u][c][j], c, best[u][j], winner[u][j], invalid[u][j]);
    } else {
      for (int c = 0; c < g.classes; ++c) {
        float val[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) load4<In>(logits + rowbase + c * g.cstride + vx[u], val[u]);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int j = 0; j < 4; ++j) argmax_step(val[u][j], c, best[u][j], winner[u][j], invalid[u][j]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (kb + 32 * u >= nvec) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        row[x_lo + vx[u] + j] = invalid[u][j] ? invalid_label : (LabelT)winner[u][j];
        invalid_voxels += invalid[u][j] ? 1 : 0;
      }
    }
  }
  for (int x = 4 * nvec + lane; x < extent; x += 32) {
    float best = 0.f;
    int winner = 0;
    bool invalid = false;
    for (int c = 0; c < g.classes; ++c)
      argmax_step(load_raw<In>(logits, rowbase + c * g.cstride + x), c, best, winner, invalid);
    row[x_lo + x] = invalid ? invalid_label : (LabelT)winner;
    invalid_voxels += invalid ? 1 : 0;
  }
  return invalid_voxels;
}

// ---------------------------------------------------------------------------
// Identity grid (source == target on every axis): the interpolant of a voxel is
// its own logit exactly (weights 1 and 0), so the label is the first argmax of
// the logits -- no float64 work.  Each lane takes kIdentityVoxels voxels of its
// warp's row per step, all their class loads in flight together.
// ---------------------------------------------------------------------------
template <int CS, typename In, typename LabelT>
__global__ void __launch_bounds__(256) restore_identity_kernel(const In* __restrict__ logits, RestoreGeometry g,
                                                                LabelT* __restrict__ labels,
                                                                int32_t* __restrict__ invalid_count,
                                                                LabelT invalid_label) {
  constexpr int V = kIdentityVoxels;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)g.out[0] * g.out[1];
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int a0 = g.axes[0], a1 = g.axes[1], a2 = g.axes[2];
  const int64_t row_step = sel3(g.sstride, a2);
  const int x_lo = sel3(g.lo, a2), x_hi = x_lo + sel3(g.tgt, a2);
  int local_invalid = 0;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int o0 = (int)(r / g.out[1]);
    const int o1 = (int)(r - (int64_t)o0 * g.out[1]);
    LabelT* row = labels + r * g.out[2];
    const int t0 = o0 - sel3(g.lo, a0), t1 = o1 - sel3(g.lo, a1);
    if (!(t0 >= 0 && t0 < sel3(g.tgt, a0) && t1 >= 0 && t1 < sel3(g.tgt, a1))) {
      for (int o2 = lane; o2 < g.out[2]; o2 += 32) row[o2] = (LabelT)0;
      continue;
    }
    if (g.vec4) {
      local_invalid += identity_row_vec<CS, In, LabelT>(logits, g, row, lane,
                                                        t0 * sel3(g.sstride, a0) + t1 * sel3(g.sstride, a1),
                                                        x_hi - x_lo, x_lo, invalid_label);
      continue;
    }
    const int64_t base = t0 * sel3(g.sstride, a0) + t1 * sel3(g.sstride, a1) - (int64_t)x_lo * row_step;
    for (int ob = lane; ob < g.out[2]; ob += 32 * V) {
      float best[V];
      int winner[V];
      bool invalid[V], inside[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int o2 = ob + 32 * v;
        inside[v] = o2 >= x_lo && o2 < x_hi;
        best[v] = 0.f;
        winner[v] = 0;
        invalid[v] = false;
      }
      // every address stays inside the logits (position clamped into the crop,
      // class into range); the value of a clamped load is never used
      int64_t pos[V];
#pragma unroll
      for (int v = 0; v < V; ++v) pos[v] = base + (int64_t)min(max(ob + 32 * v, x_lo), x_hi - 1) * row_step;
      if constexpr (CS > 0) {
        float val[V][CS];
#pragma unroll
        for (int v = 0; v < V; ++v)
#pragma unroll
          for (int c = 0; c < CS; ++c) {
            const float x = load_raw<In>(logits, pos[v] + min(c, g.classes - 1) * g.cstride);
            val[v][c] = (inside[v] && c < g.classes) ? x : 0.f;
          }
#pragma unroll
        for (int v = 0; v < V; ++v)
#pragma unroll
          for (int c = 0; c < CS; ++c)
            if (c < g.classes) argmax_step(val[v][c], c, best[v], winner[v], invalid[v]);
      } else {
        for (int c = 0; c < g.classes; ++c) {
          float val[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float x = load_raw<In>(logits, pos[v] + c * g.cstride);
            val[v] = inside[v] ? x : 0.f;
          }
#pragma unroll
          for (int v = 0; v < V; ++v) argmax_step(val[v], c, best[v], winner[v], invalid[v]);
        }
      }
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int o2 = ob + 32 * v;
        if (o2 >= g.out[2]) break;
        if (!inside[v]) {
          row[o2] = (LabelT)0;
        } else {
          row[o2] = invalid[v] ? invalid_label : (LabelT)winner[v];
          local_invalid += invalid[v] ? 1 : 0;
        }
      }
    }
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

// ---------------------------------------------------------------------------
// Resampling grid.  An axis whose upper weight is exactly 0 (every index of an
// axis that is not resampled) drops out of a voxel's sum: its lower weight is
// exactly 1 and the dropped corners contribute +-0, so the sum equals the host
// path's eight-corner sum for finite logits.  A dropped corner is never read:
// a non-finite value there (which the host sum would turn into NaN, 0 * inf,
// and flag invalid) leaves this voxel's label finite and uncounted.  Finite
// logits are the contract here as in the reference's fused path (reference
// kernels/metal_restore.py:298-316 validates them before its launch).  Each of the 8 patterns of active axes has its own
// unrolled code (Z1, Y1, X1), so only the needed corners are loaded and
// multiplied; within a warp the pattern is nearly always uniform.
// ---------------------------------------------------------------------------

// The interpolant of one class: the corners' float64 terms ((v * w_0) * w_1) *
// w_2 (active axes only, one rounding per operation) summed in (axis 0, axis 1,
// axis 2) binary corner order, axis 2 fastest, rounded to the logits' dtype.
template <bool Z1, bool Y1, bool X1, typename In>
__device__ __forceinline__ float interpolant(const In* __restrict__ p, const int64_t (&zo)[2], const int64_t (&yo)[2],
                                             const int64_t (&xo)[2], const double (&wz)[2], const double (&wy)[2],
                                             const double (&wx)[2]) {
  constexpr int NZ = Z1 ? 2 : 1, NY = Y1 ? 2 : 1, NX = X1 ? 2 : 1;
  float raw[NZ][NY][NX];
#pragma unroll
  for (int bz = 0; bz < NZ; ++bz)
#pragma unroll
    for (int by = 0; by < NY; ++by)
#pragma unroll
      for (int bx = 0; bx < NX; ++bx) raw[bz][by][bx] = load_raw<In>(p, zo[bz] + yo[by] + xo[bx]);
  double s = 0.0;
#pragma unroll
  for (int bz = 0; bz < NZ; ++bz)
#pragma unroll
    for (int by = 0; by < NY; ++by)
#pragma unroll
      for (int bx = 0; bx < NX; ++bx) {
        double term = (double)raw[bz][by][bx];
        if (Z1) term = __dmul_rn(term, wz[bz]);
        if (Y1) term = __dmul_rn(term, wy[by]);
        if (X1) term = __dmul_rn(term, wx[bx]);
        s = __dadd_rn(s, term);
      }
  return round_to_input<In>(s);
}

template <bool Z1, bool Y1, bool X1, typename In>
__device__ __forceinline__ void classify(const In* __restrict__ logits, int classes, int64_t cstride,
                                         const int64_t (&zo)[2], const int64_t (&yo)[2], const int64_t (&xo)[2],
                                         const double (&wz)[2], const double (&wy)[2], const double (&wx)[2],
                                         float& best, int& winner, bool& invalid) {
  for (int c = 0; c < classes; ++c)
    argmax_step(interpolant<Z1, Y1, X1, In>(logits + c * cstride, zo, yo, xo, wz, wy, wx), c, best, winner,
                invalid);
}

// One output row whose voxels step along volume axis RA; the taps of the two
// other volume axes (crop coordinates c_a, c_b in increasing axis order) are
// fixed for the row.  Returns the row's count of non-finite voxels.
template <int RA, typename In, typename LabelT>
__device__ __forceinline__ int restore_row(const In* __restrict__ logits, const RestoreGeometry g,
                                           LabelT* __restrict__ row, int lane, int c_a, int c_b,
                                           LabelT invalid_label) {
  constexpr int A = RA == 0 ? 1 : 0;  // the two row-constant volume axes, A < B
  constexpr int B = RA == 2 ? 1 : 2;
  const AxisTap ta = axis_tap(c_a, g.src[A], g.ratio[A]);
  const AxisTap tb = axis_tap(c_b, g.src[B], g.ratio[B]);
  const int64_t ao[2] = {ta.i0 * g.sstride[A], ta.i1 * g.sstride[A]};
  const int64_t bo[2] = {tb.i0 * g.sstride[B], tb.i1 * g.sstride[B]};
  const double aw[2] = {ta.w0, ta.w1}, bw[2] = {tb.w0, tb.w1};
  const int x_lo = g.lo[RA], x_hi = g.lo[RA] + g.tgt[RA];  // crop extent along the row
  int invalid_voxels = 0;
  for (int o2 = lane; o2 < g.out[2]; o2 += 32) {
    if (o2 < x_lo || o2 >= x_hi) {
      row[o2] = (LabelT)0;
      continue;
    }
    const AxisTap tv = axis_tap(o2 - x_lo, g.src[RA], g.ratio[RA]);
    const int64_t vo[2] = {tv.i0 * g.sstride[RA], tv.i1 * g.sstride[RA]};
    const double vw[2] = {tv.w0, tv.w1};
    // offsets and weights by volume axis 0, 1, 2
    const int64_t(&zo)[2] = RA == 0 ? vo : ao;
    const int64_t(&yo)[2] = RA == 1 ? vo : (RA == 0 ? ao : bo);
    const int64_t(&xo)[2] = RA == 2 ? vo : bo;
    const double(&wz)[2] = RA == 0 ? vw : aw;
    const double(&wy)[2] = RA == 1 ? vw : (RA == 0 ? aw : bw);
    const double(&wx)[2] = RA == 2 ? vw : bw;
    const int pattern = (wz[1] != 0.0 ? 4 : 0) | (wy[1] != 0.0 ? 2 : 0) | (wx[1] != 0.0 ? 1 : 0);
    float best = 0.f;
    int winner = 0;
    bool invalid = false;
    const int C = g.classes;
    const int64_t cs = g.cstride;
    switch (pattern) {
      case 0: classify<false, false, false, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 1: classify<false, false, true, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 2: classify<false, true, false, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 3: classify<false, true, true, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 4: classify<true, false, false, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 5: classify<true, false, true, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      case 6: classify<true, true, false, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
      default: classify<true, true, true, In>(logits, C, cs, zo, yo, xo, wz, wy, wx, best, winner, invalid); break;
    }
    row[o2] = invalid ? invalid_label : (LabelT)winner;
    invalid_voxels += invalid ? 1 : 0;
  }
  return invalid_voxels;
}

// One output row (the fastest output axis, volume axis axes[2]) per warp,
// lanes stepping along it: no per-voxel integer division, and the taps of the
// row's two other volume axes are computed once per row.
template <typename In, typename LabelT>
__global__ void __launch_bounds__(256, 3) restore_resample_kernel(const In* __restrict__ logits, RestoreGeometry g,
                                                                LabelT* __restrict__ labels,
                                                                int32_t* __restrict__ invalid_count,
                                                                LabelT invalid_label) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)g.out[0] * g.out[1];
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int a0 = g.axes[0], a1 = g.axes[1], a2 = g.axes[2];
  int local_invalid = 0;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int o0 = (int)(r / g.out[1]);
    const int o1 = (int)(r - (int64_t)o0 * g.out[1]);
    LabelT* row = labels + r * g.out[2];
    // crop coordinates of the two row-constant volume axes
    const int t0 = o0 - sel3(g.lo, a0), t1 = o1 - sel3(g.lo, a1);
    if (!(t0 >= 0 && t0 < sel3(g.tgt, a0) && t1 >= 0 && t1 < sel3(g.tgt, a1))) {
      for (int o2 = lane; o2 < g.out[2]; o2 += 32) row[o2] = (LabelT)0;
      continue;
    }
    // the row-constant crop coordinates in increasing volume-axis order
    const int c_a = a0 < a1 ? t0 : t1, c_b = a0 < a1 ? t1 : t0;
    if (a2 == 2)
      local_invalid += restore_row<2, In, LabelT>(logits, g, row, lane, c_a, c_b, invalid_label);
    else if (a2 == 1)
      local_invalid += restore_row<1, In, LabelT>(logits, g, row, lane, c_a, c_b, invalid_label);
    else
      local_invalid += restore_row<0, In, LabelT>(logits, g, row, lane, c_a, c_b, invalid_label);
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

template <int CS, typename In, typename LabelT>
static void launch_restore_typed(const void* logits, const RestoreGeometry& g, bool identity, void* labels,
                                 int32_t* invalid_count, int blocks, cudaStream_t stream) {
  const In* in = static_cast<const In*>(logits);
  LabelT* out = static_cast<LabelT*>(labels);
  const LabelT invalid = (LabelT)~(LabelT)0;
  if (identity)
    restore_identity_kernel<CS, In, LabelT><<<blocks, 256, 0, stream>>>(in, g, out, invalid_count, invalid);
  else
    restore_resample_kernel<In, LabelT><<<blocks, 256, 0, stream>>>(in, g, out, invalid_count, invalid);
}

template <typename In, typename LabelT>
static void launch_restore_classes(const void* logits, const RestoreGeometry& g, bool identity, void* labels,
                                   int32_t* invalid_count, int blocks, cudaStream_t stream) {
  if (identity && g.classes <= kSmallClasses)
    launch_restore_typed<kSmallClasses, In, LabelT>(logits, g, identity, labels, invalid_count, blocks, stream);
  else
    launch_restore_typed<0, In, LabelT>(logits, g, identity, labels, invalid_count, blocks, stream);
}

int launch_restore_labels(const nnb_restore_args& a, cudaStream_t stream) {
  RestoreGeometry g;
  for (int i = 0; i < 3; ++i) {
    g.src[i] = a.source_dims[i];
    g.tgt[i] = a.target_dims[i];
    g.ratio[i] = (double)a.source_dims[i] / (double)a.target_dims[i];
    g.sstride[i] = a.source_strides[i];
    g.lo[i] = a.crop_lo[i];
    g.axes[i] = a.axes[i];
  }
  for (int i = 0; i < 3; ++i) g.out[i] = a.volume_dims[a.axes[i]];
  g.cstride = a.class_stride;
  g.classes = a.classes;
  bool identity = true;
  for (int i = 0; i < 3; ++i) identity &= a.source_dims[i] == a.target_dims[i];
  // vector rows: the row axis is contiguous and every row start (any class) is 4-element aligned
  const int row_axis = a.axes[2];
  bool aligned = a.source_strides[row_axis] == 1 && a.class_stride % 4 == 0 &&
                 ((uintptr_t)a.logits % (a.half ? 8 : 16)) == 0;
  for (int i = 0; i < 3; ++i)
    if (i != row_axis) aligned &= a.source_strides[i] % 4 == 0;
  g.vec4 = identity && aligned ? 1 : 0;
  const int64_t rows = (int64_t)g.out[0] * g.out[1];
  const int blocks = (int)std::min<int64_t>((rows + 7) / 8, 148 * 8);  // 8 warps (rows) per block
  NNB_CUDA_CHECK(cudaMemsetAsync(a.invalid_count, 0, sizeof(int32_t), stream));
  if (a.half) {
    if (a.label_bytes == 1)
      launch_restore_classes<__half, uint8_t>(a.logits, g, identity, a.labels, a.invalid_count, blocks, stream);
    else
      launch_restore_classes<__half, uint16_t>(a.logits, g, identity, a.labels, a.invalid_count, blocks, stream);
  } else {
    if (a.label_bytes == 1)
      launch_restore_classes<float, uint8_t>(a.logits, g, identity, a.labels, a.invalid_count, blocks, stream);
    else
      launch_restore_classes<float, uint16_t>(a.logits, g, identity, a.labels, a.invalid_count, blocks, stream);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

}  // namespace nnb
