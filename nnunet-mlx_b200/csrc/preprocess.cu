// Raw-case preprocessing on the device: nonzero bounding box, hole filling of
// the nonzero mask, fused transpose + crop + per-channel normalisation,
// upstream's torch-grid resampler (image values and labels), and the spline
// resampler of nnU-Net's default plans (edge padding, cubic B-spline
// prefilter, order-1/3 sampling on the half-pixel grid, the out-of-plane
// order-0 pass of separate-axis resampling).  The streaming kernels give one
// warp to each row of their output (row coordinates and the outer axes'
// interpolation taps from one division per row, coalesced loads and stores
// along the row), the plans' transpose is folded into the source strides, and
// partial reductions are combined by warp shuffles and per-block shared memory
// before their atomics.  The C entry points (declared in include/nnb.h)
// validate their arguments here and allocate nothing.
//
// Reference: src/nnunet_mlx/data/preprocessing.py:60-163 (step order),
// :166-217 (crop_to_nonzero), :222-319 (normalisation), :340-343 (hole filling
// via scipy); src/nnunet_mlx/kernels/metal_torch_resample.py:51-131 (torch-grid
// kernel), :154-216 (launch and separate-axis composition);
// src/nnunet_mlx/data/resampling.py:87-172, 175-244 (policy), 268-306 and
// 379-427 (separate-axis spline path), 476-502 (skimage resize = scipy zoom).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <climits>
#include <type_traits>
#include <stdint.h>

#include "common.cuh"

namespace nnb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxChannels = 32;

int grid_for(int64_t n, int per_sm = 16) {
  int64_t blocks = (n + kThreads - 1) / kThreads;
  const int64_t cap = 148LL * per_sm;
  if (blocks > cap) blocks = cap;
  return (int)(blocks < 1 ? 1 : blocks);
}

template <typename T>
__device__ __forceinline__ float as_f32(T v) { return (float)v; }

// Whether a raw value is nonzero after conversion to float32, counting values
// that are not finite after it.  Integers convert exactly and are finite, so
// they are tested directly.
template <typename T>
__device__ __forceinline__ bool nonzero_f32(T v, int& bad) {
  if constexpr (std::is_integral<T>::value) {
    return v != 0;
  } else {
    const float f = (float)v;
    bad += isfinite(f) ? 0 : 1;
    return f != 0.f;
  }
}

// Where the raw case is and how the plans' axes map onto it.
struct RawView {
  const void* data;
  int64_t cstride;        // elements per channel (R0 R1 R2)
  int64_t pstride[3];     // raw element stride of plans axis i
  int32_t pdims[3];       // plans-order dims
  int32_t rdims[3];
  int32_t tr[3];          // plans axis i = raw axis tr[i]
  int32_t channels;
};

RawView make_view(const nnb_raw_case& r) {
  RawView v;
  v.data = r.data;
  v.channels = r.channels;
  const int64_t rs[3] = {(int64_t)r.raw_dims[1] * r.raw_dims[2], (int64_t)r.raw_dims[2], 1};
  v.cstride = (int64_t)r.raw_dims[0] * r.raw_dims[1] * r.raw_dims[2];
  for (int i = 0; i < 3; ++i) {
    v.rdims[i] = r.raw_dims[i];
    v.tr[i] = r.transpose[i];
    v.pstride[i] = rs[r.transpose[i]];
    v.pdims[i] = r.raw_dims[r.transpose[i]];
  }
  return v;
}

// Order-preserving int key of a float (signed comparison), and its inverse.
__device__ __forceinline__ int float_key(float f) {
  const int k = __float_as_int(f);
  return k >= 0 ? k : k ^ 0x7fffffff;
}
__device__ __forceinline__ float key_float(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff); }

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_double(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---- nonzero bounding box -------------------------------------------------

__global__ void bounds_init_kernel(int32_t* bounds) {
  if (threadIdx.x < 8) bounds[threadIdx.x] = threadIdx.x < 3 ? INT_MAX : (threadIdx.x < 6 ? -1 : 0);
}

// One warp per raw row (R0, R1 fixed, R2 along the lanes): the row's two
// outer coordinates come from one division per row, the lanes read the row
// with 16-byte vectors when it is 16-byte aligned (else coalesced scalars),
// and each channel is tested after conversion to float32 (the reference's
// mask is taken on the float32 transposed array).  Bounds are kept per raw
// axis and stored per plans axis.
template <typename T>
__global__ void __launch_bounds__(kThreads, 5) nonzero_bounds_kernel(RawView v, int vec, int32_t* bounds) {
  const T* data = static_cast<const T*>(v.data);
  const int lane = threadIdx.x & 31;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t rows = (int64_t)v.rdims[0] * v.rdims[1];
  const int len = v.rdims[2];
  int lo[3] = {INT_MAX, INT_MAX, INT_MAX}, hi[3] = {-1, -1, -1};
  int bad = 0;
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const int64_t base = row * len;
    int rlo = INT_MAX, rhi = -1;
    if (vec) {
      constexpr int N = 16 / sizeof(T);
      constexpr int kBatch = 4;
      const int chunks = len / N;
      for (int j0 = 0; j0 < chunks; j0 += 32 * kBatch) {
        unsigned mask[kBatch] = {};  // bit k: element k of the chunk is nonzero in some channel
        for (int c = 0; c < v.channels; ++c) {
          uint4 q[kBatch];
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int j = j0 + u * 32 + lane;
            q[u] = j < chunks ? *reinterpret_cast<const uint4*>(data + c * v.cstride + base + (int64_t)j * N)
                              : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            T e[N];
            memcpy(e, &q[u], 16);
#pragma unroll
            for (int k = 0; k < N; ++k) mask[u] |= (unsigned)nonzero_f32(e[k], bad) << k;
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (mask[u]) {
            const int j = j0 + u * 32 + lane;
            rlo = min(rlo, j * N + __ffs(mask[u]) - 1);
            rhi = max(rhi, j * N + 31 - __clz(mask[u]));
          }
        }
      }
    } else {
#pragma unroll 4
      for (int i = lane; i < len; i += 32) {
        bool nz = false;
        for (int c = 0; c < v.channels; ++c) nz |= nonzero_f32(data[c * v.cstride + base + i], bad);
        if (nz) {
          rlo = min(rlo, i);
          rhi = max(rhi, i);
        }
      }
    }
    rlo = __reduce_min_sync(0xffffffffu, rlo);
    rhi = __reduce_max_sync(0xffffffffu, rhi);
    if (rhi >= 0) {
      const int r0 = (int)(row / v.rdims[1]);
      const int r1 = (int)(row - (int64_t)r0 * v.rdims[1]);
      lo[0] = min(lo[0], r0);
      hi[0] = max(hi[0], r0);
      lo[1] = min(lo[1], r1);
      hi[1] = max(hi[1], r1);
      lo[2] = min(lo[2], rlo);
      hi[2] = max(hi[2], rhi);
    }
  }
  // combine the block's warps in shared memory, then one set of atomics per block
  __shared__ int part[kThreads / 32][7];
  bad = warp_sum_int(bad);
  const int warp_in_block = threadIdx.x >> 5;
  if (lane == 0) {
    for (int r = 0; r < 3; ++r) {
      part[warp_in_block][r] = lo[r];
      part[warp_in_block][3 + r] = hi[r];
    }
    part[warp_in_block][6] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int blo[3] = {INT_MAX, INT_MAX, INT_MAX}, bhi[3] = {-1, -1, -1}, bbad = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      for (int r = 0; r < 3; ++r) {
        blo[r] = min(blo[r], part[w][r]);
        bhi[r] = max(bhi[r], part[w][3 + r]);
      }
      bbad += part[w][6];
    }
    for (int a = 0; a < 3; ++a) {
      const int r = v.tr[a];
      if (bhi[r] >= 0) {
        atomicMin(&bounds[a], blo[r]);
        atomicMax(&bounds[3 + a], bhi[r]);
      }
    }
    if (bbad) atomicAdd(&bounds[6], bbad);
  }
}

// ---- crop-box geometry ----------------------------------------------------

struct Box {
  int32_t lo[3];
  int32_t dims[3];
  int64_t voxels;
};

// Raw element offset (channel 0) of crop voxel o (contiguous in plans order).
__device__ __forceinline__ int64_t raw_offset(const RawView& v, const Box& b, int64_t o, int c[3]) {
  const int64_t d12 = (int64_t)b.dims[1] * b.dims[2];
  c[0] = (int)(o / d12);
  c[1] = (int)((o / b.dims[2]) % b.dims[1]);
  c[2] = (int)(o % b.dims[2]);
  return (b.lo[0] + c[0]) * v.pstride[0] + (b.lo[1] + c[1]) * v.pstride[1] + (b.lo[2] + c[2]) * v.pstride[2];
}

// Row form of the crop box: output row `row` = (c0, c1) of the box, its raw
// element offset (channel 0) at c2 = 0, computed with one division per row.
__device__ __forceinline__ int64_t raw_row_base(const RawView& v, const Box& b, int64_t row) {
  const int c0 = (int)(row / b.dims[1]);
  const int c1 = (int)(row - (int64_t)c0 * b.dims[1]);
  return (b.lo[0] + c0) * v.pstride[0] + (b.lo[1] + c1) * v.pstride[1] + b.lo[2] * v.pstride[2];
}

#define NNB_WARP_ROWS(rows)                                                                       \
  for (int64_t row = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5,                        \
               row_step_ = ((int64_t)gridDim.x * blockDim.x) >> 5;                                  \
       row < (rows); row += row_step_)

template <typename T>
__global__ void __launch_bounds__(kThreads) fill_init_kernel(RawView v, Box b, int8_t* state) {
  const T* data = static_cast<const T*>(v.data);
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < b.voxels;
       o += (int64_t)gridDim.x * blockDim.x) {
    int c[3];
    const int64_t off = raw_offset(v, b, o, c);
    bool nonzero = false;
    for (int ch = 0; ch < v.channels; ++ch) nonzero |= as_f32(data[ch * v.cstride + off]) != 0.f;
    const bool face = c[0] == 0 || c[1] == 0 || c[2] == 0 || c[0] == b.dims[0] - 1 || c[1] == b.dims[1] - 1 ||
                      c[2] == b.dims[2] - 1;
    state[o] = nonzero ? 1 : (face ? 2 : 0);
  }
}

// One thread per line along `axis`: forward then backward, background voxels
// after reached background become reached.  Lines of one launch are disjoint.
__global__ void __launch_bounds__(kThreads) fill_sweep_kernel(int8_t* state, Box b, int axis, int32_t* changed) {
  const int64_t d0 = b.dims[0], d1 = b.dims[1], d2 = b.dims[2];
  const int64_t len = axis == 0 ? d0 : axis == 1 ? d1 : d2;
  const int64_t step = axis == 0 ? d1 * d2 : axis == 1 ? d2 : 1;
  const int64_t lines = b.voxels / len;
  int marked = 0;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < lines; t += (int64_t)gridDim.x * blockDim.x) {
    int64_t base;
    if (axis == 0) base = t;                                   // t over (i1, i2)
    else if (axis == 1) base = (t / d2) * d1 * d2 + t % d2;    // t over (i0, i2)
    else base = t * d2;                                        // t over (i0, i1)
    bool carry = false;
    for (int64_t k = 0; k < len; ++k) {
      int8_t* s = state + base + k * step;
      const int8_t val = *s;
      if (val == 1) carry = false;
      else if (val == 2) carry = true;
      else if (carry) { *s = 2; ++marked; }
    }
    carry = false;
    for (int64_t k = len - 1; k >= 0; --k) {
      int8_t* s = state + base + k * step;
      const int8_t val = *s;
      if (val == 1) carry = false;
      else if (val == 2) carry = true;
      else if (carry) { *s = 2; ++marked; }
    }
  }
  marked = warp_sum_int(marked);
  if ((threadIdx.x & 31) == 0 && marked) atomicAdd(changed, marked);
}

__global__ void __launch_bounds__(kThreads) crop_labels_kernel(const int32_t* labels, RawView v, Box b,
                                                              const int8_t* state, int32_t* out) {
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < b.voxels;
       o += (int64_t)gridDim.x * blockDim.x) {
    int c[3];
    const int32_t l = labels[raw_offset(v, b, o, c)];
    out[o] = (l == 0 && state[o] == 2) ? -1 : l;
  }
}

// ---- crop + normalisation --------------------------------------------------

// Per-channel statistics and the resolved affine, in the caller's workspace.
struct ChannelStats {
  double sum;
  double m2;
  unsigned long long count;
  int min_key;
  int max_key;
  float lower, upper, shift, divisor;
  int32_t pad[4];
};
static_assert(sizeof(ChannelStats) == 64, "workspace record is 64 bytes");

struct NormTable {
  nnb_norm_channel ch[kMaxChannels];
};

__global__ void stats_init_kernel(ChannelStats* st, int channels) {
  const int c = threadIdx.x;
  if (c < channels) {
    st[c].sum = 0.0;
    st[c].m2 = 0.0;
    st[c].count = 0ull;
    st[c].min_key = INT_MAX;
    st[c].max_key = INT_MIN;
  }
}

__device__ __forceinline__ bool zscore_selected(const nnb_norm_channel& n, const int8_t* state,
                                                const int32_t* labels, int64_t o) {
  if (!n.use_mask) return true;
  return labels ? labels[o] >= 0 : state[o] != 2;
}

// The CT affine, float32 operations in NumPy's order (clip, subtract, divide).
__device__ __forceinline__ float ct_apply(float x, const nnb_norm_channel& n) {
  x = fminf(fmaxf(x, n.lower), n.upper);
  return __fdiv_rn(__fsub_rn(x, n.mean), n.divisor);
}

// Fused path (no statistics needed): crop and normalise in one pass, one
// warp per output row (coalesced reads when the plans' last axis is the raw
// contiguous axis, coalesced row stores).
template <typename T>
__device__ __forceinline__ void crop_apply_row(const T* src, int64_t step, int len, int lane,
                                               const nnb_norm_channel& n, float* dst, int& bad) {
  const bool ct = n.scheme == NNB_NORM_CT;
  if (step == 1) {
    // 8 independent loads per lane in flight before any is used
    constexpr int kBatch = 8;
    for (int i0 = 0; i0 < len; i0 += 32 * kBatch) {
      float x[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int i = i0 + k * 32 + lane;
        x[k] = i < len ? as_f32(src[i]) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int i = i0 + k * 32 + lane;
        if (i < len) {
          float y = ct ? ct_apply(x[k], n) : x[k];
          bad += isfinite(y) ? 0 : 1;
          dst[i] = y;
        }
      }
    }
  } else {
#pragma unroll 4
    for (int i = lane; i < len; i += 32) {
      float x = as_f32(src[i * step]);
      if (ct) x = ct_apply(x, n);
      bad += isfinite(x) ? 0 : 1;
      dst[i] = x;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 5) crop_apply_kernel(RawView v, Box b, NormTable t, float* out,
                                                             int32_t* errors) {
  const T* data = static_cast<const T*>(v.data);
  const int lane = threadIdx.x & 31;
  const int len = b.dims[2];
  int bad = 0;
  NNB_WARP_ROWS((int64_t)b.dims[0] * b.dims[1]) {
    const int64_t base = raw_row_base(v, b, row);
    for (int ch = 0; ch < v.channels; ++ch) {
      const nnb_norm_channel n = t.ch[ch];
      crop_apply_row(data + ch * v.cstride + base, v.pstride[2], len, lane, n,
                     out + ch * b.voxels + row * len, bad);
    }
  }
  bad = warp_sum_int(bad);
  if (lane == 0 && bad) atomicAdd(&errors[0], bad);
}

// Statistics path, pass 1 (blockIdx.y = channel): write the cropped float32
// values and accumulate the sums, counts and extrema the channel's scheme needs.
template <typename T>
__global__ void __launch_bounds__(kThreads) crop_stats_kernel(RawView v, Box b, NormTable t, const int8_t* state,
                                                             const int32_t* labels, float* out, ChannelStats* st) {
  const T* data = static_cast<const T*>(v.data);
  const int ch = blockIdx.y;
  const nnb_norm_channel n = t.ch[ch];
  double sum = 0.0;
  unsigned long long count = 0;
  float mn = __int_as_float(0x7f800000), mx = -__int_as_float(0x7f800000);
  const int lane = threadIdx.x & 31;
  const int len = b.dims[2];
  NNB_WARP_ROWS((int64_t)b.dims[0] * b.dims[1]) {
    const T* src = data + ch * v.cstride + raw_row_base(v, b, row);
#pragma unroll 4
    for (int i = lane; i < len; i += 32) {
      const int64_t o = row * len + i;
      const float x = as_f32(src[i * v.pstride[2]]);
      out[ch * b.voxels + o] = x;
      if (n.scheme == NNB_NORM_ZSCORE) {
        if (zscore_selected(n, state, labels, o)) {
          sum += (double)x;
          ++count;
        }
      } else if (n.scheme == NNB_NORM_RESCALE01 || n.scheme == NNB_NORM_RGB01) {
        mn = fminf(mn, x);
        mx = fmaxf(mx, x);
      }
    }
  }
  if (n.scheme == NNB_NORM_ZSCORE) {
    sum = warp_sum_double(sum);
    count = warp_sum_u64(count);
    if ((threadIdx.x & 31) == 0 && count) {
      atomicAdd(&st[ch].sum, sum);
      atomicAdd(&st[ch].count, count);
    }
  } else if (n.scheme == NNB_NORM_RESCALE01 || n.scheme == NNB_NORM_RGB01) {
    const int kmn = __reduce_min_sync(0xffffffffu, float_key(mn));
    const int kmx = __reduce_max_sync(0xffffffffu, float_key(mx));
    if ((threadIdx.x & 31) == 0) {
      atomicMin(&st[ch].min_key, kmn);
      atomicMax(&st[ch].max_key, kmx);
    }
  }
}

// The float32 mean NumPy returns for the selection (rounded once here).
__device__ __forceinline__ float zscore_mean(const ChannelStats& s) {
  return s.count ? __double2float_rn(s.sum / (double)s.count) : 0.f;
}

// Statistics path, pass 2: squared deviations from the float32 mean (the
// difference taken in float32, as NumPy's var does for float32 data).
__global__ void __launch_bounds__(kThreads) zscore_m2_kernel(Box b, NormTable t, const int8_t* state,
                                                            const int32_t* labels, const float* out,
                                                            ChannelStats* st) {
  const int ch = blockIdx.y;
  const nnb_norm_channel n = t.ch[ch];
  if (n.scheme != NNB_NORM_ZSCORE) return;
  const float mean = zscore_mean(st[ch]);
  double m2 = 0.0;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < b.voxels;
       o += (int64_t)gridDim.x * blockDim.x) {
    if (zscore_selected(n, state, labels, o)) {
      const double d = (double)__fsub_rn(out[ch * b.voxels + o], mean);
      m2 += d * d;
    }
  }
  m2 = warp_sum_double(m2);
  if ((threadIdx.x & 31) == 0 && m2 != 0.0) atomicAdd(&st[ch].m2, m2);
}

// Resolve each channel's affine from its statistics; flag empty selections and
// RGB values outside [0, 255].
__global__ void stats_finalize_kernel(NormTable t, int channels, ChannelStats* st, int32_t* errors) {
  const int ch = threadIdx.x;
  if (ch >= channels) return;
  const nnb_norm_channel n = t.ch[ch];
  ChannelStats& s = st[ch];
  s.lower = n.lower;
  s.upper = n.upper;
  s.shift = n.mean;
  s.divisor = n.divisor;
  if (n.scheme == NNB_NORM_ZSCORE) {
    if (s.count == 0) {
      atomicAdd(&errors[2], 1);
      s.shift = 0.f;
      s.divisor = 1.f;
      return;
    }
    const float mean = zscore_mean(s);
    const float stdev = __double2float_rn(sqrt(s.m2 / (double)s.count));
    s.shift = mean;
    s.divisor = __double2float_rn(fmax((double)stdev, 1e-8));
  } else if (n.scheme == NNB_NORM_RESCALE01) {
    const float mn = key_float(s.min_key), mx = key_float(s.max_key);
    s.shift = mn;
    s.divisor = __double2float_rn(fmax((double)__fsub_rn(mx, mn), 1e-8));
  } else if (n.scheme == NNB_NORM_RGB01) {
    const float mn = key_float(s.min_key), mx = key_float(s.max_key);
    if (mn < 0.f || mx > 255.f) atomicAdd(&errors[1], 1);
    s.shift = 0.f;
    s.divisor = 255.f;
  }
}

// Statistics path, pass 3 (in place): apply every channel's affine.
__global__ void __launch_bounds__(kThreads) norm_apply_kernel(Box b, NormTable t, const int8_t* state,
                                                             const int32_t* labels, const ChannelStats* st,
                                                             float* out, int32_t* errors) {
  const int ch = blockIdx.y;
  const nnb_norm_channel n = t.ch[ch];
  const float shift = st[ch].shift, divisor = st[ch].divisor;
  int bad = 0;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < b.voxels;
       o += (int64_t)gridDim.x * blockDim.x) {
    float x = out[ch * b.voxels + o];
    switch (n.scheme) {
      case NNB_NORM_CT: x = ct_apply(x, n); break;
      case NNB_NORM_ZSCORE:
        if (zscore_selected(n, state, labels, o)) x = __fdiv_rn(__fsub_rn(x, shift), divisor);
        break;
      case NNB_NORM_RESCALE01: x = __fdiv_rn(__fsub_rn(x, shift), divisor); break;
      case NNB_NORM_RGB01: x = __fdiv_rn(x, 255.f); break;
      default: break;
    }
    bad += isfinite(x) ? 0 : 1;
    out[ch * b.voxels + o] = x;
  }
  bad = warp_sum_int(bad);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(&errors[0], bad);
}

// ---- torch-grid resampling -------------------------------------------------

struct ResizeGeom {
  int32_t src[3];
  int32_t tgt[3];
  float scale[3];        // float32(S / T)
  int64_t cstride;
  int64_t sstride[3];
  int32_t channels;
  int32_t mode;
  int32_t tiebreak;
};

struct Tap {
  int nearest, lo, hi;
  double w0, w1;
};

// One axis of the torch grid in float32 with one rounding per operation.
__device__ __forceinline__ Tap resize_tap(int t, int size, float scale, int mode) {
  Tap a;
  const float tf = (float)t;
  const float scaled_n = __fmul_rn(scale, mode == NNB_RESIZE_NEAREST ? tf : __fadd_rn(tf, 0.5f));
  a.nearest = min((int)scaled_n, size - 1);
  const float scaled = __fmul_rn(scale, __fadd_rn(tf, 0.5f));
  const float coord = fmaxf(__fsub_rn(scaled, 0.5f), 0.f);
  a.lo = min((int)coord, size - 1);
  a.hi = min(a.lo + 1, size - 1);
  a.w1 = (double)__fsub_rn(coord, floorf(coord));
  a.w0 = __dsub_rn(1.0, a.w1);
  return a;
}

template <bool kLabels>
__global__ void __launch_bounds__(kThreads, 4) torch_resize_kernel(ResizeGeom g, const void* source, void* target) {
  // one warp per output row (c, t0, t1): the outer two axes' taps once per row
  const int lane = threadIdx.x & 31;
  NNB_WARP_ROWS((int64_t)g.channels * g.tgt[0] * g.tgt[1]) {
    const int64_t ct0 = row / g.tgt[1];
    const int t1 = (int)(row - ct0 * g.tgt[1]);
    const int64_t c = ct0 / g.tgt[0];
    const int t0 = (int)(ct0 - c * g.tgt[0]);
    Tap a[3];
    a[0] = resize_tap(t0, g.src[0], g.scale[0], g.mode);
    a[1] = resize_tap(t1, g.src[1], g.scale[1], g.mode);
    const int64_t base = c * g.cstride;
    const int64_t corner_row[4] = {base + a[0].lo * g.sstride[0] + a[1].lo * g.sstride[1],
                                   base + a[0].lo * g.sstride[0] + a[1].hi * g.sstride[1],
                                   base + a[0].hi * g.sstride[0] + a[1].lo * g.sstride[1],
                                   base + a[0].hi * g.sstride[0] + a[1].hi * g.sstride[1]};
    // whether the (axis 0, axis 1) corner pair has a nonzero weight product (row-uniform)
    const bool row_active[4] = {true, a[1].w1 != 0.0, a[0].w1 != 0.0, a[0].w1 != 0.0 && a[1].w1 != 0.0};
#pragma unroll 2
    for (int t2 = lane; t2 < g.tgt[2]; t2 += 32) {
    const int64_t e = row * g.tgt[2] + t2;
    a[2] = resize_tap(t2, g.src[2], g.scale[2], g.mode);
    const int64_t nearest = base + a[0].nearest * g.sstride[0] + a[1].nearest * g.sstride[1] +
                            a[2].nearest * g.sstride[2];
    if (!kLabels) {
      const float* src = static_cast<const float*>(source);
      float* dst = static_cast<float*>(target);
      if (g.mode != NNB_RESIZE_LINEAR) {
        dst[e] = src[nearest];
        continue;
      }
      // Corners whose weight product is exactly 0 are not read: their term
      // is +-0, and the running sum starts at +0 and is never -0 (x + y is -0
      // only for two -0 operands), so adding +-0 leaves it unchanged.  The
      // lower weight 1 - f of an axis is never 0; the upper weight f is 0 on
      // axes that keep their size (row-uniform for axes 0 and 1).
      const bool h2 = a[2].w1 != 0.0;
      const int64_t o_lo = a[2].lo * g.sstride[2], o_hi = a[2].hi * g.sstride[2];
      float v[8];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const bool on = row_active[q];
        v[2 * q] = on ? src[corner_row[q] + o_lo] : 0.f;
        v[2 * q + 1] = on && h2 ? src[corner_row[q] + o_hi] : 0.f;
      }
      double sum = 0.0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (!row_active[q]) continue;
        const double wa = (q >> 1) ? a[0].w1 : a[0].w0, wb = (q & 1) ? a[1].w1 : a[1].w0;
        double t = __dmul_rn(__dmul_rn(__dmul_rn((double)v[2 * q], wa), wb), a[2].w0);
        sum = __dadd_rn(sum, t);
        if (h2) {
          t = __dmul_rn(__dmul_rn(__dmul_rn((double)v[2 * q + 1], wa), wb), a[2].w1);
          sum = __dadd_rn(sum, t);
        }
      }
      dst[e] = __double2float_rn(sum);
    } else {
      const int32_t* src = static_cast<const int32_t*>(source);
      int32_t* dst = static_cast<int32_t*>(target);
      if (g.mode != NNB_RESIZE_LINEAR) {
        dst[e] = src[nearest];
        continue;
      }
      int label[8];
      double weight[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int b0 = (k >> 2) & 1, b1 = (k >> 1) & 1, b2 = k & 1;
        label[k] = src[corner_row[(b0 << 1) | b1] + (b2 ? a[2].hi : a[2].lo) * g.sstride[2]];
        double w = __dmul_rn(1000.0, b0 ? a[0].w1 : a[0].w0);
        w = __dmul_rn(w, b1 ? a[1].w1 : a[1].w0);
        weight[k] = __dmul_rn(w, b2 ? a[2].w1 : a[2].w0);
      }
      const int near_label = src[nearest];
      float best = -1.f;
      int winner = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        bool seen = false;
#pragma unroll
        for (int p = 0; p < k; ++p) seen |= label[p] == label[k];
        if (seen) continue;
        double score = 0.0;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (label[q] == label[k]) score = __dadd_rn(score, weight[q]);
        const float rounded = __half2float(__float2half_rn(__double2float_rn(score)));
        bool preferred;
        if (g.tiebreak == NNB_TIE_LOWEST) preferred = label[k] < winner;
        else if (g.tiebreak == NNB_TIE_HIGHEST) preferred = label[k] > winner;
        else preferred = label[k] == near_label || (winner != near_label && label[k] < winner);
        if (rounded > best || (rounded == best && preferred)) {
          best = rounded;
          winner = label[k];
        }
      }
      dst[e] = winner;
    }
    }
  }
}

// ---- spline resampling (resample_data_or_seg_to_shape) --------------------

constexpr int kSplinePad = 12;   // edge samples scipy adds before prefiltering (mode "nearest")

struct SplineGeom {
  int32_t src[3];       // source dims
  int32_t pdim[3];      // coefficient dims: src + 2 * pad
  int32_t pad[3];       // kSplinePad on prefiltered axes, else 0
  int32_t tgt[3];
  int32_t axes;         // bit a: axis a is resampled
  int64_t cstride;      // source element strides
  int64_t sstride[3];
  int32_t channels;
};

// coef[c][p] = source[c][clamp(p - pad)] as float64 (edge padding).
template <typename S>
__global__ void __launch_bounds__(kThreads) spline_pad_kernel(const S* src, SplineGeom g, double* coef) {
  const int lane = threadIdx.x & 31;
  NNB_WARP_ROWS((int64_t)g.channels * g.pdim[0] * g.pdim[1]) {
    const int64_t c0 = row / g.pdim[1];
    const int p1 = (int)(row - c0 * g.pdim[1]);
    const int64_t c = c0 / g.pdim[0];
    const int p0 = (int)(c0 - c * g.pdim[0]);
    const int s0 = min(max(p0 - g.pad[0], 0), g.src[0] - 1);
    const int s1 = min(max(p1 - g.pad[1], 0), g.src[1] - 1);
    const S* line = src + c * g.cstride + s0 * g.sstride[0] + s1 * g.sstride[1];
    double* out = coef + row * g.pdim[2];
    for (int p2 = lane; p2 < g.pdim[2]; p2 += 32) {
      const int s2 = min(max(p2 - g.pad[2], 0), g.src[2] - 1);
      out[p2] = (double)line[s2 * g.sstride[2]];
    }
  }
}

// Mirror index of j on the half-sample-symmetric extension of n samples.
__device__ __forceinline__ int mirror_index(int j, int n) {
  const int period = 2 * n;
  j %= period;
  if (j < 0) j += period;
  return j < n ? j : period - 1 - j;
}

// Cubic B-spline prefilter of every line along `axis`: gain, causal pass with
// the half-sample-symmetric initial value c+(0) = sum_k z^k x(-k), anticausal
// pass with c-(n-1) = z / (z - 1) c+(n-1), each operation rounded separately
// as the host implementation computes it.  A block of 32 threads filters 32
// lines that are neighbours in memory; the lines stream through shared memory
// in chunks of kChunk samples (coalesced loads and stores), and each thread
// runs its line's serial recursion out of shared memory, carrying the last
// value between chunks.
constexpr int kChunk = 64;

// Element offset of (line lane, position j) and the stride between positions.
__device__ __forceinline__ void filter_line_geometry(const SplineGeom& g, int axis, int64_t group, int lane,
                                                     int64_t* base, int64_t* step, bool* valid) {
  const int64_t d0 = g.pdim[0], d1 = g.pdim[1], d2 = g.pdim[2];
  const int64_t per_channel = d0 * d1 * d2;
  if (axis == 2) {
    // 32 consecutive rows (c, p0, p1); positions along p2 (stride 1)
    const int64_t row = group * 32 + lane;
    *valid = row < (int64_t)g.channels * d0 * d1;
    *base = row * d2;
    *step = 1;
  } else {
    // lines (c, q, p2) with p2 = 32 b + lane; q is the other non-filtered axis
    const int64_t blocks2 = (d2 + 31) / 32;
    const int64_t q_count = axis == 0 ? d1 : d0;
    const int64_t cq = group / blocks2;
    const int64_t p2 = (group - cq * blocks2) * 32 + lane;
    const int64_t c = cq / q_count, q = cq - c * q_count;
    *valid = c < g.channels && p2 < d2;
    *base = c * per_channel + (axis == 0 ? q * d2 : q * d1 * d2) + p2;
    *step = axis == 0 ? d1 * d2 : d2;
  }
}

__global__ void __launch_bounds__(32) spline_filter_kernel(double* coef, SplineGeom g, int axis, int64_t groups) {
  __shared__ double tile[32][kChunk + 1];
  const double z = sqrt(3.0) - 2.0;
  const double gain = __dmul_rn(1.0 - z, 1.0 - 1.0 / z);
  const double anti = z / (z - 1.0);
  const int lane = threadIdx.x;
  const int n = g.pdim[axis];
  const int chunks = (n + kChunk - 1) / kChunk;
  for (int64_t group = blockIdx.x; group < groups; group += gridDim.x) {
    int64_t my_base, step;
    bool my_valid;
    filter_line_geometry(g, axis, group, lane, &my_base, &step, &my_valid);
    // Load chunk k of all 32 lines into the tile (coalesced along the memory-contiguous direction).
    auto load = [&](int k) {
      const int j0 = k * kChunk;
      const int len = min(kChunk, n - j0);
      if (axis == 2) {
        for (int i = 0; i < 32; ++i) {
          const int64_t b = __shfl_sync(0xffffffffu, my_base, i);
          const bool v = __shfl_sync(0xffffffffu, my_valid, i);
          for (int j = lane; j < len; j += 32) tile[i][j] = v ? coef[b + j0 + j] : 0.0;
        }
      } else {
        for (int j = 0; j < len; ++j) tile[lane][j] = my_valid ? coef[my_base + (int64_t)(j0 + j) * step] : 0.0;
      }
      __syncwarp();
    };
    auto store = [&](int k) {
      __syncwarp();
      const int j0 = k * kChunk;
      const int len = min(kChunk, n - j0);
      if (axis == 2) {
        for (int i = 0; i < 32; ++i) {
          const int64_t b = __shfl_sync(0xffffffffu, my_base, i);
          const bool v = __shfl_sync(0xffffffffu, my_valid, i);
          for (int j = lane; j < len; j += 32)
            if (v) coef[b + j0 + j] = tile[i][j];
        }
      } else {
        for (int j = 0; j < len; ++j)
          if (my_valid) coef[my_base + (int64_t)(j0 + j) * step] = tile[lane][j];
      }
      __syncwarp();
    };
    double* t = tile[lane];
    // causal pass, chunk by chunk
    double carry = 0.0;
    for (int k = 0; k < chunks; ++k) {
      load(k);
      const int len = min(kChunk, n - k * kChunk);
      for (int j = 0; j < len; ++j) t[j] = __dmul_rn(t[j], gain);
      int j = 0;
      if (k == 0) {
        // initial value from the first samples (mirror indices of -k lie in the first chunk while
        // n > kChunk; a line of at most kChunk samples is whole in the tile)
        double acc = t[0], zk = z;
        for (int m = 1; m < 64 && fabs(zk) > 1e-30; ++m) {
          const int src = mirror_index(-m, n);
          acc = __dadd_rn(acc, __dmul_rn(zk, src < kChunk ? t[src] : 0.0));
          zk = __dmul_rn(zk, z);
        }
        t[0] = acc;
        carry = acc;
        j = 1;
      }
      for (; j < len; ++j) {
        carry = __dadd_rn(t[j], __dmul_rn(z, carry));
        t[j] = carry;
      }
      store(k);
    }
    // anticausal pass, last chunk first
    for (int k = chunks - 1; k >= 0; --k) {
      load(k);
      const int len = min(kChunk, n - k * kChunk);
      int j = len - 1;
      if (k == chunks - 1) {
        t[j] = __dmul_rn(t[j], anti);
        carry = t[j];
        --j;
      }
      for (; j >= 0; --j) {
        carry = __dmul_rn(z, __dsub_rn(carry, t[j]));
        t[j] = carry;
      }
      store(k);
    }
  }
}

struct SplineTaps {
  int idx[4];
  double w[4];
};

// Taps of output index t on one axis: a resampled axis samples the half-pixel
// grid (order 3: four cubic B-spline weights from floor(c) - 1; order 1: two
// linear weights), clamped into the coefficient array; a kept axis reads t.
template <int kOrder>
__device__ __forceinline__ SplineTaps spline_taps(const SplineGeom& g, int axis, int t) {
  SplineTaps a;
  if (!((g.axes >> axis) & 1)) {
    a.idx[0] = t + g.pad[axis];
    a.w[0] = 1.0;
#pragma unroll
    for (int k = 1; k < 4; ++k) { a.idx[k] = a.idx[0]; a.w[k] = 0.0; }
    return a;
  }
  const double ratio = (double)g.src[axis] / (double)g.tgt[axis];
  const double c = __dadd_rn(__dsub_rn(__dmul_rn((double)t + 0.5, ratio), 0.5), (double)g.pad[axis]);
  const double fl = floor(c);
  const double f = __dsub_rn(c, fl);
  const int i = (int)fl;
  const int hi = g.pdim[axis] - 1;
  if (kOrder == 3) {
    // cubic B-spline weights of taps floor(c) - 1 .. floor(c) + 2, one rounding per operation
    const double s = __dsub_rn(1.0, f);
    const double f2 = __dmul_rn(f, f), s2 = __dmul_rn(s, s);
    const double f3 = __dmul_rn(f2, f), s3 = __dmul_rn(s2, s);
    a.w[0] = s3 / 6.0;
    a.w[1] = __dadd_rn(__dsub_rn(2.0 / 3.0, f2), f3 / 2.0);
    a.w[2] = __dadd_rn(__dsub_rn(2.0 / 3.0, s2), s3 / 2.0);
    a.w[3] = f3 / 6.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) a.idx[k] = min(max(i - 1 + k, 0), hi);
  } else {
    a.w[0] = __dsub_rn(1.0, f);
    a.w[1] = f;
    a.w[2] = a.w[3] = 0.0;
    a.idx[0] = min(max(i, 0), hi);
    a.idx[1] = min(max(i + 1, 0), hi);
    a.idx[2] = a.idx[3] = a.idx[1];
  }
  return a;
}

// One warp per output row (c, t0, t1); per output the sum over the taps
// (axis 0 outermost) of ((v * w0) * w1) * w2 in float64, rounded once.
template <int kOrder, typename O>
__global__ void __launch_bounds__(kThreads) spline_interp_kernel(const double* coef, SplineGeom g, O* out) {
  const int lane = threadIdx.x & 31;
  constexpr int K = kOrder == 3 ? 4 : 2;
  const int k0 = ((g.axes >> 0) & 1) ? K : 1, k1 = ((g.axes >> 1) & 1) ? K : 1, k2 = ((g.axes >> 2) & 1) ? K : 1;
  const int64_t per_channel = (int64_t)g.pdim[0] * g.pdim[1] * g.pdim[2];
  NNB_WARP_ROWS((int64_t)g.channels * g.tgt[0] * g.tgt[1]) {
    const int64_t ct0 = row / g.tgt[1];
    const int t1 = (int)(row - ct0 * g.tgt[1]);
    const int64_t c = ct0 / g.tgt[0];
    const int t0 = (int)(ct0 - c * g.tgt[0]);
    const SplineTaps a0 = spline_taps<kOrder>(g, 0, t0), a1 = spline_taps<kOrder>(g, 1, t1);
    const double* base = coef + c * per_channel;
    for (int t2 = lane; t2 < g.tgt[2]; t2 += 32) {
      const SplineTaps a2 = spline_taps<kOrder>(g, 2, t2);
      double sum = 0.0;
      for (int i = 0; i < k0; ++i) {
        for (int j = 0; j < k1; ++j) {
          const double* r = base + ((int64_t)a0.idx[i] * g.pdim[1] + a1.idx[j]) * g.pdim[2];
#pragma unroll
          for (int k = 0; k < K; ++k) {
            if (k < k2) {
              const double v = __dmul_rn(__dmul_rn(__dmul_rn(r[a2.idx[k]], a0.w[i]), a1.w[j]), a2.w[k]);
              sum = __dadd_rn(sum, v);
            }
          }
        }
      }
      out[row * g.tgt[2] + t2] = (O)sum;
    }
  }
}

// Out-of-plane order-0 pass: gather along the one changed axis, round once.
__global__ void __launch_bounds__(kThreads) nearest_axis_kernel(const double* src, int channels, Box in,
                                                               Box outb, int axis, float* out) {
  const double ratio = (double)in.dims[axis] / (double)outb.dims[axis];
  const int lane = threadIdx.x & 31;
  NNB_WARP_ROWS((int64_t)channels * outb.dims[0] * outb.dims[1]) {
    const int64_t ct0 = row / outb.dims[1];
    const int t1 = (int)(row - ct0 * outb.dims[1]);
    const int64_t c = ct0 / outb.dims[0];
    const int t0 = (int)(ct0 - c * outb.dims[0]);
    int s[2] = {t0, t1};
    for (int a = 0; a < 2; ++a) {
      if (a == axis) {
        const double x = __dadd_rn(__dsub_rn(__dmul_rn(ratio, (double)s[a] + 0.5), 0.5), 0.5);
        s[a] = min(max((int)floor(x), 0), in.dims[a] - 1);
      }
    }
    const double* line = src + c * in.voxels + ((int64_t)s[0] * in.dims[1] + s[1]) * in.dims[2];
    float* dst = out + row * outb.dims[2];
    for (int t2 = lane; t2 < outb.dims[2]; t2 += 32) {
      int s2 = t2;
      if (axis == 2) {
        const double x = __dadd_rn(__dsub_rn(__dmul_rn(ratio, (double)t2 + 0.5), 0.5), 0.5);
        s2 = min(max((int)floor(x), 0), in.dims[2] - 1);
      }
      dst[t2] = __double2float_rn(line[s2]);
    }
  }
}

int check_raw(const nnb_raw_case* r, const char* what) {
  NNB_REQUIRE(r != nullptr && r->data != nullptr, "%s: null raw case", what);
  NNB_REQUIRE(r->dtype >= NNB_DTYPE_F32 && r->dtype <= NNB_DTYPE_I32, "%s: unsupported dtype %d", what, r->dtype);
  NNB_REQUIRE(r->channels >= 1, "%s: channels must be positive", what);
  int seen = 0;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(r->raw_dims[i] >= 1, "%s: raw dims must be positive", what);
    NNB_REQUIRE(r->transpose[i] >= 0 && r->transpose[i] < 3 && !(seen & (1 << r->transpose[i])),
                "%s: transpose must be a permutation of (0, 1, 2)", what);
    seen |= 1 << r->transpose[i];
  }
  return NNB_OK;
}

int check_box(const RawView& v, const int32_t lo[3], const int32_t dims[3], Box* b, const char* what) {
  NNB_REQUIRE(lo != nullptr && dims != nullptr, "%s: null crop box", what);
  b->voxels = 1;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(lo[i] >= 0 && dims[i] >= 1 && (int64_t)lo[i] + dims[i] <= v.pdims[i],
                "%s: crop box outside the transposed case on axis %d", what, i);
    b->lo[i] = lo[i];
    b->dims[i] = dims[i];
    b->voxels *= dims[i];
  }
  return NNB_OK;
}

#define NNB_DISPATCH_RAW(dtype, KERNEL, grid, block, stream, ...)                                   \
  switch (dtype) {                                                                                \
    case NNB_DTYPE_F32: KERNEL<float><<<grid, block, 0, stream>>>(__VA_ARGS__); break;           \
    case NNB_DTYPE_F64: KERNEL<double><<<grid, block, 0, stream>>>(__VA_ARGS__); break;          \
    case NNB_DTYPE_I16: KERNEL<int16_t><<<grid, block, 0, stream>>>(__VA_ARGS__); break;         \
    case NNB_DTYPE_U8: KERNEL<uint8_t><<<grid, block, 0, stream>>>(__VA_ARGS__); break;          \
    case NNB_DTYPE_U16: KERNEL<uint16_t><<<grid, block, 0, stream>>>(__VA_ARGS__); break;        \
    default: KERNEL<int32_t><<<grid, block, 0, stream>>>(__VA_ARGS__); break;                    \
  }

}  // namespace
}  // namespace nnb

using namespace nnb;

extern "C" {

int32_t nnb_nonzero_bounds(const nnb_raw_case* raw, int32_t* bounds, void* stream) {
  if (int rc = check_raw(raw, "nonzero_bounds")) return rc;
  NNB_REQUIRE(bounds != nullptr, "nonzero_bounds: null bounds");
  const RawView v = make_view(*raw);
  cudaStream_t s = (cudaStream_t)stream;
  bounds_init_kernel<<<1, 32, 0, s>>>(bounds);
  static const int kElementBytes[] = {4, 8, 2, 1, 2, 4};
  const int vec = ((int64_t)raw->raw_dims[2] * kElementBytes[raw->dtype]) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(raw->data) % 16 == 0;
  const int64_t rows = (int64_t)raw->raw_dims[0] * raw->raw_dims[1];
  // resident blocks only (5 per SM at this kernel's register use): every block stays to the end
  NNB_DISPATCH_RAW(raw->dtype, nonzero_bounds_kernel, grid_for(rows * 32, 5), kThreads, s, v, vec, bounds);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int32_t nnb_fill_holes_init(const nnb_raw_case* raw, const int32_t crop_lo[3], const int32_t crop_dims[3],
                            int8_t* state, void* stream) {
  if (int rc = check_raw(raw, "fill_holes_init")) return rc;
  NNB_REQUIRE(state != nullptr, "fill_holes_init: null state");
  const RawView v = make_view(*raw);
  Box b;
  if (int rc = check_box(v, crop_lo, crop_dims, &b, "fill_holes_init")) return rc;
  NNB_DISPATCH_RAW(raw->dtype, fill_init_kernel, grid_for(b.voxels), kThreads, (cudaStream_t)stream, v, b, state);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int32_t nnb_fill_holes_sweep(int8_t* state, const int32_t crop_dims[3], int32_t* changed, void* stream) {
  NNB_REQUIRE(state != nullptr && changed != nullptr && crop_dims != nullptr, "fill_holes_sweep: null pointer");
  Box b;
  b.voxels = 1;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(crop_dims[i] >= 1, "fill_holes_sweep: dims must be positive");
    b.lo[i] = 0;
    b.dims[i] = crop_dims[i];
    b.voxels *= crop_dims[i];
  }
  cudaStream_t s = (cudaStream_t)stream;
  for (int axis = 0; axis < 3; ++axis) {
    const int64_t lines = b.voxels / b.dims[axis];
    fill_sweep_kernel<<<grid_for(lines), kThreads, 0, s>>>(state, b, axis, changed);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int32_t nnb_crop_labels(const int32_t* labels, const nnb_raw_case* raw, const int32_t crop_lo[3],
                        const int32_t crop_dims[3], const int8_t* state, int32_t* out, void* stream) {
  if (int rc = check_raw(raw, "crop_labels")) return rc;
  NNB_REQUIRE(labels != nullptr && state != nullptr && out != nullptr, "crop_labels: null pointer");
  const RawView v = make_view(*raw);
  Box b;
  if (int rc = check_box(v, crop_lo, crop_dims, &b, "crop_labels")) return rc;
  crop_labels_kernel<<<grid_for(b.voxels), kThreads, 0, (cudaStream_t)stream>>>(labels, v, b, state, out);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int64_t nnb_crop_normalize_workspace_bytes(int32_t channels) {
  return channels < 1 ? 0 : (int64_t)channels * (int64_t)sizeof(ChannelStats);
}

int32_t nnb_crop_normalize(const nnb_raw_case* raw, const int32_t crop_lo[3], const int32_t crop_dims[3],
                           const nnb_norm_channel* norm, const int8_t* state, const int32_t* labels,
                           void* workspace, float* out, int32_t* errors, void* stream) {
  if (int rc = check_raw(raw, "crop_normalize")) return rc;
  NNB_REQUIRE(norm != nullptr && out != nullptr && errors != nullptr, "crop_normalize: null pointer");
  if (raw->channels > kMaxChannels) {
    set_error("crop_normalize: %d channels exceed the supported %d", raw->channels, kMaxChannels);
    return NNB_E_UNSUPPORTED;
  }
  const RawView v = make_view(*raw);
  Box b;
  if (int rc = check_box(v, crop_lo, crop_dims, &b, "crop_normalize")) return rc;
  NormTable t;
  bool stats = false;
  for (int c = 0; c < raw->channels; ++c) {
    const nnb_norm_channel& n = norm[c];
    NNB_REQUIRE(n.scheme >= NNB_NORM_NONE && n.scheme <= NNB_NORM_RGB01, "crop_normalize: bad scheme %d", n.scheme);
    if (n.scheme == NNB_NORM_CT)
      NNB_REQUIRE(n.lower <= n.upper && n.divisor > 0.f, "crop_normalize: bad CT parameters on channel %d", c);
    if (n.scheme == NNB_NORM_ZSCORE && n.use_mask)
      NNB_REQUIRE(state != nullptr || labels != nullptr, "crop_normalize: masked z-score needs the crop mask");
    stats |= n.scheme == NNB_NORM_ZSCORE || n.scheme == NNB_NORM_RESCALE01 || n.scheme == NNB_NORM_RGB01;
    t.ch[c] = n;
  }
  cudaStream_t s = (cudaStream_t)stream;
  NNB_CUDA_CHECK(cudaMemsetAsync(errors, 0, 4 * sizeof(int32_t), s));
  if (!stats) {
    const int64_t rows = (int64_t)b.dims[0] * b.dims[1];
    NNB_DISPATCH_RAW(raw->dtype, crop_apply_kernel, grid_for(rows * 32), kThreads, s, v, b, t, out, errors);
    NNB_LAUNCH_CHECK();
    return NNB_OK;
  }
  NNB_REQUIRE(workspace != nullptr, "crop_normalize: statistics need the workspace");
  ChannelStats* st = static_cast<ChannelStats*>(workspace);
  stats_init_kernel<<<1, kMaxChannels, 0, s>>>(st, raw->channels);
  const dim3 grid(grid_for(b.voxels, 8), raw->channels);
  const dim3 row_grid(grid_for((int64_t)b.dims[0] * b.dims[1] * 32, 8), raw->channels);
  NNB_DISPATCH_RAW(raw->dtype, crop_stats_kernel, row_grid, kThreads, s, v, b, t, state, labels, out, st);
  zscore_m2_kernel<<<grid, kThreads, 0, s>>>(b, t, state, labels, out, st);
  stats_finalize_kernel<<<1, kMaxChannels, 0, s>>>(t, raw->channels, st, errors);
  norm_apply_kernel<<<grid, kThreads, 0, s>>>(b, t, state, labels, st, out, errors);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int32_t nnb_torch_resize(const nnb_torch_resize_args* a, void* stream) {
  NNB_REQUIRE(a != nullptr && a->source != nullptr && a->target != nullptr, "torch_resize: null pointer");
  NNB_REQUIRE(a->labels == 0 || a->labels == 1, "torch_resize: labels must be 0 or 1");
  NNB_REQUIRE(a->channels >= 1, "torch_resize: channels must be positive");
  NNB_REQUIRE(a->mode >= NNB_RESIZE_LINEAR && a->mode <= NNB_RESIZE_NEAREST_EXACT, "torch_resize: bad mode");
  NNB_REQUIRE(a->tiebreak >= NNB_TIE_LOWEST && a->tiebreak <= NNB_TIE_NEAREST, "torch_resize: bad tiebreak");
  NNB_REQUIRE(a->channel_stride >= 0, "torch_resize: strides must be non-negative");
  ResizeGeom g;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(a->source_dims[i] >= 1 && a->target_dims[i] >= 1, "torch_resize: dims must be positive");
    NNB_REQUIRE(a->source_strides[i] >= 0, "torch_resize: strides must be non-negative");
    g.src[i] = a->source_dims[i];
    g.tgt[i] = a->target_dims[i];
    g.scale[i] = (float)((double)a->source_dims[i] / (double)a->target_dims[i]);
    g.sstride[i] = a->source_strides[i];
  }
  g.cstride = a->channel_stride;
  g.channels = a->channels;
  g.mode = a->mode;
  g.tiebreak = a->tiebreak;
  const int64_t rows = (int64_t)a->channels * a->target_dims[0] * a->target_dims[1];
  cudaStream_t s = (cudaStream_t)stream;
  if (a->labels) torch_resize_kernel<true><<<grid_for(rows * 32), kThreads, 0, s>>>(g, a->source, a->target);
  else torch_resize_kernel<false><<<grid_for(rows * 32), kThreads, 0, s>>>(g, a->source, a->target);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int64_t nnb_spline_workspace_bytes(int32_t channels, const int32_t source_dims[3], int32_t axes, int32_t order) {
  if (channels < 1 || source_dims == nullptr) return 0;
  int64_t n = channels;
  for (int a = 0; a < 3; ++a) n *= source_dims[a] + ((order == 3 && ((axes >> a) & 1)) ? 2 * kSplinePad : 0);
  return n * (int64_t)sizeof(double);
}

int32_t nnb_spline_resize(const nnb_spline_resize_args* a, void* stream) {
  NNB_REQUIRE(a != nullptr && a->source && a->target && a->coefficients, "spline_resize: null pointer");
  NNB_REQUIRE(a->order == 1 || a->order == 3, "spline_resize: order must be 1 or 3");
  NNB_REQUIRE(a->channels >= 1 && a->channel_stride >= 0, "spline_resize: bad channels");
  NNB_REQUIRE(a->axes >= 0 && a->axes <= 7, "spline_resize: axes must be a 3-bit mask");
  SplineGeom g;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(a->source_dims[i] >= 1 && a->target_dims[i] >= 1 && a->source_strides[i] >= 0,
                "spline_resize: dims must be positive and strides non-negative");
    const bool on = (a->axes >> i) & 1;
    NNB_REQUIRE(on || a->source_dims[i] == a->target_dims[i], "spline_resize: axis %d is kept but changes size", i);
    g.src[i] = a->source_dims[i];
    g.tgt[i] = a->target_dims[i];
    g.pad[i] = (a->order == 3 && on) ? kSplinePad : 0;
    g.pdim[i] = g.src[i] + 2 * g.pad[i];
    g.sstride[i] = a->source_strides[i];
  }
  g.axes = a->axes;
  g.cstride = a->channel_stride;
  g.channels = a->channels;
  cudaStream_t s = (cudaStream_t)stream;
  const int64_t pad_rows = (int64_t)g.channels * g.pdim[0] * g.pdim[1];
  if (a->source_f64)
    spline_pad_kernel<double><<<grid_for(pad_rows * 32), kThreads, 0, s>>>(static_cast<const double*>(a->source), g,
                                                                            a->coefficients);
  else
    spline_pad_kernel<float><<<grid_for(pad_rows * 32), kThreads, 0, s>>>(static_cast<const float*>(a->source), g,
                                                                           a->coefficients);
  if (a->order == 3) {
    for (int axis = 0; axis < 3; ++axis) {
      if (!((a->axes >> axis) & 1)) continue;
      const int64_t groups = axis == 2 ? ((int64_t)g.channels * g.pdim[0] * g.pdim[1] + 31) / 32
                                       : (int64_t)g.channels * (axis == 0 ? g.pdim[1] : g.pdim[0]) *
                                             ((g.pdim[2] + 31) / 32);
      const int64_t cap = 148LL * 32;  // 32 resident 32-thread blocks per SM
      spline_filter_kernel<<<(int)(groups < cap ? groups : cap), 32, 0, s>>>(a->coefficients, g, axis, groups);
    }
  }
  const int64_t rows = (int64_t)g.channels * g.tgt[0] * g.tgt[1];
  if (a->order == 3) {
    if (a->target_f64) spline_interp_kernel<3, double><<<grid_for(rows * 32), kThreads, 0, s>>>(
        a->coefficients, g, static_cast<double*>(a->target));
    else spline_interp_kernel<3, float><<<grid_for(rows * 32), kThreads, 0, s>>>(
        a->coefficients, g, static_cast<float*>(a->target));
  } else {
    if (a->target_f64) spline_interp_kernel<1, double><<<grid_for(rows * 32), kThreads, 0, s>>>(
        a->coefficients, g, static_cast<double*>(a->target));
    else spline_interp_kernel<1, float><<<grid_for(rows * 32), kThreads, 0, s>>>(
        a->coefficients, g, static_cast<float*>(a->target));
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int32_t nnb_nearest_axis_resize(const double* source, int32_t channels, const int32_t source_dims[3],
                                const int32_t target_dims[3], float* target, void* stream) {
  NNB_REQUIRE(source && target && source_dims && target_dims && channels >= 1, "nearest_axis_resize: bad arguments");
  Box in, outb;
  in.voxels = outb.voxels = 1;
  int axis = -1;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(source_dims[i] >= 1 && target_dims[i] >= 1, "nearest_axis_resize: dims must be positive");
    in.lo[i] = outb.lo[i] = 0;
    in.dims[i] = source_dims[i];
    outb.dims[i] = target_dims[i];
    in.voxels *= source_dims[i];
    outb.voxels *= target_dims[i];
    if (source_dims[i] != target_dims[i]) {
      NNB_REQUIRE(axis < 0, "nearest_axis_resize: more than one axis changes size");
      axis = i;
    }
  }
  const int64_t rows = (int64_t)channels * outb.dims[0] * outb.dims[1];
  nearest_axis_kernel<<<grid_for(rows * 32), kThreads, 0, (cudaStream_t)stream>>>(source, channels, in, outb, axis,
                                                                                  target);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

}  // extern "C"
