// CUDA-core kernels of the path: the any-shape float32 convolution (used for
// the few-channel first layer and for shapes outside the tensor-core
// envelope), the transposed convolution, instance-norm finalisation and the
// residual join.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"

namespace nnb {

// ---------------------------------------------------------------------------
// Direct convolution: one thread per output voxel, CO output channels per
// block column; lazy input activation; per-tile (sum, M2) of the output.
// Reference semantics: `_unbiased_convolution` (network.py:240-269) with the
// tap order of the single-channel kernel (metal_single_channel_conv.py:32-59).
// ---------------------------------------------------------------------------
template <int CO>
__global__ void __launch_bounds__(kTileRows) conv3d_simt_kernel(nnb_conv3d_args a, int tps) {
  __shared__ float red[kTileRows][CO + 1];
  const int t = blockIdx.x % tps;
  const int b = blockIdx.x / tps;
  const int co0 = blockIdx.y * CO;
  const int nco = min(CO, a.cout - co0);
  const int r = threadIdx.x;
  const int OD = a.out_dims[0], OH = a.out_dims[1], OW = a.out_dims[2];
  const int ID = a.in_dims[0], IH = a.in_dims[1], IW = a.in_dims[2];
  const int64_t ovox = (int64_t)OD * OH * OW;
  const int64_t m = (int64_t)t * kTileRows + r;
  const bool valid = m < ovox;
  const int ox = (int)(m % OW), oy = (int)((m / OW) % OH), oz = (int)(m / ((int64_t)OW * OH));
  const int kvol = a.kernel[0] * a.kernel[1] * a.kernel[2];
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) cin_total += a.seg[s].channels;
  const int64_t wstride = (int64_t)kvol * cin_total;  // distance between output channels

  float acc[CO];
#pragma unroll
  for (int j = 0; j < CO; ++j) acc[j] = 0.f;

  if (valid) {
    int tap = 0;
    for (int kz = 0; kz < a.kernel[0]; ++kz) {
      const int iz = oz * a.stride[0] - a.pad[0] + kz;
      for (int ky = 0; ky < a.kernel[1]; ++ky) {
        const int iy = oy * a.stride[1] - a.pad[1] + ky;
        for (int kx = 0; kx < a.kernel[2]; ++kx, ++tap) {
          const int ix = ox * a.stride[2] - a.pad[2] + kx;
          if (iz < 0 || iz >= ID || iy < 0 || iy >= IH || ix < 0 || ix >= IW) continue;
          int cbase = 0;
          for (int s = 0; s < a.num_segments; ++s) {
            const nnb_segment seg = a.seg[s];
            const float* src = seg.data + ((((int64_t)b * ID + iz) * IH + iy) * IW + ix) * seg.channels;
            const float* wp = a.weight + (int64_t)co0 * wstride + (int64_t)tap * cin_total + cbase;
            for (int ci = 0; ci < seg.channels; ++ci) {
              const float v = activate(__ldg(src + ci), seg.scale, seg.shift, seg.leaky, a.slope,
                                       b * seg.channels + ci);
#pragma unroll
              for (int j = 0; j < CO; ++j)
                if (j < nco) acc[j] = fmaf(v, __ldg(wp + j * wstride + ci), acc[j]);
            }
            cbase += seg.channels;
          }
        }
      }
    }
  }
  if (a.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < CO; ++j)
      if (j < nco) acc[j] += __ldg(a.bias + co0 + j);
  }
  if (valid) {
    float* dst = a.out + ((int64_t)b * ovox + m) * a.cout + co0;
#pragma unroll
    for (int j = 0; j < CO; ++j)
      if (j < nco) dst[j] = acc[j];
  }
  if (a.partials == nullptr) return;
#pragma unroll
  for (int j = 0; j < CO; ++j) red[r][j] = valid ? acc[j] : 0.f;
  __syncthreads();
  if (r < nco) {
    const int rows = (int)min((int64_t)kTileRows, ovox - (int64_t)t * kTileRows);
    float sum = 0.f;
    for (int i = 0; i < rows; ++i) sum += red[i][r];
    const float mean = sum / rows;
    float m2 = 0.f;
    for (int i = 0; i < rows; ++i) {
      const float d = red[i][r] - mean;
      m2 = fmaf(d, d, m2);
    }
    float* p = a.partials + (((int64_t)b * a.cout + co0 + r) * tps + t) * 3;
    p[0] = sum;
    p[1] = m2;
    p[2] = (float)rows;
  }
}

// ---------------------------------------------------------------------------
// Few-input-channel convolution (the first layer: 1..8 input channels):
// memory-bound on its output, so one thread per output voxel computes a
// 32-channel group from weights held in shared memory (broadcast reads), the
// 128 x 32 output tile is staged in shared memory and written with coalesced
// 16-byte stores, and the tile's (sum, M2) partials come from the same stage.
// Tap order (kd, kh, kw) and zero padding as the reference's single-channel
// kernel (metal_single_channel_conv.py:32-59).
// ---------------------------------------------------------------------------
constexpr int kSmallCin = 8;
constexpr int kSmallMaxTaps = 27;

__global__ void __launch_bounds__(kTileRows) conv3d_small_cin_kernel(nnb_conv3d_args a, int tps) {
  __shared__ float w_s[kSmallMaxTaps * kSmallCin * 32];  // [tap][ci][co]
  __shared__ float out_s[kTileRows][33];
  const int t = blockIdx.x % tps;
  const int b = blockIdx.x / tps;
  const int co0 = blockIdx.y * 32;
  const int r = threadIdx.x;
  const int cin = a.seg[0].channels;
  const int kvol = a.kernel[0] * a.kernel[1] * a.kernel[2];
  for (int i = threadIdx.x; i < kvol * cin * 32; i += blockDim.x) {
    const int co = i % 32, ci = (i / 32) % cin, tap = i / (32 * cin);
    w_s[i] = co0 + co < a.cout ? a.weight[((int64_t)(co0 + co) * kvol + tap) * cin + ci] : 0.f;
  }
  __syncthreads();
  const int OD = a.out_dims[0], OH = a.out_dims[1], OW = a.out_dims[2];
  const int ID = a.in_dims[0], IH = a.in_dims[1], IW = a.in_dims[2];
  const int64_t ovox = (int64_t)OD * OH * OW;
  const int64_t m = (int64_t)t * kTileRows + r;
  const bool valid = m < ovox;
  const int ox = (int)(m % OW), oy = (int)((m / OW) % OH), oz = (int)(m / ((int64_t)OW * OH));
  const nnb_segment seg = a.seg[0];
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  if (valid) {
    int tap = 0;
    for (int kz = 0; kz < a.kernel[0]; ++kz) {
      const int iz = oz * a.stride[0] - a.pad[0] + kz;
      for (int ky = 0; ky < a.kernel[1]; ++ky) {
        const int iy = oy * a.stride[1] - a.pad[1] + ky;
        for (int kx = 0; kx < a.kernel[2]; ++kx, ++tap) {
          const int ix = ox * a.stride[2] - a.pad[2] + kx;
          if (iz < 0 || iz >= ID || iy < 0 || iy >= IH || ix < 0 || ix >= IW) continue;
          const float* src = seg.data + ((((int64_t)b * ID + iz) * IH + iy) * IW + ix) * cin;
          for (int ci = 0; ci < cin; ++ci) {
            const float v = activate(__ldg(src + ci), seg.scale, seg.shift, seg.leaky, a.slope, b * cin + ci);
            const float* wp = w_s + (tap * cin + ci) * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[j] = fmaf(v, wp[j], acc[j]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (a.bias != nullptr && co0 + j < a.cout) acc[j] += __ldg(a.bias + co0 + j);
    out_s[r][j] = valid ? acc[j] : 0.f;
  }
  __syncthreads();
  // coalesced store of the valid rows: 8 threads per row, 16 bytes each
  const int rows = (int)min((int64_t)kTileRows, ovox - (int64_t)t * kTileRows);
  const int ncols = min(32, a.cout - co0);
  float* base = a.out + ((int64_t)b * ovox + (int64_t)t * kTileRows) * a.cout + co0;
  if (ncols == 32 && (a.cout % 4) == 0) {
    for (int i = threadIdx.x; i < rows * 8; i += blockDim.x) {
      const int row = i >> 3, c4 = (i & 7) * 4;
      *reinterpret_cast<float4*>(base + (int64_t)row * a.cout + c4) =
          make_float4(out_s[row][c4], out_s[row][c4 + 1], out_s[row][c4 + 2], out_s[row][c4 + 3]);
    }
  } else {
    for (int i = threadIdx.x; i < rows * 32; i += blockDim.x) {
      const int row = i >> 5, c = i & 31;
      if (c < ncols) base[(int64_t)row * a.cout + c] = out_s[row][c];
    }
  }
  if (a.partials == nullptr) return;
  if (r < ncols) {
    float sum = 0.f;
    for (int i = 0; i < rows; ++i) sum += out_s[i][r];
    const float mean = sum / rows;
    float m2 = 0.f;
    for (int i = 0; i < rows; ++i) {
      const float d = out_s[i][r] - mean;
      m2 = fmaf(d, d, m2);
    }
    float* p = a.partials + (((int64_t)b * a.cout + co0 + r) * tps + t) * 3;
    p[0] = sum;
    p[1] = m2;
    p[2] = (float)rows;
  }
}

// ---------------------------------------------------------------------------
// The first layer's shape (1, 2 or 4 raw input channels, 3x3x3, stride 1,
// padding 1, 32-channel output groups): compile-time taps and channels, each
// of 64 threads computes two voxels of a 128-voxel tile (rows r and r + 64)
// so every float4 weight read from shared memory feeds 8 FMAs, and the padding
// test is three per-axis 3-bit masks computed once.  Persistent blocks (the
// weights are staged once per block, not per tile); the (sum, M2, n) partials
// come from warp transpose-reductions; rows leave through a swizzled shared
// buffer as whole 128-byte rows.
// ---------------------------------------------------------------------------
template <int CIN>
__global__ void __launch_bounds__(64) conv3d_first_kernel(nnb_conv3d_args a, int tps, int64_t total_tiles) {
  __shared__ float4 w_s[27 * CIN * 8];       // [tap][ci][co/4]
  __shared__ float4 out_s[kTileRows * 8];    // 128 rows x 32 floats, 16-byte chunks XOR-swizzled by row % 8
  __shared__ float red_s[2][32];
  __shared__ float mean_s[32], sum_s[32];
  const int co0 = blockIdx.y * 32;
  for (int i = threadIdx.x; i < 27 * CIN * 32; i += blockDim.x) {
    const int co = i % 32, ci = (i / 32) % CIN, tap = i / (32 * CIN);
    reinterpret_cast<float*>(w_s)[i] = co0 + co < a.cout ? a.weight[((int64_t)(co0 + co) * 27 + tap) * CIN + ci] : 0.f;
  }
  __syncthreads();
  const int D = a.out_dims[0], H = a.out_dims[1], W = a.out_dims[2];
  const int64_t ovox = (int64_t)D * H * W;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ncols = min(32, a.cout - co0);
  for (int64_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
    const int t = (int)(tile % tps);
    const int b = (int)(tile / tps);
    const float* x = a.seg[0].data + (int64_t)b * ovox * CIN;
    // accumulators as float pairs (channels 2j, 2j+1) for packed f32x2 FMAs: each pair is two fmaf's with
    // the same operands and rounding, so the result equals the scalar FMA chain's bit for bit
    unsigned long long acc2[2][16];
    float acc[2][32];
    int base[2];
    uint32_t mask[2];  // bits 0-8: kx, ky, kz validity (3 bits each)
    bool valid[2];
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const int64_t m = (int64_t)t * kTileRows + threadIdx.x + 64 * v;
      valid[v] = m < ovox;
      const int ox = (int)(m % W), oy = (int)((m / W) % H), oz = (int)(m / ((int64_t)W * H));
      uint32_t mk = 0;
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        mk |= (uint32_t)(valid[v] && ox + k - 1 >= 0 && ox + k - 1 < W) << k;
        mk |= (uint32_t)(valid[v] && oy + k - 1 >= 0 && oy + k - 1 < H) << (3 + k);
        mk |= (uint32_t)(valid[v] && oz + k - 1 >= 0 && oz + k - 1 < D) << (6 + k);
      }
      mask[v] = mk;
      base[v] = valid[v] ? (int)((((int64_t)(oz - 1) * H + (oy - 1)) * W + (ox - 1)) * CIN) : 0;
#pragma unroll
      for (int j = 0; j < 16; ++j) acc2[v][j] = 0ull;
    }
#pragma unroll
    for (int kz = 0; kz < 3; ++kz) {
#pragma unroll
      for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int tap = (kz * 3 + ky) * 3 + kx;
          const int off = ((kz * H + ky) * W + kx) * CIN;
          unsigned long long xv[2][CIN];
#pragma unroll
          for (int v = 0; v < 2; ++v) {
            const bool in = (mask[v] >> kx & 1) & (mask[v] >> (3 + ky) & 1) & (mask[v] >> (6 + kz) & 1);
#pragma unroll
            for (int ci = 0; ci < CIN; ++ci) {
              const float xs = in ? __ldg(x + base[v] + off + ci) : 0.f;
              asm("mov.b64 %0, {%1, %1};" : "=l"(xv[v][ci]) : "f"(xs));
            }
          }
#pragma unroll
          for (int ci = 0; ci < CIN; ++ci) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const ulonglong2 w = reinterpret_cast<const ulonglong2*>(w_s)[(tap * CIN + ci) * 8 + q];
#pragma unroll
              for (int v = 0; v < 2; ++v) {
                asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc2[v][2 * q]) : "l"(xv[v][ci]), "l"(w.x));
                asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc2[v][2 * q + 1]) : "l"(xv[v][ci]), "l"(w.y));
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int v = 0; v < 2; ++v)
#pragma unroll
      for (int j = 0; j < 16; ++j) asm("mov.b64 {%0, %1}, %2;" : "=f"(acc[v][2 * j]), "=f"(acc[v][2 * j + 1]) : "l"(acc2[v][j]));
    if (a.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float bj = co0 + j < a.cout ? __ldg(a.bias + co0 + j) : 0.f;
        acc[0][j] += bj;
        acc[1][j] += bj;
      }
    }
#pragma unroll
    for (int v = 0; v < 2; ++v)
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[v][j] = valid[v] ? acc[v][j] : 0.f;
    const int rows = (int)min((int64_t)kTileRows, ovox - (int64_t)t * kTileRows);
    // rows leave through the staging buffer (the previous tile's readers finished at its last barrier)
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const int r = threadIdx.x + 64 * v;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        out_s[r * 8 + (q ^ (r & 7))] = make_float4(acc[v][4 * q], acc[v][4 * q + 1], acc[v][4 * q + 2], acc[v][4 * q + 3]);
    }
    if (a.partials != nullptr) {
      float xs[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) xs[j] = acc[0][j] + acc[1][j];
      const float s = warp_column_sums(xs);
      red_s[warp][lane] = s;
    }
    __syncthreads();
    float* dst = a.out + ((int64_t)b * ovox + (int64_t)t * kTileRows) * a.cout + co0;
    if (ncols == 32 && (a.cout % 4) == 0) {
      for (int i = threadIdx.x; i < rows * 8; i += blockDim.x) {
        const int row = i >> 3, c = i & 7;
        *reinterpret_cast<float4*>(dst + (int64_t)row * a.cout + 4 * c) = out_s[row * 8 + (c ^ (row & 7))];
      }
    } else {
      for (int i = threadIdx.x; i < rows * 32; i += blockDim.x) {
        const int row = i >> 5, c = i & 31;
        if (c < ncols) dst[(int64_t)row * a.cout + c] = reinterpret_cast<const float*>(out_s)[row * 32 + (((c >> 2) ^ (row & 7)) << 2) + (c & 3)];
      }
    }
    if (a.partials != nullptr) {
      if (threadIdx.x < 32) {
        const float sum = red_s[0][threadIdx.x] + red_s[1][threadIdx.x];
        sum_s[threadIdx.x] = sum;
        mean_s[threadIdx.x] = sum / (float)rows;
      }
      __syncthreads();
      float xs[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float m = mean_s[j];
        const float d0 = valid[0] ? acc[0][j] - m : 0.f, d1 = valid[1] ? acc[1][j] - m : 0.f;
        xs[j] = fmaf(d0, d0, d1 * d1);
      }
      const float m2w = warp_column_sums(xs);
      __syncthreads();  // every thread has read mean_s / red_s of this tile
      red_s[warp][lane] = m2w;
      __syncthreads();
      if (threadIdx.x < ncols) {
        const int c = threadIdx.x;
        float* p = a.partials + (((int64_t)b * a.cout + co0 + c) * tps + t) * 3;
        p[0] = sum_s[c];
        p[1] = red_s[0][c] + red_s[1][c];
        p[2] = (float)rows;
      }
    }
    __syncthreads();  // staging and reduction buffers are free for the next tile
  }
}

// ---------------------------------------------------------------------------
// Pointwise head (1x1x1, one lazy segment of <= 64 channels, <= 8 outputs, no
// statistics): the segmentation head of the network's tile-callable seam.  One
// thread per voxel reads its features with 16-byte loads, applies the lazy
// affine + LeakyReLU, and writes its logits; HBM-bound on the feature read.
// ---------------------------------------------------------------------------
constexpr int kPointMaxCin = 64;
constexpr int kPointMaxCout = 8;

__global__ void __launch_bounds__(256) conv3d_pointwise_kernel(nnb_conv3d_args a, int64_t ovox) {
  __shared__ float w_s[kPointMaxCout][kPointMaxCin];
  __shared__ float b_s[kPointMaxCout];
  const nnb_segment seg = a.seg[0];
  const int cin = seg.channels, cout = a.cout;
  const int b = blockIdx.y;
  for (int i = threadIdx.x; i < kPointMaxCout * kPointMaxCin; i += blockDim.x) {
    const int co = i / kPointMaxCin, ci = i % kPointMaxCin;
    w_s[co][ci] = (co < cout && ci < cin) ? a.weight[(int64_t)co * cin + ci] : 0.f;
  }
  if (threadIdx.x < kPointMaxCout)
    b_s[threadIdx.x] = (a.bias != nullptr && (int)threadIdx.x < cout) ? a.bias[threadIdx.x] : 0.f;
  __syncthreads();
  const float* sc = seg.scale ? seg.scale + (int64_t)b * cin : nullptr;
  const float* sh = seg.scale ? seg.shift + (int64_t)b * cin : nullptr;
  for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < ovox; m += (int64_t)gridDim.x * blockDim.x) {
    const float4* src = reinterpret_cast<const float4*>(seg.data + ((int64_t)b * ovox + m) * cin);
    float y[kPointMaxCout];
#pragma unroll
    for (int co = 0; co < kPointMaxCout; ++co) y[co] = b_s[co];
    for (int c4 = 0; c4 < cin / 4; ++c4) {
      const float4 x4 = __ldg(src + c4);
      const float xs[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ci = c4 * 4 + e;
        float v = xs[e];
        if (sc != nullptr) {
          v = fmaf(v, __ldg(sc + ci), __ldg(sh + ci));
          if (seg.leaky) v = leaky(v, a.slope);
        }
#pragma unroll
        for (int co = 0; co < kPointMaxCout; ++co) y[co] = fmaf(v, w_s[co][ci], y[co]);
      }
    }
    float* dst = a.out + ((int64_t)b * ovox + m) * cout;
#pragma unroll
    for (int co = 0; co < kPointMaxCout; ++co)
      if (co < cout) dst[co] = y[co];
  }
}

static bool pointwise_shape(const nnb_conv3d_args& a) {
  if (a.num_segments != 1 || a.partials != nullptr) return false;
  if (a.seg[0].channels % 4 != 0 || a.seg[0].channels > kPointMaxCin || a.cout > kPointMaxCout) return false;
  if ((reinterpret_cast<uintptr_t>(a.seg[0].data) & 15) != 0) return false;
  for (int i = 0; i < 3; ++i)
    if (a.kernel[i] != 1 || a.stride[i] != 1 || a.pad[i] != 0) return false;
  return true;
}

static bool first_layer_shape(const nnb_conv3d_args& a) {
  if (a.num_segments != 1 || a.seg[0].scale != nullptr) return false;
  const int c = a.seg[0].channels;
  if (c != 1 && c != 2 && c != 4) return false;
  for (int i = 0; i < 3; ++i)
    if (a.kernel[i] != 3 || a.stride[i] != 1 || a.pad[i] != 1 || a.in_dims[i] != a.out_dims[i]) return false;
  // per-sample element offsets fit in int (base[] arithmetic)
  return (int64_t)a.out_dims[0] * a.out_dims[1] * a.out_dims[2] * c < (1LL << 31);
}

int launch_conv3d_simt(const nnb_conv3d_args& a, cudaStream_t stream) {
  const int64_t ovox = (int64_t)a.out_dims[0] * a.out_dims[1] * a.out_dims[2];
  const int tps = tiles_per_sample(ovox);
  if (pointwise_shape(a)) {
    NNB_REQUIRE(a.batch < 65536, "conv3d: batch too large for the pointwise grid");
    const int blocks = (int)std::min<int64_t>((ovox + 255) / 256, 148 * 8);
    conv3d_pointwise_kernel<<<dim3((unsigned)blocks, (unsigned)a.batch), 256, 0, stream>>>(a, ovox);
    NNB_LAUNCH_CHECK();
    return NNB_OK;
  }
  if (first_layer_shape(a)) {
    const int64_t total_tiles = (int64_t)tps * a.batch;
    const int groups = (a.cout + 31) / 32;
    // persistent blocks: as many as are resident at once over all SMs, split across the channel groups
    int per_sm = 0, sms = 148, dev = 0;
    NNB_CUDA_CHECK(cudaGetDevice(&dev));
    NNB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    switch (a.seg[0].channels) {
      case 1: NNB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv3d_first_kernel<1>, 64, 0)); break;
      case 2: NNB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv3d_first_kernel<2>, 64, 0)); break;
      default: NNB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, conv3d_first_kernel<4>, 64, 0)); break;
    }
    const int64_t resident = std::max<int64_t>(1, (int64_t)std::max(per_sm, 1) * sms / groups);
    dim3 grid((unsigned)std::min<int64_t>(total_tiles, resident), (unsigned)groups);
    switch (a.seg[0].channels) {
      case 1: conv3d_first_kernel<1><<<grid, 64, 0, stream>>>(a, tps, total_tiles); break;
      case 2: conv3d_first_kernel<2><<<grid, 64, 0, stream>>>(a, tps, total_tiles); break;
      default: conv3d_first_kernel<4><<<grid, 64, 0, stream>>>(a, tps, total_tiles); break;
    }
    NNB_LAUNCH_CHECK();
    return NNB_OK;
  }
  if (a.num_segments == 1 && a.seg[0].channels <= kSmallCin &&
      a.kernel[0] * a.kernel[1] * a.kernel[2] <= kSmallMaxTaps) {
    dim3 grid((unsigned)((int64_t)tps * a.batch), (unsigned)((a.cout + 31) / 32));
    NNB_REQUIRE((int64_t)tps * a.batch < (1LL << 31), "conv3d: too many tiles");
    conv3d_small_cin_kernel<<<grid, kTileRows, 0, stream>>>(a, tps);
    NNB_LAUNCH_CHECK();
    return NNB_OK;
  }
  constexpr int CO = 16;
  dim3 grid((unsigned)((int64_t)tps * a.batch), (unsigned)((a.cout + CO - 1) / CO));
  NNB_REQUIRE((int64_t)tps * a.batch < (1LL << 31), "conv3d: too many tiles");
  conv3d_simt_kernel<CO><<<grid, kTileRows, 0, stream>>>(a, tps);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

// ---------------------------------------------------------------------------
// Instance-norm finalisation: one block per (channel, sample) over its
// contiguous run of per-tile (sum, M2, n) records, in float64 and one pass.
// With K the first record's mean and d_t = sum_t - n_t K, the parallel-variance
// identity M2 = sum_t [ M2_t + (sum_t - n_t mean)^2 / n_t ] expands to
//   M2 = sum_t M2_t + sum_t d_t^2 / n_t - D^2 / N,   D = sum_t d_t, N = sum_t n_t,
// so every record is read once and contributes four independent terms.  The
// shift keeps the cancellation harmless: (mean - K)^2 <= (N / n_0) var, so the
// relative error of the difference is at most (tiles) x 2^-52.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) norm_finalize_kernel(const float* __restrict__ partials,
                                                            int channels, int tps,
                                                            const float* __restrict__ gamma,
                                                            const float* __restrict__ beta, float eps,
                                                            float* __restrict__ scale,
                                                            float* __restrict__ shift) {
  __shared__ double red[4][32];
  const int c = blockIdx.x;
  const int b = blockIdx.y;
  const float* run = partials + ((int64_t)b * channels + c) * tps * 3;
  const double n0 = (double)run[2];
  const double K = n0 > 0.0 ? (double)run[0] / n0 : 0.0;
  double v[4] = {0.0, 0.0, 0.0, 0.0};  // sum_t sum_t, sum_t n_t, sum_t M2_t, sum_t d_t^2 / n_t
#pragma unroll 4
  for (int t = threadIdx.x; t < tps; t += blockDim.x) {
    const double st = (double)run[3 * t], mt = (double)run[3 * t + 1], nt = (double)run[3 * t + 2];
    if (nt <= 0.0) continue;
    const double d = st - nt * K;
    v[0] += st;
    v[1] += nt;
    v[2] += mt;
    v[3] += d * d / nt;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v[k] += __shfl_xor_sync(0xffffffffu, v[k], off);
    if (lane == 0) red[k][warp] = v[k];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot[4] = {0.0, 0.0, 0.0, 0.0};
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
#pragma unroll
      for (int k = 0; k < 4; ++k) tot[k] += red[k][w];
    const double count = tot[1];
    const double mean = count > 0.0 ? tot[0] / count : 0.0;
    const double D = tot[0] - count * K;
    const double m2 = count > 0.0 ? tot[2] + tot[3] - D * D / count : 0.0;
    double var = count > 0.0 ? m2 / count : 0.0;
    if (var < 0) var = 0;
    const double inv = 1.0 / sqrt(var + (double)eps);
    const double sc = gamma != nullptr ? (double)gamma[c] * inv : inv;
    const double sh = (beta != nullptr ? (double)beta[c] : 0.0) - mean * sc;
    scale[(int64_t)b * channels + c] = (float)sc;
    shift[(int64_t)b * channels + c] = (float)sh;
  }
}

int launch_norm_finalize(const float* partials, int batch, int tiles, int channels, const float* gamma,
                         const float* beta, float eps, float* scale, float* shift, cudaStream_t stream) {
  dim3 grid((unsigned)channels, (unsigned)batch);
  // 1024 threads: a 128^3 layer's 16384 records per (sample, channel) are 16 loads per thread, in flight together
  norm_finalize_kernel<<<grid, tiles >= 4096 ? 1024 : 256, 0, stream>>>(partials, channels, tiles, gamma, beta, eps,
                                                                          scale, shift);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

// ---------------------------------------------------------------------------
// Transposed convolution with kernel == stride (non-overlapping blocks):
// one thread per output voxel and 32-channel output group.
// Reference: NonOverlappingConvTranspose3d (network.py:139-174).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) conv_transpose_simt_kernel(nnb_segment in, int batch, int ID, int IH,
                                                                  int IW, int KD, int KH, int KW, float slope,
                                                                  const float* __restrict__ weight,
                                                                  const float* __restrict__ bias, int cout,
                                                                  float* __restrict__ out) {
  const int OD = ID * KD, OH = IH * KH, OW = IW * KW;
  const int64_t total = (int64_t)batch * OD * OH * OW;
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= total) return;
  const int ox = (int)(o % OW), oy = (int)((o / OW) % OH), oz = (int)((o / ((int64_t)OW * OH)) % OD);
  const int b = (int)(o / ((int64_t)OW * OH * OD));
  const int ix = ox / KW, iy = oy / KH, iz = oz / KD;
  const int tap = ((oz % KD) * KH + (oy % KH)) * KW + (ox % KW);
  const int kvol = KD * KH * KW;
  const int cin = in.channels;
  const float* src = in.data + ((((int64_t)b * ID + iz) * IH + iy) * IW + ix) * cin;
  const int co0 = blockIdx.y * 32;
  const int nco = min(32, cout - co0);
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  for (int ci = 0; ci < cin; ++ci) {
    const float v = activate(__ldg(src + ci), in.scale, in.shift, in.leaky, slope, b * cin + ci);
    const float* wp = weight + ((int64_t)co0 * kvol + tap) * cin + ci;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nco) acc[j] = fmaf(v, __ldg(wp + (int64_t)j * kvol * cin), acc[j]);
  }
  float* dst = out + o * cout + co0;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < nco) dst[j] = acc[j] + (bias != nullptr ? __ldg(bias + co0 + j) : 0.f);
}

int launch_conv_transpose_simt(const nnb_segment& in, int batch, const int32_t in_dims[3], const int32_t k[3],
                               float slope, const float* weight, const float* bias, int cout, float* out,
                               cudaStream_t stream) {
  const int64_t total = (int64_t)batch * in_dims[0] * k[0] * in_dims[1] * k[1] * in_dims[2] * k[2];
  dim3 grid((unsigned)((total + 127) / 128), (unsigned)((cout + 31) / 32));
  NNB_REQUIRE((total + 127) / 128 < (1LL << 31), "conv_transpose3d: output too large");
  conv_transpose_simt_kernel<<<grid, 128, 0, stream>>>(in, batch, in_dims[0], in_dims[1], in_dims[2], k[0], k[1],
                                                       k[2], slope, weight, bias, cout, out);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

// ---------------------------------------------------------------------------
// Residual join: out = LeakyReLU(act(branch) + act(skip)), float4 vectorised.
// One float4 per thread step covers 4 channels of one voxel (channels % 4 == 0), so the sample and channel
// indices come from one division of the float4 index and the per-(sample, channel) affine is read as float4s;
// 32-bit index arithmetic when the element count allows it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float4 affine4(const nnb_segment& s, int idx, float4 x, float slope) {
  if (s.scale == nullptr) return x;
  const float4 sc = __ldg(reinterpret_cast<const float4*>(s.scale + idx));
  const float4 sh = __ldg(reinterpret_cast<const float4*>(s.shift + idx));
  float4 y = make_float4(fmaf(x.x, sc.x, sh.x), fmaf(x.y, sc.y, sh.y), fmaf(x.z, sc.z, sh.z), fmaf(x.w, sc.w, sh.w));
  if (s.leaky) y = make_float4(leaky(y.x, slope), leaky(y.y, slope), leaky(y.z, slope), leaky(y.w, slope));
  return y;
}

template <typename Index>
__global__ void residual_join_kernel(nnb_segment br, nnb_segment sk, Index voxels, int channels, Index total4,
                                     float slope, float* __restrict__ out) {
  const Index c4n = (Index)(channels / 4);
  for (Index i4 = (Index)blockIdx.x * blockDim.x + threadIdx.x; i4 < total4; i4 += (Index)gridDim.x * blockDim.x) {
    const Index vox = i4 / c4n;                   // voxel over all samples
    const int c = (int)(i4 - vox * c4n) * 4;      // first of the float4's channels
    const int b = (int)(vox / voxels);            // sample
    const int idx = b * channels + c;
    const float4 u = affine4(br, idx, __ldg(reinterpret_cast<const float4*>(br.data) + i4), slope);
    const float4 w = affine4(sk, idx, __ldg(reinterpret_cast<const float4*>(sk.data) + i4), slope);
    reinterpret_cast<float4*>(out)[i4] = make_float4(leaky(u.x + w.x, slope), leaky(u.y + w.y, slope),
                                                     leaky(u.z + w.z, slope), leaky(u.w + w.w, slope));
  }
}

// Channel counts that are not a multiple of 4 (or unaligned tensors): one element per thread step.
__global__ void residual_join_scalar_kernel(nnb_segment br, nnb_segment sk, int64_t per_sample, int channels,
                                            int64_t total, float slope, float* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int idx = (int)(i / per_sample) * channels + (int)(i % channels);
    const float u = activate(__ldg(br.data + i), br.scale, br.shift, br.leaky, slope, idx);
    const float w = activate(__ldg(sk.data + i), sk.scale, sk.shift, sk.leaky, slope, idx);
    out[i] = leaky(u + w, slope);
  }
}

int launch_residual_join(const nnb_segment& br, const nnb_segment& sk, int batch, int64_t voxels, float slope,
                         float* out, cudaStream_t stream) {
  NNB_REQUIRE(br.channels == sk.channels, "residual_join: channel mismatch");
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  bool vec = br.channels % 4 == 0 && aligned(br.data) && aligned(sk.data) && aligned(out);
  for (const nnb_segment* s : {&br, &sk})
    vec = vec && (s->scale == nullptr || (aligned(s->scale) && aligned(s->shift)));
  if (!vec) {
    const int64_t total = voxels * batch * br.channels;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    residual_join_scalar_kernel<<<blocks, 256, 0, stream>>>(br, sk, voxels * br.channels, br.channels, total, slope,
                                                            out);
    NNB_LAUNCH_CHECK();
    return NNB_OK;
  }
  const int64_t total4 = voxels * batch * (br.channels / 4);
  const int blocks = (int)std::min<int64_t>((total4 + 255) / 256, 148 * 16);
  if (total4 + (int64_t)blocks * 256 < (1LL << 31))
    residual_join_kernel<int32_t><<<blocks, 256, 0, stream>>>(br, sk, (int32_t)voxels, br.channels, (int32_t)total4,
                                                              slope, out);
  else
    residual_join_kernel<int64_t><<<blocks, 256, 0, stream>>>(br, sk, voxels, br.channels, total4, slope, out);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

}  // namespace nnb

namespace nnb {

// ---------------------------------------------------------------------------
// Operand preparation for the tensor-core convolution: one pass over a lazy
// activation that applies its instance-norm affine + LeakyReLU once per
// element (instead of once per tap inside the convolution) and writes the
// form the MMA consumes:
//   kOperandF16x2   per voxel and 32-channel group [hi(32) | lo(32)] as
//                   halves, hi = fp16(x), lo = fp16(x - hi); an element
//                   with |x| >= 65504 (no finite fp16 hi) increments
//                   g_operand_range_events.  4 bytes read, 4 written.
//   kOperandTf32x2  per voxel [hi(C) | lo(C)], hi = x with the 13 low mantissa
//                   bits cleared, lo = x - hi (both exact).  4 read, 8 written.
//   kOperandTf32    x rounded to TF32 (nearest).  4 read, 4 written.
//   kOperandBf16    per voxel and 32-channel group [bf16(x)(32) | (32)] as
//                   bf16 halves (the fp16 pair's row layout); the MMA reads
//                   only the first half, so the second is not written.
//                   4 read, 2 written.
// ---------------------------------------------------------------------------
__device__ unsigned long long g_operand_range_events = 0;

__global__ void prepare_operand_kernel(nnb_segment in, int64_t voxels_total, int64_t per_sample_vox, float slope,
                                       int op, float* __restrict__ out, unsigned long long* range_events) {
  const int C = in.channels;
  const int c8n = C / 8;  // 8 channels per thread
  const int64_t total = voxels_total * c8n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t vox = i / c8n;
    const int c8 = (int)(i - vox * c8n) * 8;
    const int b = (int)(vox / per_sample_vox);
    const float4 x0 = __ldg(reinterpret_cast<const float4*>(in.data) + 2 * i);
    const float4 x1 = __ldg(reinterpret_cast<const float4*>(in.data) + 2 * i + 1);
    float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = activate(v[e], in.scale, in.shift, in.leaky, slope, b * C + c8 + e);
    if (op == kOperandF16x2) {
      uint32_t hi[4], lo[4];
      int over = 0;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const __half h0 = __float2half_rn(v[e]), h1 = __float2half_rn(v[e + 1]);
        const __half l0 = __float2half_rn(v[e] - __half2float(h0));
        const __half l1 = __float2half_rn(v[e + 1] - __half2float(h1));
        hi[e / 2] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
        lo[e / 2] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        over += (fabsf(v[e]) >= 65504.f) + (fabsf(v[e + 1]) >= 65504.f);
      }
      if (over) atomicAdd(range_events, (unsigned long long)over);
      // group g = c8 / 32 occupies halves [64 g, 64 g + 64) of the voxel's 2 C
      __half* base = reinterpret_cast<__half*>(out) + vox * 2 * C + (c8 / 32) * 64 + (c8 % 32);
      *reinterpret_cast<uint4*>(base) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      *reinterpret_cast<uint4*>(base + 32) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    } else if (op == kOperandBf16) {
      uint32_t hb[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const __nv_bfloat162 bb = __floats2bfloat162_rn(v[e], v[e + 1]);
        hb[e / 2] = *reinterpret_cast<const uint32_t*>(&bb);
      }
      __half* base = reinterpret_cast<__half*>(out) + vox * 2 * C + (c8 / 32) * 64 + (c8 % 32);
      *reinterpret_cast<uint4*>(base) = make_uint4(hb[0], hb[1], hb[2], hb[3]);
    } else if (op == kOperandTf32x2) {
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        hi[e] = __uint_as_float(__float_as_uint(v[e]) & 0xFFFFE000u);
        lo[e] = v[e] - hi[e];
      }
      float* dst = out + vox * 2 * C + c8;
      reinterpret_cast<float4*>(dst)[0] = make_float4(hi[0], hi[1], hi[2], hi[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(hi[4], hi[5], hi[6], hi[7]);
      reinterpret_cast<float4*>(dst + C)[0] = make_float4(lo[0], lo[1], lo[2], lo[3]);
      reinterpret_cast<float4*>(dst + C)[1] = make_float4(lo[4], lo[5], lo[6], lo[7]);
    } else {
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint32_t t;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(v[e]));
        r[e] = __uint_as_float(t);
      }
      float* dst = out + vox * C + c8;
      reinterpret_cast<float4*>(dst)[0] = make_float4(r[0], r[1], r[2], r[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
  }
}

unsigned long long* operand_range_events_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_operand_range_events) != cudaSuccess) return nullptr;
  return static_cast<unsigned long long*>(p);
}

int launch_prepare_operand(const nnb_segment& in, int batch, int64_t voxels, float slope, int op, float* out,
                           cudaStream_t stream) {
  NNB_REQUIRE(in.channels % (half_rows(op) ? 32 : 8) == 0,
              "prepare_operand: channels must be a multiple of %d", half_rows(op) ? 32 : 8);
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(in.data) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
              "prepare_operand: 16-byte aligned tensors required");
  unsigned long long* events = operand_range_events_ptr();
  NNB_REQUIRE(events != nullptr, "prepare_operand: range-event counter unavailable: %s",
              cudaGetErrorString(cudaGetLastError()));
  const int64_t total = (int64_t)batch * voxels * (in.channels / 8);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
  prepare_operand_kernel<<<blocks, 256, 0, stream>>>(in, (int64_t)batch * voxels, voxels, slope, op, out, events);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int64_t operand_range_events(int reset) {
  unsigned long long count = 0;
  // every stream's preparation kernels, not only those ordered with the legacy default stream
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(&count, g_operand_range_events, sizeof(count)) != cudaSuccess) {
    set_error("operand_range_events: %s", cudaGetErrorString(cudaGetLastError()));
    return NNB_E_CUDA;
  }
  if (reset) {
    const unsigned long long zero = 0;
    if (cudaMemcpyToSymbol(g_operand_range_events, &zero, sizeof(zero)) != cudaSuccess) {
      set_error("operand_range_events: %s", cudaGetErrorString(cudaGetLastError()));
      return NNB_E_CUDA;
    }
  }
  return count > (unsigned long long)INT64_MAX ? INT64_MAX : (int64_t)count;
}

}  // namespace nnb
