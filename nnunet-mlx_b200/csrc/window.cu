// Sliding-window kernels: mirrored tile gather, fused segmentation head +
// flip-back + Gaussian accumulation (float32 or float16 accumulator), and
// normalise + label reduction (float32 accumulator, or the float16 per-fold
// normalise / fold sum / fold average of the nnunet-fp16 mode).  All are
// HBM-bound streaming kernels.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"

namespace nnb {

struct Dims3 {
  int d[3];
};

// ---------------------------------------------------------------------------
// Tile gather: item t of the batch is the patch at offset off[t] (coordinates
// of the zero-padded volume) of a (cin, Z, Y, X) volume, flipped along axis a
// when bit a of mask[t] is set, written channels-last (items, P0, P1, P2, cin).
// The volume is read unpadded: padded coordinate c maps to c - pad_lo, and
// positions outside the volume load 0 (the reference's _pad_minimum zeros).
// Every loaded value is checked for finiteness (the reference validates the
// input before inference, sliding_window.py:463-486): each thread that met a
// non-finite value adds 1 to *nonfinite.
// Reference: tile slice + mx.flip (sliding_window.py:408-411,517-518).
// ---------------------------------------------------------------------------
// Up to 8 items (every subset of 3 mirroring axes, or tiles mixed in a batch); carried by value.
struct ViewMasks {
  int m[8];
};

struct ItemTable {
  int off[8][3];
  int mask[8];
};

__global__ void gather_tiles_kernel(const float* __restrict__ vol, int cin, Dims3 vd, Dims3 pad_lo, Dims3 patch,
                                    int items, ItemTable tab, float* __restrict__ out, int* __restrict__ nonfinite) {
  // one warp per output row (item t, i, j): the row's source row and flips are resolved once, lanes walk k
  const int64_t rows = (int64_t)items * patch.d[0] * patch.d[1];
  const int64_t vstride = (int64_t)vd.d[0] * vd.d[1] * vd.d[2];
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  bool bad = false;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const int j = (int)(r % patch.d[1]);
    const int64_t ti = r / patch.d[1];
    const int i = (int)(ti % patch.d[0]);
    const int t = (int)(ti / patch.d[0]);
    const int mask = tab.mask[t];
    const int z = tab.off[t][0] + ((mask & 1) ? patch.d[0] - 1 - i : i) - pad_lo.d[0];
    const int y = tab.off[t][1] + ((mask & 2) ? patch.d[1] - 1 - j : j) - pad_lo.d[1];
    const bool row_in = (unsigned)z < (unsigned)vd.d[0] && (unsigned)y < (unsigned)vd.d[1];
    const int64_t src_row = row_in ? ((int64_t)z * vd.d[1] + y) * vd.d[2] : 0;
    const int x0 = tab.off[t][2] - pad_lo.d[2];
    const bool flip_x = (mask & 4) != 0;
    float* dst_row = out + r * patch.d[2] * cin;
    for (int k = lane; k < patch.d[2]; k += 32) {
      const int x = x0 + (flip_x ? patch.d[2] - 1 - k : k);
      float* dst = dst_row + (int64_t)k * cin;
      if (!row_in || (unsigned)x >= (unsigned)vd.d[2]) {
        for (int c = 0; c < cin; ++c) dst[c] = 0.f;
        continue;
      }
      for (int c = 0; c < cin; ++c) {
        const float v = __ldg(vol + (int64_t)c * vstride + src_row + x);
        bad |= !isfinite(v);
        dst[c] = v;
      }
    }
  }
  if (bad && nonfinite != nullptr) atomicAdd(nonfinite, 1);
}

int launch_gather_tiles(const float* vol, int cin, const int32_t vd[3], const int32_t pad_lo[3], int items,
                        const int32_t* offsets, const int32_t* masks, const int32_t patch[3], float* out,
                        int32_t* nonfinite, cudaStream_t stream) {
  NNB_REQUIRE(items >= 1 && items <= 8, "gather_tiles: 1..8 items per batch, got %d", items);
  ItemTable tab{};
  for (int t = 0; t < items; ++t) {
    NNB_REQUIRE(masks[t] >= 0 && masks[t] < 8, "gather_tiles: bad flip mask");
    tab.mask[t] = masks[t];
    for (int a = 0; a < 3; ++a) {
      // the patch must lie inside the padded extent [0, pad_lo + vd + pad_lo + 1)
      NNB_REQUIRE(offsets[3 * t + a] >= 0 && offsets[3 * t + a] + patch[a] <= vd[a] + 2 * pad_lo[a] + 1,
                  "gather_tiles: item %d lies outside the padded volume on axis %d", t, a);
      tab.off[t][a] = offsets[3 * t + a];
    }
  }
  Dims3 dvd{{vd[0], vd[1], vd[2]}}, dpad{{pad_lo[0], pad_lo[1], pad_lo[2]}}, dp{{patch[0], patch[1], patch[2]}};
  const int64_t rows = (int64_t)patch[0] * patch[1] * items;
  const int blocks = (int)std::min<int64_t>((rows + 7) / 8, 148 * 32);  // 8 warps (rows) per block
  gather_tiles_kernel<<<blocks, 256, 0, stream>>>(vol, cin, dvd, dpad, dp, items, tab, out, nonfinite);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_gather_views(const float* vol, int cin, const int32_t vd[3], const int32_t off[3],
                        const int32_t patch[3], int views, const int32_t* masks, float* out, cudaStream_t stream) {
  NNB_REQUIRE(views >= 1 && views <= 8, "gather_views: 1..8 views supported, got %d", views);
  for (int a = 0; a < 3; ++a)
    NNB_REQUIRE(off[a] >= 0 && off[a] + patch[a] <= vd[a], "gather_views: tile outside the volume on axis %d", a);
  int32_t offsets[24];
  for (int v = 0; v < views; ++v)
    for (int a = 0; a < 3; ++a) offsets[3 * v + a] = off[a];
  const int32_t zero[3] = {0, 0, 0};
  return launch_gather_tiles(vol, cin, vd, zero, views, offsets, masks, patch, out, nullptr, stream);
}

// ---------------------------------------------------------------------------
// Fused seg head + flip-back + view mean + Gaussian accumulation (one tile).
// features: (views, P0, P1, P2, F) lazy; seg_w: (C, F); acc: (AD, AH, AW, C).
// One thread per tile voxel; per view it reads the F features of the
// flipped source voxel with 16-byte loads, applies the view's lazy affine
// (staged in shared memory with the head weights), computes the C logits and
// adds them to the running view sum in view order.  HBM-bound on the feature
// read (views * P^3 * F * 4 bytes per tile).
// ---------------------------------------------------------------------------
constexpr int kAccMaxC = 8;        // classes per pass

// Accumulator update: float32 add, or the float16 window update of the
// nnunet-fp16 mode -- the float32 sum of the stored half value and the float32
// weighted prediction, rounded to nearest-even half (reference
// sliding_window.py:421-426: (logits.astype(f32) + weighted).astype(f16)).
__device__ __forceinline__ void acc_add(float* p, float w) { *p += w; }
__device__ __forceinline__ void acc_add(__half* p, float w) { *p = __float2half_rn(__half2float(*p) + w); }

template <int FV, typename AccT>  // FV = F / 4 (float4 chunks), compile-time for register arrays
__global__ void __launch_bounds__(256) accumulate_tile_vec_kernel(
    nnb_segment feat, int views, ViewMasks masks, Dims3 patch, float slope, const float* __restrict__ seg_w,
    const float* __restrict__ seg_b, int classes, const float* __restrict__ gauss, AccT* __restrict__ acc,
    AccT* __restrict__ normalizer, Dims3 ad, Dims3 off, int add_normalizer, float view_div) {
  constexpr int F = FV * 4;
  __shared__ float s_sc[8][F];
  __shared__ float s_sh[8][F];
  __shared__ float s_w[kAccMaxC][F];
  __shared__ float s_b[kAccMaxC];
  __shared__ int s_mask[8];
  if (threadIdx.x < 8) s_mask[threadIdx.x] = masks.m[threadIdx.x];
  for (int i = threadIdx.x; i < views * F; i += blockDim.x) {
    const int v = i / F, f = i % F;
    s_sc[v][f] = feat.scale ? feat.scale[v * F + f] : 1.f;
    s_sh[v][f] = feat.scale ? feat.shift[v * F + f] : 0.f;
  }
  const bool lazy = feat.scale != nullptr;
  const int64_t pvox = (int64_t)patch.d[0] * patch.d[1] * patch.d[2];
  for (int c0 = 0; c0 < classes; c0 += kAccMaxC) {
    const int nc = min(kAccMaxC, classes - c0);
    __syncthreads();
    for (int i = threadIdx.x; i < kAccMaxC * F; i += blockDim.x) {
      const int c = i / F, f = i % F;
      s_w[c][f] = c < nc ? seg_w[(int64_t)(c0 + c) * F + f] : 0.f;
    }
    if (threadIdx.x < kAccMaxC) s_b[threadIdx.x] = threadIdx.x < nc ? seg_b[c0 + threadIdx.x] : 0.f;
    __syncthreads();
    for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pvox;
         p += (int64_t)gridDim.x * blockDim.x) {
      const int k = (int)(p % patch.d[2]);
      const int j = (int)((p / patch.d[2]) % patch.d[1]);
      const int i = (int)(p / ((int64_t)patch.d[2] * patch.d[1]));
      float pred[kAccMaxC];
#pragma unroll
      for (int c = 0; c < kAccMaxC; ++c) pred[c] = 0.f;
      for (int v = 0; v < views; ++v) {
        const int mask = s_mask[v];
        const int si = (mask & 1) ? patch.d[0] - 1 - i : i;
        const int sj = (mask & 2) ? patch.d[1] - 1 - j : j;
        const int sk = (mask & 4) ? patch.d[2] - 1 - k : k;
        const int64_t q = (((int64_t)v * patch.d[0] + si) * patch.d[1] + sj) * patch.d[2] + sk;
        const float4* src = reinterpret_cast<const float4*>(feat.data + q * F);
        float logit[kAccMaxC];
#pragma unroll
        for (int c = 0; c < kAccMaxC; ++c) logit[c] = 0.f;
#pragma unroll
        for (int f4 = 0; f4 < FV; ++f4) {
          const float4 x = __ldg(src + f4);
          float z[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int f = f4 * 4 + e;
            if (lazy) {
              const float y = fmaf(z[e], s_sc[v][f], s_sh[v][f]);
              z[e] = feat.leaky ? leaky(y, slope) : y;
            }
#pragma unroll
            for (int c = 0; c < kAccMaxC; ++c) logit[c] = fmaf(z[e], s_w[c][f], logit[c]);
          }
        }
#pragma unroll
        for (int c = 0; c < kAccMaxC; ++c) pred[c] += logit[c] + s_b[c];
      }
      const float g = __ldg(gauss + p);
      const int64_t dst = ((int64_t)(off.d[0] + i) * ad.d[1] + (off.d[1] + j)) * ad.d[2] + (off.d[2] + k);
      AccT* a = acc + dst * classes + c0;
#pragma unroll
      for (int c = 0; c < kAccMaxC; ++c)
        if (c < nc) acc_add(a + c, (pred[c] / view_div) * g);
      if (add_normalizer && c0 == 0) acc_add(normalizer + dst, g);
    }
  }
}

template <int CC, typename AccT>
__global__ void __launch_bounds__(256) accumulate_tile_kernel(
    nnb_segment feat, int views, ViewMasks masks, Dims3 patch, float slope, const float* __restrict__ seg_w,
    const float* __restrict__ seg_b, int classes, const float* __restrict__ gauss, AccT* __restrict__ acc,
    AccT* __restrict__ normalizer, Dims3 ad, Dims3 off, int add_normalizer, float view_div) {
  const int64_t pvox = (int64_t)patch.d[0] * patch.d[1] * patch.d[2];
  const int F = feat.channels;
  for (int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; p < pvox;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(p % patch.d[2]);
    const int j = (int)((p / patch.d[2]) % patch.d[1]);
    const int i = (int)(p / ((int64_t)patch.d[2] * patch.d[1]));
    const float g = __ldg(gauss + p);
    const int64_t dst = ((int64_t)(off.d[0] + i) * ad.d[1] + (off.d[1] + j)) * ad.d[2] + (off.d[2] + k);
    for (int c0 = 0; c0 < classes; c0 += CC) {
      float pred[CC];
#pragma unroll
      for (int c = 0; c < CC; ++c) pred[c] = 0.f;
      for (int v = 0; v < views; ++v) {
        const int mask = masks.m[v];
        const int si = (mask & 1) ? patch.d[0] - 1 - i : i;
        const int sj = (mask & 2) ? patch.d[1] - 1 - j : j;
        const int sk = (mask & 4) ? patch.d[2] - 1 - k : k;
        const int64_t q = (((int64_t)v * patch.d[0] + si) * patch.d[1] + sj) * patch.d[2] + sk;
        const float* src = feat.data + q * F;
        float logit[CC];
#pragma unroll
        for (int c = 0; c < CC; ++c) logit[c] = 0.f;
        for (int f = 0; f < F; ++f) {
          const float z = activate(__ldg(src + f), feat.scale, feat.shift, feat.leaky, slope, v * F + f);
#pragma unroll
          for (int c = 0; c < CC; ++c)
            if (c0 + c < classes) logit[c] = fmaf(z, __ldg(seg_w + (int64_t)(c0 + c) * F + f), logit[c]);
        }
#pragma unroll
        for (int c = 0; c < CC; ++c)
          if (c0 + c < classes) pred[c] += logit[c] + __ldg(seg_b + c0 + c);
      }
#pragma unroll
      for (int c = 0; c < CC; ++c)
        if (c0 + c < classes) acc_add(acc + dst * classes + c0 + c, (pred[c] / view_div) * g);
    }
    if (add_normalizer) acc_add(normalizer + dst, g);
  }
}

// Row-staged variant (32 features, x extent <= 128, <= 8 classes): one block per
// output x-row (i, j) of the patch.  For each view the source row -- the same
// voxels, flipped -- is 128 contiguous bytes per voxel in HBM: cp.async copies it
// whole-line into a shared buffer (16-byte chunks XOR-swizzled by voxel % 8;
// two buffers, so the next view's copy overlaps this view's arithmetic), and
// thread k reads its (x-flipped) voxel from shared memory.  Replaces per-thread
// 128-byte reads whose every warp instruction touched 32 separate lines.
constexpr int kRowMax = 128;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem_src) : "memory");
}

template <typename AccT>
__global__ void __launch_bounds__(kRowMax) accumulate_tile_rows_kernel(
    nnb_segment feat, int views, ViewMasks masks, Dims3 patch, float slope, const float* __restrict__ seg_w,
    const float* __restrict__ seg_b, int classes, const float* __restrict__ gauss, AccT* __restrict__ acc,
    AccT* __restrict__ normalizer, Dims3 ad, Dims3 off, int add_normalizer, float view_div) {
  constexpr int F = 32;
  __shared__ float4 rows[2][kRowMax * 8];
  __shared__ float s_sc[8][F], s_sh[8][F];
  __shared__ float s_w[kAccMaxC][F];
  __shared__ float s_b[kAccMaxC];
  const int PX = patch.d[2];
  const int i = blockIdx.x / patch.d[1], j = blockIdx.x - i * patch.d[1];
  for (int t = threadIdx.x; t < views * F; t += blockDim.x) {
    const int v = t / F, f = t % F;
    s_sc[v][f] = feat.scale ? feat.scale[v * F + f] : 1.f;
    s_sh[v][f] = feat.scale ? feat.shift[v * F + f] : 0.f;
  }
  for (int t = threadIdx.x; t < kAccMaxC * F; t += blockDim.x) {
    const int c = t / F, f = t % F;
    s_w[c][f] = c < classes ? seg_w[c * F + f] : 0.f;
  }
  if (threadIdx.x < kAccMaxC) s_b[threadIdx.x] = threadIdx.x < classes ? seg_b[threadIdx.x] : 0.f;
  // source row of view v: voxels (v, si, sj, 0 .. PX-1), x flipped on read
  auto issue = [&](int v) {
    const int m = masks.m[v];
    const int si = (m & 1) ? patch.d[0] - 1 - i : i;
    const int sj = (m & 2) ? patch.d[1] - 1 - j : j;
    const float4* src = reinterpret_cast<const float4*>(
        feat.data + ((((int64_t)v * patch.d[0] + si) * patch.d[1] + sj) * PX) * F);
    float4* dst = rows[v & 1];
    for (int c = threadIdx.x; c < PX * 8; c += blockDim.x) {
      const int vox = c >> 3, part = c & 7;
      cp_async16(dst + vox * 8 + (part ^ (vox & 7)), src + c);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue(0);
  __syncthreads();  // tables ready
  const bool lazy = feat.scale != nullptr;
  const int k = threadIdx.x;
  float pred[kAccMaxC];
#pragma unroll
  for (int c = 0; c < kAccMaxC; ++c) pred[c] = 0.f;
  for (int v = 0; v < views; ++v) {
    if (v + 1 < views) {
      issue(v + 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // view v's row has landed for every thread
    if (k < PX) {
      const int sk = (masks.m[v] & 4) ? PX - 1 - k : k;
      const float4* r = rows[v & 1] + sk * 8;
      float logit[kAccMaxC];
#pragma unroll
      for (int c = 0; c < kAccMaxC; ++c) logit[c] = s_b[c];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 x4 = r[q ^ (sk & 7)];
        const float z4[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int f = 4 * q + e;
          float z = z4[e];
          if (lazy) {
            z = fmaf(z, s_sc[v][f], s_sh[v][f]);
            if (feat.leaky) z = leaky(z, slope);
          }
#pragma unroll
          for (int c = 0; c < kAccMaxC; ++c) logit[c] = fmaf(z, s_w[c][f], logit[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < kAccMaxC; ++c) pred[c] += logit[c];
    }
    __syncthreads();  // buffer v & 1 is free for view v + 2
  }
  if (k >= PX) return;
  const int64_t p = ((int64_t)i * patch.d[1] + j) * PX + k;
  const float g = __ldg(gauss + p);
  const int64_t dst = ((int64_t)(off.d[0] + i) * ad.d[1] + (off.d[1] + j)) * ad.d[2] + (off.d[2] + k);
  AccT* a = acc + dst * classes;
#pragma unroll
  for (int c = 0; c < kAccMaxC; ++c)
    if (c < classes) acc_add(a + c, (pred[c] / view_div) * g);
  if (add_normalizer) acc_add(normalizer + dst, g);
}

template <typename AccT>
int launch_accumulate_tile_t(const nnb_segment& feat, int views, const int32_t* masks, const int32_t patch[3],
                             float slope, const float* seg_w, const float* seg_b, int classes, const float* gauss,
                             AccT* acc, AccT* normalizer, const int32_t ad[3], const int32_t off[3],
                             int add_normalizer, int view_divisor, cudaStream_t stream) {
  NNB_REQUIRE(views >= 1 && views <= 8, "accumulate_tile: 1..8 views supported");
  NNB_REQUIRE(view_divisor >= views && view_divisor <= 8, "accumulate_tile: view_divisor %d outside [views, 8]",
              view_divisor);
  // the view mean divides the view sum by the tile's full view count (reference sliding_window.py:527), also
  // when this call adds only some of the tile's views (a batch mixing tiles)
  const float view_div = (float)view_divisor;
  ViewMasks vm{};
  for (int v = 0; v < views; ++v) vm.m[v] = masks[v];
  Dims3 dp{{patch[0], patch[1], patch[2]}}, dad{{ad[0], ad[1], ad[2]}}, doff{{off[0], off[1], off[2]}};
  const int64_t pvox = (int64_t)patch[0] * patch[1] * patch[2];
  const int blocks = (int)std::min<int64_t>((pvox + 255) / 256, 148 * 16);
  const bool aligned = (reinterpret_cast<uintptr_t>(feat.data) & 15) == 0;
  if (aligned && feat.channels == 32 && patch[2] <= kRowMax && classes <= kAccMaxC &&
      (int64_t)patch[0] * patch[1] < (1LL << 31)) {
    accumulate_tile_rows_kernel<AccT><<<(unsigned)((int64_t)patch[0] * patch[1]), kRowMax, 0, stream>>>(
        feat, views, vm, dp, slope, seg_w, seg_b, classes, gauss, acc, normalizer, dad, doff, add_normalizer,
        view_div);
  } else if (aligned && feat.channels == 32) {
    accumulate_tile_vec_kernel<8, AccT><<<blocks, 256, 0, stream>>>(feat, views, vm, dp, slope, seg_w, seg_b,
                                                                    classes, gauss, acc, normalizer, dad, doff,
                                                                    add_normalizer, view_div);
  } else {
    accumulate_tile_kernel<4, AccT><<<blocks, 256, 0, stream>>>(feat, views, vm, dp, slope, seg_w, seg_b, classes,
                                                                gauss, acc, normalizer, dad, doff, add_normalizer,
                                                                view_div);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_accumulate_tile(const nnb_segment& feat, int views, const int32_t* masks, const int32_t patch[3],
                           float slope, const float* seg_w, const float* seg_b, int classes, const float* gauss,
                           void* acc, void* normalizer, int fp16, const int32_t ad[3], const int32_t off[3],
                           int add_normalizer, int view_divisor, cudaStream_t stream) {
  if (fp16)
    return launch_accumulate_tile_t<__half>(feat, views, masks, patch, slope, seg_w, seg_b, classes, gauss,
                                            static_cast<__half*>(acc), static_cast<__half*>(normalizer), ad, off,
                                            add_normalizer, view_divisor, stream);
  return launch_accumulate_tile_t<float>(feat, views, masks, patch, slope, seg_w, seg_b, classes, gauss,
                                         static_cast<float*>(acc), static_cast<float*>(normalizer), ad, off,
                                         add_normalizer, view_divisor, stream);
}

// ---------------------------------------------------------------------------
// Normalise + first-argmax labels + channel-first logits over the crop.
// Reference: metal_normalized_labels.py:19-40 (first max, invalid flag).
// ---------------------------------------------------------------------------
template <typename LabelT>
__global__ void normalize_labels_kernel(const float* __restrict__ acc, const float* __restrict__ normalizer,
                                        int classes, Dims3 ad, Dims3 lo, Dims3 cd, float fold_divisor,
                                        float* __restrict__ logits, LabelT* __restrict__ labels,
                                        int* __restrict__ invalid_count, LabelT invalid_label) {
  const int64_t total = (int64_t)cd.d[0] * cd.d[1] * cd.d[2];
  int local_invalid = 0;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int x = (int)(o % cd.d[2]);
    const int y = (int)((o / cd.d[2]) % cd.d[1]);
    const int z = (int)(o / ((int64_t)cd.d[2] * cd.d[1]));
    const int64_t src = ((int64_t)(lo.d[0] + z) * ad.d[1] + (lo.d[1] + y)) * ad.d[2] + (lo.d[2] + x);
    const float den = __ldg(normalizer + src);
    bool invalid = !isfinite(den) || den <= 0.f;
    float best = -INFINITY;
    int winner = 0;
    bool have = false;
    for (int c = 0; c < classes; ++c) {
      float q = __ldg(acc + src * classes + c) / den;
      if (fold_divisor != 1.0f) q = q / fold_divisor;
      invalid |= !isfinite(q);
      if (logits != nullptr) logits[(int64_t)c * total + o] = q;
      if (!have || q > best) {
        best = q;
        winner = c;
        have = true;
      }
    }
    if (labels != nullptr) labels[o] = invalid ? invalid_label : (LabelT)winner;
    local_invalid += invalid ? 1 : 0;
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

int launch_normalize_labels(const float* acc, const float* normalizer, int classes, const int32_t ad[3],
                            const int32_t lo[3], const int32_t cd[3], float fold_divisor, float* logits,
                            void* labels, int label_bytes, int32_t* invalid_count, cudaStream_t stream) {
  Dims3 dad{{ad[0], ad[1], ad[2]}}, dlo{{lo[0], lo[1], lo[2]}}, dcd{{cd[0], cd[1], cd[2]}};
  const int64_t total = (int64_t)cd[0] * cd[1] * cd[2];
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  NNB_CUDA_CHECK(cudaMemsetAsync(invalid_count, 0, sizeof(int32_t), stream));
  if (label_bytes == 1) {
    NNB_REQUIRE(classes <= 255, "normalize_labels: uint8 labels need <= 255 classes");
    normalize_labels_kernel<uint8_t><<<blocks, 256, 0, stream>>>(acc, normalizer, classes, dad, dlo, dcd,
                                                                 fold_divisor, logits, (uint8_t*)labels,
                                                                 invalid_count, (uint8_t)0xFF);
  } else {
    NNB_REQUIRE(label_bytes == 2, "normalize_labels: label_bytes must be 1 or 2");
    NNB_REQUIRE(classes <= 65535, "normalize_labels: too many classes for uint16 labels");
    normalize_labels_kernel<uint16_t><<<blocks, 256, 0, stream>>>(acc, normalizer, classes, dad, dlo, dcd,
                                                                  fold_divisor, logits, (uint16_t*)labels,
                                                                  invalid_count, (uint16_t)0xFFFF);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

// ---------------------------------------------------------------------------
// nnunet-fp16 fold handling.  One fold's window -> normalised half logits over
// the crop, n = half(f32(acc) / f32(norm)) (reference sliding_window.py:185,
// 289: (logits.astype(f32) / normalizer.astype(f32)).astype(f16)), added into
// the channel-first half total: the first fold stores n, later folds
// half(f32(total) + f32(n)) in fold order (inference.py:75-85, IEEE half adds).
// Non-finite fold logits are counted.
// ---------------------------------------------------------------------------
__global__ void fold_add_fp16_kernel(const __half* __restrict__ acc, const __half* __restrict__ normalizer,
                                     int classes, Dims3 ad, Dims3 lo, Dims3 cd, __half* __restrict__ total,
                                     int first, int* __restrict__ invalid_count) {
  const int64_t vox = (int64_t)cd.d[0] * cd.d[1] * cd.d[2];
  int local_invalid = 0;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < vox;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int x = (int)(o % cd.d[2]);
    const int y = (int)((o / cd.d[2]) % cd.d[1]);
    const int z = (int)(o / ((int64_t)cd.d[2] * cd.d[1]));
    const int64_t src = ((int64_t)(lo.d[0] + z) * ad.d[1] + (lo.d[1] + y)) * ad.d[2] + (lo.d[2] + x);
    const float den = __half2float(normalizer[src]);
    bool invalid = false;
    for (int c = 0; c < classes; ++c) {
      const __half n = __float2half_rn(__half2float(acc[src * classes + c]) / den);
      const float nf = __half2float(n);
      invalid |= !isfinite(nf);
      __half* t = total + (int64_t)c * vox + o;
      *t = first ? n : __float2half_rn(__half2float(*t) + nf);
    }
    local_invalid += invalid ? 1 : 0;
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

// Fold average of the half total: half(f32(total) / folds) in place
// (inference.py:86-90, total /= float32(n)), then float32 logits of the half
// values and first-argmax labels (invalid label for non-finite values).
template <typename LabelT>
__global__ void fold_finalize_fp16_kernel(__half* __restrict__ total, int classes, int64_t vox, float folds,
                                          float* __restrict__ logits, LabelT* __restrict__ labels,
                                          int* __restrict__ invalid_count, LabelT invalid_label) {
  int local_invalid = 0;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < vox;
       o += (int64_t)gridDim.x * blockDim.x) {
    bool invalid = false;
    float best = 0.f;
    int winner = 0;
    for (int c = 0; c < classes; ++c) {
      __half* t = total + (int64_t)c * vox + o;
      const __half q = __float2half_rn(__half2float(*t) / folds);
      *t = q;
      const float qf = __half2float(q);
      invalid |= !isfinite(qf);
      if (logits != nullptr) logits[(int64_t)c * vox + o] = qf;
      if (c == 0 || qf > best) {
        best = qf;
        winner = c;
      }
    }
    if (labels != nullptr) labels[o] = invalid ? invalid_label : (LabelT)winner;
    local_invalid += invalid ? 1 : 0;
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

// One fold's normalised half logits (channel-first, as fold_add_fp16 stored them for a first fold) added into
// the half total in fold order: total = half(f32(total) + f32(part)) -- the same IEEE half add fold_add_fp16
// performs for a later fold, for folds computed on other devices.  Non-finite sums are counted.
__global__ void fold_sum_fp16_kernel(__half* __restrict__ total, const __half* __restrict__ part, int64_t n,
                                     int* __restrict__ invalid_count) {
  int local_invalid = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = __half2float(total[i]) + __half2float(part[i]);
    const __half h = __float2half_rn(v);
    local_invalid += isfinite(__half2float(h)) ? 0 : 1;
    total[i] = h;
  }
  if (local_invalid) atomicAdd(invalid_count, local_invalid);
}

int launch_fold_sum_fp16(void* total, const void* part, int64_t n, int32_t* invalid_count, cudaStream_t stream) {
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
  fold_sum_fp16_kernel<<<blocks, 256, 0, stream>>>(static_cast<__half*>(total), static_cast<const __half*>(part), n,
                                                   invalid_count);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_fold_add_fp16(const void* acc, const void* normalizer, int classes, const int32_t ad[3],
                         const int32_t lo[3], const int32_t cd[3], void* total, int first, int32_t* invalid_count,
                         cudaStream_t stream) {
  Dims3 dad{{ad[0], ad[1], ad[2]}}, dlo{{lo[0], lo[1], lo[2]}}, dcd{{cd[0], cd[1], cd[2]}};
  const int64_t vox = (int64_t)cd[0] * cd[1] * cd[2];
  const int blocks = (int)std::min<int64_t>((vox + 255) / 256, 148 * 16);
  fold_add_fp16_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __half*>(acc),
                                                   static_cast<const __half*>(normalizer), classes, dad, dlo, dcd,
                                                   static_cast<__half*>(total), first, invalid_count);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_fold_finalize_fp16(void* total, int classes, int64_t vox, int folds, float* logits, void* labels,
                              int label_bytes, int32_t* invalid_count, cudaStream_t stream) {
  const int blocks = (int)std::min<int64_t>((vox + 255) / 256, 148 * 16);
  __half* t = static_cast<__half*>(total);
  if (labels == nullptr || label_bytes == 1) {
    NNB_REQUIRE(labels == nullptr || classes <= 255, "fold_finalize_fp16: uint8 labels need <= 255 classes");
    fold_finalize_fp16_kernel<uint8_t><<<blocks, 256, 0, stream>>>(t, classes, vox, (float)folds, logits,
                                                                   (uint8_t*)labels, invalid_count, (uint8_t)0xFF);
  } else {
    NNB_REQUIRE(label_bytes == 2, "fold_finalize_fp16: label_bytes must be 1 or 2");
    fold_finalize_fp16_kernel<uint16_t><<<blocks, 256, 0, stream>>>(t, classes, vox, (float)folds, logits,
                                                                    (uint16_t*)labels, invalid_count,
                                                                    (uint16_t)0xFFFF);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

}  // namespace nnb
