// Shared helpers for the nnb CUDA sources: error reporting, lazy-activation
// loads and the per-tile instance-norm partial statistics format.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/nnb.h"

namespace nnb {

// Rows (output voxels) per statistics tile.  Tiles never straddle samples:
// tile t of sample b covers sample-local voxels [128 t, 128 t + 128).
constexpr int kTileRows = 128;

void set_error(const char* fmt, ...);

#define NNB_REQUIRE(cond, ...)                 \
  do {                                         \
    if (!(cond)) {                             \
      ::nnb::set_error(__VA_ARGS__);           \
      return NNB_E_INVALID;                    \
    }                                          \
  } while (0)

#define NNB_CUDA_CHECK(expr)                                                        \
  do {                                                                              \
    cudaError_t nnb_err_ = (expr);                                                  \
    if (nnb_err_ != cudaSuccess) {                                                  \
      ::nnb::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(nnb_err_), \
                       __FILE__, __LINE__);                                         \
      return NNB_E_CUDA;                                                            \
    }                                                                               \
  } while (0)

#define NNB_LAUNCH_CHECK()                                                          \
  do {                                                                              \
    cudaError_t nnb_err_ = cudaGetLastError();                                      \
    if (nnb_err_ != cudaSuccess) {                                                  \
      ::nnb::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(nnb_err_), \
                       __FILE__, __LINE__);                                         \
      return NNB_E_CUDA;                                                            \
    }                                                                               \
  } while (0)

// Tensor-core operand formats (see nnb_prepare_operand).
constexpr int kOperandTf32 = 0;    // one TF32 value per element
constexpr int kOperandTf32x2 = 1;  // TF32 hi/lo pair
constexpr int kOperandF16x2 = 2;   // fp16 hi + lo pair
constexpr int kOperandBf16 = 3;    // one bf16 value per element (in the fp16 pair's row layout, lo half unused)

inline bool tensor_precision(int precision) {
  return precision == NNB_PREC_FP32 || precision == NNB_PREC_TF32 || precision == NNB_PREC_FP32_TF32 ||
         precision == NNB_PREC_BF16;
}

inline int operand_kind(int precision) {
  return precision == NNB_PREC_FP32        ? kOperandF16x2
         : precision == NNB_PREC_FP32_TF32 ? kOperandTf32x2
         : precision == NNB_PREC_BF16      ? kOperandBf16
                                           : kOperandTf32;
}

// 16-bit operand formats: 128-byte A rows of 64 halves per 32 channels, 64-byte B rows.
constexpr bool half_rows(int op) { return op == kOperandF16x2 || op == kOperandBf16; }

inline int tiles_per_sample(int64_t voxels) { return (int)((voxels + kTileRows - 1) / kTileRows); }

__device__ __forceinline__ float leaky(float v, float slope) { return v >= 0.f ? v : v * slope; }

// Transpose-reduce: lane j ends with the sum over the warp's lanes of x[j] (x is clobbered).
__device__ __forceinline__ float warp_column_sums(float (&x)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {
    const bool up = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? x[i] : x[i + h];
      const float keep = up ? x[i + h] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  return x[0];
}

// Apply a segment's lazy affine + activation to one raw value.
__device__ __forceinline__ float activate(float raw, const float* scale, const float* shift,
                                          int leaky_flag, float slope, int idx) {
  if (scale == nullptr) return raw;
  float v = fmaf(raw, __ldg(scale + idx), __ldg(shift + idx));
  return leaky_flag ? leaky(v, slope) : v;
}

}  // namespace nnb
