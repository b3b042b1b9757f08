// nnb_conv3d_norm_static: convolution + instance-norm statistics without any
// device allocation.  The per-tile (sum, M2, n) partials that nnb_conv3d
// writes and nnb_instance_norm_finalize reads live in a fixed device array of
// this library instead of a caller-provided buffer.
//
// Contract (also stated in include/nnb.h):
//  * scratch capacity NNB_STATIC_PARTIALS_FLOATS floats (16 MiB); a request
//    needing batch x tiles x cout x 3 floats beyond it is rejected with
//    NNB_E_UNSUPPORTED before anything is launched;
//  * nothing in the scratch needs to start at zero: the convolution writes
//    every (sample, tile, channel) triple before the finalize reads it;
//  * one scratch per device: calls that overlap on the same device (other
//    streams or threads) race on it and must be ordered by the caller;
//  * the first call on a device looks the scratch address up with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture begins.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"

namespace nnb {
namespace {

__device__ __align__(256) float g_partials_scratch[NNB_STATIC_PARTIALS_FLOATS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

// Address of this device's scratch, looked up once per device.
int scratch_for_current_device(float** out) {
  int dev = 0;
  NNB_CUDA_CHECK(cudaGetDevice(&dev));
  NNB_REQUIRE(dev >= 0 && dev < kMaxDevices, "conv3d_norm_static: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_partials_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("conv3d_norm_static: cudaGetSymbolAddress of the partials scratch failed: %s",
                cudaGetErrorString(err));
      return NNB_E_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return NNB_OK;
}

}  // namespace
}  // namespace nnb

extern "C" int32_t nnb_conv3d_norm_static(const nnb_conv3d_args* args, const float* gamma, const float* beta,
                                          float eps, float* scale, float* shift, void* stream) {
  using namespace nnb;
  NNB_REQUIRE(args != nullptr && scale != nullptr && shift != nullptr, "conv3d_norm_static: null pointer");
  NNB_REQUIRE(args->partials == nullptr, "conv3d_norm_static: args->partials must be NULL (the library's "
              "static scratch holds the partials)");
  NNB_REQUIRE(args->batch >= 1 && args->cout >= 1, "conv3d_norm_static: bad shape");
  const int64_t tiles = nnb_conv3d_partial_tiles(args);
  if (tiles < 0) return (int32_t)tiles;
  const int64_t need = (int64_t)args->batch * tiles * args->cout * 3;
  if (need > (int64_t)NNB_STATIC_PARTIALS_FLOATS) {
    set_error("conv3d_norm_static: this convolution needs %lld partial floats (batch %d x %lld tiles x %d "
              "channels x 3) but the static scratch holds %d; use nnb_conv3d with a caller buffer",
              (long long)need, args->batch, (long long)tiles, args->cout, NNB_STATIC_PARTIALS_FLOATS);
    return NNB_E_UNSUPPORTED;
  }
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  nnb_conv3d_args a = *args;
  a.partials = scratch;
  rc = nnb_conv3d(&a, stream);
  if (rc) return rc;
  return nnb_instance_norm_finalize(scratch, args->batch, (int32_t)tiles, args->cout, gamma, beta, eps, scale,
                                    shift, stream);
}
