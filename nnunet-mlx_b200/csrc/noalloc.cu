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
//  * the first call on a device (and the first after that device's context
//    was replaced, e.g. by cudaDeviceReset) looks the scratch address up with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture begins.
#include <cuda.h>
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
CUcontext g_scratch_ctx[kMaxDevices] = {nullptr};  // context the cached address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The driver's cuCtxGetCurrent through the runtime's entry-point query (no link against libcuda).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Address of this device's scratch in the current context, looked up once per device and again whenever the
// device's current context is no longer the one the cached address was taken in.
int scratch_for_current_device(float** out) {
  int dev = 0;
  NNB_CUDA_CHECK(cudaGetDevice(&dev));
  NNB_REQUIRE(dev >= 0 && dev < kMaxDevices, "conv3d_norm_static: device ordinal %d out of range", dev);
  const CtxGetCurrentFn get = ctx_get_current();
  NNB_REQUIRE(get != nullptr, "conv3d_norm_static: cuCtxGetCurrent is not available from the driver");
  CUcontext ctx = nullptr;  // stays null until the runtime has made a context current on this thread
  NNB_REQUIRE(get(&ctx) == CUDA_SUCCESS, "conv3d_norm_static: cannot read the current CUDA context");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr || ctx == nullptr || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_partials_scratch);  // makes the context current if needed
    if (err != cudaSuccess || p == nullptr) {
      set_error("conv3d_norm_static: cudaGetSymbolAddress of the partials scratch failed: %s",
                cudaGetErrorString(err));
      return NNB_E_CUDA;
    }
    NNB_REQUIRE(get(&ctx) == CUDA_SUCCESS && ctx != nullptr, "conv3d_norm_static: no current CUDA context");
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_scratch_ctx[dev] = ctx;
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
