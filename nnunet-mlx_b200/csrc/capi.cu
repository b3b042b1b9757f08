// extern "C" entry points declared in include/nnb.h: argument validation,
// per-thread error messages and dispatch to the kernels.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>

#include "common.cuh"

namespace nnb {

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

// kernels implemented in the other translation units
int launch_conv3d_simt(const nnb_conv3d_args& a, cudaStream_t stream);
bool conv3d_tc_supported(const nnb_conv3d_args& a);
bool conv3d_tc_raw_operands(const nnb_conv3d_args& a);
int launch_conv3d_tc(const nnb_conv3d_args& a, cudaStream_t stream);
int64_t conv3d_tc_packed_bytes(int cout, int kvol, int cin_total, int precision);
int launch_conv3d_pack(const float* w, int cout, int kvol, int cin_total, int precision, void* packed,
                       cudaStream_t stream);
int conv3d_tc_partial_tiles(const nnb_conv3d_args& a);
int conv3d_tc_mode(const nnb_conv3d_args& a);
int launch_norm_finalize(const float* partials, int batch, int tiles, int channels, const float* gamma,
                         const float* beta, float eps, float* scale, float* shift, cudaStream_t stream);
int launch_conv_transpose_simt(const nnb_segment& in, int batch, const int32_t in_dims[3], const int32_t k[3],
                               float slope, const float* weight, const float* bias, int cout, float* out,
                               cudaStream_t stream);
int launch_conv_transpose_tc(const nnb_segment& in, int batch, const int32_t in_dims[3], const int32_t k[3],
                             float slope, const float* bias, int cout, const void* packed, int precision, float* out,
                             int out_operand, cudaStream_t stream);
int launch_conv3d_pack_rows(const float* w, int rows, int kvol, int cin_total, int precision, int row_taps,
                            int up_cout, void* packed, cudaStream_t stream);
int launch_prepare_operand(const nnb_segment& in, int batch, int64_t voxels, float slope, int op, float* out,
                           cudaStream_t stream);
int64_t operand_range_events(int reset);
int launch_residual_join(const nnb_segment& br, const nnb_segment& sk, int batch, int64_t voxels, float slope,
                         float* out, cudaStream_t stream);
int launch_gather_views(const float* vol, int cin, const int32_t vd[3], const int32_t off[3],
                        const int32_t patch[3], int views, const int32_t* masks, float* out, cudaStream_t stream);
int launch_gather_tiles(const float* vol, int cin, const int32_t vd[3], const int32_t pad_lo[3], int items,
                        const int32_t* offsets, const int32_t* masks, const int32_t patch[3], float* out,
                        int32_t* nonfinite, cudaStream_t stream);
int launch_accumulate_tile(const nnb_segment& feat, int views, const int32_t* masks, const int32_t patch[3],
                           float slope, const float* seg_w, const float* seg_b, int classes, const float* gauss,
                           void* acc, void* normalizer, int fp16, const int32_t ad[3], const int32_t off[3],
                           int add_normalizer, int view_divisor, cudaStream_t stream);
int launch_fold_add_fp16(const void* acc, const void* normalizer, int classes, const int32_t ad[3],
                         const int32_t lo[3], const int32_t cd[3], void* total, int first, int32_t* invalid_count,
                         cudaStream_t stream);
int launch_fold_sum_fp16(void* total, const void* part, int64_t n, int32_t* invalid_count, cudaStream_t stream);
int launch_fold_finalize_fp16(void* total, int classes, int64_t vox, int folds, float* logits, void* labels,
                              int label_bytes, int32_t* invalid_count, cudaStream_t stream);
int launch_normalize_labels(const float* acc, const float* normalizer, int classes, const int32_t ad[3],
                            const int32_t lo[3], const int32_t cd[3], float fold_divisor, float* logits,
                            void* labels, int label_bytes, int32_t* invalid_count, cudaStream_t stream);
int launch_restore_labels(const nnb_restore_args& a, cudaStream_t stream);

static int check_segment(const nnb_segment& s, const char* what) {
  NNB_REQUIRE(s.data != nullptr, "%s: null data", what);
  NNB_REQUIRE(s.channels >= 1, "%s: channels must be positive", what);
  NNB_REQUIRE(s.scale == nullptr || s.shift != nullptr, "%s: scale without shift", what);
  return NNB_OK;
}

static bool positive3(const int32_t d[3]) { return d[0] > 0 && d[1] > 0 && d[2] > 0; }

}  // namespace nnb

using namespace nnb;

extern "C" {

int32_t nnb_abi_version(void) { return NNB_ABI_VERSION; }

const char* nnb_last_error(void) { return g_error; }

int32_t nnb_conv3d(const nnb_conv3d_args* a, void* stream) {
  NNB_REQUIRE(a != nullptr, "conv3d: null args");
  NNB_REQUIRE(a->batch >= 1, "conv3d: batch must be positive");
  NNB_REQUIRE(positive3(a->in_dims) && positive3(a->out_dims) && positive3(a->kernel) && positive3(a->stride),
              "conv3d: dims, kernel and stride must be positive");
  NNB_REQUIRE(a->num_segments == 1 || a->num_segments == 2, "conv3d: 1 or 2 input segments");
  for (int s = 0; s < a->num_segments; ++s) {
    int rc = check_segment(a->seg[s], "conv3d segment");
    if (rc) return rc;
  }
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(a->pad[i] >= 0, "conv3d: negative padding");
    const int expect = (a->in_dims[i] + 2 * a->pad[i] - a->kernel[i]) / a->stride[i] + 1;
    NNB_REQUIRE(a->out_dims[i] == expect, "conv3d: out_dims[%d]=%d, expected %d", i, a->out_dims[i], expect);
  }
  NNB_REQUIRE(a->cout >= 1 && a->weight != nullptr && a->out != nullptr, "conv3d: missing weight/output");
  const cudaStream_t st = (cudaStream_t)stream;
  NNB_REQUIRE(tensor_precision(a->precision) || a->precision == NNB_PREC_SIMT, "conv3d: unknown precision %d",
              a->precision);
  if (a->operand_format == 1) {
    NNB_REQUIRE(a->precision != NNB_PREC_SIMT && a->packed != nullptr, "conv3d: prepared operands need a packed "
                "weight image and a tensor-core precision");
    for (int s = 0; s < a->num_segments; ++s)
      NNB_REQUIRE(a->seg[s].scale == nullptr, "conv3d: prepared operands carry no lazy affine");
    NNB_REQUIRE(conv3d_tc_supported(*a), "conv3d: shape outside the tensor-core envelope");
    return launch_conv3d_tc(*a, st);
  }
  if (a->operand_format == 2) {
    NNB_REQUIRE(a->packed != nullptr && conv3d_tc_supported(*a) && conv3d_tc_raw_operands(*a),
                "conv3d: raw tensor-core operands are outside the z-streaming envelope");
    for (int s = 0; s < a->num_segments; ++s) {
      NNB_REQUIRE(a->seg[s].scale == nullptr || a->seg[s].shift != nullptr, "conv3d: lazy segment without shift");
      NNB_REQUIRE(!a->seg[s].prepared || a->seg[s].scale == nullptr, "conv3d: prepared segments carry no lazy affine");
    }
    return launch_conv3d_tc(*a, st);
  }
  NNB_REQUIRE(a->operand_format == 0, "conv3d: unknown operand_format %d", a->operand_format);
  // Raw float32 operands run on the CUDA-core kernel in plain float32 (used for
  // the few-channel first layer and shapes outside the tensor-core envelope),
  // which also satisfies the requested accuracy.
  return launch_conv3d_simt(*a, st);
}

int32_t nnb_conv3d_raw_operands(const nnb_conv3d_args* a) {
  if (a == nullptr || a->num_segments < 1 || a->num_segments > 2) return 0;
  for (int i = 0; i < 3; ++i)
    if (a->in_dims[i] < 1 || a->out_dims[i] < 1 || a->kernel[i] < 1 || a->stride[i] < 1) return 0;
  return conv3d_tc_raw_operands(*a) ? 1 : 0;
}

int32_t nnb_prepare_operand(const nnb_segment* input, int32_t batch, int64_t voxels, float slope, int32_t precision,
                            float* out, void* stream) {
  NNB_REQUIRE(input != nullptr && out != nullptr, "prepare_operand: null pointer");
  int rc = check_segment(*input, "prepare_operand input");
  if (rc) return rc;
  NNB_REQUIRE(batch >= 1 && voxels >= 1, "prepare_operand: bad shape");
  NNB_REQUIRE(tensor_precision(precision), "prepare_operand: precision %d has no prepared operand", precision);
  return launch_prepare_operand(*input, batch, voxels, slope, operand_kind(precision), out, (cudaStream_t)stream);
}

int64_t nnb_operand_range_events(int32_t reset) { return operand_range_events(reset); }

int64_t nnb_conv3d_packed_bytes(int32_t cout, int32_t kvol, int32_t cin_total, int32_t precision) {
  return conv3d_tc_packed_bytes(cout, kvol, cin_total, precision);
}

int32_t nnb_conv3d_pack(const float* weight, int32_t cout, int32_t kvol, int32_t cin_total, int32_t precision,
                        void* packed, void* stream) {
  NNB_REQUIRE(weight != nullptr && packed != nullptr, "conv3d_pack: null pointer");
  NNB_REQUIRE(cout >= 1 && kvol >= 1 && cin_total >= 1, "conv3d_pack: bad shape");
  return launch_conv3d_pack(weight, cout, kvol, cin_total, precision, packed, (cudaStream_t)stream);
}

int64_t nnb_conv3d_partial_tiles(const nnb_conv3d_args* a) {
  NNB_REQUIRE(a != nullptr, "conv3d_partial_tiles: null args");
  NNB_REQUIRE(positive3(a->out_dims) && positive3(a->kernel) && positive3(a->stride),
              "conv3d_partial_tiles: dims, kernel and stride must be positive");
  if (a->operand_format == 1 || a->operand_format == 2) {
    NNB_REQUIRE(a->num_segments == 1 || a->num_segments == 2, "conv3d_partial_tiles: 1 or 2 input segments");
    return conv3d_tc_partial_tiles(*a);
  }
  return tiles_per_sample((int64_t)a->out_dims[0] * a->out_dims[1] * a->out_dims[2]);
}

int32_t nnb_conv3d_kernel_mode(const nnb_conv3d_args* a) {
  NNB_REQUIRE(a != nullptr, "conv3d_kernel_mode: null args");
  NNB_REQUIRE(positive3(a->in_dims) && positive3(a->out_dims) && positive3(a->kernel) && positive3(a->stride),
              "conv3d_kernel_mode: dims, kernel and stride must be positive");
  if (a->operand_format != 1 && a->operand_format != 2) return 0;
  NNB_REQUIRE(a->num_segments == 1 || a->num_segments == 2, "conv3d_kernel_mode: 1 or 2 input segments");
  return conv3d_tc_mode(*a);
}

int32_t nnb_instance_norm_finalize(const float* partials, int32_t batch, int32_t tiles, int32_t channels,
                                   const float* gamma, const float* beta, float eps, float* scale, float* shift,
                                   void* stream) {
  NNB_REQUIRE(partials && scale && shift, "instance_norm_finalize: null pointer");
  NNB_REQUIRE(batch >= 1 && tiles >= 1 && channels >= 1, "instance_norm_finalize: bad shape");
  NNB_REQUIRE(eps > 0.f, "instance_norm_finalize: eps must be positive");
  return launch_norm_finalize(partials, batch, tiles, channels, gamma, beta, eps, scale, shift,
                              (cudaStream_t)stream);
}

int32_t nnb_conv_transpose3d(const nnb_segment* input, int32_t batch, const int32_t in_dims[3],
                             const int32_t kernel[3], float slope, const float* weight, const float* bias,
                             int32_t cout, const void* packed, int32_t precision, float* out, void* stream) {
  NNB_REQUIRE(input != nullptr, "conv_transpose3d: null input");
  int rc = check_segment(*input, "conv_transpose3d input");
  if (rc) return rc;
  NNB_REQUIRE(batch >= 1 && positive3(in_dims) && positive3(kernel), "conv_transpose3d: bad shape");
  NNB_REQUIRE(weight && out && cout >= 1, "conv_transpose3d: missing weight/output");
  if (packed != nullptr && tensor_precision(precision) && input->channels % 32 == 0 && cout % 32 == 0)
    return launch_conv_transpose_tc(*input, batch, in_dims, kernel, slope, bias, cout, packed, precision, out, 0,
                                    (cudaStream_t)stream);
  return launch_conv_transpose_simt(*input, batch, in_dims, kernel, slope, weight, bias, cout, out,
                                    (cudaStream_t)stream);
}

int32_t nnb_conv_transpose3d_operand(const nnb_segment* input, int32_t batch, const int32_t in_dims[3],
                                     const int32_t kernel[3], float slope, const float* bias, int32_t cout,
                                     const void* packed, int32_t precision, void* out, void* stream) {
  NNB_REQUIRE(input != nullptr, "conv_transpose3d_operand: null input");
  int rc = check_segment(*input, "conv_transpose3d_operand input");
  if (rc) return rc;
  NNB_REQUIRE(batch >= 1 && positive3(in_dims) && positive3(kernel), "conv_transpose3d_operand: bad shape");
  NNB_REQUIRE(out != nullptr && cout >= 1, "conv_transpose3d_operand: missing output");
  const bool operand_precision = precision == NNB_PREC_FP32 || precision == NNB_PREC_BF16 ||
                                 precision == NNB_PREC_TF32;
  if (packed == nullptr || !operand_precision || input->channels % 32 != 0 || cout % 32 != 0) {
    set_error("conv_transpose3d_operand: needs the NNB_PREC_FP32, NNB_PREC_BF16 or NNB_PREC_TF32 tensor-core path "
              "(packed weights, 32-multiple channels)");
    return NNB_E_UNSUPPORTED;
  }
  return launch_conv_transpose_tc(*input, batch, in_dims, kernel, slope, bias, cout, packed, precision,
                                  static_cast<float*>(out), 1, (cudaStream_t)stream);
}

int64_t nnb_conv_transpose3d_packed_bytes(int32_t cout, int32_t ktaps, int32_t cin, int32_t precision) {
  if (cout % 32 != 0) return 0;
  return conv3d_tc_packed_bytes(cout * ktaps, 1, cin, precision);
}

int32_t nnb_conv_transpose3d_pack(const float* weight, int32_t cout, int32_t ktaps, int32_t cin, int32_t precision,
                                  void* packed, void* stream) {
  NNB_REQUIRE(weight != nullptr && packed != nullptr, "conv_transpose3d_pack: null pointer");
  NNB_REQUIRE(cout % 32 == 0 && ktaps >= 1 && cin >= 1, "conv_transpose3d_pack: bad shape");
  return launch_conv3d_pack_rows(weight, cout * ktaps, 1, cin, precision, ktaps, cout, packed, (cudaStream_t)stream);
}

int32_t nnb_residual_join(const nnb_segment* branch, const nnb_segment* skip, int32_t batch, int64_t voxels,
                          float slope, float* out, void* stream) {
  NNB_REQUIRE(branch && skip && out, "residual_join: null pointer");
  int rc = check_segment(*branch, "residual branch");
  if (rc) return rc;
  rc = check_segment(*skip, "residual skip");
  if (rc) return rc;
  NNB_REQUIRE(branch->channels == skip->channels, "residual_join: channel mismatch");
  NNB_REQUIRE(batch >= 1 && voxels >= 1, "residual_join: bad shape");
  return launch_residual_join(*branch, *skip, batch, voxels, slope, out, (cudaStream_t)stream);
}

int32_t nnb_gather_views(const float* volume, int32_t cin, const int32_t vol_dims[3], const int32_t offset[3],
                         const int32_t patch[3], int32_t views, const int32_t* flip_masks, float* out,
                         void* stream) {
  NNB_REQUIRE(volume && out && flip_masks && cin >= 1, "gather_views: bad arguments");
  for (int i = 0; i < 3; ++i)
    NNB_REQUIRE(offset[i] >= 0 && patch[i] >= 1 && offset[i] + patch[i] <= vol_dims[i],
                "gather_views: tile [%d, %d) outside axis %d of size %d", offset[i], offset[i] + patch[i], i,
                vol_dims[i]);
  return launch_gather_views(volume, cin, vol_dims, offset, patch, views, flip_masks, out, (cudaStream_t)stream);
}

int32_t nnb_gather_tiles(const float* volume, int32_t cin, const int32_t vol_dims[3], const int32_t pad_lo[3],
                         int32_t items, const int32_t* offsets, const int32_t* flip_masks, const int32_t patch[3],
                         float* out, int32_t* nonfinite_count, void* stream) {
  NNB_REQUIRE(volume && out && offsets && flip_masks && cin >= 1, "gather_tiles: bad arguments");
  NNB_REQUIRE(positive3(vol_dims) && positive3(patch), "gather_tiles: dimensions must be positive");
  for (int i = 0; i < 3; ++i)
    NNB_REQUIRE(pad_lo[i] >= 0 && pad_lo[i] < patch[i], "gather_tiles: pad_lo[%d] = %d outside [0, patch)", i,
                pad_lo[i]);
  return launch_gather_tiles(volume, cin, vol_dims, pad_lo, items, offsets, flip_masks, patch, out, nonfinite_count,
                             (cudaStream_t)stream);
}

static int check_accumulate(const nnb_segment* features, const int32_t* flip_masks, const int32_t patch[3],
                            const float* seg_weight, const float* seg_bias, int32_t classes, const float* gaussian,
                            const void* acc, const void* normalizer, const int32_t acc_dims[3],
                            const int32_t offset[3], int32_t add_normalizer) {
  NNB_REQUIRE(features && flip_masks && seg_weight && seg_bias && gaussian && acc, "accumulate_tile: null pointer");
  int rc = check_segment(*features, "accumulate features");
  if (rc) return rc;
  NNB_REQUIRE(classes >= 1, "accumulate_tile: classes must be positive");
  NNB_REQUIRE(!add_normalizer || normalizer != nullptr, "accumulate_tile: missing normalizer");
  for (int i = 0; i < 3; ++i)
    NNB_REQUIRE(offset[i] >= 0 && patch[i] >= 1 && offset[i] + patch[i] <= acc_dims[i],
                "accumulate_tile: tile outside accumulator on axis %d", i);
  return NNB_OK;
}

int32_t nnb_accumulate_tile(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                            const int32_t patch[3], float slope, const float* seg_weight, const float* seg_bias,
                            int32_t classes, const float* gaussian, float* acc, float* normalizer,
                            const int32_t acc_dims[3], const int32_t offset[3], int32_t add_normalizer,
                            void* stream) {
  int rc = check_accumulate(features, flip_masks, patch, seg_weight, seg_bias, classes, gaussian, acc, normalizer,
                            acc_dims, offset, add_normalizer);
  if (rc) return rc;
  return launch_accumulate_tile(*features, views, flip_masks, patch, slope, seg_weight, seg_bias, classes, gaussian,
                                acc, normalizer, 0, acc_dims, offset, add_normalizer, views, (cudaStream_t)stream);
}

int32_t nnb_accumulate_views(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                             int32_t view_divisor, const int32_t patch[3], float slope, const float* seg_weight,
                             const float* seg_bias, int32_t classes, const float* gaussian, float* acc,
                             float* normalizer, const int32_t acc_dims[3], const int32_t offset[3],
                             int32_t add_normalizer, void* stream) {
  int rc = check_accumulate(features, flip_masks, patch, seg_weight, seg_bias, classes, gaussian, acc, normalizer,
                            acc_dims, offset, add_normalizer);
  if (rc) return rc;
  return launch_accumulate_tile(*features, views, flip_masks, patch, slope, seg_weight, seg_bias, classes, gaussian,
                                acc, normalizer, 0, acc_dims, offset, add_normalizer, view_divisor,
                                (cudaStream_t)stream);
}

int32_t nnb_accumulate_tile_fp16(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                                 const int32_t patch[3], float slope, const float* seg_weight,
                                 const float* seg_bias, int32_t classes, const float* gaussian, void* acc16,
                                 void* normalizer16, const int32_t acc_dims[3], const int32_t offset[3],
                                 int32_t add_normalizer, void* stream) {
  int rc = check_accumulate(features, flip_masks, patch, seg_weight, seg_bias, classes, gaussian, acc16,
                            normalizer16, acc_dims, offset, add_normalizer);
  if (rc) return rc;
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(acc16) & 1) == 0 && (reinterpret_cast<uintptr_t>(normalizer16) & 1) == 0,
              "accumulate_tile_fp16: half buffers must be 2-byte aligned");
  return launch_accumulate_tile(*features, views, flip_masks, patch, slope, seg_weight, seg_bias, classes, gaussian,
                                acc16, normalizer16, 1, acc_dims, offset, add_normalizer, views,
                                (cudaStream_t)stream);
}

int32_t nnb_fold_add_fp16(const void* acc16, const void* normalizer16, int32_t classes, const int32_t acc_dims[3],
                          const int32_t crop_lo[3], const int32_t crop_dims[3], void* total16, int32_t first_fold,
                          int32_t* invalid_count, void* stream) {
  NNB_REQUIRE(acc16 && normalizer16 && total16 && invalid_count && classes >= 1, "fold_add_fp16: bad arguments");
  for (int i = 0; i < 3; ++i)
    NNB_REQUIRE(crop_lo[i] >= 0 && crop_dims[i] >= 1 && crop_lo[i] + crop_dims[i] <= acc_dims[i],
                "fold_add_fp16: crop outside accumulator on axis %d", i);
  return launch_fold_add_fp16(acc16, normalizer16, classes, acc_dims, crop_lo, crop_dims, total16, first_fold,
                              invalid_count, (cudaStream_t)stream);
}

int32_t nnb_fold_sum_fp16(void* total16, const void* part16, int64_t elements, int32_t* invalid_count,
                          void* stream) {
  NNB_REQUIRE(total16 && part16 && invalid_count && elements >= 1, "fold_sum_fp16: bad arguments");
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(total16) & 1) == 0 && (reinterpret_cast<uintptr_t>(part16) & 1) == 0,
              "fold_sum_fp16: half buffers must be 2-byte aligned");
  return launch_fold_sum_fp16(total16, part16, elements, invalid_count, (cudaStream_t)stream);
}

int32_t nnb_fold_finalize_fp16(void* total16, int32_t classes, int64_t voxels, int32_t folds, float* logits,
                               void* labels, int32_t label_bytes, int32_t* invalid_count, void* stream) {
  NNB_REQUIRE(total16 && invalid_count && classes >= 1 && voxels >= 1 && folds >= 1,
              "fold_finalize_fp16: bad arguments");
  NNB_CUDA_CHECK(cudaMemsetAsync(invalid_count, 0, sizeof(int32_t), (cudaStream_t)stream));
  return launch_fold_finalize_fp16(total16, classes, voxels, folds, logits, labels, label_bytes, invalid_count,
                                   (cudaStream_t)stream);
}

int32_t nnb_normalize_labels(const float* acc, const float* normalizer, int32_t classes, const int32_t acc_dims[3],
                             const int32_t crop_lo[3], const int32_t crop_dims[3], float fold_divisor,
                             float* logits, void* labels, int32_t label_bytes, int32_t* invalid_count,
                             void* stream) {
  NNB_REQUIRE(acc && normalizer && invalid_count && classes >= 1, "normalize_labels: bad arguments");
  NNB_REQUIRE(fold_divisor > 0.f, "normalize_labels: fold_divisor must be positive");
  for (int i = 0; i < 3; ++i)
    NNB_REQUIRE(crop_lo[i] >= 0 && crop_dims[i] >= 1 && crop_lo[i] + crop_dims[i] <= acc_dims[i],
                "normalize_labels: crop outside accumulator on axis %d", i);
  return launch_normalize_labels(acc, normalizer, classes, acc_dims, crop_lo, crop_dims, fold_divisor, logits,
                                 labels, label_bytes, invalid_count, (cudaStream_t)stream);
}

int32_t nnb_restore_class_labels(const nnb_restore_args* a, void* stream) {
  NNB_REQUIRE(a != nullptr, "restore_class_labels: null arguments");
  NNB_REQUIRE(a->logits && a->labels && a->invalid_count, "restore_class_labels: null pointer");
  NNB_REQUIRE(a->half == 0 || a->half == 1, "restore_class_labels: half must be 0 or 1");
  NNB_REQUIRE(a->label_bytes == 1 || a->label_bytes == 2, "restore_class_labels: label_bytes must be 1 or 2");
  // 1-byte labels keep 255 free for the invalid label; 2-byte labels accept the reference's 65536 classes, where
  // the invalid label 65535 is also the top class and only invalid_count tells them apart
  NNB_REQUIRE(a->classes >= 1 && a->classes <= (a->label_bytes == 1 ? 255 : 65536),
              "restore_class_labels: %d classes do not fit %d-byte labels", a->classes, a->label_bytes);
  NNB_REQUIRE(positive3(a->source_dims) && positive3(a->target_dims) && positive3(a->volume_dims),
              "restore_class_labels: dimensions must be positive");
  NNB_REQUIRE(a->class_stride >= 0 && a->source_strides[0] >= 0 && a->source_strides[1] >= 0 &&
                  a->source_strides[2] >= 0,
              "restore_class_labels: strides must be non-negative");
  int seen = 0;
  for (int i = 0; i < 3; ++i) {
    NNB_REQUIRE(a->axes[i] >= 0 && a->axes[i] < 3 && !(seen & (1 << a->axes[i])),
                "restore_class_labels: axes must be a permutation of (0, 1, 2)");
    seen |= 1 << a->axes[i];
    NNB_REQUIRE(a->crop_lo[i] >= 0 && (int64_t)a->crop_lo[i] + a->target_dims[i] <= a->volume_dims[i],
                "restore_class_labels: crop box outside the volume on axis %d", i);
  }
  return launch_restore_labels(*a, (cudaStream_t)stream);
}

}  // extern "C"
