/*
 * nnb.h -- C ABI of the B200 (sm_100a) inference path for nnU-Net 3-D U-Nets.
 *
 * The reference (MedMLX/nnunet-mlx v0.9.0) runs this path through MLX ops and
 * Metal kernels held in Python strings; its "FFI" is `mx.fast.metal_kernel`
 * plus MLX's built-in `mx.conv3d` / `mx.matmul`.  Each entry point below
 * replaces one of those call sites; the citation names the reference file and
 * lines (paths relative to the reference project root).
 *
 * Conventions
 *  - All pointers are device pointers owned by the caller (PyTorch tensors in
 *    the Python host).  The library allocates no memory.
 *  - `stream` is a `cudaStream_t` passed as `void*`; every call is
 *    asynchronous on that stream.
 *  - Every function returns 0 on success or a negative NNB_E* code;
 *    nnb_last_error() returns a message for the calling thread's last error.
 *  - Activations are channels-last float32 (B, D, H, W, C).  An activation
 *    read by a convolution may be "lazy": the raw output of the previous
 *    convolution plus per-(sample, channel) `scale`/`shift` from its instance
 *    norm and a LeakyReLU flag.  Consumers apply y = act(x * scale + shift)
 *    while loading and load 0 for zero-padding taps, so normalised
 *    activations never make an extra round trip through HBM.
 */
#ifndef NNB_H
#define NNB_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NNB_ABI_VERSION 13

enum nnb_status {
  NNB_OK = 0,
  NNB_E_INVALID = -1,     /* bad argument (shape, pointer, alignment) */
  NNB_E_UNSUPPORTED = -2, /* valid request outside the implemented envelope */
  NNB_E_CUDA = -3,        /* a CUDA runtime call failed */
  NNB_E_DEVICE = -4,      /* a device-side check failed (bounded wait expired, bad index) */
  NNB_E_NONFINITE = -5    /* non-finite or non-positive normaliser found */
};

/* Arithmetic of the convolution contractions. */
enum nnb_precision {
  NNB_PREC_FP32 = 0,      /* split fp16 pairs (hi + lo, 3 products): float32-level
                             accuracy; activations must stay below 65504 in magnitude
                             (out-of-range values are counted, see nnb_operand_range_events) */
  NNB_PREC_TF32 = 1,      /* single-pass TF32 tensor cores (fast, looser bound)     */
  NNB_PREC_SIMT = 2,      /* plain float32 FMA on CUDA cores (any shape)            */
  NNB_PREC_FP32_TF32 = 3, /* split TF32 (hi/lo products): float32-level accuracy at any
                             float32 magnitude; half the speed of NNB_PREC_FP32      */
  NNB_PREC_BF16 = 4       /* BF16 inputs, float32 accumulation: activations and weights
                             rounded to bf16, one tensor product per useful product
                             (fast, looser bound)                                    */
};

/* One channel segment of a convolution input (two segments = decoder concat). */
typedef struct nnb_segment {
  const float* data;   /* (B, D, H, W, channels) float32 */
  const float* scale;  /* (B, channels) or NULL for identity */
  const float* shift;  /* (B, channels), required when scale != NULL */
  int32_t channels;
  int32_t leaky;       /* 1: LeakyReLU(slope) after the affine */
  int32_t prepared;    /* operand_format 2 only: 1 = `data` holds nnb_prepare_operand output of the
                          activation for the call's precision (scale must be NULL); 0 = raw */
  int32_t reserved;    /* 0 */
} nnb_segment;

typedef struct nnb_conv3d_args {
  int32_t batch;
  int32_t in_dims[3];   /* D, H, W of every segment */
  int32_t out_dims[3];
  int32_t kernel[3];
  int32_t stride[3];
  int32_t pad[3];
  int32_t num_segments; /* 1 or 2 */
  nnb_segment seg[2];
  float slope;          /* LeakyReLU negative slope used by lazy segments */
  int32_t cout;
  const float* weight;  /* converted layout (cout, kD, kH, kW, cin_total) */
  const void* packed;   /* tensor-core weight image from nnb_conv3d_pack, or NULL */
  const float* bias;    /* (cout) added to the output, or NULL */
  float* out;           /* (B, oD, oH, oW, cout) */
  float* partials;      /* (B, cout, nnb_conv3d_partial_tiles(args), 3) per-tile
                           (sum, M2, n) of the output, or NULL */
  int32_t precision;    /* enum nnb_precision */
  int32_t operand_format; /* 0: raw float32 segments (lazy affine allowed; CUDA-core kernel);
                             1: segments prepared by nnb_prepare_operand for `precision`
                             (tensor-core kernel; scale/shift must be NULL);
                             2: raw float32 segments (lazy affine allowed) read by the
                             tensor-core kernel, which prepares them itself, or segments
                             flagged `prepared` -- only where nnb_conv3d_raw_operands(args)
                             returns 1 */
} nnb_conv3d_args;

/* Library identity. */
int32_t nnb_abi_version(void);
const char* nnb_last_error(void);

/*
 * First device-side error recorded by a kernel since the last reset (0 when
 * none), e.g. a bounded mbarrier wait that expired; `where` receives the wait
 * site.  Synchronises with the device.  No reference counterpart: the
 * reference's Metal kernels have no device-side waits.
 */
int32_t nnb_device_status(int32_t* where, int32_t reset);

/*
 * 3-D convolution with padding, stride and up to two concatenated input
 * segments, optional lazy instance-norm + LeakyReLU per segment, optional
 * bias, and per-tile instance-norm partial statistics of the output.  The
 * tensor-core path (operand_format 1) needs 32-multiple segment channels,
 * 16-byte aligned segments, cout % 16 == 0, kernel <= 15 and stride <= 8 per
 * axis, and at most 1024 K-steps (taps x cin_total / 32).  Replaces `ConvNorm._conv_norm` -> `_unbiased_convolution`
 * (`mx.conv3d`, and the split-K decoder concat) in
 * src/nnunet_mlx/model/network.py:214-269,305-322 and the single-channel
 * Metal kernel src/nnunet_mlx/kernels/metal_single_channel_conv.py:32-97.
 */
int32_t nnb_conv3d(const nnb_conv3d_args* args, void* stream);

/*
 * 1 when the tensor-core path for `args` (shape fields, precision,
 * num_segments and segment channels read) takes raw lazy segments
 * (operand_format 2): NNB_PREC_FP32, NNB_PREC_BF16 or NNB_PREC_TF32 3x3x3
 * stride-1 padding-1 convolutions with <= 32 output channels and a LeakyReLU
 * slope in [0, 1], whose kernel applies the affine + LeakyReLU and the
 * operand conversion (fp16 pair, bf16 or TF32) to each input plane in shared
 * memory (replacing the nnb_prepare_operand pass); 0 otherwise.  Replaces nothing in the reference
 * (MLX materialises the normalised activation,
 * src/nnunet_mlx/kernels/metal_native_norm.py:62-70).
 */
int32_t nnb_conv3d_raw_operands(const nnb_conv3d_args* args);

/*
 * Tensor-core operand preparation: apply a lazy activation's affine +
 * LeakyReLU once per element and write the form the tensor-core convolution
 * gathers:
 *   NNB_PREC_FP32       per voxel and 32-channel group, 64 halves
 *                       [hi(32) | lo(32)], hi = fp16(x), lo = fp16(x - hi);
 *                       |x| >= 65504 increments the range-event counter
 *                       (C % 32 == 0; out holds batch * voxels * C floats' bytes);
 *   NNB_PREC_FP32_TF32  per voxel [hi(C) | lo(C)], hi = x with the 13 low
 *                       mantissa bits cleared, lo = x - hi (2 C floats);
 *   NNB_PREC_TF32       x rounded to TF32 (C floats);
 *   NNB_PREC_BF16       per voxel and 32-channel group, 64 bf16 halves
 *                       [bf16(x)(32) | (32)] (C % 32 == 0; the fp16 pair's
 *                       layout, of which the convolution reads the first half;
 *                       the second half is left unwritten).
 * Replaces the affine pass of
 * src/nnunet_mlx/kernels/metal_native_norm.py:62-70,155-168 (there the
 * normalised activation is materialised in float32).
 */
int32_t nnb_prepare_operand(const nnb_segment* input, int32_t batch, int64_t voxels, float slope,
                            int32_t precision, float* out, void* stream);

/*
 * Count of out-of-range fp16-pair operands on the current device since the
 * last reset: activation elements nnb_prepare_operand(NNB_PREC_FP32) found at
 * or above 65504 in magnitude, plus at least one per affected thread where a
 * tensor-core convolution prepared raw operands itself (operand_format 2);
 * reset != 0 zeroes the counter.
 * Synchronises with the device.  A non-zero count means results computed with
 * NNB_PREC_FP32 since the reset must be recomputed with NNB_PREC_FP32_TF32.
 * No reference counterpart (the reference computes in float32).
 */
int64_t nnb_operand_range_events(int32_t reset);

/*
 * Tiles per sample of the partials nnb_conv3d writes for `args` (only the
 * shape fields, operand_format and num_segments are read): bricks of at most
 * 128 output voxels on the tensor-core path, 128-voxel runs otherwise.
 * Negative: an nnb_status error.  No reference counterpart (MLX reduces
 * statistics in its own norm pass).
 */
int64_t nnb_conv3d_partial_tiles(const nnb_conv3d_args* args);

/*
 * Which kernel nnb_conv3d launches for `args` (the fields nnb_conv3d_partial_tiles
 * reads, plus precision): 0 the CUDA-core kernel (operand_format 0), 1 the
 * tensor-core box kernel, 2 the halo kernel, 3 the z-streaming kernel.
 * Negative: an nnb_status error.  For reporting and profiling; no reference
 * counterpart (MLX chooses its conv3d algorithm internally).
 */
int32_t nnb_conv3d_kernel_mode(const nnb_conv3d_args* args);

/* Bytes of the tensor-core weight image for (cout, kvol, cin_total, precision). */
int64_t nnb_conv3d_packed_bytes(int32_t cout, int32_t kvol, int32_t cin_total, int32_t precision);

/*
 * Build the tensor-core weight image from converted-layout weights: per N-tile
 * and K-step, [W_hi; W_lo] stacked along N -- NNB_PREC_FP32: fp16 rows
 * W0 = fp16(s w), W1 = fp16(s w - W0) in 64-byte swizzled K-major
 * rows, s a power of two per output column (max |s w| < 2^14), followed by
 * the float 1/s of every column; NNB_PREC_FP32_TF32: TF32 hi/lo rows;
 * NNB_PREC_TF32: TF32 rows (128-byte swizzled K-major rows); NNB_PREC_BF16:
 * bf16(w) rows (64-byte swizzled, no column scales).  The image must start on a 1024-byte boundary.  Replaces the
 * weight layout work MLX does inside `mx.conv3d` for
 * src/nnunet_mlx/model/network.py:261-269.
 */
int32_t nnb_conv3d_pack(const float* weight, int32_t cout, int32_t kvol, int32_t cin_total,
                        int32_t precision, void* packed, void* stream);

/*
 * Instance-norm statistics from `tiles` per-tile (sum, M2, n) partials per
 * (sample, channel), laid out (batch, channels, tiles, 3) (Chan's parallel
 * combination in float64) -> per-(sample, channel) scale = gamma*rsqrt(var+eps)
 * and shift = beta - mean*scale.  Replaces the reduction passes of
 * src/nnunet_mlx/kernels/metal_native_norm.py:32-60,92-153 (the affine pass
 * 62-70,155-168 is applied lazily by consumers).
 */
int32_t nnb_instance_norm_finalize(const float* partials, int32_t batch, int32_t tiles,
                                   int32_t channels, const float* gamma, const float* beta,
                                   float eps, float* scale, float* shift, void* stream);

/*
 * No-allocation variant of nnb_conv3d + nnb_instance_norm_finalize (no
 * counterpart in the reference): the per-tile partials live in a fixed
 * device array of NNB_STATIC_PARTIALS_FLOATS floats (16 MiB) inside the
 * library, so the call allocates no device memory.  For callers that cannot
 * allocate between launches -- an FFI host with no device allocator of its
 * own, or a service that reserves all device memory up front (cudaMalloc
 * synchronises the device and can fail under memory pressure).
 *  - args->partials must be NULL; writes args->out plus per-(sample, channel)
 *    scale/shift exactly as nnb_conv3d followed by nnb_instance_norm_finalize.
 *  - Requests needing batch x nnb_conv3d_partial_tiles(args) x cout x 3 floats
 *    beyond the scratch are rejected with NNB_E_UNSUPPORTED (e.g. a batch-8
 *    128^3 32-channel layer needs 12.6 M floats: use nnb_conv3d).
 *  - Nothing needs to start at zero (every partial is written before read).
 *  - One scratch per device: calls overlapping on one device (other streams
 *    or threads) race on it; order them.
 *  - The first call on a device looks the scratch address up
 *    (cudaGetSymbolAddress, with that device current); make it before any
 *    stream capture begins.  The address is looked up again when the
 *    device's current context is not the one it was taken in (after
 *    cudaDeviceReset, for instance), so that first-call rule applies again
 *    after a context change.
 */
#define NNB_STATIC_PARTIALS_FLOATS (4 * 1024 * 1024)
int32_t nnb_conv3d_norm_static(const nnb_conv3d_args* args, const float* gamma, const float* beta,
                               float eps, float* scale, float* shift, void* stream);

/*
 * Non-overlapping transposed convolution (kernel == stride) with lazy input
 * segment and bias.  Replaces `NonOverlappingConvTranspose3d`
 * src/nnunet_mlx/model/network.py:101-174 (matmul + interleave + bias).
 * weight: (cout, kD, kH, kW, cin).  With `packed` (from
 * nnb_conv_transpose3d_pack) and 32-multiple channel counts it runs as a
 * tensor-core GEMM whose epilogue scatters every (tap, channel) block to its
 * up-sampled voxel, and `input` must then be an operand prepared by
 * nnb_prepare_operand for `precision`; otherwise it runs on CUDA cores over
 * the raw (lazy) input.
 */
int32_t nnb_conv_transpose3d(const nnb_segment* input, int32_t batch, const int32_t in_dims[3],
                             const int32_t kernel[3], float slope, const float* weight,
                             const float* bias, int32_t cout, const void* packed, int32_t precision,
                             float* out, void* stream);

/*
 * nnb_conv_transpose3d on the tensor-core path whose output is written
 * directly as the tensor-core operand of the up-sampled activation (the
 * nnb_prepare_operand layout of `precision`, 4 bytes per channel:
 * NNB_PREC_FP32 [hi(32) | lo(32)] halves per 32-channel group, whose
 * out-of-range values count in nnb_operand_range_events; NNB_PREC_BF16
 * [bf16(32) | (32)], the second half left unwritten; NNB_PREC_TF32 TF32
 * values) instead of float32, so the
 * decoder's concat convolution reads it without a preparation pass.
 * Requires `packed`, 32-multiple channel counts and one of those three
 * precisions (else NNB_E_UNSUPPORTED).  Same reference call site as
 * nnb_conv_transpose3d.
 */
int32_t nnb_conv_transpose3d_operand(const nnb_segment* input, int32_t batch, const int32_t in_dims[3],
                                     const int32_t kernel[3], float slope, const float* bias, int32_t cout,
                                     const void* packed, int32_t precision, void* out, void* stream);

/* Bytes of the tensor-core image of a transposed-convolution weight (0: not eligible). */
int64_t nnb_conv_transpose3d_packed_bytes(int32_t cout, int32_t ktaps, int32_t cin, int32_t precision);

/* Build that image (rows = tap * cout + channel) from a (cout, kD, kH, kW, cin) weight. */
int32_t nnb_conv_transpose3d_pack(const float* weight, int32_t cout, int32_t ktaps, int32_t cin,
                                  int32_t precision, void* packed, void* stream);

/*
 * Residual join of `ResidualBlock` / `BottleneckResidualBlock`:
 * out = LeakyReLU(act(branch) + act(skip)) over (rows, channels), where act
 * applies the segment's lazy affine.  Replaces
 * src/nnunet_mlx/model/network.py:511-516,568-573.
 */
int32_t nnb_residual_join(const nnb_segment* branch, const nnb_segment* skip, int32_t batch,
                          int64_t voxels, float slope, float* out, void* stream);

/*
 * Gather one tile of a channel-first (cin, Z, Y, X) volume at `offset` into a
 * channels-last batch of `views` mirrored copies (B = views): view v is
 * flipped along the axes whose bits are set in flip_masks[v].  Replaces the
 * tile slicing and `mx.flip` + `mx.contiguous` of
 * src/nnunet_mlx/prediction/sliding_window.py:408-411,517-518.
 */
int32_t nnb_gather_views(const float* volume, int32_t cin, const int32_t vol_dims[3],
                         const int32_t offset[3], const int32_t patch[3], int32_t views,
                         const int32_t* flip_masks, float* out, void* stream);

/*
 * Gather a batch of `items` (1..8) patches of a channel-first (cin, Z, Y, X)
 * volume into a channels-last (items, P0, P1, P2, cin) batch: item t is the
 * patch at offsets[3t .. 3t+2] of the volume zero-padded by pad_lo before each
 * axis (the reference's _pad_minimum, sliding_window.py:542-562; positions
 * outside the unpadded volume load 0, nothing is materialised), flipped along
 * the axes whose bits are set in flip_masks[t].  Items may come from different
 * tiles (a batch of (tile, view) work units).  Every value read is checked:
 * each thread that read a non-finite value adds 1 to *nonfinite_count (NULL:
 * no check), the reference's finite-input check (sliding_window.py:463-486)
 * folded into the read.  Host arrays: offsets (3 x items), flip_masks (items).
 * Replaces the padding, the tile slicing and `mx.flip` of
 * src/nnunet_mlx/prediction/sliding_window.py:408-411,517-518,542-562.
 */
int32_t nnb_gather_tiles(const float* volume, int32_t cin, const int32_t vol_dims[3],
                         const int32_t pad_lo[3], int32_t items, const int32_t* offsets,
                         const int32_t* flip_masks, const int32_t patch[3], float* out,
                         int32_t* nonfinite_count, void* stream);

/*
 * Fused segmentation head + mirror flip-back + view average + Gaussian-weighted
 * accumulation of one tile: for each tile voxel, logits_v = W . act(x_v[flip_v(p)]) + b
 * for every view in order, pred = (sum_v logits_v) / views, and
 * acc[offset + p] += pred * g[p]; normalizer[offset + p] += g[p] when
 * add_normalizer != 0.  Replaces the seg head (network.py:875-876),
 * `mirrored_prediction` (sliding_window.py:489-527) and the scatter-add of
 * `_accumulate_logits` (sliding_window.py:435-436).
 */
int32_t nnb_accumulate_tile(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                            const int32_t patch[3], float slope, const float* seg_weight,
                            const float* seg_bias, int32_t classes, const float* gaussian,
                            float* acc, float* normalizer, const int32_t acc_dims[3],
                            const int32_t offset[3], int32_t add_normalizer, void* stream);

/*
 * nnb_accumulate_tile for some of a tile's views: the `views` given are summed
 * in order and divided by view_divisor (the tile's full view count, >= views)
 * before the Gaussian weighting, so calls over disjoint groups of a tile's
 * views add up to that tile's mirrored prediction (the groups' float32 sums
 * round separately).  Used when (tile, view) work units are sharded across
 * GPUs.  Replaces the same reference lines as nnb_accumulate_tile.
 */
int32_t nnb_accumulate_views(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                             int32_t view_divisor, const int32_t patch[3], float slope,
                             const float* seg_weight, const float* seg_bias, int32_t classes,
                             const float* gaussian, float* acc, float* normalizer,
                             const int32_t acc_dims[3], const int32_t offset[3],
                             int32_t add_normalizer, void* stream);

/*
 * nnunet-fp16 accumulation mode (reference sliding_window.py:96-113,415-433,
 * 185-186, inference.py:75-90; the mode MedMLX runs and the predict CLI use,
 * medmlx.py:41-42,121-134).  acc16 (AD, AH, AW, C) and normalizer16 (AD, AH, AW)
 * are IEEE half; gaussian holds the float32 values of the half Gaussian
 * (upstream's scaled impulse response).  Per tile voxel the window update is
 * half(f32(acc) + pred * g) and the normaliser half(f32(n) + g), round to
 * nearest even -- the float32 seg head / flip-back / view mean being
 * nnb_accumulate_tile's.
 */
int32_t nnb_accumulate_tile_fp16(const nnb_segment* features, int32_t views, const int32_t* flip_masks,
                                 const int32_t patch[3], float slope, const float* seg_weight,
                                 const float* seg_bias, int32_t classes, const float* gaussian, void* acc16,
                                 void* normalizer16, const int32_t acc_dims[3], const int32_t offset[3],
                                 int32_t add_normalizer, void* stream);

/*
 * One fold of the nnunet-fp16 mode: normalised half logits over the crop,
 * n = half(f32(acc) / f32(norm)), into the channel-first half total
 * (C, crop_dims): the first fold stores n, later folds half(f32(total) + n) in
 * fold order.  invalid_count accumulates voxels with a non-finite n (the
 * caller zeroes it once per fold ensemble).
 */
int32_t nnb_fold_add_fp16(const void* acc16, const void* normalizer16, int32_t classes,
                          const int32_t acc_dims[3], const int32_t crop_lo[3], const int32_t crop_dims[3],
                          void* total16, int32_t first_fold, int32_t* invalid_count, void* stream);

/*
 * nnunet-fp16 fold sum for folds computed on other devices: total16[i] =
 * half(f32(total16[i]) + f32(part16[i])) over `elements` halves, where part16
 * is one fold's normalised half logits (what nnb_fold_add_fp16 stores for a
 * first fold) -- the same IEEE half add nnb_fold_add_fp16 performs for a later
 * fold, so folds summed here in fold order give the single-device total bit
 * for bit.  Non-finite sums add to *invalid_count (not reset).  Replaces the
 * fold accumulation of src/nnunet_mlx/prediction/inference.py:75-85 when the
 * folds run on several GPUs (the reference runs them on one device).
 */
int32_t nnb_fold_sum_fp16(void* total16, const void* part16, int64_t elements, int32_t* invalid_count,
                          void* stream);

/*
 * Fold average of the half total in place, half(f32(total) / folds), then
 * optional float32 channel-first logits of the half values and first-argmax
 * labels (1 or 2 bytes; all-ones for a voxel with a non-finite value, counted
 * in invalid_count, which this call zeroes first).
 */
int32_t nnb_fold_finalize_fp16(void* total16, int32_t classes, int64_t voxels, int32_t folds, float* logits,
                               void* labels, int32_t label_bytes, int32_t* invalid_count, void* stream);

/*
 * Normalise accumulated logits and reduce them to labels over the crop
 * window: q = (acc / normalizer) / fold_divisor; label = first argmax of q;
 * writes channel-first float32 logits (classes, cD, cH, cW) when `logits` is
 * non-NULL and labels (uint8 when label_bytes == 1, uint16 when 2) when
 * `labels` is non-NULL.  A non-finite or non-positive normaliser or a
 * non-finite quotient stores the invalid label (all ones) and sets
 * *invalid_count.  Replaces src/nnunet_mlx/kernels/metal_normalized_labels.py:19-98
 * and the finalize divide of sliding_window.py:169-176.
 */
int32_t nnb_normalize_labels(const float* acc, const float* normalizer, int32_t classes,
                             const int32_t acc_dims[3], const int32_t crop_lo[3],
                             const int32_t crop_dims[3], float fold_divisor, float* logits,
                             void* labels, int32_t label_bytes, int32_t* invalid_count,
                             void* stream);

/*
 * Device restoration of class labels: class logits on the network's grid ->
 * resampled to the cropped original grid -> first-argmax labels -> written
 * into the uncropped volume in the output axis order, in one pass.
 *
 * Interpolation is order-1 (trilinear) on a half-pixel grid with edge-clamped
 * indices: per target index t of an axis with source size S and target size T,
 * c = (t + 0.5) * (S / T) - 0.5, i0 = clamp(floor(c)), i1 = clamp(floor(c) + 1),
 * w1 = c - floor(c), w0 = 1 - w1; the value is the float64 sum over the eight
 * corners, axis-0 corner outermost, of ((v * w_0) * w_1) * w_2, rounded once to
 * the logits' precision (float32, or IEEE half for half logits); the label is
 * the first class with the largest rounded value.  This is the arithmetic of
 * the host spline path at order 1 (scipy.ndimage.zoom, grid_mode, mode
 * "nearest", as called through skimage resize), reproduced operation for
 * operation, so values and labels equal that path's bit for bit.  Voxels of
 * the volume outside the crop box get label 0.  Equal source and target grids
 * reduce to the argmax of the logits.
 *
 * Replaces the fused Metal restoration
 * src/nnunet_mlx/kernels/metal_restore.py:71-139 (kernel), :404-427 (launch),
 * :462-495 (per-axis metadata), its callers :292-334 and :363-401, and the host
 * uncrop + inverse transpose of src/nnunet_mlx/prediction/export.py:363-373.
 * Unlike the Metal kernel (double-single arithmetic, logits limited to
 * FLT_MAX / 16) any finite float32 or half logits are accepted.  Logits must be
 * finite: corners of interpolation weight exactly 0 (every corner of an axis
 * that is not resampled) are not read, so a non-finite value there is not
 * counted in invalid_count, where the host path's sum would turn it into NaN.
 */
typedef struct nnb_restore_args {
  const void* logits;           /* class logits on the source grid (device)                  */
  int32_t half;                 /* 0: float32 logits, 1: IEEE half logits                    */
  int32_t classes;              /* 1 .. 65536 (1 .. 255 for 1-byte labels); with 65536 classes
                                   the invalid label 65535 is also a class: read invalid_count */
  int32_t source_dims[3];       /* source grid (S0, S1, S2)                                  */
  int32_t target_dims[3];       /* resampled grid = crop box extent (T0, T1, T2)             */
  int64_t class_stride;         /* element strides of the logits: class, then axes 0..2      */
  int64_t source_strides[3];    /*   (any layout: (C, S0, S1, S2), (S0, S1, S2, C), views)   */
  int32_t volume_dims[3];       /* uncropped volume in the source axis order                 */
  int32_t crop_lo[3];           /* start of the crop box in the volume                       */
  int32_t axes[3];              /* output axis i is volume axis axes[i] (a permutation)      */
  int32_t label_bytes;          /* 2: uint16 labels, 1: uint8                                */
  void* labels;                 /* output, contiguous, shape volume_dims[axes[i]] (device)    */
  int32_t* invalid_count;       /* device counter: += voxels whose interpolated value is not
                                   finite (their label is all ones); zeroed by the call      */
} nnb_restore_args;

int32_t nnb_restore_class_labels(const nnb_restore_args* args, void* stream);

/* ---------------------------------------------------------------------------
 * Raw-case preprocessing on the device: the step before the sliding window
 * (reference src/nnunet_mlx/data/preprocessing.py:60-163, upstream
 * DefaultPreprocessor.run_case_npy order): transpose to the plans' axis order,
 * crop to the nonzero bounding box, normalise each channel, resample to the
 * target spacing on the torch sampling grid.  All entry points are
 * stream-ordered and allocate nothing; the transpose is folded into the reads
 * of the raw volume (no transposed copy is made).
 * ------------------------------------------------------------------------ */

enum {
  NNB_DTYPE_F32 = 0, NNB_DTYPE_F64 = 1, NNB_DTYPE_I16 = 2,
  NNB_DTYPE_U8 = 3, NNB_DTYPE_U16 = 4, NNB_DTYPE_I32 = 5
};

/* A raw case as read from the image file: contiguous (C, R0, R1, R2) values of
 * `dtype`; plans axis i is raw axis transpose[i] (the plans' transpose_forward). */
typedef struct nnb_raw_case {
  const void* data;        /* device */
  int32_t dtype;           /* NNB_DTYPE_*                                      */
  int32_t channels;
  int32_t raw_dims[3];
  int32_t transpose[3];    /* a permutation of (0, 1, 2)                        */
} nnb_raw_case;

/* Nonzero bounding box of the transposed case.  `bounds` (device int32[8]) gets
 * lo[3], hi[3] (inclusive, plans axis order; lo > hi when no voxel is nonzero),
 * [6] = values that are not finite after conversion to float32, [7] = 0.
 * Replaces the bound projections of crop_to_nonzero,
 * src/nnunet_mlx/data/preprocessing.py:166-217 (and the float32 finiteness
 * check of :104-118). */
int32_t nnb_nonzero_bounds(const nnb_raw_case* raw, int32_t* bounds, void* stream);

/* Hole filling of the nonzero mask inside a crop box (scipy binary_fill_holes,
 * 6-connected background, as resolved at preprocessing.py:340-343).  The box
 * holds every nonzero voxel, so the background outside it is one component
 * that touches every face of the box.  `state` (device int8, contiguous crop
 * box in plans order): 1 = nonzero voxel, 2 = background connected to the
 * outside, 0 = background not (yet) reached.
 *   nnb_fill_holes_init: state of every voxel, background on the box faces = 2.
 *   nnb_fill_holes_sweep: one forward + backward line sweep along each axis,
 *   marking background next to marked background; adds the number of voxels it
 *   marked to *changed (device int32).  Repeat until a sweep marks nothing; the
 *   filled mask is then state != 2. */
int32_t nnb_fill_holes_init(const nnb_raw_case* raw, const int32_t crop_lo[3], const int32_t crop_dims[3],
                            int8_t* state, void* stream);
int32_t nnb_fill_holes_sweep(int8_t* state, const int32_t crop_dims[3], int32_t* changed, void* stream);

/* Cropped, transposed previous-stage labels (cascade input, contiguous int32
 * (1, R0, R1, R2) on the device) with background (0) outside the filled mask set
 * to -1 (preprocessing.py:209-215). */
int32_t nnb_crop_labels(const int32_t* labels, const nnb_raw_case* raw, const int32_t crop_lo[3],
                        const int32_t crop_dims[3], const int8_t* state, int32_t* out, void* stream);

enum {
  NNB_NORM_NONE = 0, NNB_NORM_CT = 1, NNB_NORM_ZSCORE = 2,
  NNB_NORM_RESCALE01 = 3, NNB_NORM_RGB01 = 4
};

/* One channel's plans normalisation (preprocessing.py:272-319).  CT: clip to
 * [lower, upper], subtract mean, divide by divisor = max(std, 1e-8), each
 * already rounded to float32.  Z-score: mean and standard deviation of the
 * selected voxels (all, or the crop mask when use_mask), applied to those
 * voxels only.  Rescale: subtract the minimum, divide by max(max - min, 1e-8).
 * RGB: divide by 255 (values must lie in [0, 255]).  All float32 arithmetic. */
typedef struct nnb_norm_channel {
  int32_t scheme;          /* NNB_NORM_*                                         */
  int32_t use_mask;        /* z-score over the crop mask                         */
  float lower, upper, mean, divisor;   /* CT parameters                          */
} nnb_norm_channel;

/* Bytes of the caller's device workspace for nnb_crop_normalize. */
int64_t nnb_crop_normalize_workspace_bytes(int32_t channels);

/* Crop the transposed raw case to the box and normalise it: `out` is the
 * contiguous float32 (C, crop_dims) result.  `norm` is a HOST array of
 * `channels` entries.  `state` (from nnb_fill_holes_*) is required when a
 * z-score channel uses the mask; with `labels` (the cropped previous stage from
 * nnb_crop_labels) the mask is labels >= 0 instead, as in the reference
 * (preprocessing.py:137, previous-stage foreground stays eligible).  Statistics
 * are float64 sums (mean and standard deviation rounded to float32, as NumPy
 * returns them for float32 data).  `errors` (device int32[4], zeroed by the
 * call): [0] non-finite outputs, [1] RGB values outside [0, 255], [2] z-score
 * channels with an empty selection, [3] = 0.  Channels that need no statistics
 * (none, CT) are normalised while they are cropped, in one pass.  Replaces
 * preprocessing.py:206-207 (crop) and :222-319 (normalisation). */
int32_t nnb_crop_normalize(const nnb_raw_case* raw, const int32_t crop_lo[3], const int32_t crop_dims[3],
                           const nnb_norm_channel* norm, const int8_t* state, const int32_t* labels,
                           void* workspace, float* out, int32_t* errors, void* stream);

enum { NNB_RESIZE_LINEAR = 0, NNB_RESIZE_NEAREST = 1, NNB_RESIZE_NEAREST_EXACT = 2 };
enum { NNB_TIE_LOWEST = 0, NNB_TIE_HIGHEST = 1, NNB_TIE_NEAREST = 2 };

/* One pass of upstream's torch-grid resampler (resample_torch_fornnunet).
 * Per axis scale = float32(S / T).  Nearest modes copy the sample at
 * min(int(scale * (t + s)), S - 1), s = 0 (nearest) or 0.5 (nearest-exact).
 * Linear: coordinate max(scale * (t + 0.5) - 0.5, 0) in float32, indices
 * floor and floor + 1 clamped to S - 1, weights (1 - f, f); image values are
 * the float64 sum over the eight corners (axis 0 outermost) of
 * ((v * w0) * w1) * w2, rounded once to float32; labels score each distinct
 * corner label by the summed 1000 * w0 * w1 * w2 of its corners, rounded
 * float64 -> float32 -> float16, and keep the best score, ties by `tiebreak`
 * (lowest label, highest label, or the nearest sample's label then the lowest).
 * Image values must be finite: corners whose weight product is exactly 0 are
 * not read (their term is +-0 and cannot change the float64 sum).
 * The source is read through element strides, so the separate-axis passes need
 * no moved copy: resample in-plane with the separate axis kept, then that axis.
 * Replaces src/nnunet_mlx/kernels/metal_torch_resample.py:51-131 (kernel),
 * :154-194 (launch) and :196-216 (separate-axis composition). */
typedef struct nnb_torch_resize_args {
  const void* source;           /* float32 image values or int32 labels (device)     */
  int32_t labels;               /* 0: image values, 1: int32 labels in [-1, 32767]  */
  int32_t channels;
  int32_t source_dims[3];
  int64_t channel_stride;       /* element strides of the source                     */
  int64_t source_strides[3];
  int32_t target_dims[3];
  int32_t mode;                 /* NNB_RESIZE_*                                      */
  int32_t tiebreak;             /* NNB_TIE_* (labels with the linear mode)           */
  void* target;                 /* contiguous (C, T0, T1, T2), the source's type     */
} nnb_torch_resize_args;

int32_t nnb_torch_resize(const nnb_torch_resize_args* args, void* stream);

/* Spline resampling of image values (resample_data_or_seg_to_shape; the
 * reference's host path: skimage resize -> scipy.ndimage.zoom(order, mode
 * "nearest", grid_mode=True), src/nnunet_mlx/data/resampling.py:476-502).
 * Every axis in `axes` is resampled as scipy does: order 3 pads it with 12
 * edge samples and prefilters it in float64 (cubic B-spline, pole sqrt(3) - 2,
 * gain 6, causal and anticausal passes with half-sample-symmetric initial
 * values), then samples the coefficients on the half-pixel grid
 * c = (t + 0.5) * (S / T) - 0.5 with the four cubic B-spline weights; order 1
 * interpolates the values with index clamping.  Per output the taps' products
 * ((v * w0) * w1) * w2 (axis 0 outermost) are summed in float64 and rounded
 * once to the target type.  Axes not in `axes` must keep their size and are
 * read plane by plane (the in-plane pass of separate-axis resampling,
 * src/nnunet_mlx/data/resampling.py:268-306).  `coefficients` is a caller
 * workspace of nnb_spline_workspace_bytes(...) bytes. */
typedef struct nnb_spline_resize_args {
  const void* source;           /* float32 or float64 values (device)                  */
  int32_t source_f64;
  int32_t channels;
  int32_t source_dims[3];
  int64_t channel_stride;       /* element strides of the source                       */
  int64_t source_strides[3];
  int32_t target_dims[3];
  int32_t axes;                 /* bit a set: axis a is resampled                       */
  int32_t order;                /* 1 or 3                                              */
  double* coefficients;         /* workspace (device)                                  */
  void* target;                 /* contiguous (C, T0, T1, T2)                          */
  int32_t target_f64;           /* 0: float32 target, 1: float64                       */
} nnb_spline_resize_args;

int64_t nnb_spline_workspace_bytes(int32_t channels, const int32_t source_dims[3], int32_t axes, int32_t order);
int32_t nnb_spline_resize(const nnb_spline_resize_args* args, void* stream);

/* Out-of-plane pass of separate-axis resampling at order 0 (reference
 * resize_out_of_plane / nearest_axis_indices, src/nnunet_mlx/data/resampling.py:379-427):
 * float64 (C, S0, S1, S2) -> float32 (C, T0, T1, T2) where at most one axis
 * changes size; that axis takes index clamp(floor(S / T * (t + 0.5) - 0.5 + 0.5),
 * 0, S - 1) (float64, one rounding per operation); the value is rounded once. */
int32_t nnb_nearest_axis_resize(const double* source, int32_t channels, const int32_t source_dims[3],
                                const int32_t target_dims[3], float* target, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NNB_H */
