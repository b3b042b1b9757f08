"""ctypes binding of the C ABI in ``include/nnb.h`` (library ``_nnb.so``).

The shared library is built in-tree by ``nnunet_mlx_b200.build.build_extension``
(``nvcc -gencode arch=compute_100a,code=sm_100a``).  There is no fallback: if
the library is missing or the GPU is not an sm_100 device, every compute call
raises ``ContractError``.  Nonzero C status codes become ``ContractError``
carrying ``nnb_last_error()``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from nnunet_mlx_b200.errors import ContractError

LIB_PATH = Path(__file__).resolve().parent / "_nnb.so"
ABI_VERSION = 13

PREC_FP32 = 0        # split fp16 pairs on the tensor cores, float32-level accuracy (|activation| < 65504)
PREC_TF32 = 1        # single-pass TF32 tensor cores
PREC_SIMT = 2        # CUDA-core float32
PREC_FP32_TF32 = 3   # split-TF32 hi/lo tensor cores, float32-level accuracy at any magnitude
PREC_BF16 = 4        # bf16 inputs, float32 accumulation (one product per useful product)
TENSOR_PRECISIONS = (PREC_FP32, PREC_TF32, PREC_FP32_TF32, PREC_BF16)
# precisions whose transposed convolution can write the next convolution's operand directly
OPERAND_OUTPUT_PRECISIONS = (PREC_FP32, PREC_TF32, PREC_BF16)
# nnb_conv3d_kernel_mode -> the kernel a convolution launches
KERNEL_MODES = {0: "conv3d_simt_kernel", 1: "conv3d_tc_kernel", 2: "conv3d_halo_kernel", 3: "conv3d_zstream_kernel"}

STATUS = {0: "ok", -1: "invalid argument", -2: "unsupported", -3: "CUDA error", -4: "device check failed",
          -5: "non-finite"}

I32x3 = ctypes.c_int32 * 3


class Segment(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("shift", ctypes.c_void_p),
                ("channels", ctypes.c_int32), ("leaky", ctypes.c_int32), ("prepared", ctypes.c_int32),
                ("reserved", ctypes.c_int32)]


class Conv3dArgs(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("in_dims", I32x3), ("out_dims", I32x3), ("kernel", I32x3),
                ("stride", I32x3), ("pad", I32x3), ("num_segments", ctypes.c_int32), ("seg", Segment * 2),
                ("slope", ctypes.c_float), ("cout", ctypes.c_int32), ("weight", ctypes.c_void_p),
                ("packed", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("partials", ctypes.c_void_p), ("precision", ctypes.c_int32),
                ("operand_format", ctypes.c_int32)]


I64x3 = ctypes.c_int64 * 3


class RestoreArgs(ctypes.Structure):
    _fields_ = [("logits", ctypes.c_void_p), ("half", ctypes.c_int32), ("classes", ctypes.c_int32),
                ("source_dims", I32x3), ("target_dims", I32x3), ("class_stride", ctypes.c_int64),
                ("source_strides", I64x3), ("volume_dims", I32x3), ("crop_lo", I32x3), ("axes", I32x3),
                ("label_bytes", ctypes.c_int32), ("labels", ctypes.c_void_p), ("invalid_count", ctypes.c_void_p)]


# raw-case dtypes, normalisation schemes, torch-grid modes and label tie rules (include/nnb.h)
RAW_DTYPES = {"float32": 0, "float64": 1, "int16": 2, "uint8": 3, "uint16": 4, "int32": 5}
NORM_SCHEMES = {"NoNormalization": 0, "CTNormalization": 1, "ZScoreNormalization": 2,
                "RescaleTo01Normalization": 3, "RGBTo01Normalization": 4}
RESIZE_MODES = {"linear": 0, "nearest": 1, "nearest-exact": 2}
TIEBREAKS = {"lowest": 0, "highest": 1, "nearest": 2}


class RawCase(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("channels", ctypes.c_int32),
                ("raw_dims", I32x3), ("transpose", I32x3)]


class NormChannel(ctypes.Structure):
    _fields_ = [("scheme", ctypes.c_int32), ("use_mask", ctypes.c_int32), ("lower", ctypes.c_float),
                ("upper", ctypes.c_float), ("mean", ctypes.c_float), ("divisor", ctypes.c_float)]


class SplineResizeArgs(ctypes.Structure):
    _fields_ = [("source", ctypes.c_void_p), ("source_f64", ctypes.c_int32), ("channels", ctypes.c_int32),
                ("source_dims", I32x3), ("channel_stride", ctypes.c_int64), ("source_strides", I64x3),
                ("target_dims", I32x3), ("axes", ctypes.c_int32), ("order", ctypes.c_int32),
                ("coefficients", ctypes.c_void_p), ("target", ctypes.c_void_p), ("target_f64", ctypes.c_int32)]


class TorchResizeArgs(ctypes.Structure):
    _fields_ = [("source", ctypes.c_void_p), ("labels", ctypes.c_int32), ("channels", ctypes.c_int32),
                ("source_dims", I32x3), ("channel_stride", ctypes.c_int64), ("source_strides", I64x3),
                ("target_dims", I32x3), ("mode", ctypes.c_int32), ("tiebreak", ctypes.c_int32),
                ("target", ctypes.c_void_p)]


SYMBOLS = {
    "nnb_abi_version": (ctypes.c_int32, []),
    "nnb_last_error": (ctypes.c_char_p, []),
    "nnb_device_status": (ctypes.c_int32, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]),
    "nnb_conv3d": (ctypes.c_int32, [ctypes.POINTER(Conv3dArgs), ctypes.c_void_p]),
    "nnb_conv3d_partial_tiles": (ctypes.c_int64, [ctypes.POINTER(Conv3dArgs)]),
    "nnb_conv3d_norm_static": (ctypes.c_int32, [ctypes.POINTER(Conv3dArgs), ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_conv3d_packed_bytes": (ctypes.c_int64, [ctypes.c_int32] * 4),
    "nnb_operand_range_events": (ctypes.c_int64, [ctypes.c_int32]),
    "nnb_conv3d_raw_operands": (ctypes.c_int32, [ctypes.POINTER(Conv3dArgs)]),
    "nnb_conv3d_kernel_mode": (ctypes.c_int32, [ctypes.POINTER(Conv3dArgs)]),
    "nnb_prepare_operand": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                                             ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_conv3d_pack": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_instance_norm_finalize": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_void_p]),
    "nnb_conv_transpose3d": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32, I32x3, I32x3,
                                              ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                              ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_conv_transpose3d_operand": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32, I32x3, I32x3,
                                                      ctypes.c_float, ctypes.c_void_p, ctypes.c_int32,
                                                      ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                                      ctypes.c_void_p]),
    "nnb_conv_transpose3d_packed_bytes": (ctypes.c_int64, [ctypes.c_int32] * 4),
    "nnb_conv_transpose3d_pack": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                   ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_residual_join": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.POINTER(Segment), ctypes.c_int32,
                                           ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_gather_views": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, I32x3, I32x3, I32x3, ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_gather_tiles": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, I32x3, I32x3, ctypes.c_int32,
                                          ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), I32x3,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_accumulate_views": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32,
                                              ctypes.POINTER(ctypes.c_int32), ctypes.c_int32, I32x3, ctypes.c_float,
                                              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_void_p, ctypes.c_void_p, I32x3, I32x3, ctypes.c_int32,
                                              ctypes.c_void_p]),
    "nnb_accumulate_tile": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32,
                                             ctypes.POINTER(ctypes.c_int32), I32x3, ctypes.c_float,
                                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                             ctypes.c_void_p, ctypes.c_void_p, I32x3, I32x3, ctypes.c_int32,
                                             ctypes.c_void_p]),
    "nnb_accumulate_tile_fp16": (ctypes.c_int32, [ctypes.POINTER(Segment), ctypes.c_int32,
                                                  ctypes.POINTER(ctypes.c_int32), I32x3, ctypes.c_float,
                                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                                  ctypes.c_void_p, ctypes.c_void_p, I32x3, I32x3, ctypes.c_int32,
                                                  ctypes.c_void_p]),
    "nnb_fold_add_fp16": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, I32x3, I32x3, I32x3,
                                           ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_fold_sum_fp16": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_void_p]),
    "nnb_fold_finalize_fp16": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                                ctypes.c_void_p]),
    "nnb_normalize_labels": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, I32x3, I32x3,
                                              I32x3, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_restore_class_labels": (ctypes.c_int32, [ctypes.POINTER(RestoreArgs), ctypes.c_void_p]),
    "nnb_nonzero_bounds": (ctypes.c_int32, [ctypes.POINTER(RawCase), ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_fill_holes_init": (ctypes.c_int32, [ctypes.POINTER(RawCase), I32x3, I32x3, ctypes.c_void_p,
                                             ctypes.c_void_p]),
    "nnb_fill_holes_sweep": (ctypes.c_int32, [ctypes.c_void_p, I32x3, ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_crop_labels": (ctypes.c_int32, [ctypes.c_void_p, ctypes.POINTER(RawCase), I32x3, I32x3, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_crop_normalize_workspace_bytes": (ctypes.c_int64, [ctypes.c_int32]),
    "nnb_crop_normalize": (ctypes.c_int32, [ctypes.POINTER(RawCase), I32x3, I32x3, ctypes.POINTER(NormChannel),
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_void_p]),
    "nnb_torch_resize": (ctypes.c_int32, [ctypes.POINTER(TorchResizeArgs), ctypes.c_void_p]),
    "nnb_spline_workspace_bytes": (ctypes.c_int64, [ctypes.c_int32, I32x3, ctypes.c_int32, ctypes.c_int32]),
    "nnb_spline_resize": (ctypes.c_int32, [ctypes.POINTER(SplineResizeArgs), ctypes.c_void_p]),
    "nnb_nearest_axis_resize": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int32, I32x3, I32x3, ctypes.c_void_p,
                                                 ctypes.c_void_p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load ``_nnb.so`` once; raise ``ContractError`` if it is missing or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("NNB_LIBRARY", LIB_PATH))
    if not path.is_file():
        raise ContractError(f"CUDA extension not built: {path} is missing "
                            "(run nnunet_mlx_b200.build.build_extension())")
    lib = ctypes.CDLL(str(path))
    for name, (restype, argtypes) in SYMBOLS.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.nnb_abi_version() != ABI_VERSION:
        raise ContractError("CUDA extension ABI version mismatch")
    _lib = lib
    return lib


def check(status: int, what: str) -> None:
    if status != 0:
        message = load().nnb_last_error().decode(errors="replace")
        raise ContractError(f"{what} failed ({STATUS.get(status, status)}): {message}")


def device_status(reset: bool = True) -> tuple[int, int]:
    where = ctypes.c_int32(0)
    status = load().nnb_device_status(ctypes.byref(where), 1 if reset else 0)
    return int(status), int(where.value)


def dims3(values) -> ctypes.Array:
    values = tuple(int(v) for v in values)
    if len(values) != 3:
        raise ContractError(f"expected three spatial sizes, got {values}")
    return I32x3(*values)
